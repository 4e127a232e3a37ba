"""Build libyue2ar_cuda.so in-tree: nvcc for sm_100a, C++20 host code, static cudart.

    python yue2-mlx_b200/build.py [--force]

Objects go to ``yue2-mlx_b200/_build/``; the library lands next to this file so it
travels with the source tree. Rebuilds only what changed (source or header mtimes).
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libyue2ar_cuda.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def _json_include() -> str:
    """Directory holding nlohmann/json.hpp (header-only; shipped inside the image)."""
    import site
    roots = list(site.getsitepackages()) + [os.path.dirname(os.path.dirname(os.__file__))]
    for r in roots:
        for sub in ("include/cudnn_frontend/thirdparty",):
            d = os.path.join(r, sub)
            if os.path.exists(os.path.join(d, "nlohmann", "json.hpp")):
                return d
    hits = glob.glob("/opt/**/nlohmann/json.hpp", recursive=True) + glob.glob("/usr/include/nlohmann/json.hpp")
    if hits:
        return os.path.dirname(os.path.dirname(hits[0]))
    raise RuntimeError("nlohmann/json.hpp not found")


def _flags() -> list[str]:
    return ARCH + ["-O3", "-lineinfo", "-std=c++20", "--expt-relaxed-constexpr",
                   "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
                   "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-I", _json_include()]


def _stale(obj: str, src: str, headers: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src] + headers)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    flags = _flags()
    jobs = []
    objs = []
    for src in sources:
        obj = os.path.join(OUT_DIR, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, src, headers):
            jobs.append([_nvcc(), *flags, "-c", src, "-o", obj])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, file=sys.stderr)
        return cmd

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(run, jobs))
    if force or jobs or not os.path.exists(LIB):
        link = [_nvcc(), *ARCH, "-shared", "-cudart=static", "-o", LIB + ".tmp", *objs, "-lpthread", "-ldl", "-lrt"]
        run(link)
        os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
