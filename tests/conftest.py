"""Shared fixtures. ``gpu`` marks tests that need a B200 (they call the CUDA library)."""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the sm_100a library")
    config.addinivalue_line("markers", "slow: takes more than ~30 s on CPU")


def _load(name, path, package_dir=None):
    if name in sys.modules:
        return sys.modules[name]
    kw = {"submodule_search_locations": [package_dir]} if package_dir else {}
    spec = importlib.util.spec_from_file_location(name, path, **kw)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_package():
    """The product package (its directory name has a hyphen, so import it by path)."""
    pkg_dir = os.path.join(ROOT, "yue2-mlx_b200")
    return _load("yue2_mlx_b200", os.path.join(pkg_dir, "__init__.py"), pkg_dir)


def load_synth():
    return _load("yue2_mlx_b200_synth", os.path.join(ROOT, "yue2-mlx_b200", "synth.py"))


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def synth():
    return load_synth()


@pytest.fixture(scope="session")
def golden():
    def get(name):
        return np.load(os.path.join(GOLDEN, name))
    return get


@pytest.fixture(scope="session")
def tiny_dir(tmp_path_factory, synth):
    """BASELINE config-1 dims, BF16, non-unit norm weights (the tiny_bf16 fixture's model)."""
    d = str(tmp_path_factory.mktemp("tiny"))
    synth.write_converted(d, synth.TINY, seed=0, norm_std=0.1, workers=1)
    return d


@pytest.fixture(scope="session")
def pinned_dir(tmp_path_factory, synth):
    """The YuE2-3B dims model in BF16 (seed 0, unit norms): the golden fixtures' model."""
    d = str(tmp_path_factory.mktemp("pinned"))
    synth.write_converted(d, synth.PINNED, seed=0)
    return d


@pytest.fixture(scope="session")
def pinned(pinned_dir):
    """The pinned model loaded on cuda:0 once for every GPU test module."""
    return load_package().ARModel(pinned_dir)
