"""Tensor parallelism: the split plan on CPU (gloo ranks) and the NCCL path on 2 GPUs.

CPU tests (no GPU; they call the library's host-only split functions):
* the plan covers every q/k/v row, O column, gate/up row and down column exactly once
  across ranks, and a rank's query heads are exactly those of its KV heads (GQA groups
  stay whole);
* the head slices cover every phase column exactly once;
* on two gloo ranks, a decoder layer computed from each rank's rows of every weight
  (attention heads, hidden rows of O and down, FFN rows of gate/up), with each output
  block all-gathered, and the LM head computed by column slices, equal the whole model's
  layer and head (FP64, to rounding: numpy's BLAS blocks products by matrix shape).

GPU test (two GPUs, torchrun): the tensor-parallel model against the one-GPU model on the
same weights — logits bit-identical (every value is computed by one rank with the one-GPU
kernels and reduction order), tokens identical on every rank and to one GPU.
"""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from tests.conftest import ROOT, load_package


@pytest.fixture(scope="module")
def yar():
    return load_package()


@pytest.mark.parametrize("dims", [(2048, 16, 8, 128, 6144), (256, 4, 2, 64, 688)])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_covers_every_row_once(yar, dims, world):
    hidden, heads, kv, hd, ffn = dims
    if kv % world or ffn % world or (ffn // world) % 8 or hidden % (8 * world):
        with pytest.raises(yar.YarError):
            yar.tp_plan(hidden, heads, kv, hd, ffn, 0, world)
        return
    seen = {k: np.zeros(n, int) for k, n in (("q", heads * hd), ("kv", kv * hd), ("ffn", ffn), ("h", hidden))}
    group = heads // kv
    for r in range(world):
        p = yar.tp_plan(hidden, heads, kv, hd, ffn, r, world)
        for k in seen:
            seen[k][p[f"{k}_row0"]:p[f"{k}_row0"] + p[f"{k}_rows"]] += 1
            assert p[f"{k}_row0"] == r * p[f"{k}_rows"]  # rank blocks in rank order
        q_heads = set(range(p["q_row0"] // hd, (p["q_row0"] + p["q_rows"]) // hd))
        kv_heads = set(range(p["kv_row0"] // hd, (p["kv_row0"] + p["kv_rows"]) // hd))
        assert {h // group for h in q_heads} == kv_heads
        assert p["q_rows"] % hd == 0 and p["kv_rows"] % hd == 0 and p["h_rows"] % 8 == 0
    assert all((v == 1).all() for v in seen.values())


@pytest.mark.parametrize("width", [32769, 151644, 4096, 5, 8])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_slices_cover_every_column_once(yar, width, world):
    seen = np.zeros(width, int)
    for r in range(world):
        b, e = yar.tp_head_slice(width, r, world)
        assert 0 <= b <= e <= width
        # Ranges start on a 128-column block (a whole tcgen05 tile of the batched head stays
        # within one rank, computed as on one GPU).
        assert b % 128 == 0 or b == width
        seen[b:e] += 1
    assert (seen == 1).all()


def test_plan_rejects_bad_ranks(yar):
    for rank, world in ((2, 2), (-1, 2), (0, 0)):
        with pytest.raises(yar.YarError):
            yar.tp_plan(2048, 16, 8, 128, 6144, rank, world)


# --- gloo decomposition (two CPU ranks) -------------------------------------------------

def _rms(x, w, eps=1e-6):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def _rope(x, pos, theta=1e6):
    d = x.shape[-1]
    inv = 1.0 / theta ** (np.arange(0, d, 2) / d)
    ang = pos[:, None] * inv[None, :]
    c, s = np.cos(ang), np.sin(ang)
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def _attention(x, w, hd, group, q_sl, kv_sl):
    """Causal attention output of the query heads in q_sl (whose KV heads are kv_sl) over
    the T rows of x, [T][heads in q_sl * hd]; FP64."""
    T = x.shape[0]
    h = _rms(x, w["ln1"])
    q = (h @ w["q"][q_sl].T).reshape(T, -1, hd)
    k = (h @ w["k"][kv_sl].T).reshape(T, -1, hd)
    v = (h @ w["v"][kv_sl].T).reshape(T, -1, hd)
    pos = np.arange(T, dtype=np.float64)
    q = np.stack([_rope(_rms(q[:, i], w["qn"]), pos) for i in range(q.shape[1])], 1)
    k = np.stack([_rope(_rms(k[:, i], w["kn"]), pos) for i in range(k.shape[1])], 1)
    mask = np.triu(np.full((T, T), -np.inf), 1)
    outs = []
    for i in range(q.shape[1]):
        sc = q[:, i] @ k[:, i // group].T / np.sqrt(hd) + mask
        p = np.exp(sc - sc.max(-1, keepdims=True))
        outs.append((p / p.sum(-1, keepdims=True)) @ v[:, i // group])
    return np.concatenate(outs, -1)


def _swiglu(x, w, f_sl):
    h = _rms(x, w["ln2"])
    g, u = h @ w["gate"][f_sl].T, h @ w["up"][f_sl].T
    return g / (1 + np.exp(-g)) * u


def _weights(heads, kv, hd, ffn, H, V, seed=0):
    rng = np.random.default_rng(seed)
    n = lambda *s: rng.normal(0, 0.05, s)  # noqa: E731
    return {"ln1": 1 + n(H), "ln2": 1 + n(H), "qn": 1 + n(hd), "kn": 1 + n(hd), "q": n(heads * hd, H),
            "k": n(kv * hd, H), "v": n(kv * hd, H), "o": n(H, heads * hd), "gate": n(ffn, H), "up": n(ffn, H),
            "down": n(H, ffn), "head": n(V, H), "norm": 1 + n(H)}


def _gloo_rank(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sys.path.insert(0, ROOT)
    from tests.conftest import load_package as lp
    yar = lp()
    heads, kv, hd, ffn, H, V, T = 4, 2, 64, 688, 256, 301, 7
    w = _weights(heads, kv, hd, ffn, H, V)
    x = np.random.default_rng(1).normal(0, 1, (T, H))
    p = yar.tp_plan(H, heads, kv, hd, ffn, rank, world)
    sl = {k: slice(p[f"{k}_row0"], p[f"{k}_row0"] + p[f"{k}_rows"]) for k in ("q", "kv", "ffn", "h")}

    def gather(block):
        """Every rank's column block (rank order) side by side: the engine's all-gather."""
        parts = [torch.zeros_like(torch.from_numpy(block)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(block)))
        return np.concatenate([t.numpy() for t in parts], axis=1)

    attn = gather(_attention(x, w, hd, heads // kv, sl["q"], sl["kv"]))
    x1 = gather(x[:, sl["h"]] + attn @ w["o"][sl["h"]].T)
    mlp = gather(_swiglu(x1, w, sl["ffn"]))
    x2 = gather(x1[:, sl["h"]] + mlp @ w["down"][sl["h"]].T)
    hn = _rms(x2, w["norm"])
    b, e = yar.tp_head_slice(V, rank, world)
    parts = [None] * world
    dist.all_gather_object(parts, (b, e, hn @ w["head"][b:e].T))
    if rank == 0:
        logits = np.zeros((T, V))
        for b2, e2, m in parts:
            logits[:, b2:e2] = m
        full = slice(None)
        y1 = x + _attention(x, w, hd, heads // kv, full, full) @ w["o"].T
        y2 = y1 + _swiglu(y1, w, full) @ w["down"].T
        ref = _rms(y2, w["norm"]) @ w["head"].T
        np.save(os.path.join(out_dir, "err.npy"), np.array([np.abs(x2 - y2).max(), np.abs(logits - ref).max()]))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_reassemble_the_whole_layer(tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(_gloo_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    err = np.load(tmp_path / "err.npy")
    assert err[0] < 1e-12 and err[1] < 1e-12, err  # FP64 BLAS blocks by shape


# --- two GPUs ---------------------------------------------------------------------------

@pytest.mark.gpu
def test_tensor_parallel_two_gpus_match_one_gpu(synth, tmp_path):
    """Run on a box with at least two GPUs (skipped on one): TP=2 against TP=1."""
    import dataclasses
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    small = str(tmp_path / "wide2")
    synth.write_converted(small, dataclasses.replace(synth.PINNED, layers=2, vocab=4096, context=4096), seed=3,
                          norm_std=0.1)
    big = str(tmp_path / "vocab")
    synth.write_converted(big, dataclasses.replace(synth.PINNED, layers=2, context=4096), seed=4, norm_std=0.1)
    out = str(tmp_path / "tp.json")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "900", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "tp_worker.py"), small, big, out]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if r.returncode != 0:
        print(r.stdout[-20000:])
        print(r.stderr[-20000:])
    assert r.returncode == 0, "the tensor-parallel ranks failed (their output is printed above)"
    res = json.load(open(out))
    assert res["dims_tp"]["heads"] == 8 and res["dims_tp"]["kv_heads"] == 4 and res["dims_tp"]["ffn"] == 3072
    print(json.dumps(res))
    for key in ("full_rows1", "full_rows2", "full_rows1_per_op", "full_rows2_per_op", "semantic", "abc", "batch"):
        assert res[key]["bit_identical"], (key, res[key])
        assert res[key].get("same_on_all_ranks", True), key
    assert res["semantic"]["width"] == 32769 and res["abc"]["width"] == 151644
    assert res["generate"]["ranks_agree"] and res["generate"]["equal_to_one_gpu"]
    assert res["generate"]["tensor_parallel"] == 2 and len(res["generate"]["tokens"]) == 24
    assert res["generate"]["tp_exchange"] == "peer_stores"
    assert res["batch"]["ranks_agree"] and res["batch"]["equal_to_one_gpu"]
    assert res["batch"]["forward"] == "batched_tcgen05"
