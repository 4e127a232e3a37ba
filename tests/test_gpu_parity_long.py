"""Parity at the benchmark configurations' shapes, through the C ABI.

* Long context on the pinned widths (2 layers, 4096-row vocabulary): decode at ~3000
  cached positions against the CPU oracle's full prefill + decode, where every split of
  the decode attention holds several 64-position chunks (the running max/sum/output is
  rescaled across chunks inside a split), for one row and a CFG-style row pair, and with
  the whole context forced into one split per (row, kv head).
* ~9000 cached positions (BASELINE config 4's decode length): every layer of a decode
  step teacher-forced — the layer's input and the cache read back from the engine, its
  output compared with the oracle's layer on those exact inputs — and the head.
* YuE2-3B dims (28 layers): the config-2 capture (512-token prefill, 16 teacher-forced
  steps; semantic logits of every step and ABC logits with the ABC_END row) and the
  config-3 CFG pair (1024-token conditional and 64-token unconditional branches on two
  rows) against upstream golden logits, and every layer of a decode step teacher-forced
  against the oracle.

Tolerances:
* a teacher-forced layer (identical inputs and cache): BASELINE's logits bound, rel-L2 <=
  1e-3, for the typical layer (median) and every head; no single layer beyond two BF16
  ulps (2^-7), the effect of a last-bit flip landing in a BF16-rounded RMSNorm scale;
* model level: twice the radius between two valid BF16 implementations measured on the
  same inputs (the numpy oracle vs upstream PyTorch, recorded with each golden fixture;
  the reference's own rule, tools/limits.py:1-79), with the short-context bounds of the
  other parity tests as the floor on the 2-layer model;
* greedy tokens equal wherever the reference's top-1/top-2 margin exceeds 0.05.
"""
import dataclasses
import json
import os

import numpy as np
import pytest

from oracle import ar_oracle as ora
from tests.conftest import load_package

pytestmark = pytest.mark.gpu


def f(b):
    return ora.bf16_from_bits(b)


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(np.asarray(b, np.float64)))


@pytest.fixture(scope="module")
def yar():
    return load_package()


@pytest.fixture(scope="module")
def wide_long(yar, synth, tmp_path_factory):
    """Pinned widths (2048 / 16x128 / 8x128 / 6144), 2 layers, 4096-row vocabulary and a
    12288-position RoPE table: the decode kernels at production shapes and long contexts."""
    dims = dataclasses.replace(synth.PINNED, layers=2, vocab=4096, context=12288)
    d = str(tmp_path_factory.mktemp("wide_long"))
    synth.write_converted(d, dims, seed=3, norm_std=0.1)
    bits = synth.read_safetensors(os.path.join(d, "ar-bf16.safetensors"))
    return yar.ARModel(d, any_dims=True), ora.OracleAR(bits, dims, bf16=True), dims


def oracle_trace(oracle, prompt, forced, capacity):
    """Oracle chunked prefill (1024-token chunks, as the engine) then teacher-forced steps:
    logits per row [1 + len(forced), vocab] and the cache."""
    cache = oracle.new_cache(capacity)
    h = None
    for s0 in range(0, len(prompt), 1024):
        h = oracle.forward(prompt[s0:s0 + 1024], cache)
    rows = [oracle.project(h[-1], None)[0]]
    for t in forced:
        rows.append(oracle.step(t, cache, None))
    return np.stack(rows), cache


@pytest.fixture(scope="module")
def long3000(wide_long):
    _, oracle, _ = wide_long
    rng = np.random.default_rng(41)
    prompts = [rng.integers(0, 4096, 2980).tolist(), rng.integers(0, 4096, 1500).tolist()]
    forced = rng.integers(0, 4096, 6).tolist()
    traces = [oracle_trace(oracle, p, forced, 3072) for p in prompts]
    return prompts, forced, traces


@pytest.mark.parametrize("rows,splits,persistent", [(1, 0, True), (2, 0, True), (1, 1, True), (2, 1, False),
                                                    (1, 0, False)])
def test_long_context_decode_vs_oracle(yar, wide_long, long3000, rows, splits, persistent):
    """~3000 positions: 47 chunks per (row, kv head). Automatic splits put 3 chunks in each
    of 16 splits (one row) or 6 chunks in each of 8 (two rows); splits=1 puts all 47 in one.
    The second row holds 1500 positions (a CFG pair with unequal branches)."""
    model, _, _ = wide_long
    prompts, forced, traces = long3000
    s = model.session(max_rows=2, max_ctx=3072)
    s.set_persistent(persistent)
    s.set_max_splits(splits)
    s.set_trace(persistent)
    for r in range(rows):
        s.reset(r, 3072)
        s.prefill(r, prompts[r], phase=None)
    got = [[f(s.logits(r, None))] for r in range(rows)]
    for t in forced:
        s.step(list(range(rows)), [t] * rows, phase=None)
        for r in range(rows):
            got[r].append(f(s.logits(r, None)))
    if persistent:
        assert np.any(s.trace()), "the persistent decode kernel did not run"
    for r in range(rows):
        want, cache = traces[r]
        mine = np.stack(got[r])
        # Radius of the pinned-width 2-layer model (oracle FP32 vs FP64 accumulation):
        # max-abs 0.031, rel-L2 0.0073; bounds are about twice that.
        assert np.abs(mine - want).max() <= 0.0625, r
        assert rel_l2(mine, want) <= 0.015, r
        n0 = len(prompts[r])
        # The decode steps' K/V: layer 0 sees identical inputs (last-bit linear flips only);
        # layer 1 sees layer 0's output, attention over the whole context included.
        for layer, flips, bound in ((0, 0.005, 1e-4), (1, 1.0, 0.02)):
            k, v = s.kv(r, layer, n0, len(forced))
            for name, mine_kv in (("k", f(k)), ("v", f(v))):
                theirs = cache[name][layer][:, n0:n0 + len(forced)]
                fl, rl = float(np.mean(mine_kv != theirs)), rel_l2(mine_kv, theirs)
                assert fl <= flips and rl <= bound, (r, layer, name, fl, rl)
        # The prefill's layer-1 K/V across the context (its layer-0 attention ran over up to
        # 2980 positions in 1024-token chunks).
        sel = np.r_[0:64, n0 // 2:n0 // 2 + 64, n0 - 64:n0]
        k, v = s.kv(r, 1, 0, n0)
        for name, mine_kv in (("k", f(k)[:, sel]), ("v", f(v)[:, sel])):
            rl = rel_l2(mine_kv, cache[name][1][:, sel])
            assert rl <= 0.02, (r, name, rl)
    s.close()


def teacher_forced_layers(oracle, s, rows, n_layers, phase):
    """Every layer of the engine's last decode step, teacher-forced: the oracle's layer l
    on the engine's input rows (hidden slot l) and the engine's cache of layer l, against
    the engine's output (slot l + 1); then the final norm + head on the engine's last
    residual rows against the engine's logits. Returns the rel-L2 of every layer (row-major
    over rows) and of every head."""
    layers, heads = [], []
    for r in rows:
        pos = s.position(r) - 1  # the position the step wrote
        for layer in range(n_layers):
            x_in = f(s.hidden(r, layer))[None]
            k, v = s.kv(r, layer, 0, pos + 1)
            kf, vf = f(k), f(v)
            cache = oracle.new_cache(pos + 1)
            cache["k"][layer, :, :pos] = kf[:, :pos]
            cache["v"][layer, :, :pos] = vf[:, :pos]
            out = oracle.layer(layer, x_in, cache, pos)[0]
            mine = f(s.hidden(r, layer + 1))
            layers.append(rel_l2(mine, out))
            # The K/V the step appended: identical inputs, last-bit linear flips only.
            for name, got in (("k", kf[:, pos]), ("v", vf[:, pos])):
                assert np.mean(got != cache[name][layer][:, pos]) <= 0.01, (r, layer, name)
        head = oracle.project(oracle.final_norm(f(s.hidden(r, n_layers))[None]), phase)[0]
        heads.append(rel_l2(f(s.logits(r, phase)), head))
    return layers, heads


def check_layers(layers, heads):
    """Teacher-forced bounds. A layer's FP32 sums in another order leave its BF16 outputs
    equal up to rare last-bit flips; BASELINE's 1e-3 rel-L2 holds for the typical layer
    (median) and the head. Rarely a flip lands in a BF16-rounded RMSNorm scale (a q/k head
    norm or a layer norm), which moves that whole row by one BF16 ulp (2^-8 relative):
    no single layer may exceed two ulps (2^-7)."""
    lay, hd = np.array(layers), np.array(heads)
    stats = dict(median=float(np.median(lay)), p90=float(np.percentile(lay, 90)), max=float(lay.max()),
                 over_1e3=int((lay > 1e-3).sum()), n=int(lay.size), head_max=float(hd.max()))
    assert stats["median"] <= 1e-3 and stats["max"] <= 2.0 ** -7 and stats["head_max"] <= 1e-3, stats
    return stats


@pytest.mark.parametrize("persistent", [True, False])
def test_9000_positions_every_layer_teacher_forced(yar, wide_long, persistent):
    """Row 0 at ~9000 positions (141 chunks per kv head, 8-9 per split) and row 1 at ~4100,
    stepped together: each layer against the oracle on identical inputs (check_layers)."""
    model, oracle, dims = wide_long
    rng = np.random.default_rng(43)
    prompts = [rng.integers(0, 4096, 8990).tolist(), rng.integers(0, 4096, 4100).tolist()]
    s = model.session(max_rows=2, max_ctx=9024)
    s.set_persistent(persistent)
    s.set_layer_dump(True)
    for r in range(2):
        s.reset(r, 9024)
        s.prefill(r, prompts[r], phase=None)
    layers, heads = [], []
    for t in rng.integers(0, 4096, 3).tolist():
        s.step([0, 1], [t, t], phase=None)
        wl, wh = teacher_forced_layers(oracle, s, (0, 1), dims.layers, None)
        layers += wl
        heads += wh
    check_layers(layers, heads)
    s.close()


def _bound(meta_radius, floor):
    """Twice the measured radius between the two valid implementations, never below `floor`."""
    return max(2 * meta_radius["max_abs"], floor[0]), max(2 * meta_radius["rel_l2"], floor[1])


def test_pinned_3b_config2_capture_vs_upstream(yar, pinned, golden):
    """Config 2's shape on the 28-layer model: 512-token prefill, 16 teacher-forced codec
    ids; semantic logits of every row and ABC logits (151,644 columns, ABC_END last) of rows
    0, 8 and 16 against upstream."""
    g = golden("config2_bf16.npz")
    meta = json.loads(str(g["meta"]))
    prompt, forced = g["prompt"].tolist(), g["forced"].tolist()
    abc_rows = meta["abc_rows"]
    for phase, ref_bits, keep in (("semantic", g["semantic_logits"], None), ("abc", g["abc_logits"], abc_rows)):
        s = pinned.session(max_rows=1, max_ctx=544)
        s.reset(0, 544)
        s.prefill(0, prompt, phase=phase)
        rows = [f(s.logits(0, phase))]
        for t in forced:
            s.step([0], [t], phase=phase)
            rows.append(f(s.logits(0, phase)))
        ours = np.stack(rows) if keep is None else np.stack(rows)[keep]
        ref = f(ref_bits)
        max_abs, rel = _bound(meta["oracle_vs_upstream"][phase], (0.0625, 0.01))
        assert np.abs(ours - ref).max() <= max_abs, phase
        assert rel_l2(ours, ref) <= rel, phase
        # Greedy choices must agree where upstream's top-1/top-2 margin exceeds twice the
        # measured radius between two valid implementations: below that either order is
        # within the logit bound (row 0 of the ABC rows has margin 0.078 against a 0.19
        # radius, and the mma.sync and tcgen05 prefill attentions pick differently there).
        srt = np.sort(ref, axis=1)
        sure = srt[:, -1] - srt[:, -2] > 2 * meta["oracle_vs_upstream"][phase]["max_abs"]
        assert sure.any(), phase
        assert (np.argmax(ours, 1)[sure] == np.argmax(ref, 1)[sure]).all(), phase
        if phase == "semantic":
            sel = g["kv_positions"]
            for layer, flips in ((0, 0.02), (27, 1.0)):
                k, v = s.kv(0, layer, 0, 528)
                for name, mine in (("k", f(k)[:, sel]), ("v", f(v)[:, sel])):
                    theirs = f(g[f"{name}_layer{layer}"])
                    assert np.mean(mine != theirs) <= flips, (layer, name)
                    assert rel_l2(mine, theirs) <= (2e-3 if layer == 0 else 0.1), (layer, name)
        s.close()


def test_pinned_3b_cfg_pair_vs_upstream(yar, pinned, golden):
    """Config 3's shape: the conditional (1024 ids) and unconditional (64 ids) branches of one
    CFG request on rows 0 and 1, stepped together with the same tokens (one two-row forward
    per token), each against upstream's own trace of that branch."""
    g = golden("cfg_pair_bf16.npz")
    meta = json.loads(str(g["meta"]))
    forced = g["forced"].tolist()
    s = pinned.session(max_rows=2, max_ctx=1040)
    for r, ids in ((0, g["cond"]), (1, g["uncond"])):
        s.reset(r, len(ids) + 16)
        s.prefill(r, ids.tolist(), phase="semantic")
    out = [[f(s.logits(0, "semantic"))], [f(s.logits(1, "semantic"))]]
    for t in forced:
        s.step([0, 1], [t, t], phase="semantic")
        for r in range(2):
            out[r].append(f(s.logits(r, "semantic")))
    for r, key, name in ((0, "cond_logits", "cond"), (1, "uncond_logits", "uncond")):
        ours, ref = np.stack(out[r]), f(g[key])
        max_abs, rel = _bound(meta["oracle_vs_upstream"][name], (0.0625, 0.01))
        assert np.abs(ours - ref).max() <= max_abs, name
        assert rel_l2(ours, ref) <= rel, name
        srt = np.sort(ref, axis=1)
        sure = srt[:, -1] - srt[:, -2] > 0.05
        assert (np.argmax(ours, 1)[sure] == np.argmax(ref, 1)[sure]).all(), name
    s.close()


def test_pinned_3b_every_layer_teacher_forced(yar, pinned, pinned_dir, golden, synth):
    """All 28 layers and the semantic head of 3B decode steps (config 2's prompt, one row;
    then the CFG pair's two rows) against the oracle on the engine's own inputs and cache
    (check_layers)."""
    bits = synth.read_safetensors(os.path.join(pinned_dir, "ar-bf16.safetensors"))
    oracle = ora.OracleAR(bits, synth.PINNED, bf16=True, lazy=True)
    g = golden("config2_bf16.npz")
    s = pinned.session(max_rows=2, max_ctx=1040)
    s.set_layer_dump(True)
    s.reset(0, 544)
    s.prefill(0, g["prompt"].tolist(), phase="semantic")
    s.step([0], [int(g["forced"][0])], phase="semantic")
    wl, wh = teacher_forced_layers(oracle, s, (0,), 28, "semantic")
    c = golden("cfg_pair_bf16.npz")
    for r, ids in ((0, c["cond"]), (1, c["uncond"])):
        s.reset(r, len(ids) + 16)
        s.prefill(r, ids.tolist(), phase="semantic")
    s.step([0, 1], [int(c["forced"][0])] * 2, phase="semantic")
    wl2, wh2 = teacher_forced_layers(oracle, s, (0, 1), 28, "semantic")
    check_layers(wl + wl2, wh + wh2)
    s.close()
