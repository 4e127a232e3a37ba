"""Generate the golden fixtures in this folder from the reference's own PyTorch AR path.

Run in a container that has the reference tree (it is read only, never modified):

    python tests/golden/make_golden.py --reference <path-to-reference-root>

The upstream package ``vendor/yue/src/yue2`` (the only AR implementation of the
reference that runs off-Mac) is imported from that tree; its model, StaticKVCache and
``distribution`` produce every expected value below. Weights come from
``yue2-mlx_b200/synth.py`` (seeded, identical bits on every machine), so the GPU tests
can rebuild the same model without the reference.

Fixtures:
* ``tiny_fp32.npz``: tiny decoder in FP32, prompt of 32 ids
  (``torch.randint`` seed 0), greedy 64 tokens; per-step full-vocab logits and tokens.
* ``tiny_bf16.npz`` — same dims in BF16 with non-unit norm weights (norm_std 0.1);
  per-step logits (BF16 bits), tokens, and K/V of layer 1 at every position.
* ``pinned_bf16.npz`` — YuE2-3B dims, BF16, seed 0: 128-id prompt (seed 1), prefill of
  124 ids then 4 teacher-forced decode steps (the capture shape of the reference's
  ``tools/oracle.py ar``); semantic-slice logits (BF16 bits), full-vocab argmax and
  K/V samples of layers 0 and 27.
* ``config2_bf16.npz`` — BASELINE config-2 shape on the same 3B model: 512-id prompt
  (seed 2), 16 teacher-forced codec ids; semantic logits of every row, ABC logits (text
  rows + ABC_END) of rows 0/8/16, K/V samples of layers 0 and 27, and the radius between
  the numpy oracle and upstream on the same inputs (``meta``).
* ``cfg_pair_bf16.npz`` — BASELINE config-3 shape: conditional prompt of 1024 ids and
  unconditional prompt of 64 ids (seed 3), each branch with its own cache, stepped with
  the same 8 codec ids; semantic logits of both branches and the oracle radius.
* ``sampler_cases.npz`` — upstream ``distribution`` outputs (phase-local) for crafted
  and random cases, plus upstream BF16 CFG mixing, ``penalty ** count`` and RoPE
  ``inv_freq`` values.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def load_synth():
    spec = importlib.util.spec_from_file_location("yar_synth", os.path.join(ROOT, "yue2-mlx_b200", "synth.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["yar_synth"] = mod
    spec.loader.exec_module(mod)
    return mod


synth = load_synth()


def upstream_model(dims, tensors: dict, dtype):
    from yue2.modeling_yue2 import YuE2Config, YuE2ForCausalLM
    cfg = YuE2Config(hidden_size=dims.hidden, intermediate_size=dims.ffn, num_hidden_layers=dims.layers,
                     num_attention_heads=dims.heads, num_key_value_heads=dims.kv_heads,
                     head_dim=dims.head_dim, vocab_size=dims.vocab, rms_norm_eps=dims.eps,
                     rope_theta=dims.theta, max_position_embeddings=dims.context,
                     max_latent_frames=64)
    with torch.device("meta"):
        model = YuE2ForCausalLM(cfg)
    model = model.to_empty(device="cpu").to(dtype)
    state = model.state_dict()
    for name in state:
        state[name].zero_()
    with torch.no_grad():
        for name, value in tensors.items():
            t = torch.from_numpy(np.ascontiguousarray(value))
            if t.dtype == torch.int16 or value.dtype == np.uint16:
                t = torch.from_numpy(np.ascontiguousarray(value).view(np.int16)).view(torch.bfloat16)
            state[name].copy_(t.to(dtype))
    model.eval()
    return model


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def greedy_trace(model, prompt, steps, capacity, dtype):
    from yue2.modeling_yue2 import StaticKVCache
    c = model.config
    cache = StaticKVCache(c.num_hidden_layers, 1, c.num_key_value_heads, capacity, c.head_dim, dtype,
                          torch.device("cpu"))
    logits, tokens = [], []
    with torch.inference_mode():
        out = model(torch.tensor([prompt]), past_key_values=cache, use_cache=True, logits_to_keep=1).logits[:, -1]
        for i in range(steps):
            logits.append(out[0].clone())
            tok = int(out[0].float().argmax())
            tokens.append(tok)
            if i + 1 < steps:
                out = model(torch.tensor([[tok]]), past_key_values=cache, use_cache=True,
                            logits_to_keep=1).logits[:, -1]
    return logits, tokens, cache


def make_tiny(out_dir):
    dims = synth.TINY
    prompt = torch.randint(0, dims.vocab, (32,), generator=torch.Generator().manual_seed(0)).tolist()
    # FP32 (config 1): unrounded float32 draws.
    tensors = synth.f32_tensors(dims, seed=0, std=0.02, norm_std=0.0)
    model = upstream_model(dims, tensors, torch.float32)
    logits, tokens, _ = greedy_trace(model, prompt, 64, 32 + 64, torch.float32)
    np.savez_compressed(os.path.join(out_dir, "tiny_fp32.npz"), prompt=np.array(prompt, np.int32),
                        tokens=np.array(tokens, np.int32),
                        logits=torch.stack(logits).numpy().astype(np.float32),
                        meta=json.dumps({"seed": 0, "std": 0.02, "norm_std": 0.0, "dims": dims.__dict__}))
    # BF16 with non-unit norms.
    with tempfile.TemporaryDirectory() as tmp:
        synth.write_converted(tmp, dims, seed=0, norm_std=0.1, workers=1)
        bits = synth.read_safetensors(os.path.join(tmp, "ar-bf16.safetensors"))
        bits = {k: np.array(v) for k, v in bits.items()}
    model = upstream_model(dims, bits, torch.bfloat16)
    # Layer-0 operator inputs/outputs of a 32-token prefill, to pin each oracle op alone.
    acts = {}
    layer = model.model.layers[0]
    hooks = []
    for name, mod in (("in_norm", layer.input_layernorm), ("q_proj", layer.self_attn.q_proj),
                      ("k_proj", layer.self_attn.k_proj), ("v_proj", layer.self_attn.v_proj),
                      ("q_norm", layer.self_attn.q_norm), ("k_norm", layer.self_attn.k_norm),
                      ("o_proj", layer.self_attn.o_proj), ("post_norm", layer.post_attention_layernorm),
                      ("gate_proj", layer.mlp.gate_proj), ("up_proj", layer.mlp.up_proj),
                      ("down_proj", layer.mlp.down_proj)):
        def hook(mod, inp, out, name=name):
            acts[f"op_{name}_in"] = bf16_bits(inp[0][0])
            acts[f"op_{name}_out"] = bf16_bits(out[0])
        hooks.append(mod.register_forward_hook(hook))
    with torch.inference_mode():
        model(torch.tensor([prompt]), use_cache=False)
    for h in hooks:
        h.remove()
    logits, tokens, cache = greedy_trace(model, prompt, 64, 32 + 64, torch.bfloat16)
    np.savez_compressed(os.path.join(out_dir, "tiny_bf16.npz"), prompt=np.array(prompt, np.int32),
                        tokens=np.array(tokens, np.int32),
                        logits=np.stack([bf16_bits(x) for x in logits]),
                        k_layer1=bf16_bits(cache.key_cache[1][0]), v_layer1=bf16_bits(cache.value_cache[1][0]),
                        meta=json.dumps({"seed": 0, "std": 0.02, "norm_std": 0.1, "dims": dims.__dict__}),
                        **acts)


def make_pinned(out_dir):
    from yue2.modeling_yue2 import StaticKVCache
    from yue2.protocol import CODEC_OFFSET, CODEC_SIZE, MUSIC_END
    dims = synth.PINNED
    prompt = torch.randint(0, dims.vocab, (128,), generator=torch.Generator().manual_seed(1)).tolist()
    with tempfile.TemporaryDirectory() as tmp:
        synth.write_converted(tmp, dims, seed=0, norm_std=0.0)
        bits = synth.read_safetensors(os.path.join(tmp, "ar-bf16.safetensors"))
        model = upstream_model(dims, bits, torch.bfloat16)
        del bits
    torch.set_num_threads(os.cpu_count())
    c = model.config
    cache = StaticKVCache(c.num_hidden_layers, 1, c.num_key_value_heads, 128, c.head_dim, torch.bfloat16,
                          torch.device("cpu"))
    rows = []
    with torch.inference_mode():
        out = model(torch.tensor([prompt[:124]]), past_key_values=cache, use_cache=True, logits_to_keep=1).logits[:, -1]
        rows.append(out[0].clone())
        for tok in prompt[124:]:
            out = model(torch.tensor([[tok]]), past_key_values=cache, use_cache=True, logits_to_keep=1).logits[:, -1]
            rows.append(out[0].clone())
    full = torch.stack(rows)
    sem = full[:, MUSIC_END:CODEC_OFFSET + CODEC_SIZE]
    sel = np.r_[0:16, 60:68, 112:128]
    np.savez_compressed(os.path.join(out_dir, "pinned_bf16.npz"), prompt=np.array(prompt, np.int32),
                        semantic_logits=bf16_bits(sem), full_argmax=full.float().argmax(-1).numpy().astype(np.int32),
                        kv_positions=sel.astype(np.int32),
                        k_layer0=bf16_bits(cache.key_cache[0][0][:, sel]), v_layer0=bf16_bits(cache.value_cache[0][0][:, sel]),
                        k_layer27=bf16_bits(cache.key_cache[27][0][:, sel]), v_layer27=bf16_bits(cache.value_cache[27][0][:, sel]),
                        meta=json.dumps({"seed": 0, "std": 0.02, "norm_std": 0.0, "prefill": 124, "decode": 4}))


def _upstream_trace(model, prefix, forced, capacity):
    """Upstream prefill of ``prefix`` then one teacher-forced step per id of ``forced``:
    the full-vocabulary logits rows (prefill's last position, then each step) and the
    StaticKVCache (modeling_yue2.py:357-400)."""
    from yue2.modeling_yue2 import StaticKVCache
    c = model.config
    cache = StaticKVCache(c.num_hidden_layers, 1, c.num_key_value_heads, capacity, c.head_dim, torch.bfloat16,
                          torch.device("cpu"))
    rows = []
    with torch.inference_mode():
        out = model(torch.tensor([prefix]), past_key_values=cache, use_cache=True, logits_to_keep=1).logits[:, -1]
        rows.append(out[0].clone())
        for tok in forced:
            out = model(torch.tensor([[tok]]), past_key_values=cache, use_cache=True, logits_to_keep=1).logits[:, -1]
            rows.append(out[0].clone())
    return torch.stack(rows), cache


def _phase_slices(full):
    from yue2.protocol import ABC_END, CODEC_OFFSET, CODEC_SIZE, EOD, MUSIC_END
    sem = full[..., MUSIC_END:CODEC_OFFSET + CODEC_SIZE]
    abc = torch.cat([full[..., :EOD], full[..., ABC_END:ABC_END + 1]], dim=-1)
    return sem, abc


def _radius(ours: np.ndarray, ref: np.ndarray) -> dict:
    return {"max_abs": float(np.abs(ours - ref).max()),
            "rel_l2": float(np.linalg.norm(ours - ref) / np.linalg.norm(ref))}


def _oracle_trace(bits, prefix, forced, capacity, phases):
    """The numpy oracle on the same weights and ids: the last prefill row and every step's
    logits per phase (to record the radius between the two valid BF16 implementations)."""
    sys.path.insert(0, ROOT)
    from oracle import ar_oracle as ora
    oracle = ora.OracleAR(bits, synth.PINNED, bf16=True)
    out = {ph: [] for ph in phases}
    cache = oracle.new_cache(capacity)
    h = None
    for s0 in range(0, len(prefix), 1024):
        h = oracle.forward(prefix[s0:s0 + 1024], cache)
    for ph in phases:
        out[ph].append(oracle.project(h[-1], ph)[0])
    for tok in forced:
        h = oracle.forward([tok], cache)
        for ph in phases:
            out[ph].append(oracle.project(h[-1], ph)[0])
    return {ph: np.stack(v) for ph, v in out.items()}


def _pinned_bits():
    with tempfile.TemporaryDirectory() as tmp:
        synth.write_converted(tmp, synth.PINNED, seed=0, norm_std=0.0)
        bits = synth.read_safetensors(os.path.join(tmp, "ar-bf16.safetensors"))
        return {k: np.array(v) for k, v in bits.items()}


ABC_ROWS = (0, 8, 16)  # steps whose ABC-phase logits are kept (151,644 columns each)


def make_config2(out_dir, bits=None):
    """BASELINE config-2 shape on YuE2-3B dims: 512 random prompt ids (full vocabulary),
    then 16 teacher-forced semantic (codec) ids; semantic logits of all 17 rows and ABC
    logits (text rows + ABC_END) of rows ABC_ROWS; layer-0 and layer-27 K/V samples."""
    dims = synth.PINNED
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, dims.vocab, (512,), generator=g).tolist()
    forced = (151853 + torch.randint(0, 32768, (16,), generator=g)).tolist()
    bits = bits if bits is not None else _pinned_bits()
    model = upstream_model(dims, bits, torch.bfloat16)
    full, cache = _upstream_trace(model, prompt, forced, 544)
    del model
    sem, abc = _phase_slices(full)
    sel = np.r_[0:8, 252:260, 504:528]
    orc = _oracle_trace(bits, prompt, forced, 544, ("semantic", "abc"))
    sem_f = sem.float().numpy()
    abc_f = abc[list(ABC_ROWS)].float().numpy()
    meta = {"seed": 0, "std": 0.02, "norm_std": 0.0, "prefill": 512, "decode": 16, "prompt_seed": 2,
            "abc_rows": list(ABC_ROWS),
            "oracle_vs_upstream": {"semantic": _radius(orc["semantic"], sem_f),
                                   "abc": _radius(orc["abc"][list(ABC_ROWS)], abc_f)}}
    print("config2 radius", meta["oracle_vs_upstream"])
    np.savez_compressed(os.path.join(out_dir, "config2_bf16.npz"), prompt=np.array(prompt, np.int32),
                        forced=np.array(forced, np.int32), semantic_logits=bf16_bits(sem),
                        abc_logits=bf16_bits(abc[list(ABC_ROWS)]), kv_positions=sel.astype(np.int32),
                        k_layer0=bf16_bits(cache.key_cache[0][0][:, sel]),
                        v_layer0=bf16_bits(cache.value_cache[0][0][:, sel]),
                        k_layer27=bf16_bits(cache.key_cache[27][0][:, sel]),
                        v_layer27=bf16_bits(cache.value_cache[27][0][:, sel]), meta=json.dumps(meta))


def make_cfg_pair(out_dir, bits=None):
    """BASELINE config-3 shape on YuE2-3B dims: the conditional branch (1024 random ids) and
    the unconditional branch (64 random ids) of one CFG request, each with its own cache,
    stepped with the same 8 teacher-forced codec ids (the loop feeds both branches the one
    sampled token; native/src/sampling.cpp:185-230). Semantic logits of both branches."""
    dims = synth.PINNED
    g = torch.Generator().manual_seed(3)
    cond = torch.randint(0, dims.vocab, (1024,), generator=g).tolist()
    uncond = torch.randint(0, dims.vocab, (64,), generator=g).tolist()
    forced = (151853 + torch.randint(0, 32768, (8,), generator=g)).tolist()
    bits = bits if bits is not None else _pinned_bits()
    model = upstream_model(dims, bits, torch.bfloat16)
    full_c, _ = _upstream_trace(model, cond, forced, 1040)
    full_u, _ = _upstream_trace(model, uncond, forced, 80)
    del model
    sem_c, _ = _phase_slices(full_c)
    sem_u, _ = _phase_slices(full_u)
    orc_c = _oracle_trace(bits, cond, forced, 1040, ("semantic",))["semantic"]
    orc_u = _oracle_trace(bits, uncond, forced, 80, ("semantic",))["semantic"]
    meta = {"seed": 0, "std": 0.02, "norm_std": 0.0, "cond": 1024, "uncond": 64, "decode": 8, "prompt_seed": 3,
            "oracle_vs_upstream": {"cond": _radius(orc_c, sem_c.float().numpy()),
                                   "uncond": _radius(orc_u, sem_u.float().numpy())}}
    print("cfg radius", meta["oracle_vs_upstream"])
    np.savez_compressed(os.path.join(out_dir, "cfg_pair_bf16.npz"), cond=np.array(cond, np.int32),
                        uncond=np.array(uncond, np.int32), forced=np.array(forced, np.int32),
                        cond_logits=bf16_bits(sem_c), uncond_logits=bf16_bits(sem_u), meta=json.dumps(meta))


def make_sampler(out_dir):
    from yue2.protocol import ABC_END, CODEC_OFFSET, CODEC_SIZE, EOD, MUSIC_END, VOCAB_SIZE, Sampling
    from yue2.sampling import distribution, window_penalty

    def project(v, phase):
        if phase == "abc":
            return np.concatenate((v[..., :EOD], v[..., ABC_END:ABC_END + 1]), axis=-1)
        return v[..., MUSIC_END:CODEC_OFFSET + CODEC_SIZE]

    cases = []
    rng = np.random.default_rng(7)

    def add(name, full_logits, sampling, history, step, phase, legacy=False):
        src = torch.from_numpy(full_logits.astype(np.float32)).to(torch.bfloat16)[None]
        out = distribution(src, sampling, history, step, phase, legacy).float().numpy()[0]
        cases.append(dict(name=name, logits=synth.f32_to_bf16_bits(project(src[0].float().numpy(), phase)),
                          expected=project(out, phase).astype(np.float32),
                          sampling=dict(temperature=sampling.temperature, top_p=sampling.top_p,
                                        top_k=sampling.top_k, repetition_penalty=sampling.repetition_penalty,
                                        penalty_window=sampling.penalty_window, min_tokens=sampling.min_tokens,
                                        max_tokens=sampling.max_tokens),
                          history=list(map(int, history)), step=step, phase=phase, legacy=legacy))

    base = np.full(VOCAB_SIZE, -20, np.float32)
    v = base.copy(); v[CODEC_OFFSET:CODEC_OFFSET + 4] = [5, 4, 4, 3]
    add("topk_ties", v, Sampling(top_k=2, top_p=1, min_tokens=0, repetition_penalty=1), [], 0, "semantic")
    v = base.copy(); v[CODEC_OFFSET:CODEC_OFFSET + 4] = [5, 4, 3, 2]
    add("nucleus_keep1", v, Sampling(top_k=4, top_p=.01, min_tokens=0, repetition_penalty=1), [], 0, "semantic")
    v = base.copy(); v[CODEC_OFFSET:CODEC_OFFSET + 3] = [4.5, -4.5, 3]
    hist = [CODEC_OFFSET + 2] * 5 + [CODEC_OFFSET, CODEC_OFFSET, CODEC_OFFSET + 1]
    add("window_expiry", v, Sampling(temperature=.7, top_p=1, top_k=20, min_tokens=0, repetition_penalty=1.2,
                                     penalty_window=3), hist, 0, "semantic")
    v = base.copy(); v[CODEC_OFFSET + CODEC_SIZE - 1] = 3; v[MUSIC_END] = 4; v[EOD] = 100
    add("min_tokens_masks_end", v, Sampling(temperature=1, top_k=1, top_p=1, min_tokens=1), [], 0, "semantic")
    add("end_allowed_after_min", v, Sampling(temperature=1, top_k=1, top_p=1, min_tokens=1), [], 1, "semantic")
    v = base.copy(); v[EOD - 1] = 3; v[ABC_END] = 4; v[EOD] = 100
    add("abc_boundaries_min", v, Sampling(temperature=1, top_k=1, top_p=1, min_tokens=1), [], 0, "abc")
    add("abc_boundaries_end", v, Sampling(temperature=1, top_k=1, top_p=1, min_tokens=1), [], 1, "abc")
    # Random realistic logits (std ~2, BF16 ties are common) with the BASELINE config-2
    # sampler and the reference defaults, with histories inside and outside the phase.
    for i in range(10):
        v = (rng.standard_normal(VOCAB_SIZE) * 2.0).astype(np.float32)
        phase = "semantic" if i < 8 else "abc"
        hist = list(rng.integers(CODEC_OFFSET, CODEC_OFFSET + 64, size=int(rng.integers(0, 120))))
        hist += [int(rng.integers(0, EOD))] * 3
        for t in range(len(hist)):
            v[hist[t]] += 1.5
        if i % 3 == 0:
            s = Sampling(temperature=1.0, top_k=50, top_p=0.93, min_tokens=400, max_tokens=400)
        elif i % 3 == 1:
            s = Sampling()
        else:
            s = Sampling(temperature=.7, top_p=.9, top_k=30, repetition_penalty=1.005, penalty_window=100,
                         min_tokens=32, max_tokens=4096)
        add(f"random_{i}", v, s, hist, int(rng.integers(0, 300)), phase)
    # legacy_off (historical BF16 sampling): the chain in BF16, nucleus keeping >= 3 rows.
    rng_legacy = np.random.default_rng(17)
    v = base.copy(); v[CODEC_OFFSET:CODEC_OFFSET + 5] = [5, 4, 3, 2, 1]
    add("legacy_nucleus_keep3", v, Sampling(top_k=5, top_p=.01, min_tokens=0, repetition_penalty=1), [], 0,
        "semantic", legacy=True)
    for i in range(6):
        v = (rng_legacy.standard_normal(VOCAB_SIZE) * 2.0).astype(np.float32)
        phase = "semantic" if i < 4 else "abc"
        hist = list(rng_legacy.integers(CODEC_OFFSET, CODEC_OFFSET + 64, size=int(rng_legacy.integers(0, 120))))
        for t in range(len(hist)):
            v[hist[t]] += 1.5
        s = (Sampling(temperature=1.0, top_k=50, top_p=0.93, min_tokens=400, max_tokens=400) if i % 2 == 0 else
             Sampling(temperature=.7, top_p=.9, top_k=30, repetition_penalty=1.005, penalty_window=100,
                      min_tokens=32, max_tokens=4096))
        add(f"legacy_random_{i}", v, s, hist, int(rng_legacy.integers(0, 300)), phase, legacy=True)
    # Greedy with penalty.
    v = (rng.standard_normal(VOCAB_SIZE) * 2.0).astype(np.float32)
    hist = list(rng.integers(CODEC_OFFSET, CODEC_OFFSET + 32, size=60))
    add("greedy_penalty", v, Sampling(temperature=0, top_k=5, top_p=.5, min_tokens=0), hist, 3, "semantic")

    # CFG BF16 arithmetic (upstream sampling.py:109).
    cond = torch.from_numpy((rng.standard_normal(4096) * 4).astype(np.float32)).to(torch.bfloat16)
    unc = torch.from_numpy((rng.standard_normal(4096) * 4).astype(np.float32)).to(torch.bfloat16)
    cfg = {}
    for scale in (1.5, 1.01, 3.0):
        cfg[str(scale)] = bf16_bits(unc + scale * (cond - unc))

    # penalty ** count in FP32 (sampling.py:22) and RoPE inv_freq (modeling_yue2.py:144-146).
    alphas = {}
    for p in (1.2, 1.005, 1.1, 0.9):
        freq = torch.arange(0, 101, dtype=torch.float32)
        alphas[str(p)] = (p ** freq).numpy().astype(np.float32)
    inv = {}
    for d, theta in ((128, 1e6), (64, 1e4)):
        inv[f"{d}_{theta}"] = (1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))).numpy()

    payload = {}
    for i, c in enumerate(cases):
        payload[f"c{i}_logits"] = c["logits"]
        finite = np.flatnonzero(np.isfinite(c["expected"]))
        payload[f"c{i}_idx"] = finite.astype(np.int32)
        payload[f"c{i}_val"] = c["expected"][finite]
    payload["cases"] = json.dumps([{k: v for k, v in c.items() if k not in ("logits", "expected")} for c in cases])
    payload["cfg_cond"] = bf16_bits(cond)
    payload["cfg_uncond"] = bf16_bits(unc)
    for k, v in cfg.items():
        payload[f"cfg_{k}"] = v
    for k, v in alphas.items():
        payload[f"alpha_{k}"] = v
    for k, v in inv.items():
        payload[f"invfreq_{k}"] = v
    np.savez_compressed(os.path.join(out_dir, "sampler_cases.npz"), **payload)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", choices=["tiny", "pinned", "sampler", "config2", "cfg"], default=None)
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "vendor", "yue", "src"))
    torch.set_num_threads(os.cpu_count())
    if args.only in (None, "sampler"):
        make_sampler(HERE)
    if args.only in (None, "tiny"):
        make_tiny(HERE)
    if args.only in (None, "pinned"):
        make_pinned(HERE)
    if args.only in (None, "config2", "cfg"):
        bits = _pinned_bits()
        if args.only in (None, "config2"):
            make_config2(HERE, bits)
        if args.only in (None, "cfg"):
            make_cfg_pair(HERE, bits)


if __name__ == "__main__":
    main()
