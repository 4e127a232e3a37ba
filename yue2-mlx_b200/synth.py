"""Seeded synthetic checkpoints in the converted AR layout.

There is no real YuE2 checkpoint on these machines, so every test, the bench and the
CPU baseline run on weights drawn here. The directory this module writes has exactly
the layout ``lyra prepare`` produces for the AR partition and which ``ARModel`` loads
(native/src/ar.cpp:133-238, native/src/conversion.cpp:203-275, :383-389, :552-565):

* ``config.json``      — the generator config (conversion.cpp:203-221);
* ``conversion.json``  — schema-1 manifest with a ``precisions.bf16`` record;
* ``ar-bf16.safetensors`` — the AR tensors only, BF16, row-major ``[out, in]``;
* ``ar-8bit.safetensors`` / ``ar-4bit.safetensors`` (``precisions`` naming "8bit" /
  "4bit") — the same tensors with every linear weight (q/k/v/o, gate/up/down, LM head;
  not the embedding) in affine group-64 form, as ``lyra prepare`` writes it
  (conversion.py:596-620, :651-735): the packed ``.weight`` as U32 ``[out, in * bits / 32]``
  (element (32 / bits) i + j in bits (bits j).. of word i; at 8 bits the words'
  little-endian bytes are the elements in order) and BF16 ``.scales`` / ``.biases``
  ``[out, in / 64]``; ``w ~= scale * q + bias`` per 64-column group.

Weights: every matrix (embedding and LM head included) is N(0, std) with std 0.02,
drawn with numpy's PCG64 ``standard_normal`` in float32, multiplied by float32(std) and
rounded to BF16 (round to nearest even). Draws are made in row blocks of at most
``BLOCK_ELEMS`` elements, each block seeded by ``[seed, tensor_index, block_index]``, so
any tensor or row range can be regenerated alone and blocks can be drawn in parallel
with identical bits on any machine running the same numpy. Norm weights are 1.0 unless
``norm_std`` > 0, in which case they are ``1 + N(0, norm_std)`` (tests use that so the
norm-weight rounding point is exercised).
"""
from __future__ import annotations

import json
from concurrent.futures import ThreadPoolExecutor
import os
from dataclasses import asdict, dataclass

import numpy as np

BLOCK_ELEMS = 1 << 22


@dataclass(frozen=True)
class Dims:
    hidden: int = 2048
    layers: int = 28
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 6144
    vocab: int = 184704
    eps: float = 1e-6
    theta: float = 1e6
    context: int = 24576


PINNED = Dims()
"""The YuE2-3B AR dims the reference pins (native/src/ar.cpp:164-169)."""

TINY = Dims(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, ffn=688,
            vocab=4096, eps=1e-6, theta=1e4, context=2048)
"""BASELINE config 1: the tiny LLaMA-style decoder used for fast parity checks."""


def tensor_specs(d: Dims) -> list[tuple[str, tuple[int, ...]]]:
    """AR tensors in canonical order; the index in this list seeds each tensor."""
    specs = [("model.embed_tokens.weight", (d.vocab, d.hidden)),
             ("lm_head.weight", (d.vocab, d.hidden)),
             ("model.norm.weight", (d.hidden,))]
    q, kv = d.heads * d.head_dim, d.kv_heads * d.head_dim
    for i in range(d.layers):
        p = f"model.layers.{i}."
        specs += [(p + "input_layernorm.weight", (d.hidden,)),
                  (p + "post_attention_layernorm.weight", (d.hidden,)),
                  (p + "self_attn.q_proj.weight", (q, d.hidden)),
                  (p + "self_attn.k_proj.weight", (kv, d.hidden)),
                  (p + "self_attn.v_proj.weight", (kv, d.hidden)),
                  (p + "self_attn.o_proj.weight", (d.hidden, q)),
                  (p + "self_attn.q_norm.weight", (d.head_dim,)),
                  (p + "self_attn.k_norm.weight", (d.head_dim,)),
                  (p + "mlp.gate_proj.weight", (d.ffn, d.hidden)),
                  (p + "mlp.up_proj.weight", (d.ffn, d.hidden)),
                  (p + "mlp.down_proj.weight", (d.hidden, d.ffn))]
    return specs


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round float32 to BF16 (nearest, ties to even) and return the uint16 bit pattern."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).copy()
    u += np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    return (u >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def _blocks(shape: tuple[int, ...]):
    rows = shape[0]
    cols = int(np.prod(shape[1:])) if len(shape) > 1 else 1
    per = max(1, BLOCK_ELEMS // cols)
    for b, r0 in enumerate(range(0, rows, per)):
        yield b, r0, min(rows, r0 + per), cols


def draw_block(seed: int, tidx: int, block: int, n: int, std: float) -> np.ndarray:
    rng = np.random.default_rng([seed, tidx, block])
    a = rng.standard_normal(n, dtype=np.float32)
    a *= np.float32(std)
    return a


def tensor_f32(shape, tidx: int, seed: int, std: float, norm_std: float,
               rows: tuple[int, int] | None = None) -> np.ndarray:
    """Float32 draws of one tensor (or rows [r0, r1) of it) before BF16 rounding."""
    if len(shape) == 1:
        if norm_std > 0:
            return np.float32(1.0) + draw_block(seed, tidx, 0, shape[0], norm_std)
        return np.ones(shape[0], dtype=np.float32)
    r0, r1 = rows if rows is not None else (0, shape[0])
    out = np.empty((r1 - r0,) + tuple(shape[1:]), dtype=np.float32)
    for b, b0, b1, cols in _blocks(tuple(shape)):
        if b1 <= r0 or b0 >= r1:
            continue
        vals = draw_block(seed, tidx, b, (b1 - b0) * cols, std).reshape((b1 - b0,) + tuple(shape[1:]))
        s0, s1 = max(b0, r0), min(b1, r1)
        out[s0 - r0:s1 - r0] = vals[s0 - b0:s1 - b0]
    return out


def tensor_bits(shape, tidx: int, seed: int, std: float, norm_std: float,
                rows: tuple[int, int] | None = None) -> np.ndarray:
    """BF16 bits of one tensor (or of rows [r0, r1) of it), as the writer produces them."""
    return f32_to_bf16_bits(tensor_f32(shape, tidx, seed, std, norm_std, rows))


def f32_tensors(dims: Dims, seed: int = 0, std: float = 0.02, norm_std: float = 0.0) -> dict:
    """All AR tensors as unrounded float32 (BASELINE config 1 runs the tiny model in FP32)."""
    return {name: tensor_f32(shape, i, seed, std, norm_std)
            for i, (name, shape) in enumerate(tensor_specs(dims))}


def config_json(d: Dims) -> dict:
    """Generator config in the shape conversion.cpp:203-221 pins."""
    return {"model_type": "yue2", "architectures": ["YuE2ForCausalLM"],
            "hidden_size": d.hidden, "num_hidden_layers": d.layers,
            "num_attention_heads": d.heads, "num_key_value_heads": d.kv_heads,
            "head_dim": d.head_dim, "intermediate_size": d.ffn, "vocab_size": d.vocab,
            "rms_norm_eps": d.eps, "rope_theta": d.theta,
            "max_position_embeddings": d.context, "tie_word_embeddings": False,
            "latent_type": "vae", "latent_dim": 64, "max_latent_frames": d.context,
            "timestep_shift": 1.0, "hidden_act": "silu", "dtype": "bfloat16"}


def _layout(d: Dims):
    specs = tensor_specs(d)
    header, off = {}, 0
    for name, shape in specs:
        n = int(np.prod(shape)) * 2
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [off, off + n]}
        off += n
    header["__metadata__"] = {"format": "mlx", "partition": "ar", "precision": "bfloat16"}
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * ((8 - (len(raw) % 8)) % 8)
    return specs, header, raw


def _fill_job(args):
    path, data_start, offset, shape, tidx, seed, std, norm_std, r0, r1 = args
    bits = tensor_bits(shape, tidx, seed, std, norm_std, rows=(r0, r1) if len(shape) > 1 else None)
    cols = int(np.prod(shape[1:])) if len(shape) > 1 else 1
    mm = np.memmap(path, dtype=np.uint16, mode="r+")
    start = (data_start + offset) // 2 + (r0 * cols if len(shape) > 1 else 0)
    mm[start:start + bits.size] = bits.reshape(-1)
    mm.flush()
    del mm
    return bits.size


QUANT_GROUP = 64


def linear_names(dims: Dims) -> list[str]:
    """The weights the 8-bit artifact quantizes: every linear layer's (linear_only), not
    the embedding table (ar.cpp:204-222 lists them)."""
    return [name for name, shape in tensor_specs(dims) if len(shape) == 2 and name != "model.embed_tokens.weight"]


def quantize_affine(w: np.ndarray, bits: int = 8) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Affine group-64 quantization of a float32 ``[rows, cols]`` matrix to ``bits`` (8 or
    4), after the published scheme of ``mlx.core.quantize`` (mode "affine"; MLX 0.32.2 is
    the version conversion.py:31 pins): per 64-column group, scale = (max - min) / (2^bits
    - 1) (at least 1e-7) and bias = min, each stored as BF16, and q = round((w - bias) /
    scale) in [0, 2^bits - 1], formed with the stored values. Returns (q uint8 [rows, cols],
    scale bits, bias bits)."""
    top = (1 << bits) - 1
    rows, cols = w.shape
    g = np.asarray(w, dtype=np.float32).reshape(rows, cols // QUANT_GROUP, QUANT_GROUP)
    lo, hi = g.min(axis=2), g.max(axis=2)
    scale = np.maximum((hi - lo) / np.float32(top), np.float32(1e-7)).astype(np.float32)
    s_bits, b_bits = f32_to_bf16_bits(scale), f32_to_bf16_bits(lo)
    s = bf16_bits_to_f32(s_bits)[:, :, None]
    b = bf16_bits_to_f32(b_bits)[:, :, None]
    q = np.clip(np.rint((g - b) / s), 0, top).astype(np.uint8).reshape(rows, cols)
    return q, s_bits, b_bits


def quantize_affine8(w: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    return quantize_affine(w, 8)


def pack_words(q: np.ndarray, bits: int) -> np.ndarray:
    """The U32 words of ``q`` [rows, cols] at ``bits`` per element: element (32 / bits) i + j
    in bits (bits j)..(bits j + bits - 1) of word i; as little-endian bytes."""
    rows, cols = q.shape
    if bits == 8:
        return np.ascontiguousarray(q, dtype=np.uint8).view(np.uint32)
    n = q.astype(np.uint32).reshape(rows, cols // 8, 8)
    return (n << (np.arange(8, dtype=np.uint32) * np.uint32(4))).sum(axis=2, dtype=np.uint32)


def _q_layout(d: Dims, bits: int):
    """Header of ar-<bits>bit.safetensors: the BF16 file's tensors in the same order, every
    linear as ``.weight`` (U32), ``.scales`` and ``.biases`` (BF16)."""
    linear = set(linear_names(d))
    header, off, parts = {}, 0, []
    for name, shape in tensor_specs(d):
        if name in linear:
            out, inp = shape
            if inp % QUANT_GROUP:  # conversion.py:610-611
                raise ValueError(f"Linear weight cannot use group-64 quantization: {name}")
            prefix = name[: -len("weight")]
            items = [(name, "U32", [out, inp * bits // 32], out * inp * bits // 8),
                     (prefix + "scales", "BF16", [out, inp // QUANT_GROUP], out * inp // QUANT_GROUP * 2),
                     (prefix + "biases", "BF16", [out, inp // QUANT_GROUP], out * inp // QUANT_GROUP * 2)]
        else:
            items = [(name, "BF16", list(shape), int(np.prod(shape)) * 2)]
        for key, dtype, shp, n in items:
            header[key] = {"dtype": dtype, "shape": shp, "data_offsets": [off, off + n]}
            off += n
        parts.append((name, shape, name in linear))
    header["__metadata__"] = {"format": "mlx", "partition": "ar", "precision": f"{bits}bit"}
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * ((8 - (len(raw) % 8)) % 8)
    return parts, header, raw


def _q_job(args):
    src, dst, data_start, header, name, shape, is_linear, r0, r1, qbits = args
    bits = read_safetensors(src)[name]
    mm = np.memmap(dst, dtype=np.uint8, mode="r+")
    if not is_linear:
        b, _ = header[name]["data_offsets"]
        view = np.ascontiguousarray(bits).view(np.uint8).reshape(-1)
        mm[data_start + b:data_start + b + view.size] = view
    else:
        q, sb, bb = quantize_affine(bf16_bits_to_f32(bits[r0:r1]), qbits)
        words = pack_words(q, qbits).view(np.uint8).reshape(-1)
        cols = shape[1]
        prefix = name[: -len("weight")]
        b = header[name]["data_offsets"][0] + r0 * cols * qbits // 8
        mm[data_start + b:data_start + b + words.size] = words
        for key, arr in ((prefix + "scales", sb), (prefix + "biases", bb)):
            b = header[key]["data_offsets"][0] + r0 * (cols // QUANT_GROUP) * 2
            v = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
            mm[data_start + b:data_start + b + v.size] = v
    mm.flush()
    del mm


def quantized_record(bits: int) -> dict:
    """The manifest record conversion.py:754-761 writes for a quantized precision."""
    return {"ar": f"ar-{bits}bit.safetensors", "bits": bits, "group_size": QUANT_GROUP, "mode": "affine",
            "linear_only": True, "embedding_dtype": "bfloat16"}


def write_quantized(directory: str, dims: Dims, workers: int | None = None, bits: int = 8) -> str:
    """ar-<bits>bit.safetensors (bits 8 or 4) from the directory's ar-bf16.safetensors (the
    BF16 weights are the source, as in conversion.py:651-735)."""
    if bits not in (8, 4):
        raise ValueError("bits must be 8 or 4")
    parts, header, raw = _q_layout(dims, bits)
    src = os.path.join(directory, "ar-bf16.safetensors")
    dst = os.path.join(directory, f"ar-{bits}bit.safetensors")
    data_start = 8 + len(raw)
    total = data_start + max(v["data_offsets"][1] for k, v in header.items() if k != "__metadata__")
    with open(dst, "wb") as f:
        f.write(np.uint64(len(raw)).tobytes())
        f.write(raw)
        f.truncate(total)
    jobs = []
    for name, shape, is_linear in parts:
        if not is_linear:
            jobs.append((src, dst, data_start, header, name, shape, False, 0, 0, bits))
            continue
        step = max(16, (1 << 23) // shape[1])
        for r0 in range(0, shape[0], step):
            jobs.append((src, dst, data_start, header, name, shape, True, r0, min(shape[0], r0 + step), bits))
    workers = workers or min(32, os.cpu_count() or 1)
    if workers > 1 and len(jobs) > 1:
        with ThreadPoolExecutor(max_workers=workers) as pool:
            for _ in pool.map(_q_job, jobs):
                pass
    else:
        for j in jobs:
            _q_job(j)
    return dst


def write_converted(directory: str, dims: Dims = PINNED, seed: int = 0, std: float = 0.02,
                    norm_std: float = 0.0, workers: int | None = None,
                    precisions: tuple[str, ...] = ("bf16",)) -> str:
    """Write config.json, conversion.json and ar-bf16.safetensors under ``directory``
    (and ar-8bit / ar-4bit.safetensors when ``precisions`` names "8bit" / "4bit")."""
    if any(p not in ("bf16", "8bit", "4bit") for p in precisions) or "bf16" not in precisions:
        raise ValueError("precisions: 'bf16', optionally with '8bit' and '4bit'")
    os.makedirs(directory, exist_ok=True)
    specs, header, raw = _layout(dims)
    path = os.path.join(directory, "ar-bf16.safetensors")
    data_start = 8 + len(raw)
    total = data_start + max(v["data_offsets"][1] for k, v in header.items() if k != "__metadata__")
    with open(path, "wb") as f:
        f.write(np.uint64(len(raw)).tobytes())
        f.write(raw)
        f.truncate(total)
    jobs = []
    for tidx, (name, shape) in enumerate(specs):
        off = header[name]["data_offsets"][0]
        if len(shape) == 1:
            jobs.append((path, data_start, off, shape, tidx, seed, std, norm_std, 0, 1))
            continue
        # One job per group of blocks (~64 MB) keeps the pool busy on the big tables.
        per = max(1, BLOCK_ELEMS // int(np.prod(shape[1:])))
        step = per * 8
        for r0 in range(0, shape[0], step):
            jobs.append((path, data_start, off, shape, tidx, seed, std, norm_std, r0, min(shape[0], r0 + step)))
    # Threads, not processes: numpy's generators and ufunc loops release the GIL, and a
    # thread pool needs no importable worker module (callers load this file by path).
    workers = workers or min(32, os.cpu_count() or 1)
    if workers > 1 and len(jobs) > 1:
        with ThreadPoolExecutor(max_workers=workers) as pool:
            for _ in pool.map(_fill_job, jobs):
                pass
    else:
        for j in jobs:
            _fill_job(j)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(config_json(dims), f, indent=1)
    manifest = {"schema": 1, "format": "lyra-yue2-mlx",
                "source": {"synthetic": True, "seed": seed, "std": std, "norm_std": norm_std,
                           "dims": asdict(dims)},
                "upstream": "synthetic", "conversion": "synthetic",
                "precisions": {"bf16": {"ar": "ar-bf16.safetensors", "nar": "nar-bf16.safetensors",
                                        "dtype": "bfloat16"}},
                "files": {}}
    for bits in (8, 4):
        if f"{bits}bit" in precisions:
            write_quantized(directory, dims, workers, bits)
            manifest["precisions"][f"{bits}bit"] = quantized_record(bits)
    with open(os.path.join(directory, "conversion.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return directory


def read_safetensors(path: str) -> dict[str, np.ndarray]:
    """Read a safetensors file into {name: array} (memory-mapped): BF16 tensors as uint16
    bits, U32 tensors as uint32."""
    with open(path, "rb") as f:
        n = int(np.frombuffer(f.read(8), dtype=np.uint64)[0])
        header = json.loads(f.read(n))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, rec in header.items():
        if name == "__metadata__":
            continue
        b, e = rec["data_offsets"]
        dt = {"BF16": np.uint16, "U32": np.uint32}[rec["dtype"]]
        out[name] = mm[8 + n + b:8 + n + e].view(dt).reshape(rec["shape"])
    return out
