"""CPU restatement (numpy) of the YuE2 AR decoder — TEST INFRASTRUCTURE ONLY.

This module is the parity oracle. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and only as
the checker or the timed CPU baseline; the CUDA product never routes through it.

It restates the upstream PyTorch AR path (the reference's only AR implementation that
runs off-Mac) with the same storage/rounding points, every contraction accumulated in
float32:

* ``RMSNorm``   vendor/yue/src/yue2/modeling_yue2.py:131-132
  ``bf16(bf16(x * bf16(rsqrt(mean(f32(x)^2) + eps))) * w)`` (also native/src/ar.cpp:30-35)
* ``RoPE``      modeling_yue2.py:142-156 — FP32 ``inv_freq = 1/(theta ** (2i/d))``,
  FP32 angles ``pos * inv_freq``, cos/sin rounded to the activation dtype, half-split
  rotation with a rounding after every product and sum (native/src/ar.cpp:52-87)
* ``Attention`` modeling_yue2.py:174-213 — q/k/v projections, per-head q/k RMSNorm, RoPE,
  append to the cache at slot = position (StaticKVCache, :383-393), GQA with q head h
  reading kv head ``h // (heads / kv_heads)``, causal (bottom-right) visibility, scale
  ``head_dim ** -0.5`` in FP32, FP32 softmax and FP32 P.V, output rounded once
* ``MLP``       modeling_yue2.py:223-224 — ``down(bf16(bf16(silu_f32(gate)) * up))``
* ``DecoderLayer`` AR-only branch modeling_yue2.py:296-303 — BF16 residual adds
* ``project``   native/src/ar.cpp:302-323 — phase-local LM-head rows
* affine 8- and 4-bit linears (the ``8bit`` / ``4bit`` precisions, ar.cpp:20-29 and
  :305-311 call ``mx::quantized_matmul(x, w, scales, biases, transpose=true, 64, bits,
  "affine")``; MLX 0.32.2, pinned by conversion.py:31, is not in the reference tree): the
  published semantics — element (32 / bits) i + j of a row in bits (bits j).. of U32 word
  i, and per 64-column group ``w = scale * q + bias`` with BF16 scale and bias — restated
  by dequantizing to float32 (``dequantize_affine``) and contracting in float32 like
  every other linear.
  Parity of this restatement with MLX itself is unpinned (MLX runs only on Apple GPUs).

In ``bf16=False`` mode no rounding is applied (BASELINE config 1 runs the tiny model in
FP32). Parity of this restatement with the upstream code is pinned by the golden vectors
under ``tests/golden/`` (produced by importing the upstream package).
"""
from __future__ import annotations

import numpy as np

EOD = 151643
ABC_END = 151848
MUSIC_END = 151852
CODEC_OFFSET, CODEC_SIZE = 151853, 32768
CONTEXT = 24576

F32 = np.float32


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest BF16 (ties to even), returned as float32."""
    a = np.ascontiguousarray(x, dtype=F32)
    u = a.view(np.uint32).copy()
    nan = np.isnan(a)
    u += np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    u &= np.uint32(0xFFFF0000)
    out = u.view(F32)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def bf16_from_bits(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(F32)


def bits_from_bf16(x) -> np.ndarray:
    return (np.ascontiguousarray(bf16_round(x)).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def rope_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    """FP32 ``1 / theta ** (arange(0, d, 2) / d)`` (modeling_yue2.py:144-146).

    The power is formed in double and rounded once to float32, then the reciprocal is
    an IEEE float32 division, matching torch's float32 pow + float32 reciprocal.
    """
    exponent = np.arange(0, head_dim, 2, dtype=F32) / F32(head_dim)
    power = np.array([float(F32(theta)) ** float(e) for e in exponent], dtype=np.float64).astype(F32)
    return (F32(1.0) / power).astype(F32)


def rope_cos_sin(positions, head_dim: int, theta: float):
    """FP32 angles, cos/sin evaluated in double and rounded once to float32."""
    inv = rope_inv_freq(head_dim, theta)
    angles = np.asarray(positions, dtype=F32)[:, None] * inv[None, :]
    angles = angles.astype(F32)
    return np.cos(angles.astype(np.float64)).astype(F32), np.sin(angles.astype(np.float64)).astype(F32)


def dequantize_affine(packed, scales_bits, biases_bits) -> np.ndarray:
    """Float32 ``scale * q + bias`` of an affine group-64 matrix: ``packed`` U32
    ``[rows, cols * bits / 32]`` (element (32 / bits) i + j in bits (bits j).. of word i;
    bits 8 or 4, known from the shapes), BF16 bits of the scales and biases
    ``[rows, cols / 64]``."""
    words = np.ascontiguousarray(packed, dtype=np.uint32)
    rows, groups = words.shape[0], np.asarray(scales_bits).shape[1]
    bits = words.shape[1] * 32 // (groups * 64)
    if bits not in (8, 4):
        raise ValueError("packed width does not match 8 or 4 bits per weight")
    per = 32 // bits
    shifts = np.arange(per, dtype=np.uint32) * np.uint32(bits)
    q = ((words[:, :, None] >> shifts[None, None, :]) & np.uint32((1 << bits) - 1)).reshape(rows, -1).astype(F32)
    s = bf16_from_bits(scales_bits)
    b = bf16_from_bits(biases_bits)
    out = q.reshape(rows, groups, -1) * s[:, :, None] + b[:, :, None]
    return out.reshape(rows, -1).astype(F32)


def dequantize_affine8(packed, scales_bits, biases_bits) -> np.ndarray:
    return dequantize_affine(packed, scales_bits, biases_bits)


def _quantized_groups(tensors) -> set:
    """Names of the ``.weight`` entries that have ``.scales`` beside them."""
    return {k[: -len("scales")] + "weight" for k in tensors if k.endswith(".scales")}


class LazyBf16Weights:
    """BF16 bit arrays (e.g. memory-mapped safetensors) whose float32 values are formed on
    each access and not kept: a 3B-parameter model then costs no resident float32 copy,
    for tests that run one layer at a time."""

    def __init__(self, bits: dict):
        self.bits = bits
        self.quantized = _quantized_groups(bits)

    def __getitem__(self, name):
        if name in self.quantized:
            p = name[: -len("weight")]
            return dequantize_affine(self.bits[name], self.bits[p + "scales"], self.bits[p + "biases"])
        return bf16_from_bits(self.bits[name])


class OracleAR:
    """The AR decoder on float32 arrays, with BF16 rounding points when ``bf16``."""

    def __init__(self, tensors: dict, dims, bf16: bool = True, prerounded: bool = False, lazy: bool = False):
        self.d = dims
        self.bf16 = bf16
        if lazy:  # BF16 bits, converted per access
            self.w = LazyBf16Weights(tensors)
            return
        self.w = {}
        quantized = _quantized_groups(tensors)
        for name, value in tensors.items():
            if name.endswith(".scales") or name.endswith(".biases"):
                continue
            if name in quantized:  # affine 8- or 4-bit: float32 scale * q + bias, not rounded
                p = name[: -len("weight")]
                self.w[name] = dequantize_affine(value, tensors[p + "scales"], tensors[p + "biases"])
                continue
            if prerounded:  # float32 arrays (or row-indexable views) already holding BF16 values, kept as given
                self.w[name] = value
                continue
            a = np.asarray(value)
            if a.dtype == np.uint16:
                self.w[name] = bf16_from_bits(a)  # already BF16 values
                continue
            a = np.ascontiguousarray(a, dtype=F32)
            self.w[name] = bf16_round(a) if bf16 else a

    # -- rounding ---------------------------------------------------------------------
    def r(self, x):
        return bf16_round(x) if self.bf16 else np.asarray(x, dtype=F32)

    # -- building blocks ----------------------------------------------------------------
    def rms_norm(self, x, weight):
        """modeling_yue2.py:131-132."""
        var = np.mean(np.square(x.astype(F32)), axis=-1, keepdims=True, dtype=F32)
        scale = self.r(F32(1.0) / np.sqrt(var + F32(self.d.eps)))
        return self.r(self.r(x * scale) * weight)

    def linear(self, x, name):
        return self.r(np.matmul(x, self.w[name].T).astype(F32))

    def rope(self, x, cos, sin):
        """modeling_yue2.py:152-156; x is [T, H, D], cos/sin are [T, D/2]."""
        half = x.shape[-1] // 2
        c = self.r(cos)[:, None, :]
        s = self.r(sin)[:, None, :]
        x1, x2 = x[..., :half], x[..., half:]
        first = self.r(self.r(x1 * c) - self.r(x2 * s))
        second = self.r(self.r(x2 * c) + self.r(x1 * s))
        return np.concatenate([first, second], axis=-1)

    def silu(self, g):
        g = g.astype(F32)
        return self.r(g / (F32(1.0) + np.exp(-g)))

    # -- cache ----------------------------------------------------------------------------
    def new_cache(self, capacity: int) -> dict:
        d = self.d
        shape = (d.layers, d.kv_heads, capacity, d.head_dim)
        return {"k": np.zeros(shape, F32), "v": np.zeros(shape, F32), "offset": 0, "capacity": capacity}

    # -- forward ----------------------------------------------------------------------------
    def layer(self, i: int, x, cache: dict, start: int) -> np.ndarray:
        """Decoder layer ``i`` (modeling_yue2.py:296-303) on residual rows ``x`` [T, H] at
        positions ``start ..``: appends their K/V to ``cache`` layer ``i`` and returns the
        layer's output rows. ``cache`` must already hold positions ``< start`` of layer ``i``."""
        d = self.d
        T = x.shape[0]
        end = start + T
        if end > cache["capacity"]:
            raise ValueError("KV cache capacity exceeded; generation was not shortened")
        cos, sin = rope_cos_sin(np.arange(start, end), d.head_dim, d.theta)
        group = d.heads // d.kv_heads
        scale = F32(float(d.head_dim) ** -0.5)
        visible = np.arange(end)[None, :] <= np.arange(start, end)[:, None]
        p = f"model.layers.{i}."
        h = self.rms_norm(x, self.w[p + "input_layernorm.weight"])
        q = self.linear(h, p + "self_attn.q_proj.weight").reshape(T, d.heads, d.head_dim)
        k = self.linear(h, p + "self_attn.k_proj.weight").reshape(T, d.kv_heads, d.head_dim)
        v = self.linear(h, p + "self_attn.v_proj.weight").reshape(T, d.kv_heads, d.head_dim)
        q = self.rms_norm(q, self.w[p + "self_attn.q_norm.weight"])
        k = self.rms_norm(k, self.w[p + "self_attn.k_norm.weight"])
        q = self.rope(q, cos, sin)
        k = self.rope(k, cos, sin)
        cache["k"][i, :, start:end] = k.transpose(1, 0, 2)
        cache["v"][i, :, start:end] = v.transpose(1, 0, 2)
        out = np.empty((T, d.heads, d.head_dim), F32)
        for hq in range(d.heads):
            kv = hq // group
            K = cache["k"][i, kv, :end]
            V = cache["v"][i, kv, :end]
            s = (q[:, hq, :] @ K.T).astype(F32) * scale
            s = np.where(visible, s, F32(-np.inf))
            m = s.max(axis=-1, keepdims=True)
            e = np.exp(s - m).astype(F32)
            l = e.sum(axis=-1, keepdims=True, dtype=F32)
            out[:, hq, :] = ((e @ V).astype(F32) / l).astype(F32)
        attn = self.r(out).reshape(T, d.heads * d.head_dim)
        x = self.r(x + self.linear(attn, p + "self_attn.o_proj.weight"))
        h2 = self.rms_norm(x, self.w[p + "post_attention_layernorm.weight"])
        g = self.linear(h2, p + "mlp.gate_proj.weight")
        u = self.linear(h2, p + "mlp.up_proj.weight")
        m = self.r(self.silu(g) * u)
        return self.r(x + self.linear(m, p + "mlp.down_proj.weight"))

    def forward(self, ids, cache: dict) -> np.ndarray:
        """Run ``ids`` at positions ``cache.offset ..``; return final-normed hidden [T, H]."""
        ids = np.asarray(ids, dtype=np.int64)
        start = cache["offset"]
        if start + len(ids) > cache["capacity"]:
            raise ValueError("KV cache capacity exceeded; generation was not shortened")
        x = self.w["model.embed_tokens.weight"][ids].copy()
        for i in range(self.d.layers):
            x = self.layer(i, x, cache, start)
        cache["offset"] = start + len(ids)
        return self.final_norm(x)

    def final_norm(self, x) -> np.ndarray:
        return self.rms_norm(x, self.w["model.norm.weight"])

    def cache_from(self, k_layers, v_layers, length: int, capacity: int) -> dict:
        """A cache holding given K/V (per layer [kv_heads][length][head_dim] float32 values,
        e.g. read back from the engine) at positions ``0 .. length``: decode steps from it
        are teacher-forced on those exact cached values."""
        cache = self.new_cache(capacity)
        for i, (k, v) in enumerate(zip(k_layers, v_layers)):
            cache["k"][i, :, :length] = k
            cache["v"][i, :, :length] = v
        cache["offset"] = length
        return cache

    def project(self, hidden, phase: str | None) -> np.ndarray:
        """Phase-local LM head (native/src/ar.cpp:302-323); ``None`` = full vocabulary."""
        head = self.w["lm_head.weight"]
        if phase is None:
            rows = head
        elif phase == "semantic":
            rows = head[MUSIC_END:CODEC_OFFSET + CODEC_SIZE]
        elif phase == "abc":
            rows = np.concatenate([head[:EOD], head[ABC_END:ABC_END + 1]])
        else:
            raise ValueError("phase must be 'abc' or 'semantic'")
        return self.r(np.matmul(np.atleast_2d(hidden), rows.T).astype(F32))

    def prefill(self, ids, capacity: int, phase: str | None, chunk: int = 1024):
        """Chunked prefill (native/src/sampling.cpp:152-183); returns (last-row logits, cache)."""
        cache = self.new_cache(capacity)
        h = None
        for s in range(0, len(ids), chunk):
            h = self.forward(ids[s:s + chunk], cache)
        return self.project(h[-1], phase)[0], cache

    def step(self, token: int, cache: dict, phase: str | None) -> np.ndarray:
        h = self.forward([token], cache)
        return self.project(h[-1], phase)[0]
