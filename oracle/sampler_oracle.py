"""CPU restatement (numpy) of the AR sampler — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import this
module, as the checker; the CUDA sampler never calls it.

Two layers:

1. The filter chain, a restatement of upstream ``distribution``
   (vendor/yue/src/yue2/sampling.py:16-53) on phase-local rows
   (native/src/sampling.cpp:8-99): FP32 upcast, end-token mask while
   ``step < min_tokens``, the frequency-powered window penalty
   ``alpha = penalty ** count``, ``s < 0 ? s * alpha : s / alpha`` (sampling.py:16-23),
   temperature division, top-k by the k-th *value* (ties kept), and the shifted nucleus
   ``cumsum(p) - p > top_p`` keeping at least one row. CFG mixing follows
   sampling.py:109 / native/src/sampling.cpp:100-115 with a BF16 rounding after the
   subtraction, the scalar multiply (FP32 scalar) and the add.

2. The draw contract of this build (the reference's RNGs differ per backend and it
   disclaims cross-backend token equality, tests/test_sampling.py:1): one FP32 uniform
   per step from Philox4x32-10 (Salmon et al., SC'11) keyed by the request seed with
   counter ``(step, stream, 0, 0)``; survivors sorted by (score desc, index asc);
   ``e_i = yexp(s_i - s_0)``; sequential FP32 sums; ``target = u * sum(e)``; the token is
   the first survivor whose running sum exceeds ``target``. ``yexp`` is Cody–Waite
   range reduction with a split ln 2 plus a degree-7 Taylor polynomial in Horner form,
   every operation a single IEEE float32 multiply/add (no FMA), so this numpy code and
   the CUDA sampler produce identical bits.

Top-p uses the same ``e_i``: ``p_i = e_i / S`` (IEEE division), a sequential FP32
running sum ``c_i`` and ``removed_i = i >= 1 and (c_i - p_i) > f32(top_p)``.

``legacy_off`` (historical BF16 sampling, sampling.py:27 with ``legacy_off=True``) keeps
the scores in BF16 as torch does: the penalty power has its base rounded to BF16 first
(``bf16(penalty) ** count``, rounded to BF16), the penalty multiply / divide and the
temperature division (by the FP32 temperature) round to BF16, the nucleus probabilities
are ``bf16(e_i / S)``, the cumulative sum is an FP32 running sum rounded to BF16 at each
row, ``preceding = bf16(cum_i - p_i)`` is compared against ``bf16(top_p)``, and the
first three rows are always kept (sampling.py:50).
"""
from __future__ import annotations

import numpy as np

from .ar_oracle import ABC_END, CODEC_OFFSET, CODEC_SIZE, EOD, MUSIC_END, bf16_round

F32 = np.float32

# Cody–Waite split of ln 2: the high part has few enough bits that n * LN2_HI is exact.
LN2_HI = F32(0.693145751953125)
LN2_LO = F32(1.428606765330187e-06)
LOG2E = F32(1.4426950408889634)
EXP_FLUSH = F32(-87.0)
TAYLOR = [F32(1.0 / f) for f in (5040.0, 720.0, 120.0, 24.0, 6.0, 2.0, 1.0, 1.0)]

PHILOX_M0, PHILOX_M1 = 0xD2511F53, 0xCD9E8D57
PHILOX_W0, PHILOX_W1 = 0x9E3779B9, 0xBB67AE85


def phase_size(phase: str | None, vocab: int | None = None) -> int:
    if phase == "abc":
        return EOD + 1
    if phase == "semantic":
        return CODEC_SIZE + 1
    if phase is None:
        return vocab
    raise ValueError("phase must be 'abc' or 'semantic'")


def end_index(phase: str | None) -> int | None:
    return EOD if phase == "abc" else 0 if phase == "semantic" else None


def local_to_native(token: int, phase: str | None) -> int:
    """native/src/sampling.cpp:33-37."""
    if phase == "abc":
        return token if token < EOD else ABC_END
    if phase == "semantic":
        return MUSIC_END + token
    return token


def native_to_local(token: int, phase: str | None):
    """native/src/sampling.cpp:19-32."""
    if phase == "abc":
        if 0 <= token < EOD:
            return token
        return EOD if token == ABC_END else None
    if phase == "semantic":
        if token == MUSIC_END:
            return 0
        if CODEC_OFFSET <= token < CODEC_OFFSET + CODEC_SIZE:
            return token - MUSIC_END
        return None
    return token


def yexp(x) -> np.ndarray:
    """exp(x) for x <= 0 in float32: Cody–Waite reduction + degree-7 Taylor (Horner)."""
    x = np.asarray(x, dtype=F32)
    flush = ~(x >= EXP_FLUSH)
    xc = np.where(flush, F32(0.0), x).astype(F32)
    n = np.rint(xc * LOG2E).astype(F32)
    r = ((xc - n * LN2_HI).astype(F32) - (n * LN2_LO).astype(F32)).astype(F32)
    p = TAYLOR[0]
    for c in TAYLOR[1:]:
        p = (p * r).astype(F32) + c
        p = np.asarray(p, dtype=F32)
    bits = ((n.astype(np.int32) + 127) << 23).astype(np.uint32)
    out = (p * bits.view(F32)).astype(F32)
    return np.where(flush, F32(0.0), out).astype(F32)


def _mulhilo(a: int, b: int):
    p = a * b
    return (p >> 32) & 0xFFFFFFFF, p & 0xFFFFFFFF


def philox4x32_10(counter, key):
    """Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) on Python ints."""
    c0, c1, c2, c3 = [int(v) & 0xFFFFFFFF for v in counter]
    k0, k1 = [int(v) & 0xFFFFFFFF for v in key]
    for rnd in range(10):
        hi0, lo0 = _mulhilo(PHILOX_M0, c0)
        hi1, lo1 = _mulhilo(PHILOX_M1, c2)
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        if rnd < 9:
            k0 = (k0 + PHILOX_W0) & 0xFFFFFFFF
            k1 = (k1 + PHILOX_W1) & 0xFFFFFFFF
    return c0, c1, c2, c3


def uniform(seed: int, step: int, stream: int = 0) -> np.float32:
    """The per-step draw: top 24 bits of Philox word 0, times 2**-24, in [0, 1)."""
    w0 = philox4x32_10((step, stream, 0, 0), (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))[0]
    return F32((w0 >> 8) * (1.0 / 16777216.0))


def penalty_alpha(penalty: float, count: int) -> np.float32:
    """FP32 ``penalty ** count``: float32 base, power in double, rounded once."""
    return F32(float(F32(penalty)) ** int(count))


def guided(conditional, unconditional, scale: float) -> np.ndarray:
    """CFG with BF16 rounding after each op (sampling.cpp:100-115, upstream sampling.py:109)."""
    c = bf16_round(conditional)
    if unconditional is None:
        return c
    u = bf16_round(unconditional)
    delta = bf16_round(c - u)
    scaled = bf16_round(delta * F32(scale))
    return bf16_round(u + scaled)


def legacy_alpha(penalty: float, count: int) -> np.float32:
    """BF16 ``penalty ** count`` of the BF16 path: base rounded to BF16, result to BF16."""
    base = float(bf16_round(np.array([penalty], F32))[0])
    return bf16_round(np.array([F32(base ** int(count))], F32))[0]


def filter_scores(logits, sampling: dict, history, step: int, phase: str | None,
                  vocab: int | None = None, legacy_off: bool = False):
    """Upstream ``distribution`` on phase-local rows; returns (scores, sorted survivors).

    ``scores`` is the FP32 filtered vector (removed rows are -inf), as the upstream
    function returns it. ``order`` lists surviving local ids sorted by (score desc,
    index asc); it is None for greedy sampling (temperature 0).
    """
    s = np.array(logits, dtype=F32, copy=True)
    n = s.shape[-1]
    end = end_index(phase)
    if step < sampling["min_tokens"] and end is not None:
        s[end] = -np.inf
    penalty = sampling["repetition_penalty"]
    window = sampling["penalty_window"]
    if penalty != 1.0 and len(history):
        recent = list(history)[-window:] if window else list(history)
        counts: dict[int, int] = {}
        for t in recent:
            loc = native_to_local(int(t), phase)
            if loc is not None and 0 <= loc < n:
                counts[loc] = counts.get(loc, 0) + 1
        for loc, c in counts.items():
            a = legacy_alpha(penalty, c) if legacy_off else penalty_alpha(penalty, c)
            v = s[loc]
            s[loc] = F32(v * a) if v < 0 else F32(v / a)
            if legacy_off:
                s[loc] = bf16_round(np.array([s[loc]], F32))[0]
    t = sampling["temperature"]
    if t == 0:
        return s, None
    if t != 1:
        s = (s / F32(t)).astype(F32)
        if legacy_off:
            s = bf16_round(s)
    k = min(int(sampling["top_k"]), n)
    threshold = np.sort(s)[::-1][k - 1]
    s = np.where(s < threshold, F32(-np.inf), s).astype(F32)
    idx = np.flatnonzero(np.isfinite(s))
    order = idx[np.lexsort((idx, -s[idx]))]
    if sampling["top_p"] < 1 and len(order):
        e = yexp((s[order] - s[order[0]]).astype(F32))
        total = F32(0.0)
        for v in e:
            total = F32(total + v)
        p = (e / total).astype(F32)
        c = F32(0.0)
        top_p = F32(sampling["top_p"])
        keep = np.ones(len(order), dtype=bool)
        if legacy_off:
            p = bf16_round(p)
            top_p = bf16_round(np.array([top_p], F32))[0]
            for i in range(len(order)):
                c = F32(c + p[i])
                cum = bf16_round(np.array([c], F32))[0]
                preceding = bf16_round(np.array([F32(cum - p[i])], F32))[0]
                if i >= 3 and preceding > top_p:
                    keep[i] = False
        else:
            for i in range(len(order)):
                c = F32(c + p[i])
                if i >= 1 and F32(c - p[i]) > top_p:
                    keep[i] = False
        s[order[~keep]] = -np.inf
        order = order[keep]
    return s, order


def draw(scores, order, u) -> int:
    """Inverse CDF over ``order`` with sequential FP32 sums of ``yexp(s_i - s_0)``."""
    e = yexp((scores[order] - scores[order[0]]).astype(F32))
    total = F32(0.0)
    for v in e:
        total = F32(total + v)
    target = F32(F32(u) * total)
    acc = F32(0.0)
    for i, v in enumerate(e):
        acc = F32(acc + v)
        if target < acc:
            return int(order[i])
    return int(order[-1])


def sample(logits, sampling: dict, history, step: int, phase: str | None, seed: int,
           stream: int = 0, unconditional=None, cfg_scale: float = 1.0, vocab: int | None = None,
           legacy_off: bool = False):
    """One sampler step on phase-local BF16 logits; returns (local token, filtered scores)."""
    mixed = guided(logits, unconditional if cfg_scale != 1.0 else None, cfg_scale)
    scores, order = filter_scores(mixed, sampling, history, step, phase, vocab, legacy_off)
    if order is None:
        return int(np.argmax(scores)), scores
    return draw(scores, order, uniform(seed, step, stream)), scores


def sampling_dict(temperature=1.0, top_p=0.95, top_k=100, repetition_penalty=1.2,
                  penalty_window=50, min_tokens=200, max_tokens=9000) -> dict:
    """lyra::Sampling defaults (native/include/lyra/types.hpp:78-87)."""
    return dict(temperature=temperature, top_p=top_p, top_k=top_k,
                repetition_penalty=repetition_penalty, penalty_window=penalty_window,
                min_tokens=min_tokens, max_tokens=max_tokens)
