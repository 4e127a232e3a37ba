"""yue2-mlx_b200 — YuE2 AR engine on B200 (sm_100a), driven through its C ABI.

The CUDA library ``libyue2ar_cuda.so`` (built from ``csrc/`` by ``build.py``) is the
product; this module is a thin ctypes mirror of the reference's AR interface
(native/include/lyra/ar.hpp:27-48, upstream vendor/yue/src/yue2/sampling.py:57) so
Python callers and the parity tests read like the reference's own:

* ``Sampling``                — lyra::Sampling / yue2.protocol.Sampling (types.hpp:78-87)
* ``ARModel(path)``           — ARModel(dir, "bf16", verify=False) (ar.cpp:133-238)
* ``ARModel.session(...)``    — device KV cache + decode state for up to N rows
* ``generate_tokens(...)``    — generate_tokens (sampling.cpp:185-288): returns
                                ``(tokens, timing, truncated)`` like the reference
* ``Session.prefill/step/logits/kv`` — ARModel::hidden + project per row

There is no CPU fallback: importing works without a GPU, but every compute call goes to
the CUDA library, and a missing library raises at import.
"""
from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libyue2ar_cuda.so")

OK, FAILURE, INVALID_INPUT, CANCELLED = 0, 1, 2, 130
PHASES = {"abc": 0, "semantic": 1, None: 2, "full": 2}
LOAD_ANY_DIMS = 1
LOAD_8BIT = 2
LOAD_4BIT = 4
PRECISIONS = ("bf16", "8bit", "4bit")

EOD, ABC_END, MUSIC_END = 151643, 151848, 151852
CODEC_OFFSET, CODEC_SIZE, CONTEXT = 151853, 32768, 24576


class YarError(Exception):
    """A failed C-ABI call: ``status`` is the lyra_status code, ``kind`` the error type."""

    def __init__(self, status: int, kind: str, message: str):
        super().__init__(f"{kind}: {message}")
        self.status, self.kind, self.message = status, kind, message


class _Sampling(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_double), ("top_p", ctypes.c_double), ("top_k", ctypes.c_int32),
                ("repetition_penalty", ctypes.c_double), ("penalty_window", ctypes.c_int32),
                ("min_tokens", ctypes.c_int32), ("max_tokens", ctypes.c_int32)]


CANCEL_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)
TOKEN_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int, ctypes.c_int32)


def _load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python yue2-mlx_b200/build.py` "
                          "(there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    P, I, U64, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_double
    i32p = ctypes.POINTER(ctypes.c_int32)
    u16p = ctypes.POINTER(ctypes.c_uint16)
    sig = {
        "yar_last_error": (ctypes.c_char_p, []),
        "yar_last_error_type": (ctypes.c_char_p, []),
        "yar_version": (ctypes.c_char_p, []),
        "yar_model_load": (I, [ctypes.c_char_p, I, ctypes.POINTER(P)]),
        "yar_model_load_ex": (I, [ctypes.c_char_p, I, ctypes.c_uint32, ctypes.POINTER(P)]),
        "yar_model_load_precision": (I, [ctypes.c_char_p, ctypes.c_char_p, I, ctypes.c_uint32, ctypes.POINTER(P)]),
        "yar_model_precision_bits": (I, [P, ctypes.POINTER(I)]),
        "yar_tp_unique_id": (I, [ctypes.c_char_p]),
        "yar_tp_plan": (I, [I, I, I, I, I, I, I, ctypes.POINTER(ctypes.c_int64)]),
        "yar_tp_head_slice": (I, [I, I, I, ctypes.POINTER(I), ctypes.POINTER(I)]),
        "yar_model_load_tp": (I, [ctypes.c_char_p, I, I, I, ctypes.c_char_p, ctypes.c_uint32, ctypes.POINTER(P)]),
        "yar_model_free": (I, [P]),
        "yar_model_dims": (I, [P, ctypes.POINTER(ctypes.c_int64)]),
        "yar_session_create": (I, [P, I, I, I, ctypes.POINTER(P)]),
        "yar_session_free": (I, [P]),
        "yar_session_set_option": (I, [P, I, I]),
        "yar_session_trace": (I, [P, ctypes.POINTER(ctypes.c_uint64), ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
        "yar_generate": (I, [P, i32p, I, ctypes.POINTER(_Sampling), U64, I, i32p, I, D, I, CANCEL_FN, P,
                             TOKEN_FN, P, i32p, ctypes.POINTER(I), ctypes.POINTER(I), ctypes.c_char_p,
                             ctypes.c_size_t]),
        "yar_generate_batch": (I, [P, I, i32p, i32p, ctypes.POINTER(_Sampling), ctypes.POINTER(ctypes.c_uint64), I, I,
                                   i32p, ctypes.POINTER(I), ctypes.POINTER(I), ctypes.c_char_p, ctypes.c_size_t]),
        "yar_generate_requests": (I, [P, I, I, i32p, i32p, ctypes.POINTER(_Sampling), ctypes.POINTER(ctypes.c_uint64),
                                      I, I, i32p, ctypes.POINTER(I), ctypes.POINTER(I), ctypes.c_char_p,
                                      ctypes.c_size_t]),
        "yar_row_reset": (I, [P, I, I]),
        "yar_row_prefill": (I, [P, I, i32p, I, I, I]),
        "yar_rows_step": (I, [P, ctypes.POINTER(I), i32p, I, I]),
        "yar_row_logits": (I, [P, I, u16p, I]),
        "yar_row_kv": (I, [P, I, I, I, I, u16p, u16p]),
        "yar_row_position": (I, [P, I, ctypes.POINTER(I)]),
        "yar_row_hidden": (I, [P, I, I, u16p, I]),
        "yar_sample_host": (I, [P, u16p, u16p, I, D, ctypes.POINTER(_Sampling), i32p, I, I, I, U64, I, i32p,
                                ctypes.POINTER(ctypes.c_float)]),
        "yar_sample_device_noalloc": (I, [P, P, ctypes.c_int64, I, I, D, ctypes.POINTER(_Sampling), i32p, I, I, I,
                                          U64, P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    return lib


lib = _load_library()


def _check(status: int):
    if status != OK:
        raise YarError(status, lib.yar_last_error_type().decode(), lib.yar_last_error().decode())


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


@dataclass(frozen=True)
class Sampling:
    """lyra::Sampling (native/include/lyra/types.hpp:78-87); validated by the library."""
    temperature: float = 1.0
    top_p: float = 0.95
    top_k: int = 100
    repetition_penalty: float = 1.2
    penalty_window: int = 50
    min_tokens: int = 200
    max_tokens: int = 9000

    def _c(self) -> _Sampling:
        return _Sampling(self.temperature, self.top_p, self.top_k, self.repetition_penalty,
                         self.penalty_window, self.min_tokens, self.max_tokens)


ABC_SAMPLING = Sampling(.7, .9, 30, 1.005, 100, 32, 4096)
"""GenerationConfig.abc defaults (types.hpp:89)."""


def tp_unique_id() -> bytes:
    """128 opaque bytes naming a new tensor-parallel group (ncclGetUniqueId); one rank
    makes it and every rank passes it to ``ARModel(..., tp=(rank, world, id))``."""
    buf = ctypes.create_string_buffer(128)
    _check(lib.yar_tp_unique_id(buf))
    return buf.raw


def tp_plan(hidden: int, heads: int, kv_heads: int, head_dim: int, ffn: int, rank: int, world: int) -> dict:
    """The loader's tensor-parallel split for one rank, in rows of the whole model's
    tensors: q_proj, k/v_proj, gate/up_proj and o/down_proj ("h") rows."""
    out = (ctypes.c_int64 * 8)()
    _check(lib.yar_tp_plan(hidden, heads, kv_heads, head_dim, ffn, rank, world, out))
    keys = ("q_row0", "q_rows", "kv_row0", "kv_rows", "ffn_row0", "ffn_rows", "h_row0", "h_rows")
    return dict(zip(keys, [int(v) for v in out]))


def tp_head_slice(width: int, rank: int, world: int) -> tuple[int, int]:
    """Columns [begin, end) of a phase projection this rank computes under tensor parallelism."""
    b, e = ctypes.c_int(), ctypes.c_int()
    _check(lib.yar_tp_head_slice(width, rank, world, ctypes.byref(b), ctypes.byref(e)))
    return b.value, e.value


class ARModel:
    """Converted AR weights resident on one GPU (ARModel, ar.cpp:133-238).

    ``precision`` is the reference's: "bf16" (ar-bf16.safetensors), "8bit" or "4bit" (affine
    8- / 4-bit group-64 linears, ar-8bit / ar-4bit.safetensors).
    ``tp=(rank, world, nccl_id)`` loads this rank's tensor-parallel share instead (BF16
    only): its KV-head groups and FFN column block, with NCCL exchanges inside every
    forward. All ranks must then make the same calls with the same arguments."""

    def __init__(self, path: str, device: int = 0, any_dims: bool = False, tp=None, precision: str = "bf16"):
        h = ctypes.c_void_p()
        flags = LOAD_ANY_DIMS if any_dims else 0
        if tp is None:
            _check(lib.yar_model_load_precision(os.fsencode(path), precision.encode(), device, flags,
                                                ctypes.byref(h)))
            self.tp_rank, self.tp_world = 0, 1
        else:
            rank, world, nccl_id = tp
            if precision not in PRECISIONS:
                raise ValueError("precision must be 'bf16', '8bit', or '4bit'")
            flags |= {"bf16": 0, "8bit": LOAD_8BIT, "4bit": LOAD_4BIT}[precision]
            if len(nccl_id) != 128:
                raise ValueError("nccl_id must be the 128 bytes of tp_unique_id()")
            _check(lib.yar_model_load_tp(os.fsencode(path), device, rank, world, bytes(nccl_id), flags,
                                         ctypes.byref(h)))
            self.tp_rank, self.tp_world = rank, world
        self._h = h
        dims = (ctypes.c_int64 * 10)()
        _check(lib.yar_model_dims(h, dims))
        keys = ("hidden", "layers", "heads", "kv_heads", "head_dim", "ffn", "vocab", "context", "weights_mib", "sms")
        self.dims = dict(zip(keys, [int(v) for v in dims]))
        self.device = device
        b = ctypes.c_int()
        _check(lib.yar_model_precision_bits(h, ctypes.byref(b)))
        self.precision = {8: "8bit", 4: "4bit"}.get(b.value, "bf16")

    def session(self, max_rows: int = 2, max_ctx: int = 4096, page_tokens: int = 256) -> "Session":
        return Session(self, max_rows, max_ctx, page_tokens)

    def close(self):
        if getattr(self, "_h", None):
            lib.yar_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def phase_width(self, phase) -> int:
        if phase == "semantic":
            return CODEC_SIZE + 1
        if phase == "abc":
            return EOD + 1
        return self.dims["vocab"]

    def sample(self, cond_bits, sampling: Sampling, history=(), step: int = 0, phase="semantic", seed: int = 0,
               uncond_bits=None, cfg_scale: float = 1.0, want_scores: bool = True, legacy_off: bool = False):
        """The device sampler on host BF16 logits: returns (local token, FP32 scores)."""
        cond = np.ascontiguousarray(np.asarray(cond_bits, dtype=np.uint16))
        n = cond.size
        unc = None if uncond_bits is None else np.ascontiguousarray(np.asarray(uncond_bits, dtype=np.uint16))
        hist = _i32(list(history)) if len(history) else np.zeros(1, np.int32)
        tok = ctypes.c_int32()
        scores = np.empty(n, np.float32) if want_scores else None
        _check(lib.yar_sample_host(self._h, _ptr(cond, ctypes.c_uint16),
                                   None if unc is None else _ptr(unc, ctypes.c_uint16), n, cfg_scale,
                                   ctypes.byref(sampling._c()), _ptr(hist, ctypes.c_int32), len(history), step,
                                   PHASES[phase], seed, int(legacy_off), ctypes.byref(tok),
                                   None if scores is None else _ptr(scores, ctypes.c_float)))
        return tok.value, scores


class Session:
    """Paged KV cache and decode state for up to ``max_rows`` rows on the model's GPU."""

    def __init__(self, model: ARModel, max_rows: int, max_ctx: int, page_tokens: int):
        h = ctypes.c_void_p()
        _check(lib.yar_session_create(model._h, max_rows, max_ctx, page_tokens, ctypes.byref(h)))
        self._h, self.model = h, model
        self.max_rows, self.max_ctx = max_rows, max_ctx

    def close(self):
        if getattr(self, "_h", None):
            lib.yar_session_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_persistent(self, on: bool):
        """Decode forward as one persistent kernel (default) or one kernel per operation."""
        _check(lib.yar_session_set_option(self._h, 1, int(bool(on))))

    def generate_batch(self, prefixes, sampling: Sampling, seeds, phase="semantic", legacy_off: bool = False):
        """Independent requests decoded together on rows 0..n-1: (token lists, timing, truncated)."""
        return _generate_batch(self, prefixes, sampling, seeds, phase, legacy_off)

    def generate_requests(self, prefixes, samplings, seeds, phase="semantic", slots: int = 0,
                          legacy_off: bool = False):
        """Continuous batching: requests served on `slots` rows (0 = as many as fit), finished
        rows refilled from the queue. Returns (token lists, timing, truncated flags)."""
        n = len(prefixes)
        lens = np.array([len(p) for p in prefixes], np.int32)
        flat = _i32(np.concatenate([np.asarray(p, np.int32) for p in prefixes]))
        sd = np.ascontiguousarray(np.asarray(seeds, np.uint64))
        arr = (_Sampling * n)(*[smp._c() for smp in samplings])
        caps = [max(1, smp.max_tokens) for smp in samplings]
        offs = np.concatenate([[0], np.cumsum(caps)]).astype(np.int64)
        out = np.zeros(int(offs[-1]), np.int32)
        n_out, trunc = np.zeros(n, np.int32), np.zeros(n, np.int32)
        timing = ctypes.create_string_buffer(4096)
        _check(lib.yar_generate_requests(self._h, n, slots, _ptr(flat, ctypes.c_int32), _ptr(lens, ctypes.c_int32),
                                         arr, _ptr(sd, ctypes.c_uint64), PHASES[phase], int(legacy_off),
                                         _ptr(out, ctypes.c_int32), _ptr(n_out, ctypes.c_int),
                                         _ptr(trunc, ctypes.c_int), timing, len(timing)))
        tokens = [out[offs[r]:offs[r] + n_out[r]].tolist() for r in range(n)]
        return tokens, json.loads(timing.value.decode()), [bool(t) for t in trunc]

    def set_prefetch_stages(self, n: int):
        """L2 prefetch distance of the persistent decode kernel, in 32 KB stages per SM."""
        _check(lib.yar_session_set_option(self._h, 3, int(n)))

    def set_prefill_attention_tc(self, on: bool):
        """Prefill attention (head_dim 128) on tcgen05 tensor cores (default) or, off, the mma.sync kernel."""
        _check(lib.yar_session_set_option(self._h, 7, int(bool(on))))

    def set_max_splits(self, n: int):
        """Cap the decode attention's splits per (row, kv head); 0 restores the automatic plan."""
        _check(lib.yar_session_set_option(self._h, 4, int(n)))

    def set_fault_inject(self, op: int):
        """Failure-path testing: operation 1 + 5 * layer + k of the persistent decode waits for
        a flag nothing writes (short limit), so the step fails with RuntimeError; 0 = off."""
        _check(lib.yar_session_set_option(self._h, 6, int(op)))

    def set_layer_dump(self, on: bool):
        """Record each decode step's residual rows after the embedding and every layer."""
        _check(lib.yar_session_set_option(self._h, 5, int(bool(on))))

    def hidden(self, row: int, slot: int) -> np.ndarray:
        """Residual row of the last decode step (BF16 bits): slot 0 embedding, l + 1 after layer l."""
        out = np.empty(self.model.dims["hidden"], np.uint16)
        _check(lib.yar_row_hidden(self._h, row, slot, _ptr(out, ctypes.c_uint16), out.size))
        return out

    def set_trace(self, on: bool):
        """Record the persistent decode kernel's per-CTA timeline (see ``trace``)."""
        _check(lib.yar_session_set_option(self._h, 2, int(bool(on))))

    def trace(self) -> np.ndarray:
        """Timeline of the last step with an active row: [sm][5 * layers + 1][8] SM-clock
        stamps per CTA and operation (slots 6/7 of the first operation and of the head:
        globaltimer ns and SM clock at the step's start and end)."""
        d = self.model.dims
        k = d["sms"] * (5 * d["layers"] + 1) * 8
        out = np.zeros(k + 16, np.uint64)
        n = ctypes.c_size_t()
        _check(lib.yar_session_trace(self._h, _ptr(out, ctypes.c_uint64), out.size, ctypes.byref(n)))
        return out[:k].reshape(d["sms"], 5 * d["layers"] + 1, 8)

    def sampler_trace(self) -> np.ndarray:
        """The last sampler launch's phase stamps (16 uint64, see yar_session_trace)."""
        return self._trace_tail()[:16]

    def step_log(self) -> np.ndarray:
        """[64][4] globaltimer ns per decode step (ring indexed by step % 64): sampler start
        and end (request 0), persistent kernel start and end (CTA 0)."""
        return self._trace_tail()[16:16 + 256].reshape(64, 4)

    def _trace_tail(self) -> np.ndarray:
        d = self.model.dims
        k = d["sms"] * (5 * d["layers"] + 1) * 8
        out = np.zeros(k + 16 + 256, np.uint64)
        n = ctypes.c_size_t()
        _check(lib.yar_session_trace(self._h, _ptr(out, ctypes.c_uint64), out.size, ctypes.byref(n)))
        return out[k:]

    def reset(self, row: int, capacity: int):
        _check(lib.yar_row_reset(self._h, row, capacity))

    def prefill(self, row: int, ids, phase="semantic", chunk: int = 0):
        a = _i32(ids)
        _check(lib.yar_row_prefill(self._h, row, _ptr(a, ctypes.c_int32), a.size, PHASES[phase], chunk))

    def step(self, rows, tokens, phase="semantic"):
        r = np.ascontiguousarray(np.asarray(rows, dtype=np.int32))
        t = _i32(tokens)
        _check(lib.yar_rows_step(self._h, _ptr(r, ctypes.c_int), _ptr(t, ctypes.c_int32), r.size, PHASES[phase]))

    def logits(self, row: int, phase="semantic") -> np.ndarray:
        """Last projected logits of ``row`` as BF16 bits (phase-local width)."""
        n = self.model.phase_width(phase)
        out = np.empty(n, np.uint16)
        _check(lib.yar_row_logits(self._h, row, _ptr(out, ctypes.c_uint16), n))
        return out

    def kv(self, row: int, layer: int, start: int, count: int):
        d = self.model.dims
        k = np.empty((d["kv_heads"], count, d["head_dim"]), np.uint16)
        v = np.empty_like(k)
        _check(lib.yar_row_kv(self._h, row, layer, start, count, _ptr(k, ctypes.c_uint16), _ptr(v, ctypes.c_uint16)))
        return k, v

    def position(self, row: int) -> int:
        p = ctypes.c_int()
        _check(lib.yar_row_position(self._h, row, ctypes.byref(p)))
        return p.value

    def generate(self, prefix, sampling: Sampling, seed: int, phase="semantic", negative=None, cfg_scale: float = 1.0,
                 legacy_off: bool = False, cancelled=None, on_token=None):
        """generate_tokens (native/src/sampling.cpp:185-288): (tokens, timing, truncated)."""
        pre = _i32(prefix)
        neg = _i32(negative) if negative is not None and len(negative) else np.zeros(1, np.int32)
        n_neg = len(negative) if negative is not None else 0
        out = np.empty(max(1, sampling.max_tokens), np.int32)
        n_out, trunc = ctypes.c_int(), ctypes.c_int()
        timing = ctypes.create_string_buffer(4096)
        cancel_cb = CANCEL_FN(lambda _ctx: 1 if cancelled and cancelled() else 0) if cancelled else CANCEL_FN()
        phase_names = {0: "abc", 1: "semantic", 2: None}
        token_cb = TOKEN_FN(lambda _ctx, ph, tok: on_token(phase_names[ph], int(tok))) if on_token else TOKEN_FN()
        _check(lib.yar_generate(self._h, _ptr(pre, ctypes.c_int32), pre.size, ctypes.byref(sampling._c()), seed,
                                PHASES[phase], _ptr(neg, ctypes.c_int32), n_neg, cfg_scale, int(legacy_off),
                                cancel_cb, None, token_cb, None, _ptr(out, ctypes.c_int32), ctypes.byref(n_out),
                                ctypes.byref(trunc), timing, len(timing)))
        return out[:n_out.value].tolist(), json.loads(timing.value.decode()), bool(trunc.value)


def _generate_batch(session, prefixes, sampling: Sampling, seeds, phase="semantic", legacy_off: bool = False):
    n = len(prefixes)
    lens = np.array([len(p) for p in prefixes], np.int32)
    flat = _i32(np.concatenate([np.asarray(p, np.int32) for p in prefixes]))
    sd = np.ascontiguousarray(np.asarray(seeds, np.uint64))
    out = np.zeros(n * max(1, sampling.max_tokens), np.int32)
    n_out, trunc = np.zeros(n, np.int32), np.zeros(n, np.int32)
    timing = ctypes.create_string_buffer(4096)
    _check(lib.yar_generate_batch(session._h, n, _ptr(flat, ctypes.c_int32), _ptr(lens, ctypes.c_int32),
                                  ctypes.byref(sampling._c()), _ptr(sd, ctypes.c_uint64), PHASES[phase],
                                  int(legacy_off), _ptr(out, ctypes.c_int32), _ptr(n_out, ctypes.c_int),
                                  _ptr(trunc, ctypes.c_int), timing, len(timing)))
    m = max(1, sampling.max_tokens)
    tokens = [out[r * m:r * m + n_out[r]].tolist() for r in range(n)]
    return tokens, json.loads(timing.value.decode()), [bool(t) for t in trunc]


def generate_tokens(model: ARModel, prefix, sampling: Sampling, seed: int, phase: str = "semantic", negative=None,
                    cfg_scale: float = 1.0, legacy_off: bool = False, cancelled=None, on_token=None,
                    session: Session | None = None):
    """Module-level mirror of the reference's ``generate_tokens`` (request-local session)."""
    cfg = cfg_scale != 1.0
    need = max(len(prefix), len(negative) if negative is not None else 0) + sampling.max_tokens
    own = session is None
    s = session or model.session(max_rows=2 if cfg else 1, max_ctx=need)
    try:
        return s.generate(prefix, sampling, seed, phase, negative, cfg_scale, legacy_off, cancelled, on_token)
    finally:
        if own:
            s.close()


def header_functions(header: str | None = None) -> list[str]:
    """Names of the functions ``include/yue2ar.h`` declares (used to check the exports)."""
    import re
    header = header or os.path.join(os.path.dirname(HERE), "include", "yue2ar.h")
    text = open(header).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(yar_\w+)\s*\(", text, re.M)))
