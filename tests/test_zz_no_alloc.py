"""yar_sample_device_noalloc against yar_sample_host and the CPU sampler oracle, through
the C ABI.

yar_sample_device_noalloc is the sampler step for callers that can't allocate device
memory: a process whose caching allocator (PyTorch's, here) already holds the GPU's free
memory, or a real-time loop that can't take cudaFree's device-wide synchronisation. It
reads the caller's device logits, writes the caller's device token and score row, and
works in one static device array shared by every call. The checks:
* the same token and the same filtered FP32 scores as yar_sample_host on the same inputs,
  bit for bit (the tolerance of the other sampler tests), on two calls in a row that
  reuse that array with different widths and settings;
* the same token and scores as the CPU restatement of the sampler (oracle/sampler_oracle),
  directly rather than through the other entry point;
* the device's free memory is the same before and after the calls (every buffer the test
  passes is allocated beforehand), so the entry point allocated nothing.
The file sorts last so that a run stopping at the first failure has already run every
other test.
"""
import ctypes

import numpy as np
import pytest

from oracle import ar_oracle as ora
from oracle import sampler_oracle as so
from tests.conftest import load_package

pytestmark = pytest.mark.gpu

MAX_COLUMNS = 196608  # the entry point's stated limit


@pytest.fixture(scope="module")
def yar():
    return load_package()


@pytest.fixture(scope="module")
def tiny(yar, tiny_dir):
    return yar.ARModel(tiny_dir, any_dims=True)


def _buffers(cond, uncond):
    """Device buffers for one call, owned by the test (torch), not by the library."""
    import torch
    n = cond.size
    rows = 1 if uncond is None else 2
    stride = n + 13  # a padded, unaligned row stride, to exercise row_stride
    host = np.zeros((rows, stride), np.uint16)
    host[0, :n] = cond
    if uncond is not None:
        host[1, :n] = uncond
    return dict(logits=torch.from_numpy(host.view(np.int16)).to("cuda:0"), rows=rows, stride=stride, n=n,
                token=torch.full((1,), -7, dtype=torch.int32, device="cuda:0"),
                scores=torch.full((n,), float("nan"), dtype=torch.float32, device="cuda:0"))


def _call(yar, model, buf, smp, history, step, phase, seed, cfg_scale):
    """One call of the entry point through the C ABI on prepared device buffers."""
    import torch
    hist = np.asarray(list(history) or [0], np.int32)
    stream = torch.cuda.current_stream("cuda:0").cuda_stream
    status = yar.lib.yar_sample_device_noalloc(
        model._h, buf["logits"].data_ptr(), buf["stride"], buf["rows"], buf["n"], cfg_scale, ctypes.byref(smp._c()),
        hist.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(history), step, yar.PHASES[phase], seed,
        buf["token"].data_ptr(), buf["scores"].data_ptr(), stream)
    yar._check(status)


def _noalloc(yar, model, cond, uncond, smp, history, step, phase, seed, cfg_scale):
    buf = _buffers(cond, uncond)
    _call(yar, model, buf, smp, history, step, phase, seed, cfg_scale)
    return int(buf["token"].item()), buf["scores"].cpu().numpy()


def _case(rng, yar, n, phase, cfg_scale, smp, hist_lo, hist_span):
    cond = ora.bits_from_bf16((rng.standard_normal(n) * 2.5).astype(np.float32))
    uncond = ora.bits_from_bf16((rng.standard_normal(n) * 2.5).astype(np.float32)) if cfg_scale != 1 else None
    history = (hist_lo + rng.integers(0, hist_span, int(rng.integers(1, 150)))).tolist()
    return dict(cond=cond, uncond=uncond, smp=yar.Sampling(**smp), raw=smp, history=history,
                step=int(rng.integers(0, 40)), phase=phase, seed=int(rng.integers(0, 2**62)), cfg_scale=cfg_scale)


def _cases(yar):
    rng = np.random.default_rng(2024)
    return [
        # Semantic phase with CFG, window penalty, top-k and nucleus.
        _case(rng, yar, 32769, "semantic", 1.5,
              dict(temperature=1.0, top_p=0.93, top_k=50, repetition_penalty=1.2, penalty_window=50,
                   min_tokens=20, max_tokens=400), 151853, 200),
        # Then the wider ABC phase, no CFG: the shared array holds the first call's rows.
        _case(rng, yar, 151644, "abc", 1.0,
              dict(temperature=0.7, top_p=0.9, top_k=30, repetition_penalty=1.005, penalty_window=100,
                   min_tokens=32, max_tokens=4096), 0, 5000),
    ]


def test_noalloc_sampler_matches_host_entry_point_on_consecutive_calls(yar, tiny):
    cases = _cases(yar)
    got = [_noalloc(yar, tiny, c["cond"], c["uncond"], c["smp"], c["history"], c["step"], c["phase"], c["seed"],
                    c["cfg_scale"]) for c in cases]
    for i, (c, (tok, scores)) in enumerate(zip(cases, got)):
        want_tok, want_scores = tiny.sample(c["cond"], c["smp"], c["history"], c["step"], c["phase"], c["seed"],
                                            uncond_bits=c["uncond"], cfg_scale=c["cfg_scale"])
        assert tok == want_tok, i
        np.testing.assert_array_equal(scores, want_scores, err_msg=f"call {i}")


def test_noalloc_sampler_matches_cpu_oracle_and_allocates_nothing(yar, tiny):
    import torch
    cases = _cases(yar)
    bufs = [_buffers(c["cond"], c["uncond"]) for c in cases]
    c0 = cases[0]
    _call(yar, tiny, bufs[0], c0["smp"], c0["history"], c0["step"], c0["phase"], c0["seed"], c0["cfg_scale"])
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(0)
    for _ in range(2):  # two rounds of calls, each round both cases in a row
        for c, b in zip(cases, bufs):
            _call(yar, tiny, b, c["smp"], c["history"], c["step"], c["phase"], c["seed"], c["cfg_scale"])
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(0)
    assert free_after == free_before, (free_before, free_after)
    for i, (c, b) in enumerate(zip(cases, bufs)):
        unc = None if c["uncond"] is None else ora.bf16_from_bits(c["uncond"])
        want_tok, want_scores = so.sample(ora.bf16_from_bits(c["cond"]), c["raw"], c["history"], c["step"],
                                          c["phase"], c["seed"], unconditional=unc, cfg_scale=c["cfg_scale"])
        assert int(b["token"].item()) == want_tok, i
        scores = b["scores"].cpu().numpy()
        fin = np.isfinite(want_scores)
        np.testing.assert_array_equal(np.isfinite(scores), fin, err_msg=f"case {i}")
        np.testing.assert_array_equal(scores[fin], want_scores[fin], err_msg=f"case {i}")


def test_noalloc_sampler_rejects_rows_beyond_its_scratch(yar, tiny):
    smp = yar.Sampling(temperature=0.0, top_p=1.0, top_k=5, repetition_penalty=1.0, penalty_window=1,
                       min_tokens=0, max_tokens=10)
    big = np.zeros(MAX_COLUMNS + 1, np.uint16)
    with pytest.raises(yar.YarError) as e:
        _noalloc(yar, tiny, big, None, smp, [], 0, "full", 0, 1.0)
    assert e.value.status == 2 and "exceed" in e.value.message
    # The widest allowed row still matches the host entry point afterwards.
    rng = np.random.default_rng(5)
    cond = ora.bits_from_bf16(rng.standard_normal(MAX_COLUMNS).astype(np.float32))
    tok, scores = _noalloc(yar, tiny, cond, None, smp, [], 0, "full", 0, 1.0)
    want_tok, want_scores = tiny.sample(cond, smp, [], 0, "full", 0)
    assert tok == want_tok
    np.testing.assert_array_equal(scores, want_scores)
