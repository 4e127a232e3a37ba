"""Failure detection without a GPU fault, through the C ABI.

* A bounded device wait that runs out: the session option YAR_OPT_FAULT_INJECT makes one
  operation of the persistent decode kernel wait for a flag that nothing writes (with a
  short poll limit). The wait expires, the kernel records an error code in the session's
  device error word and finishes its step without computing; the call returns
  RuntimeError, and the next call on the same session succeeds with the same result as a
  fresh session (the failed step left no state behind). No trap, fault or endless loop is
  involved.
* A tensor-parallel rank that never joins: a rank-0 load for a world of two whose peer
  never calls in gives up after the join deadline (YAR_TP_JOIN_TIMEOUT_S), aborts its
  communicator and returns RuntimeError, in a child process so no state is shared.
"""
import dataclasses
import os
import subprocess
import sys
import time

import numpy as np
import pytest

from tests.conftest import ROOT, load_package

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def yar():
    return load_package()


@pytest.fixture(scope="module")
def wide2(yar, synth, tmp_path_factory):
    dims = dataclasses.replace(synth.PINNED, layers=2, vocab=4096, context=4096)
    d = str(tmp_path_factory.mktemp("wide2f"))
    synth.write_converted(d, dims, seed=3, norm_std=0.1)
    return yar.ARModel(d, any_dims=True)


@pytest.mark.parametrize("op,rows", [(1 + 5 * 1 + 3, 1), (1 + 5 * 0 + 1, 2), (1 + 5 * 1 + 0, 2)])
def test_expired_device_wait_is_an_error_and_the_session_recovers(yar, wide2, op, rows):
    """op: layer 1 gate/up (1 row), layer 0 attention (2 rows), layer 1 QKV (2 rows)."""
    rng = np.random.default_rng(71)
    prompts = [rng.integers(0, 4096, 100).tolist(), rng.integers(0, 4096, 57).tolist()]
    s = wide2.session(max_rows=2, max_ctx=256)
    s.set_trace(True)
    for r in range(rows):
        s.reset(r, 256)
        s.prefill(r, prompts[r], phase=None)
    s.set_fault_inject(op)
    t0 = time.time()
    with pytest.raises(yar.YarError) as e:
        s.step(list(range(rows)), [5] * rows, phase=None)
    assert e.value.kind == "RuntimeError" and "device error" in e.value.message
    assert time.time() - t0 < 30
    assert np.any(s.trace()), "the persistent decode kernel did not run"
    assert [s.position(r) for r in range(rows)] == [len(p) for p in prompts[:rows]]
    s.set_fault_inject(0)
    s.step(list(range(rows)), [5] * rows, phase=None)
    got = [s.logits(r, None) for r in range(rows)]
    fresh = wide2.session(max_rows=2, max_ctx=256)
    for r in range(rows):
        fresh.reset(r, 256)
        fresh.prefill(r, prompts[r], phase=None)
    fresh.step(list(range(rows)), [5] * rows, phase=None)
    for r in range(rows):
        np.testing.assert_array_equal(got[r], fresh.logits(r, None))
    s.close()
    fresh.close()


CHILD = r"""
import os, sys, time
sys.path.insert(0, sys.argv[1])
from tests.conftest import load_package
yar = load_package()
uid = yar.tp_unique_id()
t0 = time.time()
try:
    yar.ARModel(sys.argv[2], device=0, any_dims=True, tp=(0, 2, uid))
    print("LOADED")
except yar.YarError as e:
    print("ERROR", e.kind, "|", e.message, "|", round(time.time() - t0, 1))
"""


def test_tensor_parallel_rank_that_never_joins_times_out(tiny_dir):
    env = dict(os.environ, YAR_TP_JOIN_TIMEOUT_S="3", NCCL_NVLS_ENABLE="0")
    out = subprocess.run([sys.executable, "-c", CHILD, ROOT, tiny_dir], env=env, capture_output=True, text=True,
                         timeout=120)
    line = [ln for ln in out.stdout.splitlines() if ln.startswith(("ERROR", "LOADED"))]
    assert line, out.stdout + out.stderr
    assert line[0].startswith("ERROR RuntimeError"), line[0]
    assert "did not join" in line[0]
    assert float(line[0].rsplit("|", 1)[1]) < 60
