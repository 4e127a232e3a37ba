"""One rank of the tensor-parallel GPU test (launched by torchrun, one process per GPU).

Every rank loads its tensor-parallel share of the model (NCCL group from the id that
rank 0 makes and broadcasts over a gloo group) and, on the same GPU, the whole model as
the one-GPU reference, then runs the same calls on both:

* teacher-forced prefill + decode steps (one row, and a CFG-style pair of rows) in the
  full-vocabulary phase of the 4096-row model: logits of the two models side by side;
* the same in the semantic and ABC phases of a 184,704-row model (the LM head split by
  columns across ranks, the ABC extra row included);
* a sampled generation and a batched generation (18 requests, the tcgen05 forward): the
  tokens every rank returns, against each other and against the one-GPU model's.

Rank 0 writes the measurements as JSON to the path given; the pytest side asserts.
"""
import datetime
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch.distributed as dist  # noqa: E402

from tests.conftest import load_package  # noqa: E402


def f(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def forced_logits(model, prompt, forced, rows, phase, ctx, persistent=True):
    s = model.session(max_rows=2, max_ctx=ctx)
    s.set_persistent(persistent)
    for r in range(rows):
        s.reset(r, ctx)
        s.prefill(r, prompt, phase=phase)
    out = [f(s.logits(0, phase))]
    for t in forced:
        s.step(list(range(rows)), [t] * rows, phase=phase)
        out.append(f(s.logits(0, phase)))
    s.close()
    return np.stack(out)


def main():
    small_dir, vocab_dir, out_path = sys.argv[1], sys.argv[2], sys.argv[3]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    device = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    yar = load_package()
    res = {"world": world}

    def gather(obj):
        objs = [None] * world
        dist.all_gather_object(objs, obj)
        return objs

    def new_group_id():
        ids = [yar.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        return ids[0]

    # 4096-row model, full-vocabulary phase.
    tp = yar.ARModel(small_dir, device=device, any_dims=True, tp=(rank, world, new_group_id()))
    one = yar.ARModel(small_dir, device=device, any_dims=True)
    res["dims_tp"], res["dims_one"] = tp.dims, one.dims
    rng = np.random.default_rng(5)
    prompt, forced = rng.integers(0, 4096, 300).tolist(), rng.integers(0, 4096, 12).tolist()
    # Decode steps of one row and of a row pair: the persistent kernel (exchanging through
    # stores into the peers' buffers) and the per-operation kernels (exchanging through NCCL).
    for rows in (1, 2):
        b = forced_logits(one, prompt, forced, rows, None, 400)
        for mode, persistent in (("", True), ("_per_op", False)):
            a = forced_logits(tp, prompt, forced, rows, None, 400, persistent)
            res[f"full_rows{rows}{mode}"] = {"max_abs": float(np.abs(a - b).max()), "rel_l2": rel_l2(a, b),
                                             "bit_identical": bool(np.array_equal(a, b)),
                                             "same_on_all_ranks": len({x.tobytes() for x in gather(a)}) == 1}

    smp = dict(temperature=1.0, top_p=0.93, top_k=50, repetition_penalty=1.2, penalty_window=50, min_tokens=24,
               max_tokens=24)
    s = tp.session(max_rows=1, max_ctx=512)
    toks, timing, _ = s.generate(prompt, yar.Sampling(**smp), seed=7, phase=None)
    s.close()
    s = one.session(max_rows=1, max_ctx=512)
    toks_one, _, _ = s.generate(prompt, yar.Sampling(**smp), seed=7, phase=None)
    s.close()
    res["generate"] = {"tokens": toks, "ranks_agree": all(t == toks for t in gather(toks)),
                       "equal_to_one_gpu": toks == toks_one, "tensor_parallel": timing["tensor_parallel"],
                       "tp_exchange": timing["tp_exchange"]}

    n = 18
    prefixes = [rng.integers(0, 4096, int(rng.integers(20, 200))).tolist() for _ in range(n)]
    seeds = [int(x) for x in rng.integers(0, 2**62, n)]
    bsmp = dict(smp, min_tokens=8, max_tokens=8)
    s = one.session(max_rows=n, max_ctx=256)
    btoks_one, _, _ = s.generate_batch(prefixes, yar.Sampling(**bsmp), seeds, phase=None)
    s.close()
    s = tp.session(max_rows=n, max_ctx=256)
    btoks, btiming, _ = s.generate_batch(prefixes, yar.Sampling(**bsmp), seeds, phase=None)
    # One teacher-forced batched step on both models: logits side by side.
    for r in range(n):
        s.reset(r, 256)
        s.prefill(r, prefixes[r], phase=None)
    s.step(list(range(n)), [btoks[r][0] for r in range(n)], phase=None)
    lb_tp = np.stack([f(s.logits(r, None)) for r in range(n)])
    s.close()
    s = one.session(max_rows=n, max_ctx=256)
    for r in range(n):
        s.reset(r, 256)
        s.prefill(r, prefixes[r], phase=None)
    s.step(list(range(n)), [btoks[r][0] for r in range(n)], phase=None)
    lb_one = np.stack([f(s.logits(r, None)) for r in range(n)])
    s.close()
    res["batch"] = {"forward": btiming["forward"], "ranks_agree": all(b == btoks for b in gather(btoks)),
                    "equal_to_one_gpu": btoks == btoks_one, "bit_identical": bool(np.array_equal(lb_tp, lb_one)),
                    "max_abs": float(np.abs(lb_tp - lb_one).max()), "rel_l2": rel_l2(lb_tp, lb_one)}
    tp.close()
    one.close()

    # 184,704-row model: the semantic and ABC phases (the LM head split by columns).
    tp = yar.ARModel(vocab_dir, device=device, any_dims=True, tp=(rank, world, new_group_id()))
    one = yar.ARModel(vocab_dir, device=device, any_dims=True)
    prompt, forced = rng.integers(0, 184704, 200).tolist(), rng.integers(0, 184704, 4).tolist()
    for phase in ("semantic", "abc"):
        a = forced_logits(tp, prompt, forced, 1, phase, 256)
        b = forced_logits(one, prompt, forced, 1, phase, 256)
        res[phase] = {"width": int(a.shape[1]), "max_abs": float(np.abs(a - b).max()), "rel_l2": rel_l2(a, b),
                      "bit_identical": bool(np.array_equal(a, b)),
                      "same_on_all_ranks": len({x.tobytes() for x in gather(a)}) == 1}
    tp.close()
    one.close()

    if rank == 0:
        with open(out_path, "w") as fh:
            json.dump(res, fh)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
