"""AR decode benchmark (BASELINE config 2 per GPU): YuE2-3B dims, BF16, synthetic seeded
weights, prompt of 512 random ids, 400 sampled semantic tokens (T 1.0, top-k 50,
top-p 0.93, reference defaults elsewhere; min_tokens = max_tokens so every run decodes
exactly 400 tokens). One bench step = one generate_tokens call through the C ABI.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU, each rank an independent song (data
parallel, no collective on the data path; NCCL only for the barrier and the max-reduce
of the timings). Prints one JSON line on rank 0.

More workloads are reported under their own keys of the same line: "cfg" (config 3: one
classifier-free-guidance song per GPU, conditional prompt 1024 / unconditional 64, scale
1.5, 3000 tokens), "bs64" (config 5: 64 independent requests per GPU, data parallel) and
"long_context" (config 4: one 9000-position song, tensor-parallel across all N ranks).

`--impl reference` times the CPU restatement of the reference's AR path (oracle/, a numpy
port: the reference's own AR engine is Apple-only MLX) decoding the same config-2 song on
all host threads: the whole 28-layer model on the bench's own weights, the semantic head
and the sampler, a bounded number of decode steps per bench step.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "AR decode tok/s (bs1/GPU; bs64 box-wide) and % of HBM roofline"
PROMPT, DECODE = 512, 400
SAMPLING = dict(temperature=1.0, top_p=0.93, top_k=50, repetition_penalty=1.2, penalty_window=50,
                min_tokens=DECODE, max_tokens=DECODE)
LAYER_BYTES = 50_331_648 * 2          # q,k,v,o,gate,up,down of one layer, BF16
NORM_BYTES = 28 * (2 * 2048 + 2 * 128) * 2 + 2048 * 2
HEAD_BYTES = 32769 * 2048 * 2         # semantic LM-head rows
KV_BYTES_PER_POS = 28 * 2 * 8 * 128 * 2
EMBED_BYTES = 2048 * 2


def step_bytes(L: int) -> int:
    """Algorithmic HBM bytes of one decode step at L visible positions (B = 1)."""
    return 28 * LAYER_BYTES + NORM_BYTES + HEAD_BYTES + EMBED_BYTES + KV_BYTES_PER_POS * (L + 1)


def q_matrix_bytes(rows: int, cols: int, bits: int = 8) -> int:
    """Bytes of one matrix in quantized form: bits / 8 bytes per weight plus a BF16 scale and
    bias per 64 weights (rows padded to the 16-row stage unit the kernel streams)."""
    return int((rows + 15) // 16 * 16 * cols * (bits / 8 + 4 / 64))


def q_step_bytes(L: int, bits: int = 8) -> int:
    """Algorithmic HBM bytes of one quantized decode step at L visible positions (B = 1)."""
    layer = sum(q_matrix_bytes(r, c, bits) for r, c in ((4096, 2048), (2048, 2048), (12288, 2048), (2048, 6144)))
    return 28 * layer + NORM_BYTES + q_matrix_bytes(32769, 2048, bits) + EMBED_BYTES + KV_BYTES_PER_POS * (L + 1)


def q8_step_bytes(L: int) -> int:
    return q_step_bytes(L, 8)


def load_module(name, path, pkg=None):
    import importlib.util
    if name in sys.modules:
        return sys.modules[name]
    kw = {"submodule_search_locations": [pkg]} if pkg else {}
    spec = importlib.util.spec_from_file_location(name, path, **kw)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi clock/throttle sampling during the timed region."""

    def __init__(self, index: int):
        self.proc = None
        self.index = index

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}",
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.summary = None
        if not self.proc:
            return
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= 7]
        if not rows:
            return
        sm = [float(r[0]) for r in rows if r[0].strip().replace(".", "").isdigit()]
        reasons = set()
        for r in rows:
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), r[3:7]):
                if v.strip() == "Active":
                    reasons.add(name)
        self.summary = {"sm_mhz": float(np.median(sm)) if sm else None,
                        "sm_max_mhz": float(rows[0][1]) if rows[0][1].strip().replace(".", "").isdigit() else None,
                        "reasons": sorted(reasons), "samples": len(rows)}


BS64_REQUESTS, BS64_DECODE = 64, 1024


def batched_throughput(yar, model, rank, barrier, maxall, per_gpu: int, label: str, rows: int = 0,
                       n_requests: int = 0, lengths=None):
    """Config 5 on each GPU: `n_requests` (default `per_gpu`) independent requests served by
    continuous batching on `rows` rows (default: one row per request) — prompt lengths
    uniform in [256, 2048] (seeded per rank), top-k 50 with per-request seeds, fixed lengths
    (1024 tokens, or `lengths` = (lo, hi) drawn per request). Value = decoded tokens over
    the device time of the decode loop (max over ranks) x ranks; e2e includes the prefills
    (a refilled row's prefill runs between decode chunks)."""
    rng = np.random.default_rng(5000 + rank)
    n_req = n_requests or per_gpu
    rows = rows or n_req
    lens = rng.integers(256, 2049, n_req)
    prompts = [rng.integers(0, 184704, int(n)).astype(np.int32) for n in lens]
    seeds = [int(x) for x in rng.integers(0, 2**62, n_req)]
    outs = ([BS64_DECODE] * n_req if lengths is None else
            [int(x) for x in rng.integers(lengths[0], lengths[1] + 1, n_req)])
    smps = [yar.Sampling(**dict(SAMPLING, min_tokens=o, max_tokens=o)) for o in outs]
    warm = yar.Sampling(**dict(SAMPLING, min_tokens=16, max_tokens=16))
    s = model.session(max_rows=rows, max_ctx=2048 + max(outs))
    s.generate_requests([p[:256] for p in prompts[:rows]], [warm] * rows, seeds[:rows], phase="semantic",
                        slots=rows)  # capture + first use
    barrier()
    t0 = time.perf_counter()
    toks, timing, _ = s.generate_requests(prompts, smps, seeds, phase="semantic", slots=rows)
    wall = time.perf_counter() - t0
    s.close()
    n = sum(len(t) for t in toks)
    dec = maxall(timing["decode_device_ms"] / 1000.0)
    wall = maxall(wall)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    steps = timing["decode_steps"]
    avg_L = float(np.mean(lens)) + float(np.mean(outs)) / 2
    step_bytes_b = 28 * LAYER_BYTES + NORM_BYTES + HEAD_BYTES + rows * (EMBED_BYTES + KV_BYTES_PER_POS * (avg_L + 1))
    peak, _ = peaks()
    achieved = step_bytes_b / (dec / steps) / 1e9
    return {"workload": label, "requests_per_gpu": n_req, "rows_per_gpu": rows,
            "value": n * world / dec, "unit": "tok/s", "e2e": n * world / wall,
            "prefill_s": timing["prefill_seconds"], "ms_per_step": 1000 * dec / steps, "decode_steps": steps,
            "refills": timing["refills"], "tokens": n * world, "bytes_per_step": int(step_bytes_b),
            "achieved_gbs": achieved, "frac_of_hbm": achieved / peak, "forward": timing["forward"]}


CFG_COND, CFG_UNCOND, CFG_DECODE, CFG_SCALE = 1024, 64, 3000, 1.5


def cfg_song(yar, model, rank, barrier, maxall):
    """Config 3 on each GPU: one classifier-free-guidance song — conditional prompt of 1024
    random ids, unconditional prompt of 64, guidance scale 1.5, 3000 sampled semantic tokens
    (fixed length) — both branches decoded together as one two-row step per token (the
    weights are read once for both rows). Value = song tokens over the decode loop's device
    time, max over ranks; e2e = song tokens over the wall time of the generate call (both
    prefills, host copies and the token read-back included)."""
    rng = np.random.default_rng(3000 + rank)
    cond = rng.integers(0, 184704, CFG_COND).astype(np.int32)
    uncond = rng.integers(0, 184704, CFG_UNCOND).astype(np.int32)
    s = model.session(max_rows=2, max_ctx=CFG_COND + CFG_DECODE + 8)
    s.generate(cond[:256], yar.Sampling(**dict(SAMPLING, min_tokens=32, max_tokens=32)), seed=1, phase="semantic",
               negative=uncond, cfg_scale=CFG_SCALE)
    barrier()
    smp = yar.Sampling(**dict(SAMPLING, min_tokens=CFG_DECODE, max_tokens=CFG_DECODE))
    t0 = time.perf_counter()
    toks, timing, _ = s.generate(cond, smp, seed=2, phase="semantic", negative=uncond, cfg_scale=CFG_SCALE)
    wall = time.perf_counter() - t0
    s.close()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    dec, wall = maxall(timing["decode_device_ms"] / 1000.0), maxall(wall)
    # Per step: the weights once, both rows' KV (average visible lengths over the song).
    kv_pos = (CFG_COND + CFG_DECODE / 2) + (CFG_UNCOND + CFG_DECODE / 2)
    step_b = 28 * LAYER_BYTES + NORM_BYTES + HEAD_BYTES + 2 * EMBED_BYTES + KV_BYTES_PER_POS * (kv_pos + 2)
    peak, _ = peaks()
    achieved = step_b / (dec / len(toks)) / 1e9
    return {"workload": "config3: one CFG song per GPU, cond prompt 1024 / uncond 64 random ids, scale 1.5, "
                        "3000 semantic tokens, T1.0 top-k50 top-p0.93",
            "value": len(toks) * world / dec, "unit": "tok/s", "e2e": len(toks) * world / wall,
            "tokens": len(toks) * world, "ms_per_token": 1000 * dec / len(toks), "prefill_s": timing["prefill_seconds"],
            "bytes_per_step": int(step_b), "achieved_gbs": achieved, "frac_of_hbm": achieved / peak,
            "cfg_branches": timing.get("cfg_branches")}


LONG_PROMPT, LONG_TOTAL = 2048, 9000


def long_context(yar, model_one, weights, rank, world, local, barrier, maxall):
    """Config 4: one song — prompt of 2048 random ids decoded to 9000 positions (6952
    sampled semantic tokens, fixed length), 256-token pages — tensor-parallel over all
    ranks (TP = N; N = 1 runs the one-GPU model, persistent kernel). Value = decoded tokens
    over the decode loop's device time, max over ranks; e2e = tokens over the wall time of
    the generate call (prefill, host copies and the token read-back included)."""
    if world > 1:
        import torch.distributed as dist
        ids = [yar.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        model = yar.ARModel(weights, device=local, tp=(rank, world, ids[0]))
    else:
        model = model_one
    n_dec = LONG_TOTAL - LONG_PROMPT
    rng = np.random.default_rng(7000)  # the same song on every rank
    prompt = rng.integers(0, 184704, LONG_PROMPT).astype(np.int32)
    s = model.session(max_rows=1, max_ctx=LONG_TOTAL, page_tokens=256)
    s.generate(prompt[:256], yar.Sampling(**dict(SAMPLING, min_tokens=32, max_tokens=32)), seed=1, phase="semantic")
    barrier()
    t0 = time.perf_counter()
    toks, timing, _ = s.generate(prompt, yar.Sampling(**dict(SAMPLING, min_tokens=n_dec, max_tokens=n_dec)), seed=2,
                                 phase="semantic")
    wall = time.perf_counter() - t0
    s.close()
    if model is not model_one:
        model.close()
    dec, wall = maxall(timing["decode_device_ms"] / 1000.0), maxall(wall)
    avg_L = LONG_PROMPT + n_dec / 2
    # Per GPU and token: its share of the layers, the head and the KV cache, plus the
    # replicated norms and embedding row.
    per_gpu = (28 * LAYER_BYTES + HEAD_BYTES + KV_BYTES_PER_POS * (avg_L + 1)) / world + NORM_BYTES + EMBED_BYTES
    peak, _ = peaks()
    achieved = per_gpu / (dec / len(toks)) / 1e9
    return {"workload": "config4: one song, prompt 2048, decoded to 9000 positions, 256-token pages",
            "parallelism": f"tp{world}", "value": len(toks) / dec, "unit": "tok/s", "e2e": len(toks) / wall,
            "tokens": len(toks), "ms_per_token": 1000 * dec / len(toks), "prefill_s": timing["prefill_seconds"],
            "bytes_per_token_per_gpu": int(per_gpu), "achieved_gbs_per_gpu": achieved, "frac_of_hbm": achieved / peak,
            "tensor_parallel": timing["tensor_parallel"], "tp_exchange": timing["tp_exchange"]}


def measured_traffic(avg_L: float, profile: str = "decode_persistent_config2.txt"):
    """DRAM bytes (read + write) of one persistent decode launch from the committed ncu
    capture, moved from the captured position to `avg_L` by the KV bytes per position
    (weights and head rows are position-independent)."""
    path = os.path.join(ROOT, "profiles", profile)
    try:
        kv = dict(line.split(":", 1) for line in open(path) if line.startswith("traffic_"))
        return int(int(kv["traffic_bytes_per_launch"]) + KV_BYTES_PER_POS * (avg_L - int(kv["traffic_position"])))
    except (OSError, KeyError, ValueError):
        return None


def ensure_weights(rank: int, world: int, barrier, q8: bool = False, q4: bool = False) -> str:
    synth = load_module("yue2_mlx_b200_synth", os.path.join(ROOT, "yue2-mlx_b200", "synth.py"))
    d = os.environ.get("YAR_BENCH_WEIGHTS", os.path.join(tempfile.gettempdir(), "yar_bench_3b_seed0"))
    marker = os.path.join(d, ".complete")
    if rank == 0 and not os.path.exists(marker):
        synth.write_converted(d, synth.PINNED, seed=0)
        open(marker, "w").write("ok")
    for bits, want in ((8, q8), (4, q4)):
        marker_q = os.path.join(d, f".complete_{bits}bit")
        if want and rank == 0 and not os.path.exists(marker_q):
            # The quantized artifact of the same weights (conversion.py:651-735 quantizes the
            # BF16 file).
            synth.write_quantized(d, synth.PINNED, bits=bits)
            man = json.load(open(os.path.join(d, "conversion.json")))
            man["precisions"][f"{bits}bit"] = synth.quantized_record(bits)
            json.dump(man, open(os.path.join(d, "conversion.json"), "w"), indent=1)
            open(marker_q, "w").write("ok")
    barrier()
    return d


def q8_song(yar, weights, rank, barrier, maxall, steps: int, local: int, peak: float, bits: int = 8):
    """Config 2 on the `8bit` (or `4bit`) precision of the same weights (affine group-64
    linears, ar-<bits>bit.safetensors): the same prompts, sampling and timing as the
    headline, decode through the quantized persistent kernel."""
    import torch
    model = yar.ARModel(weights, device=local, precision=f"{bits}bit")
    session = model.session(max_rows=1, max_ctx=PROMPT + DECODE)
    smp = yar.Sampling(**SAMPLING)
    rng = np.random.default_rng(3000 + rank)
    prompts = [rng.integers(0, 184704, PROMPT).astype(np.int32) for _ in range(2 + steps)]
    for i in range(2):
        session.generate(prompts[i], smp, seed=i, phase="semantic")
    barrier()
    decode_ms, wall, tokens = 0.0, 0.0, 0
    for i in range(steps):
        t0 = time.perf_counter()
        toks, timing, _ = session.generate(prompts[2 + i], smp, seed=2 + i, phase="semantic")
        wall += time.perf_counter() - t0
        decode_ms += timing["decode_device_ms"]
        tokens += len(toks)
    torch.cuda.synchronize()
    barrier()
    decode_s, wall_s = maxall(decode_ms / 1000.0), maxall(wall)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    per_token_s = decode_s / tokens
    bytes_per_step = q_step_bytes(int(PROMPT + DECODE / 2), bits)
    achieved = bytes_per_step / per_token_s / 1e9
    session.close()
    model.close()
    return {"workload": f"config2 on the {bits}bit precision of the bench weights (affine {bits}-bit group-64 "
                        "linears, BF16 embedding and norms), same prompts/sampling/timing as the headline",
            "value": tokens * world / decode_s, "unit": "tok/s", "ms_per_token": 1000 * per_token_s,
            "e2e": {"value": tokens * world / wall_s, "unit": "tok/s"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "bytes_per_step": bytes_per_step}}


class CpuDecoder:
    """The CPU restatement of the reference's AR path (oracle/ar_oracle.py + the sampler
    oracle) decoding config 2 on the host cores: every one of the 28 layers on the bench's
    own weights (BF16 values held as float32, float32 BLAS on every host thread), the
    semantic head rows and the sampler, after a 512-token prefill. The embedding rows are
    formed from the BF16 bits as they are looked up."""

    def __init__(self, weights_dir: str, threads: int):
        import threadpoolctl
        synth = load_module("yue2_mlx_b200_synth", os.path.join(ROOT, "yue2-mlx_b200", "synth.py"))
        from oracle import ar_oracle as ora
        from oracle import sampler_oracle as so
        self.ora, self.so = ora, so
        self.limits = threadpoolctl.threadpool_limits(threads)  # torchrun sets OMP_NUM_THREADS=1
        self.threads = threads
        bits = synth.read_safetensors(os.path.join(weights_dir, "ar-bf16.safetensors"))

        class EmbedRows:
            def __init__(self, b):
                self.b = b

            def __getitem__(self, ids):
                return ora.bf16_from_bits(self.b[ids])

        tensors = {}
        for name, arr in bits.items():
            if name == "model.embed_tokens.weight":
                tensors[name] = EmbedRows(arr)
            elif name == "lm_head.weight":
                t = np.zeros(arr.shape, np.float32)  # untouched pages are never materialized
                r0, r1 = ora.MUSIC_END, ora.CODEC_OFFSET + ora.CODEC_SIZE
                t[r0:r1] = ora.bf16_from_bits(arr[r0:r1])
                tensors[name] = t
            else:
                tensors[name] = ora.bf16_from_bits(arr)
        synth_dims = synth.PINNED
        self.model = ora.OracleAR(tensors, synth_dims, bf16=True, prerounded=True)
        rng = np.random.default_rng(1000)
        self.prompt = rng.integers(0, 184704, PROMPT).tolist()
        self.cache = self.model.new_cache(PROMPT + DECODE)
        t0 = time.perf_counter()
        h = self.model.forward(self.prompt, self.cache)
        self.prefill_s = time.perf_counter() - t0
        self.logits = self.model.project(h[-1], "semantic")[0]
        self.history: list[int] = []
        self.decoded = 0

    def decode(self, n: int) -> float:
        """Sample and forward n tokens (the GPU arm's sampler settings); returns seconds."""
        t0 = time.perf_counter()
        for _ in range(n):
            if self.cache["offset"] >= PROMPT + DECODE:  # keep the window at config-2 positions
                self.cache["offset"] = PROMPT
                self.history = []
            tok, _ = self.so.sample(self.logits, SAMPLING, self.history, len(self.history), "semantic", 7)
            native = self.so.local_to_native(tok, "semantic")
            self.history.append(native)
            h = self.model.forward([native], self.cache)
            self.logits = self.model.project(h[-1], "semantic")[0]
            self.decoded += 1
        return time.perf_counter() - t0

    def sample_desc(self, n: int) -> str:
        return (f"numpy port of the reference AR path (oracle/), config-2 song: all 28 layers on the bench weights "
                f"(float32 math on BF16 values), semantic head, sampler; {n} decode steps at positions "
                f"{PROMPT}..{PROMPT + DECODE} after a {PROMPT}-token prefill ({self.prefill_s:.1f} s), float32 BLAS "
                f"on {self.threads} host threads")


def cpu_decode_sample(weights_dir: str, seconds_budget: float = 20.0):
    """Bounded CPU baseline: decode steps of CpuDecoder until ~seconds_budget has passed."""
    dec = CpuDecoder(weights_dir, os.cpu_count() or 1)
    dec.decode(1)  # first touch of every weight page
    spent, n = 0.0, 0
    while spent < seconds_budget and n < 64:
        spent += dec.decode(1)
        n += 1
    return {"value": n / spent, "unit": "tok/s", "cores": dec.threads, "kind": "port", "sample": dec.sample_desc(n)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-bs64", action="store_true", help="skip the config-5 batched throughput measurement")
    ap.add_argument("--no-long", action="store_true", help="skip the config-4 long-context tensor-parallel song")
    ap.add_argument("--no-cfg", action="store_true", help="skip the config-3 classifier-free-guidance song")
    ap.add_argument("--no-q8", action="store_true", help="skip the config-2 song on 8-bit weights")
    ap.add_argument("--no-q4", action="store_true", help="skip the config-2 song on 4-bit weights")
    ap.add_argument("--precision", choices=["bf16", "8bit", "4bit"], default="bf16",
                    help="weights of the headline song (quantized: that precision's line is the headline)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    config = {"workload": "config2: YuE2-3B dims (28L, H2048, 16/8 heads, FFN 6144, vocab 184704), bs1 per GPU, "
                          "prompt 512 random ids, 400 semantic tokens, T1.0 top-k50 top-p0.93",
              "batch_per_gpu": 1, "prompt": PROMPT, "decode": DECODE, "phase": "semantic",
              "parallelism": f"dp{args.gpus}", "l2": "inputs larger than L2 (2.95 GB of weights per step)"}

    if args.impl == "reference":
        if rank != 0:
            return  # rank 0 alone times the CPU arm; the other ranks exit without work
        weights = ensure_weights(0, 1, lambda: None)
        dec = CpuDecoder(weights, os.cpu_count() or 1)
        per_step = 4  # decode steps per bench step (a bounded sample of the config-2 song)
        for _ in range(args.warmup):
            dec.decode(per_step)
        times = [dec.decode(per_step) for _ in range(args.steps)]
        v = per_step * args.steps / sum(times)
        print(json.dumps({"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s",
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": 1000 * sum(times) / args.steps, "ms_per_token": 1000 * sum(times) / (per_step * args.steps),
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "bf16 storage, f32 math", "data": "synthetic (the bench weights, random prompt ids)",
                          "config": dict(config, bench_step=f"{per_step} decode tokens of the config-2 song"),
                          "cpu_baseline": {"value": v, "unit": "tok/s", "cores": dec.threads, "kind": "port",
                                           "sample": dec.sample_desc(per_step * args.steps)},
                          "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        barrier = lambda: (torch.cuda.synchronize(), dist.barrier(device_ids=[local]))

        def maxall(v):
            t = torch.tensor([v], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
    else:
        barrier = lambda: torch.cuda.synchronize()
        maxall = lambda v: v

    q8_head = args.precision != "bf16"
    head_bits = {"bf16": 0, "8bit": 8, "4bit": 4}[args.precision]
    weights = ensure_weights(rank, world, barrier, q8=head_bits == 8, q4=head_bits == 4)
    yar = load_module("yue2_mlx_b200", os.path.join(ROOT, "yue2-mlx_b200", "__init__.py"),
                      os.path.join(ROOT, "yue2-mlx_b200"))
    model = yar.ARModel(weights, device=local, precision=args.precision)
    if q8_head:
        config = dict(config, workload=config["workload"] + f", {args.precision} precision (affine {head_bits}-bit "
                                                            "group-64 linears)",
                      l2=f"inputs larger than L2 ({q_step_bytes(0, head_bits) / 1e9:.2f} GB of weights per step)")
    session = model.session(max_rows=1, max_ctx=PROMPT + DECODE)
    smp = yar.Sampling(**SAMPLING)
    rng = np.random.default_rng(1000 + rank)
    prompts = [rng.integers(0, 184704, PROMPT).astype(np.int32) for _ in range(args.warmup + args.steps)]

    for i in range(args.warmup):
        session.generate(prompts[i], smp, seed=i, phase="semantic")
    barrier()
    decode_ms, wall, prefill_s, tokens = 0.0, 0.0, 0.0, 0
    with Clocks(local) as clk:
        t_start = time.perf_counter()
        for i in range(args.steps):
            t0 = time.perf_counter()
            toks, timing, _ = session.generate(prompts[args.warmup + i], smp, seed=args.warmup + i, phase="semantic")
            wall += time.perf_counter() - t0
            decode_ms += timing["decode_device_ms"]
            prefill_s += timing["prefill_seconds"]
            tokens += len(toks)
        torch.cuda.synchronize()
        t_total = time.perf_counter() - t_start
    barrier()
    decode_s = maxall(decode_ms / 1000.0)
    wall_s = maxall(wall)
    total_tokens = tokens * world
    value = total_tokens / decode_s
    e2e = total_tokens / wall_s
    per_token_s = decode_s / (tokens)
    avg_L = PROMPT + DECODE / 2
    bytes_per_step = q_step_bytes(int(avg_L), head_bits) if q8_head else step_bytes(int(avg_L))
    peak, peak_kind = peaks()
    achieved = bytes_per_step / per_token_s / 1e9
    layers = 28
    # Per decoded token: the persistent decode kernel (embedding, 28 layers, LM head) and
    # the sampler. Per song: the prefill's embedding, 10 kernels per layer, the head GEMV.
    launches_per_token = 2
    # Prefill of 512 tokens per layer: RMSNorm, QKV GEMM, q/k post, attention, O GEMM and
    # its split-K reduction, RMSNorm, gate/up GEMM, down GEMM and its reduction.
    prefill_launches = 1 + 10 * layers + 1
    traffic = measured_traffic(avg_L, f"decode_q{head_bits}_config2.txt" if q8_head else "decode_persistent_config2.txt")
    cfg = None if args.no_cfg else cfg_song(yar, model, rank, barrier, maxall)
    bs64 = bs64_weak = bs64_cont = None
    if not args.no_bs64:
        # Config 5 as BASELINE states it: 64 requests in all, sharded across the N GPUs.
        per = max(1, BS64_REQUESTS // world)
        bs64 = batched_throughput(yar, model, rank, barrier, maxall, per,
                                  f"config5: 64 requests sharded across {world} GPU(s) ({per} per GPU, one row "
                                  "each), prompts U[256,2048], 1024 tokens each, top-k 50")
        if world > 1:  # weak-scaling variant: 64 requests on every GPU
            bs64_weak = batched_throughput(yar, model, rank, barrier, maxall, BS64_REQUESTS,
                                           "config5 weak variant: 64 requests per GPU, prompts U[256,2048], "
                                           "1024 tokens each, top-k 50")
        # Continuous batching: 96 requests per GPU with lengths U[512,1536] on 64 rows, finished
        # rows refilled from the queue between decode chunks.
        bs64_cont = batched_throughput(yar, model, rank, barrier, maxall, 96,
                                       "config5 continuous batching: 96 requests per GPU on 64 rows, prompts "
                                       "U[256,2048], U[512,1536] tokens each, top-k 50", rows=64,
                                       n_requests=96, lengths=(512, 1536))
    quant = {}
    for bits, skip in ((8, args.no_q8), (4, args.no_q4)):
        if skip or q8_head:
            quant[bits] = None
            continue
        try:
            ensure_weights(rank, world, barrier, q8=bits == 8, q4=bits == 4)
            quant[bits] = q8_song(yar, weights, rank, barrier, maxall, args.steps, local, peak, bits)
        except Exception as e:
            quant[bits] = {"error": f"{type(e).__name__}: {e}"[:300]}
    long = None
    if not args.no_long:
        # Every rank takes the same path, so a failure here is raised on every rank alike:
        # it is reported in the line instead of losing the data-parallel measurement.
        try:
            long = long_context(yar, model, weights, rank, world, local, barrier, maxall)
        except Exception as e:
            long = {"error": f"{type(e).__name__}: {e}"[:300]}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_decode_sample(weights)
        except Exception as e:  # reported, not fatal
            cpu = {"error": str(e)}
    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000 * decode_s / args.steps, "ms_per_token": 1000 * per_token_s,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": f"u{head_bits} weights, bf16 activations" if q8_head else "bf16",
            "data": "synthetic (seeded N(0,0.02) weights, random prompt ids)", "config": config,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": PROMPT * 4,
                    "d2h_bytes_per_step": DECODE * 4 + 20 * ((DECODE + 15) // 16),
                    "prefill_s_per_step": prefill_s / args.steps},
            "roofline": {"bound": "hbm",
                         "kernel": "k_decode_persistent (whole decode forward, one CTA per SM) + k_sampler; "
                                   "achieved = algorithmic bytes / device time per decoded token (both kernels)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_kind, "bytes_per_step": bytes_per_step, "traffic": traffic},
            "gpu_launches": args.steps * (DECODE * launches_per_token + prefill_launches),
            "clocks": clk.summary,
            "cpu_baseline": cpu,
            "cfg": cfg,
            "bs64": bs64,
            "bs64_per_gpu": bs64_weak,
            "bs64_continuous": bs64_cont,
            "long_context": long,
            "q8": quant[8],
            "q4": quant[4],
        }
        print(json.dumps(out))
    session.close()
    model.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
