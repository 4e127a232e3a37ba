// kernels_persistent.cu — the whole decode forward of one token (1 or 2 rows) as one
// persistent kernel: embedding, 28 x (QKV, attention, O, gate/up, down), LM head.
//
// Why: bs1 decode streams 2.95 GB of weights per token through ~143 dependent operations;
// as separate kernels every boundary costs a ramp and a tail (several us), far more than
// the bandwidth time of the small projections. Here each CTA's producer lane streams the
// CTA's weight rows for every task of the step, in order, through a 6-stage (192 KB)
// shared-memory ring, waiting only for ring space — never for activations — so HBM keeps
// streaming while the consumer warps wait at operation boundaries.
//
// Grid: one CTA per SM, co-resident by cooperative launch. Block: 8 consumer warps + a
// producer warpgroup (one lane issues the copies; see kPersistThreads). Operation boundaries are flagged words: every output is stored as an
// 8-byte word of two BF16 values and a flag naming the step and the operation, and the
// next operation polls (bounded) the words it reads until they carry the expected flag.
// Global counters remain for the position latch at the step's start and, under tensor
// parallelism, for the head; `epoch` counts completed steps (the last action of a step is
// CTA 0 advancing it), so neither flags nor counters need a reset between steps.
//
// The GEMV and attention code is the same device code as the standalone kernels
// (tma_ring.cuh, attn_decode.cuh): both paths produce identical logits.
//
// Failure: every wait is bounded and also gives up as soon as any CTA has recorded an
// error; a CTA that gave up keeps releasing ring stages and taking every barrier (so its
// producer finishes and no copy is left in flight) and keeps signalling counters (so
// other CTAs do not wait for it), without computing.
//
// Tensor parallelism (tp_world ranks, one GPU each, every rank running this kernel for the
// same step): each rank's operations compute its rows (its heads' attention, its hidden
// rows of O and down, its FFN rows of gate/up, its columns of the head) and the epilogues
// store every flagged word both locally and into each peer's mapped copy of the buffer
// (x, attn, mlp, logits: one exchange region per session, mapped by CUDA IPC); a reader
// polls its local copy for the flag. The all-gather is the epilogue's stores, and the
// flag wait is the only synchronization. The head's counter is released to every rank at
// system scope and counts all ranks' contributions. QKV stays rank-local.
#include "attn_decode.cuh"
#include "tma_ring.cuh"

namespace yar {

constexpr int kPersistStages = 6;
// 8-bit weights: 34,816-byte stages (16 rows x 2048 columns and their scale/bias words); a
// KV chunk (32 KB) fits one. Five of them leave the shared memory the two-row kernel needs
// (a sixth for one row measured no faster: 0.833 vs 0.827 ms per token at config 2).
constexpr int kPersistStagesQ8 = 5;
// Block: two consumer warpgroups (warps 0..7) and a producer warpgroup (warps 8..11; lane
// 0 of warp 8 issues the copies). The launch gives every thread 168 registers (65536 / 384,
// rounded down to 8); the producer warpgroup then returns registers (setmaxnreg.dec to
// 40) and the consumer warpgroups take them (setmaxnreg.inc to 232): 4 x 32 x 40 +
// 8 x 32 x 232 = 64,512, the launch's total, and per scheduler partition (warps k, k+4,
// k+8) 40 + 2 x 232 = 504 x 32 <= 16,384. With 168 the one-row kernel spilled; with 232 it
// does not. The host launches only a build whose kernels use exactly kPersistLaunchRegs
// (an increase beyond the launch's total would never be granted).
constexpr int kPersistProducerWarps = 4;
constexpr int kPersistThreads = (kRingConsumers + kPersistProducerWarps) * 32;
constexpr int kPersistLaunchRegs = 168, kPersistProducerRegs = 40, kPersistConsumerRegs = 232;
static_assert(kPersistProducerWarps * 32 * kPersistProducerRegs + kRingConsumers * 32 * kPersistConsumerRegs <=
                  kPersistThreads * kPersistLaunchRegs,
              "register split exceeds the launch's registers");
static_assert(kPersistProducerRegs + 2 * kPersistConsumerRegs <= 512, "register split exceeds a scheduler partition");
constexpr int kPersistMaxK = 6144;
constexpr long long kCounterWaitLimit = 1ll << 22;  // polls of ~100 ns: under a second

constexpr int kMaxTpWorld = 8;
constexpr int kMaxPersistGrid = 256;

struct PersistParams {
  CUtensorMap head_map;        // stage map of this rank's phase rows of the head (`head`, `head_rows`)
  const CUtensorMap *wmaps;    // device array [layer][4]: stage maps of qkv, o, gu, down
  // Quantized weights (the kernel's QB = 8 or 4): stage images per layer and of this rank's phase
  // rows of the head (rows [0, head_rows) as `head`).
  const QLayer *qlayers;
  const unsigned char *qhead;
  const LayerWeights *layers;  // device array, one entry per layer
  // QKV: this rank's q/k/v rows; QD, F: the model's query and FFN widths (the K of O and
  // down); HS, h0: this rank's hidden rows of O and down; FL, f0: its FFN rows.
  int n_layers, H, QKV, QD, F, vocab, HS, h0, FL, f0;
  float eps;
  const bf16 *embed, *final_norm, *head;
  int head_rows, extra_row;  // phase rows [0, head_rows) of `head`, plus one extra row or -1
  bf16 *x, *qkv, *attn, *mlp, *logits;
  int logit_stride;
  // Flagged-word copies of the activations (two BF16 values + a flag per 8-byte word),
  // [rows][stride words]: the residual rows, raw q/k/v, attention heads, FFN activations.
  uint2 *x_ll, *qkv_ll, *attn_ll, *mlp_ll;
  int x_lls, qkv_lls, attn_lls, mlp_lls;
  DecodeAttnParams ap;
  int *token, *pos, *cur_pos, *capacity, *active, *error;
  int *ctr, *epoch;
  int prefetch_stages;        // L2 prefetch distance beyond the ring, in stages
  unsigned long long *trace;  // optional [cta][op][8] SM-clock stamps (clock64), op = 5*layer + k
  bf16 *layer_dump;           // optional [n_layers + 1][dump_stride rows][H]: x after embedding / each layer
  int dump_stride;
  // Failure-path testing: operation `inject_op` (1 + 5 l + k; 0 = none) waits for a flag
  // nothing writes, and every flagged wait gives up after `ll_limit` polls.
  int inject_op;
  long long ll_limit;
  // Tensor parallelism: ranks, and the byte offsets from this rank's exchange region to
  // each peer's (as mapped here).
  int tp_world, tp_ndst;
  long long tp_dst[kMaxTpWorld - 1];
  // CTA c runs attention units attn_rank[c], + grid, ...: rank 0 is the CTA with the
  // fewest GEMV stages per layer (attention_ranks below).
  unsigned char attn_rank[kMaxPersistGrid];
};
static_assert(sizeof(PersistParams) <= 4096, "kernel parameters must fit the 4 KB launch limit");

__device__ __forceinline__ unsigned long long sm_clock() { return (unsigned long long)clock64(); }
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Release-add at GPU scope: orders this thread's earlier writes, and those of the CTA made
// visible to it by a preceding barrier, before the count.
__device__ __forceinline__ void red_release_add(int *p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// System scope, for the counters of exchanged operations (peer GPUs add to them after
// storing into this GPU's memory over NVLink). A system-scope fence costs microseconds, so
// the publisher takes one fence and then adds relaxed to every rank's counter (a release
// pattern), and a waiter polls relaxed and fences once the count is reached (an acquire
// pattern).
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void red_relaxed_add_sys(int *p, int v) {
  asm volatile("red.relaxed.sys.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_relaxed_sys(const int *p) {
  int v;
  asm volatile("ld.relaxed.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// True on every consumer thread when `v` is true on any of them (barrier `bar_id`).
__device__ __forceinline__ bool team_any(int bar_id, bool v) {
  int r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.s32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"(int(v)), "r"(bar_id), "n"(kAttnThreads)
      : "memory");
  return r != 0;
}

// The attention units of one step: rows in order; an active row has kv_heads x n_splits
// units (kv head major), an inactive row kv_heads units without work, each standing in for
// its kv head's arrival. Unit u runs on the CTA of attention rank u % grid, on all its
// consumer warps.
// Its chunks travel through the CTA's weight ring as stages (K rows, then V rows),
// issued right after the layer's QKV stages.
template <int NB>
struct StepRows {
  int active[NB], pos[NB];
};
struct UnitInfo {
  int row, kvh, split, n_splits, c0, c1;
  bool active;
};
template <int NB>
__device__ __forceinline__ int step_units(const StepRows<NB> &r, int kvh_n, int max_splits) {
  int U = 0;
  for (int b = 0; b < NB; ++b) U += kvh_n * (r.active[b] ? split_plan(r.pos[b] + 1, max_splits).n_splits : 1);
  return U;
}
template <int NB>
__device__ __forceinline__ UnitInfo step_unit(const StepRows<NB> &r, int kvh_n, int max_splits, int u) {
  UnitInfo ui{};
  for (int b = 0; b < NB; ++b) {
    const bool act = r.active[b] != 0;
    const SplitPlan sp = act ? split_plan(r.pos[b] + 1, max_splits) : SplitPlan{0, 1, 1};
    const int ub = kvh_n * sp.n_splits;
    if (u < ub || b == NB - 1) {
      ui.row = b;
      ui.active = act;
      ui.kvh = u / sp.n_splits;
      ui.split = u % sp.n_splits;
      ui.n_splits = sp.n_splits;
      ui.c0 = act ? ui.split * sp.cps : 0;
      ui.c1 = act ? min(ui.c0 + sp.cps, sp.nchunks) : 0;
      return ui;
    }
    u -= ub;
  }
  return ui;
}

constexpr int kMaxCtaChunks = 64;  // KV chunks of one CTA in one layer

// Rotation of the group ranges per operation (o: 0 QKV, 2 O, 3 gate/up, 4 down), as
// fractions of the grid: the CTAs holding one more group than the even share differ from
// operation to operation, so no CTA carries the most stages of every operation of a layer
// (on 148 SMs a CTA streams at most 22 GEMV stages per layer instead of 23) and every
// producer gets ahead of its consumers somewhere in the layer.
__host__ __device__ __forceinline__ int op_rotation(int o, int grid) {
  const int num = o == 2 ? 125 : o == 3 ? 108 : o == 4 ? 75 : 0;
  return num * grid / 148;
}

// Stages CTA `cta` streams of an N x K operation o (the split task_groups and the
// producer use; units of `urows` rows: 8 for BF16 stages, 16 for 8-bit ones).
__host__ __device__ __forceinline__ int op_cta_stages(int N, int K, int o, int cta, int grid, int urows = 8) {
  const int groups = (N + urows - 1) / urows, pos = (cta + op_rotation(o, grid)) % grid;
  return ((pos + 1) * groups / grid - pos * groups / grid) * (K / kRingPiece);
}

// Attention ranks: CTAs ordered by the GEMV stages they stream per layer (fewest first,
// then by index). A KV chunk is one more stage in its CTA's ring, and every operation
// waits for the CTA that finishes it last, so the units go to the CTAs with the fewest
// stages: at 96 one-chunk units on 148 SMs no CTA streams more than 22 stages per layer
// (23 with units on CTAs 0..95).
inline void attention_ranks(PersistParams &p, int grid, int urows) {
  int order[kMaxPersistGrid], total[kMaxPersistGrid];
  for (int c = 0; c < grid; ++c) {
    total[c] = op_cta_stages(p.QKV, p.H, 0, c, grid, urows) + op_cta_stages(p.HS, p.QD, 2, c, grid, urows) +
               op_cta_stages(2 * p.FL, p.H, 3, c, grid, urows) + op_cta_stages(p.HS, p.F, 4, c, grid, urows);
    int i = c;  // insertion sort by (total, index)
    for (; i > 0 && total[order[i - 1]] > total[c]; --i) order[i] = order[i - 1];
    order[i] = c;
  }
  for (int i = 0; i < grid; ++i) p.attn_rank[order[i]] = static_cast<unsigned char>(i);
}

__device__ __forceinline__ void prefetch_l2(const void *src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// The flag of operation `op` of step `epoch` (op 0: the embedding; 1 + 5 l + k: operation
// k of layer l — 0 QKV, 1 attention, 2 O, 3 gate/up, 4 down): unique per step and
// operation (the epoch restarts with zeroed words), never zero.
__device__ __forceinline__ uint32_t ll_flag(int epoch, int op, int n_layers) {
  return uint32_t(epoch + 1) * uint32_t(5 * n_layers + 2) + uint32_t(op) + 1u;
}

// `dst`: the peer offsets (tp_ndst of them) the exchanged outputs are also stored at.
// Operations read and write the flagged words: the residual rows x carry the flag of
// their last writer (the embedding, O or down).
__device__ __forceinline__ GemvTask layer_task(const PersistParams &p, int l, int k, const long long *dst, int epoch) {
  const LayerWeights &w = p.layers[l];
  const int H = p.H, nd = p.tp_ndst, nL = p.n_layers;
  auto fl = [&](int op) { return ll_flag(epoch, op, nL); };
  const uint32_t x_in = l == 0 ? fl(0) : fl(1 + 5 * (l - 1) + 4);  // x as the layer receives it
  GemvTask t;
  switch (k) {
    case 0:
      t = GemvTask{w.qkv, p.QKV, H, p.x, H, w.ln1, p.eps, p.qkv, p.QKV, kEpiStore, 0, nullptr};
      t.in_ll = p.x_ll, t.in_ll_stride = p.x_lls, t.in_flag = x_in;
      t.out_ll = p.qkv_ll, t.out_ll_stride = p.qkv_lls, t.out_flag = fl(1 + 5 * l);
      return t;
    case 1:
      t = GemvTask{w.o, p.HS, p.QD, p.attn, p.QD, nullptr, p.eps, p.x + p.h0, H, kEpiResidual, nd, dst};
      t.in_ll = p.attn_ll, t.in_ll_stride = p.attn_lls, t.in_flag = fl(1 + 5 * l + 1);
      t.out_ll = p.x_ll + p.h0 / 2, t.out_ll_stride = p.x_lls, t.out_flag = fl(1 + 5 * l + 2), t.res_flag = x_in;
      return t;
    case 2:
      t = GemvTask{w.gu, 2 * p.FL, H, p.x, H, w.ln2, p.eps, p.mlp + p.f0, p.F, kEpiSwiGLU, nd, dst};
      t.in_ll = p.x_ll, t.in_ll_stride = p.x_lls, t.in_flag = fl(1 + 5 * l + 2);
      t.out_ll = p.mlp_ll + p.f0 / 2, t.out_ll_stride = p.mlp_lls, t.out_flag = fl(1 + 5 * l + 3);
      return t;
    default:
      t = GemvTask{w.down, p.HS, p.F, p.mlp, p.F, nullptr, p.eps, p.x + p.h0, H, kEpiResidual, nd, dst};
      t.in_ll = p.mlp_ll, t.in_ll_stride = p.mlp_lls, t.in_flag = fl(1 + 5 * l + 3);
      t.out_ll = p.x_ll + p.h0 / 2, t.out_ll_stride = p.x_lls, t.out_flag = fl(1 + 5 * l + 4),
      t.res_flag = fl(1 + 5 * l + 2);
      return t;
  }
}
// The head reads the final residual rows (flagged) and writes plain logits (read by the
// next kernel).
__device__ __forceinline__ GemvTask head_task(const PersistParams &p, const long long *dst, int epoch) {
  GemvTask t{p.head,   p.head_rows, p.H, p.x, p.H, p.final_norm, p.eps, p.logits, p.logit_stride, kEpiStore,
             p.tp_ndst, dst};
  t.in_ll = p.x_ll, t.in_ll_stride = p.x_lls, t.in_flag = ll_flag(epoch, 1 + 5 * (p.n_layers - 1) + 4, p.n_layers);
  return t;
}

struct KvChunkRef {
  int page, kvh, base, n_main;
};
// A stage of the producer's sequence: stage i of operation o (0 QKV, 1 this CTA's KV
// chunks, 2 O, 3 gate/up, 4 down) of layer l; layer n_layers is the LM head (o = 0). The
// operation's constants are loaded once on entering it.
struct ProdCursor {
  int l, o, i, len;
  const CUtensorMap *map;    // GEMV operations: weight stage map (BF16) or stage image (8-bit),
  const unsigned char *img;  // K, this CTA's first group (unit), stages per group
  int K, N, g, ks, KS;
};

// The producer lane's view of one step. It walks the stage sequence twice: once to copy
// stages into the ring, and `prefetch_stages` stages ahead of that to pull the same
// bytes into L2 (cp.async.bulk.prefetch), so HBM keeps streaming while the consumers wait
// at operation boundaries and the ring copies of those stages then hit L2.
template <int NB, int QB>
struct Producer {
  static constexpr bool kQ8 = QB != 0;  // quantized weights (8 or 4 bits)
  static constexpr int kQStage = kQ8 ? q_stage_bytes<(QB ? QB : 8)>() : 0;
  const LayerWeights *layers;
  const CUtensorMap *wmaps, *head_map;
  const QLayer *qlayers;
  const unsigned char *qhead;
  int head_rows, H, QKV, QD, F, HS, FL, nL, epoch;
  bf16 *pool;
  AttnGeom g;
  int max_splits;
  const int *page_table, *ctr, *active, *pos, *capacity;
  int *error;
  int nkv, arank;
  bool planned, failed;
  KvChunkRef *kv;  // this CTA's chunk list (shared memory, kMaxCtaChunks entries)

  __device__ Producer(const PersistParams &p, int ep, KvChunkRef *kv_smem)
      : layers(p.layers), wmaps(p.wmaps), head_map(&p.head_map), qlayers(p.qlayers), qhead(p.qhead), head_rows(p.head_rows), H(p.H), QKV(p.QKV), QD(p.QD), F(p.F), HS(p.HS),
        FL(p.FL), nL(p.n_layers), epoch(ep), pool(p.ap.pool), g(p.ap.g), max_splits(p.ap.max_splits),
        page_table(p.ap.page_table), ctr(p.ctr), active(p.active), pos(p.pos), capacity(p.capacity), error(p.error), nkv(0),
        arank(p.attn_rank[blockIdx.x]), planned(false), failed(false), kv(kv_smem) {}

  // This CTA's KV chunks. The step's rows are computed here as every CTA computes them
  // (step_row): no CTA waits for another to latch them.
  __device__ bool plan() {
    StepRows<NB> rows;
    for (int b = 0; b < NB; ++b) {
      const int a = __ldcg(active + b), q = __ldcg(pos + b);
      rows.active[b] = a && q < __ldcg(capacity + b);
      rows.pos[b] = q;
    }
    const int U = step_units(rows, g.kv_heads, max_splits);
    for (int u = arank; u < U; u += gridDim.x) {
      const UnitInfo ui = step_unit(rows, g.kv_heads, max_splits, u);
      for (int c = ui.c0; c < ui.c1; ++c) {
        if (nkv == kMaxCtaChunks) {
          atomicOr(error, 32);
          return false;
        }
        const int base = c * kKvChunk;
        kv[nkv++] = KvChunkRef{__ldcg(page_table + size_t(ui.row) * g.pages_per_row + (base >> g.page_shift)),
                               ui.kvh, base, min(kKvChunk, rows.pos[ui.row] - base)};
      }
    }
    return true;
  }

  // Load operation (c.l, c.o)'s constants and stage count into the cursor.
  __device__ void enter(ProdCursor &c) {
    c.i = 0;
    if (c.l < nL && c.o == 1) {
      if (!planned) {
        planned = true;
        failed = !plan();
      }
      c.len = failed ? 0 : nkv;
      return;
    }
    if (c.l == nL) {
      c.map = head_map, c.img = qhead, c.N = head_rows, c.K = H;
    } else {
      const CUtensorMap *m = wmaps + 4 * c.l;
      const QLayer q = kQ8 ? qlayers[c.l] : QLayer{};
      switch (c.o) {
        case 0: c.map = m, c.img = q.qkv, c.N = QKV, c.K = H; break;
        case 2: c.map = m + 1, c.img = q.o, c.N = HS, c.K = QD; break;
        case 3: c.map = m + 2, c.img = q.gu, c.N = 2 * FL, c.K = H; break;
        default: c.map = m + 3, c.img = q.down, c.N = HS, c.K = F; break;
      }
    }
    const int groups = kQ8 ? (c.N + kQ8Rows - 1) / kQ8Rows : (c.N + 7) / 8;
    const int pos = (int(blockIdx.x) + (c.l == nL ? 0 : op_rotation(c.o, int(gridDim.x)))) % int(gridDim.x);
    const int g0 = pos * groups / int(gridDim.x), g1 = (pos + 1) * groups / int(gridDim.x);
    c.KS = c.K / kRingPiece;
    c.g = g0;
    c.ks = 0;
    c.len = (g1 - g0) * c.KS;
  }
  __device__ bool valid(const ProdCursor &c) const { return c.l < nL || (c.l == nL && c.o == 0); }
  __device__ void begin(ProdCursor &c) {
    c.l = 0;
    c.o = 0;
    enter(c);
    skip_empty(c);
  }
  __device__ void skip_empty(ProdCursor &c) {
    while (!failed && valid(c) && c.i >= c.len) {
      if (c.l == nL) {
        c.o = 1;  // past the head
        return;
      }
      if (++c.o == 5) {
        c.o = 0;
        ++c.l;
      }
      enter(c);
    }
  }
  // Advance to the next stage; false past the last stage.
  __device__ bool next(ProdCursor &c) {
    ++c.i;
    if (++c.ks == c.KS) {
      c.ks = 0;
      ++c.g;
    }
    skip_empty(c);
    return !failed && valid(c);
  }
  // Copy the stage into ring slot `dst`, completing on `bar`.
  __device__ void issue(const ProdCursor &c, bf16 *dst, uint64_t *bar, uint64_t pol) const {
    if (c.l < nL && c.o == 1) {
      const KvChunkRef r = kv[c.i];
      const unsigned bytes = r.n_main > 0 ? unsigned(r.n_main) * 128 * 2 : 0u;
      mbar_arrive_expect_tx(bar, 2 * bytes);
      if (bytes) {
        const size_t blk = (size_t(c.l) * g.num_pages + r.page) * 2;
        const size_t off = (size_t(r.kvh) * g.page_tokens + (r.base & (g.page_tokens - 1))) * 128;
        bulk_g2s(dst, pool + blk * g.page_elems + off, bytes, bar);
        bulk_g2s(dst + kKvChunk * 128, pool + (blk + 1) * g.page_elems + off, bytes, bar);
      }
      return;
    }
    if (kQ8) {
      mbar_arrive_expect_tx(bar, unsigned(kQStage));
      bulk_g2s_hint(dst, c.img + (size_t(c.g) * c.KS + c.ks) * kQStage, unsigned(kQStage), bar, pol);
      return;
    }
    mbar_arrive_expect_tx(bar, unsigned(kRingStageBytes));
    stage_load(dst, c.map, c.g * 8, c.ks, bar, pol);
  }
  // Pull the stage's bytes into L2.
  __device__ void prefetch(const ProdCursor &c) const {
    if (c.l < nL && c.o == 1) {
      const KvChunkRef r = kv[c.i];
      if (r.n_main <= 0) return;
      const size_t blk = (size_t(c.l) * g.num_pages + r.page) * 2;
      const size_t off = (size_t(r.kvh) * g.page_tokens + (r.base & (g.page_tokens - 1))) * 128;
      prefetch_l2(pool + blk * g.page_elems + off, unsigned(r.n_main) * 256);
      prefetch_l2(pool + (blk + 1) * g.page_elems + off, unsigned(r.n_main) * 256);
      return;
    }
    if (kQ8)
      prefetch_l2(c.img + (size_t(c.g) * c.KS + c.ks) * kQStage, unsigned(kQStage));
    else
      stage_prefetch(c.map, c.g * 8, c.ks);
  }
};

// QB: the weights' precision — 0 (BF16, stage-map copies), 8 or 4 (affine 8- or 4-bit stage
// images, ring_consume_q8); everything else is shared.
template <int NB, int QB>
__global__ void __launch_bounds__(kPersistThreads, 1) k_decode_persistent(const __grid_constant__ PersistParams p) {
  // 1024-byte alignment: the weight stages are 128-byte-swizzled tensor copies.
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  constexpr bool kQ8 = QB != 0;  // quantized weights (8 or 4 bits)
  constexpr int kBits = QB ? QB : 8;
  constexpr int NS = kQ8 ? kPersistStagesQ8 : kPersistStages;
  constexpr int kSlot = kQ8 ? kQ8StageBytes : kRingStageBytes;  // bytes of a ring slot (a 4-bit stage uses 18,432)
  constexpr int kUrows = kQ8 ? kQ8Rows : 8;                       // weight rows of a stage
  using ASm = AttnTeamSmem<128, 2>;
  // Layout: ring | act (GEMV activations) aliased with the attention teams' scratch (the
  // two are never live at once) | group partials.
  constexpr size_t kActBytes = size_t(NB) * kPersistMaxK * 2;
  constexpr size_t kUnion = kActBytes > sizeof(ASm) ? kActBytes : sizeof(ASm);
  unsigned char *ringb = smem_raw;
  bf16 *ring = reinterpret_cast<bf16 *>(smem_raw);
  bf16 *act = reinterpret_cast<bf16 *>(smem_raw + NS * kSlot);
  ASm *team_sm = reinterpret_cast<ASm *>(smem_raw + NS * kSlot);  // attention scratch
  float *gred = reinterpret_cast<float *>(smem_raw + NS * kSlot + kUnion);
  // Quantized: the group sums, FP16 factors and offset shares of the staged rows (q8_stage_chunk).
  __shared__ __align__(16) float s_sumx[kQ8 ? NB * (kPersistMaxK / 64) : 4];
  __shared__ __align__(16) float s_qfac[kQ8 ? NB * (kPersistMaxK / 64) : 4];
  __shared__ __align__(16) float s_qneg[kQ8 ? NB * (kPersistMaxK / 64) : 4];
  __shared__ __align__(8) uint64_t full[NS], empty[NS];
  __shared__ float red[NB * kRingConsumers];
  __shared__ AttnRow<128> rowst[NB];
  __shared__ int s_epoch, s_bad, s_trace;
  __shared__ int s_row[NB][4];  // this step's rows: active, position, token, active before the room check
  __shared__ KvChunkRef kv_chunks[kMaxCtaChunks];
  __shared__ uint4 s_keep[2][NB * kResKeepCols / 8];  // kept residual columns for O and down
  __shared__ long long s_dst[kMaxTpWorld - 1];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nL = p.n_layers, H = p.H;
  const bool tp = p.tp_world > 1;
  const int W = p.tp_world;
  if (threadIdx.x < kMaxTpWorld - 1) s_dst[threadIdx.x] = threadIdx.x < p.tp_ndst ? p.tp_dst[threadIdx.x] : 0;
  if ((smem_u32(ring) & 1023) != 0) {  // never copy into a misaligned ring (every CTA alike)
    if (threadIdx.x == 0) atomicOr(p.error, 1);
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRingConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_epoch = ld_acquire(p.epoch);
    s_bad = 0;
    // The timeline records steps with an active row only (the sampler that ran before this
    // kernel has set this step's activity), so it keeps the last step that did work.
    int any_active = 0;
    for (int b = 0; b < NB; ++b) any_active |= __ldcg(p.active + b);
    s_trace = p.trace != nullptr && any_active != 0;
  }
  __syncthreads();
  const int epoch = s_epoch;
  unsigned long long *const trace = s_trace ? p.trace : nullptr;
  const int all = int(gridDim.x);
  // The op's task; an injected fault makes its input wait for a flag that is never written.
  auto task = [&](int l, int k) {
    GemvTask t = layer_task(p, l, k, s_dst, epoch);
    t.ll_limit = p.ll_limit;
    const int op = 1 + 5 * l + (k == 0 ? 0 : k + 1);
    if (p.inject_op == op) t.in_flag ^= 0x80000000u;
    // O and down (no RMSNorm): each consumer warp stages its own k-range, so a warp starts
    // as soon as its inputs (for O: its kv head's outputs) are written.
    if (k == 1 || k == 3) t.stage_per_warp = true;
    if (kQ8) {
      const QLayer &q = p.qlayers[l];
      t.qimg = k == 0 ? q.qkv : k == 1 ? q.o : k == 2 ? q.gu : q.down;
      t.sumx = s_sumx;
      t.qfac = s_qfac;
      t.qneg = s_qneg;
    }
    if (l == 0 && k == 0 && p.inject_op != op) {
      // The first QKV reads each row's token embedding itself (an inactive row: zeros).
      t.in_ll = nullptr;
      t.in_gather = true;
      for (int b = 0; b < NB; ++b) t.in_row[b] = s_row[b][0] ? p.embed + size_t(s_row[b][2]) * H : nullptr;
    }
    return t;
  };
  auto fl = [&](int op) { return ll_flag(epoch, op, nL); };

  if (warp >= kRingConsumers) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPersistProducerRegs));
    if (warp == kRingConsumers && lane == 0) {
      auto pstamp = [&](int o, int k) {
        if (trace) trace[(size_t(blockIdx.x) * (5 * nL + 1) + o) * 8 + k] = sm_clock();
      };
      Producer<NB, QB> pr(p, epoch, kv_chunks);
      ProdCursor ic, pc;
      pr.begin(ic);
      pc = ic;
      bool iv = !pr.failed && pr.valid(ic), pv = iv;
      long long it = 0, pf = 0;
      const uint64_t pol = weight_stream_policy();
      const int ahead = p.prefetch_stages;
      while (iv) {
        while (pv && pf < it + ahead) {
          pr.prefetch(pc);
          pv = pr.next(pc);
          ++pf;
        }
        const int s = int(it % NS);
        if (it >= NS && !mbar_wait(&empty[s], unsigned((it / NS) - 1) & 1u)) {
          atomicOr(p.error, 4);
          break;
        }
        const int op = 5 * ic.l + ic.o, so = ic.o == 1 ? 6 : 4;  // attention op slots 4/5 hold unit stamps
        if (ic.i == 0) pstamp(op, so);
        pr.issue(ic, reinterpret_cast<bf16 *>(ringb + size_t(s) * kSlot), &full[s], pol);
        ++it;
        iv = pr.next(ic);
        if (!iv || 5 * ic.l + ic.o != op) pstamp(op, so + 1);
      }
      ring_drain<NS>(full, it);
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPersistConsumerRegs));
  const int ctid = threadIdx.x;
  bool bad = false, dead = false;  // dead: a ring wait expired (the producer is presumed stuck)
  long long it = 0;
  auto stamp = [&](int o, int k) {
    if (trace && ctid == 0) trace[(size_t(blockIdx.x) * (5 * nL + 1) + o) * 8 + k] = sm_clock();
  };
  // Thread 0 publishes one share of counter idx: to this rank only (GPU scope), or
  // (exchanged operations under tensor parallelism) to every rank at system scope.
  auto publish = [&](int idx, bool all_ranks) {
    if (!tp || !all_ranks) {
      red_release_add(p.ctr + idx, 1);
      return;
    }
    fence_acq_rel_sys();
    red_relaxed_add_sys(p.ctr + idx, 1);
    for (int i = 0; i < p.tp_ndst; ++i)
      red_relaxed_add_sys(reinterpret_cast<int *>(reinterpret_cast<char *>(p.ctr + idx) + s_dst[i]), 1);
  };
  // One barrier orders every consumer thread's writes before thread 0's release-add, which
  // publishes the CTA's share; the same barrier makes a recorded failure CTA-wide.
  auto signal = [&](int idx, bool all_ranks) {
    if (bad) s_bad = 1;
    consumer_sync();
    bad = s_bad != 0;
    if (ctid == 0) publish(idx, all_ranks);
  };
  // Wait until counter idx reaches target; gives up on expiry or once any CTA failed.
  // `exchanged`: a counter every rank adds to (system scope under tensor parallelism).
  auto wait_for = [&](int idx, int target, bool exchanged) {
    if (ctid == 0 && !s_bad) {
      const bool sys = tp && exchanged;
      long long i = 0;
      for (; i < kCounterWaitLimit; ++i) {
        if ((sys ? ld_relaxed_sys(p.ctr + idx) : ld_acquire(p.ctr + idx)) >= target) {
          if (sys) fence_acq_rel_sys();
          break;
        }
        if (ld_acquire(p.error) != 0) {
          i = kCounterWaitLimit;
          break;
        }
        __nanosleep(64);
      }
      if (i >= kCounterWaitLimit) {
        atomicOr(p.error, 16);
        s_bad = 1;
      }
    }
    consumer_sync();
    bad = s_bad != 0;
  };
  const int kvh_n = p.ap.g.kv_heads, nsplit = p.ap.max_splits;
  const int c_head = 1 + 5 * nL;  // counter 0 (the old position latch) is unused
  auto c_op = [&](int l, int k) { return 1 + 5 * l + k; };  // k: 0 qkv, 1 attn, 2 o, 3 gu, 4 down

  // The step's rows, computed alike by every CTA from what the sampler and the previous
  // step left (no latch between CTAs): a row is active when the sampler left it active and
  // it has room for one more position; it forwards position pos[b] and token token[b]. CTA
  // 0 advances the positions at the step's end, when every CTA has read them (each CTA's
  // layer-0 outputs, which CTA 0 waits for, come after its reads). CTA 0 also records the
  // errors (a full row, a token out of range: token 0 is used) and writes each row's
  // embedding as flagged residual words (an inactive row: zeros) for the readers that poll
  // x after the embedding (the hidden-state record, residual epilogues without kept
  // columns); the first QKV reads the embedding rows directly.
  if (ctid == 0)
    for (int b = 0; b < NB; ++b) {
      const int a = __ldcg(p.active + b), q = __ldcg(p.pos + b);
      const bool full = a && q >= __ldcg(p.capacity + b);
      int tok = a && !full ? __ldcg(p.token + b) : 0;
      const bool bad_tok = tok < 0 || tok >= p.vocab;
      if (bad_tok) tok = 0;
      s_row[b][0] = a && !full;
      s_row[b][1] = q;
      s_row[b][2] = tok;
      s_row[b][3] = a;
      if (blockIdx.x == 0 && (full || bad_tok)) atomicOr(p.error, full ? 2 : 1);
    }
  consumer_sync();
  if (blockIdx.x == 0)
    for (int b = 0; b < NB; ++b) {
      const uint32_t *src = reinterpret_cast<const uint32_t *>(p.embed + size_t(s_row[b][2]) * H);
      for (int c = ctid; c < H / 2; c += kRingConsumers * 32)
        ll_store_all(p.x_ll + size_t(b) * p.x_lls + c, s_row[b][0] ? __ldg(src + c) : 0u, fl(0), 0, nullptr);
    }
  // Trace calibration: globaltimer (ns) and the SM clock at the step's start and end.
  auto calib = [&](int o) {
    if (trace && ctid == 0) {
      trace[(size_t(blockIdx.x) * (5 * nL + 1) + o) * 8 + 6] = globaltimer();
      trace[(size_t(blockIdx.x) * (5 * nL + 1) + o) * 8 + 7] = sm_clock();
    }
  };
  // Hidden-state record (optional): CTA 0 copies the residual rows once they carry the flag
  // of the operation that completed them (`slot` 0: the embedding, l + 1: after layer l).
  auto dump_x = [&](int slot) {
    if (!p.layer_dump || blockIdx.x != 0 || bad) return;
    const uint32_t want = slot == 0 ? fl(0) : fl(c_op(slot - 1, 4));
    for (int b = 0; b < NB; ++b) {
      uint32_t *dst = reinterpret_cast<uint32_t *>(p.layer_dump + (size_t(slot) * p.dump_stride + b) * H);
      for (int c = ctid; c < H / 2; c += kRingConsumers * 32) {
        uint32_t w = 0;
        if (!ll_wait1(p.x_ll + size_t(b) * p.x_lls + c, want, w, p.error)) atomicOr(p.error, 64);
        dst[c] = w;
      }
    }
  };
  calib(0);
  // Step log (tracing only): CTA 0's start and end ns of this step (64-step ring after the
  // per-CTA timeline and the sampler's 16 stamps; slots 2 and 3 of the step's entry).
  unsigned long long *step_log =
      p.trace ? p.trace + size_t(gridDim.x) * (5 * nL + 1) * 8 + 16 + size_t(epoch & 63) * 4 : nullptr;
  if (step_log && blockIdx.x == 0 && ctid == 0) step_log[2] = globaltimer();
  dump_x(0);
  // This step's row state (activity, position, cos/sin, page table) for the attention units.
  for (int b = 0; b < NB; ++b)
    attn_row_load_at<128>(rowst[b], p.ap, b, s_row[b][0], s_row[b][1], ctid, kRingConsumers * 32);
  consumer_sync();
  StepRows<NB> srows;
  for (int b = 0; b < NB; ++b) {
    srows.active[b] = rowst[b].active;
    srows.pos[b] = rowst[b].pos;
  }
  const int U = step_units(srows, kvh_n, nsplit), arank = p.attn_rank[blockIdx.x];
  // Merge jobs of this step: rows that are active and split their context.
  bool merge_row[NB];
  int merge_splits[NB], n_merges = 0;
  for (int b = 0; b < NB; ++b) {
    merge_splits[b] = srows.active[b] ? split_plan(srows.pos[b] + 1, nsplit).n_splits : 1;
    merge_row[b] = srows.active[b] && merge_splits[b] > 1;
    if (merge_row[b]) n_merges += kvh_n;
  }

  // One GEMV operation: stage the flagged input rows (the wait for the producing
  // operation), consume this CTA's stages, write its flagged outputs.
  // A CTA without rows of the operation (possible under tensor parallelism) skips it: it
  // neither waits for nor reads the input words, which a later operation may overwrite.
  // `keep`, [keep_lo, keep_hi): raw input columns the staging keeps (RMSNorm operations).
  // Returns whether the CTA took part.
  auto gemv_op = [&](const GemvTask &t, int op_slot, const uint4 (*wn)[4], int o, uint4 *keep = nullptr,
                     int keep_lo = 0, int keep_hi = 0) {
    int g0, g1;
    task_groups(t.N, blockIdx.x, gridDim.x, g0, g1, op_rotation(o, int(gridDim.x)), kUrows);
    if (g0 == g1) return false;
    if (!t.stage_per_warp &&
        !ring_stage_act<NB, kPersistMaxK / kRingPiece>(t, act, red, ctid, wn, p.error, keep, keep_lo, keep_hi))
      bad = true;
    stamp(op_slot, 1);
    if constexpr (kQ8)
      ring_consume_q8<NB, NS, kPersistMaxK / kRingPiece, kBits>(t, g0, g1, ringb, act, full, empty, it, gred,
                                                                p.error, bad, dead, ctid);
    else
      ring_consume<NB, NS, kPersistMaxK / kRingPiece>(t, g0, g1, ring, act, full, empty, it, gred, p.error, bad, dead,
                                                      ctid);
    stamp(op_slot, 2);
    return true;
  };
  // The residual operations (O, down) add this CTA's output columns [8 g0, 8 g1) of x (from
  // h0): the RMSNorm staging before each (QKV, gate/up) reads all of x and keeps those
  // columns in s_keep[0] (for O) and s_keep[1] (for down), so their epilogues read the old
  // residual from shared memory instead of polling it through L2.
  int keep_lo[2], keep_hi[2];
  for (int i = 0; i < 2; ++i) {
    int g0, g1;
    task_groups(p.HS, blockIdx.x, gridDim.x, g0, g1, op_rotation(i == 0 ? 2 : 4, int(gridDim.x)), kUrows);
    keep_lo[i] = kUrows * g0;
    keep_hi[i] = (g1 - g0) * kUrows <= kResKeepCols ? kUrows * g1 : kUrows * g0;  // too wide: poll instead
  }
  auto with_kept = [&](GemvTask t, bool kept, int i) {
    if (kept && keep_hi[i] > keep_lo[i]) {
      t.res_smem = reinterpret_cast<const uint32_t *>(s_keep[i]);
      t.res_lo = keep_lo[i];
    }
    return t;
  };

  uint4 wn_next[4];  // RMSNorm weight chunks of the next norm-prologue GEMV, loaded before its wait
  ring_norm_w_load(task(0, 0), wn_next, ctid);
  for (int l = 0; l < nL; ++l) {
    // The layer's five operations in one rolled loop: the four GEMVs share one instance of
    // the GEMV code (the copies of an unrolled loop each ran cold once per launch, and the
    // first layer paid for every one of them).
    bool kept_o = false, kept_d = false;
#pragma unroll 1
    for (int k = 0; k < 5; ++k) {
      stamp(5 * l + k, 0);
      if (k == 1) {
        // Attention: the CTA's units, one after another on all consumer warps; each unit waits
        // for its own kv head's projections (flagged words) and streams its KV chunks as ring
        // stages (every consumer warp releases each once).
        float wv[4];
        if (arank < U) attn_load_norm_w<128, 2>(p.layers[l].qn, p.layers[l].kn, wv, ctid);
        stamp(5 * l + 1, 0);
        {
          DecodeAttnParams ap = p.ap;
          ap.layer = l;
          ap.out_ndst = p.tp_ndst;
          ap.out_dst = s_dst;
          ap.qkv_ll = p.qkv_ll;
          ap.qkv_ll_stride = p.qkv_lls;
          ap.qkv_flag = fl(c_op(l, 0));
          ap.out_ll = p.attn_ll + (ap.out - p.attn) / 2;  // this rank's heads within the whole width
          ap.out_ll_stride = p.attn_lls;
          ap.out_flag = fl(c_op(l, 1));
          ap.part_flag = ap.out_flag;  // another buffer: the same step and operation
          ap.ll_limit = p.ll_limit;
          if (p.inject_op == c_op(l, 1)) ap.qkv_flag ^= 0x80000000u;
          long long itk = it;
          for (int ku = 0, u = arank; u < U; ++ku, u += gridDim.x) {
            const UnitInfo ui = step_unit(srows, kvh_n, nsplit, u);
            const int nch = ui.c1 - ui.c0;
            unsigned long long *st =
                (trace && ku == 0) ? trace + (size_t(blockIdx.x) * (5 * nL + 1) + 5 * l + 1) * 8 : nullptr;
            const AttnRow<128> &rs = rowst[ui.row];
            if (ui.active && !bad &&
                !attn_qk<128, 2>(ap, *team_sm, rs, ui.row, ui.kvh, ui.split == ui.n_splits - 1, wv, ctid, 1))
              bad = true;
            attn_stamp(st, 3, ctid);
            AttnWarpAcc<128, 2> wacc;
            attn_warp_init(wacc);
            // Each warp waits for, computes and releases its share of every chunk on its own; a
            // failure is voted once per unit (the barrier below). After a failure elsewhere the
            // chunks are still waited for and released; an expired ring wait stops both.
            bool wbad = bad;
            for (int j = 0; j < nch; ++j) {
              const long long ij = itk + j;
              const int sidx = int(ij % NS);
              bool landed = false;
              if (!dead) {
                landed = mbar_wait(&full[sidx], unsigned(ij / NS) & 1u);
                if (!landed) {
                  if (lane == 0) atomicOr(p.error, 8);
                  dead = wbad = true;
                }
              }
              wbad = __any_sync(0xFFFFFFFFu, wbad);
              if (j == 0) attn_stamp(st, 1, ctid);  // the unit's first chunk has landed
              if (!wbad) {
                const bf16 *ks = reinterpret_cast<const bf16 *>(ringb + size_t(sidx) * kSlot);
                const int base = (ui.c0 + j) * kKvChunk, n_main = min(kKvChunk, rs.pos - base);
                attn_chunk<128, 2>(team_sm->q_b, team_sm->knew, team_sm->vnew, ks, ks + kKvChunk * 128, n_main,
                                   rs.pos - base < kKvChunk, ap.g.scale, wacc, ctid);
              }
              __syncwarp();
              if (lane == 0 && landed) mbar_arrive(&empty[sidx]);
            }
            if (team_any(1, wbad)) bad = true;
            attn_stamp(st, 4, ctid);
            if (ui.active && !bad) {
              const AttnAcc<128> acc = attn_combine<128, 2>(*team_sm, wacc, ctid, 1);
              if (ui.n_splits == 1)
                attn_single_out<128, 2>(ap, acc, ui.row, ui.kvh, ctid);
              else
                attn_partial_ll<128, 2>(ap, acc, ui.row, ui.kvh, ui.split, ctid);
            } else if (!ui.active && ui.split == 0) {
              attn_write_inactive<128, 2>(ap, ui.row, ui.kvh, ctid);  // an inactive row's heads: zero words
            }
            attn_stamp(st, 5, ctid);
            itk += nch;
          }
          it = itk;
          // Merge jobs: one per (active row with more than one split, kv head), on the CTAs of
          // attention ranks U, U + 1, ... (those without units while the grid has room): each
          // polls its splits' flagged partials and writes the head outputs. No split waits for
          // another, and no arrival counter is taken.
          if (!bad) {
            const int G = int(gridDim.x);
            for (int j = ((arank - U) % G + G) % G; j < n_merges; j += G) {
              int b = 0, jj = j;
              for (; b < NB; ++b) {
                if (!merge_row[b]) continue;
                if (jj < kvh_n) break;
                jj -= kvh_n;
              }
              if (b == NB) break;
              unsigned long long *st = (trace && arank >= U && j < G) ? trace + (size_t(blockIdx.x) * (5 * nL + 1) + 5 * l + 1) * 8
                                                                    : nullptr;  // a CTA without units: free slots
              if (!attn_merge_ll<128, 2>(ap, b, jj, merge_splits[b], ctid, st)) bad = true;
            }
          }
        }
        stamp(5 * l + 1, 2);
        continue;
      }
      // k: 0 QKV (RMSNorm of x fused), 2 O (+ residual), 3 gate/up (RMSNorm, SwiGLU),
      // 4 down (+ residual); the GEMV task index is k, or k - 1 after attention.
      const int tk = k == 0 ? 0 : k - 1;
      const bool norm_op = k == 0 || k == 3, res_op = k == 2 || k == 4;
      const int ki = k <= 2 ? 0 : 1;  // kept residual columns: for O (0) or down (1)
      GemvTask t = task(l, tk);
      if (res_op) t = with_kept(t, ki == 0 ? kept_o : kept_d, ki);
      const bool took = gemv_op(t, 5 * l + k, norm_op ? &wn_next : nullptr, k, norm_op ? s_keep[ki] : nullptr,
                                p.h0 + keep_lo[ki], p.h0 + keep_hi[ki]);
      if (k == 0) kept_o = took;
      if (k == 3) kept_d = took;
      stamp(5 * l + k, 3);
      if (k == 2) ring_norm_w_load(task(l, 2), wn_next, ctid);  // gate/up's norm weights
      if (k == 4 && l + 1 < nL) ring_norm_w_load(task(l + 1, 0), wn_next, ctid);
    }
    dump_x(l + 1);
  }
  // Final RMSNorm + phase rows of the LM head.
  {
    GemvTask head = head_task(p, s_dst, epoch);
    head.ll_limit = p.ll_limit;
    if (kQ8) {
      head.qimg = p.qhead;
      head.sumx = s_sumx;
      head.qfac = s_qfac;
      head.qneg = s_qneg;
    }
    int g0, g1;
    stamp(5 * nL, 0);
    task_groups(head.N, blockIdx.x, gridDim.x, g0, g1, 0, kUrows);
    const bool extra_cta = p.extra_row >= 0 && blockIdx.x == gridDim.x - 1;  // uses `act` below
    if ((g0 < g1 || extra_cta) && !ring_stage_act<NB, kPersistMaxK / kRingPiece>(head, act, red, ctid, nullptr, p.error))
      bad = true;
    stamp(5 * nL, 1);
    if constexpr (kQ8)
      ring_consume_q8<NB, NS, kPersistMaxK / kRingPiece, kBits>(head, g0, g1, ringb, act, full, empty, it, gred,
                                                                p.error, bad, dead, ctid);
    else
      ring_consume<NB, NS, kPersistMaxK / kRingPiece>(head, g0, g1, ring, act, full, empty, it, gred, p.error, bad,
                                                      dead, ctid);
    stamp(5 * nL, 2);
    if (p.extra_row >= 0 && blockIdx.x == gridDim.x - 1 && warp < NB && !bad) {
      // The ABC phase's extra row (ABC_END), from the normalized activations in `act` (8-bit
      // weights: the row's BF16 dequantized copy, and `act` holds FP16 values times the
      // group's factor, exactly the BF16 values).
      const bf16 *wr = p.head + size_t(p.extra_row - 0) * H;
      float v = 0.f;
      for (int c = lane; c < H / 8; c += 32) {
        uint4 av = act_load_chunk(act + warp * H, c * 8);
        if constexpr (kQ8) {
          const float f = s_qfac[warp * (H / 64) + c / 8];
          uint32_t *w4 = reinterpret_cast<uint32_t *>(&av);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 h = __half22float2(*reinterpret_cast<const __half2 *>(&w4[q]));
            w4[q] = pack_bf16x2(__float2bfloat16_rn(h.x * f), __float2bfloat16_rn(h.y * f));
          }
        }
        const uint4 wq = ldg16(wr + c * 8);
        v = fmaf(bf_lo(wq.x), bf_lo(av.x), v);
        v = fmaf(bf_hi(wq.x), bf_hi(av.x), v);
        v = fmaf(bf_lo(wq.y), bf_lo(av.y), v);
        v = fmaf(bf_hi(wq.y), bf_hi(av.y), v);
        v = fmaf(bf_lo(wq.z), bf_lo(av.z), v);
        v = fmaf(bf_hi(wq.z), bf_hi(av.z), v);
        v = fmaf(bf_lo(wq.w), bf_lo(av.w), v);
        v = fmaf(bf_hi(wq.w), bf_hi(av.w), v);
      }
      v = warp_sum(v);
      if (lane == 0) store_all(p.logits + size_t(warp) * p.logit_stride + p.head_rows, f2bf(v), p.tp_ndst, s_dst);
    }
    // Under tensor parallelism the head columns of every rank must be in before the step
    // ends (the sampler, launched after this kernel, reads the whole logits rows).
    if (tp) signal(c_head, true);
    calib(5 * nL);
  }
  if (blockIdx.x == 0) {
    if (tp) wait_for(c_head, (epoch + 1) * all * W, true);
    if (ctid == 0) {
      // The positions advance (a full row is deactivated instead); the host reads them after
      // the step, and the next step's CTAs after this kernel.
      for (int b = 0; b < NB; ++b) {
        if (!s_row[b][3]) continue;
        p.cur_pos[b] = s_row[b][1];
        if (s_row[b][0])
          p.pos[b] = s_row[b][1] + 1;
        else
          p.active[b] = 0;
      }
      __threadfence();
      atomicExch(p.epoch, epoch + 1);
      if (step_log) step_log[3] = globaltimer();
    }
  }
}

size_t persistent_smem(int NB, int QB) {
  const size_t act = size_t(NB) * kPersistMaxK * 2, teams = sizeof(AttnTeamSmem<128, 2>);
  const size_t ring = QB ? size_t(kPersistStagesQ8) * kQ8StageBytes : size_t(kPersistStages) * kRingStageBytes;
  return ring + (act > teams ? act : teams) + size_t(ring_gred_floats(NB)) * 4;
}

// The kernel instance for a row count and precision.
static const void *persistent_kernel(int n_rows, int bits) {
  if (bits == 8) return n_rows == 1 ? (const void *)k_decode_persistent<1, 8> : (const void *)k_decode_persistent<2, 8>;
  if (bits == 4) return n_rows == 1 ? (const void *)k_decode_persistent<1, 4> : (const void *)k_decode_persistent<2, 4>;
  return n_rows == 1 ? (const void *)k_decode_persistent<1, 0> : (const void *)k_decode_persistent<2, 0>;
}

void configure_persistent_kernels() {
  for (int bits : {0, 8, 4})
    for (int rows = 1; rows <= 2; ++rows)
      YAR_CUDA(cudaFuncSetAttribute(persistent_kernel(rows, bits), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(persistent_smem(rows, bits))));
}

// True when the persistent kernel handles this model and row count.
void build_stage_maps(Model &m) {
  const Dims &d = m.d, &f = m.full;
  if (d.hidden % kRingPiece || f.qdim() % kRingPiece || f.ffn % kRingPiece) return;
  // The shapes launch_persistent gives the kernel (this rank's rows).
  const int QKV = d.qkv_rows(), HS = m.tp.h_rows, FL = d.ffn;
  std::vector<CUtensorMap> maps(size_t(d.layers) * 4);
  for (int l = 0; l < d.layers; ++l) {
    const LayerWeights &w = m.layers[l];
    encode_stage_map(&maps[4 * l + 0], w.qkv, QKV, d.hidden);
    encode_stage_map(&maps[4 * l + 1], w.o, HS, f.qdim());
    encode_stage_map(&maps[4 * l + 2], w.gu, 2 * FL, d.hidden);
    encode_stage_map(&maps[4 * l + 3], w.down, HS, f.ffn);
  }
  YAR_CUDA(cudaMalloc(&m.d_wmaps, maps.size() * sizeof(CUtensorMap)));
  YAR_CUDA(cudaMemcpy(m.d_wmaps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice));
}

bool persistent_supported(const Model &m, int n_rows) {
  // The ring GEMVs need every K (hidden, and the model's query and FFN widths: O and down
  // keep their whole input width under tensor parallelism) a multiple of 2048, and the
  // stage maps of the layers' weights.
  const Dims &d = m.d, &f = m.full;
  if (n_rows < 1 || n_rows > 2 || m.tp_world > kMaxTpWorld || !m.d_wmaps) return false;
  if (d.head_dim != 128 || d.heads != 2 * d.kv_heads) return false;
  if (d.hidden % kRingPiece || f.qdim() % kRingPiece || f.ffn % kRingPiece || f.ffn > kPersistMaxK ||
      d.hidden > kPersistMaxK || f.qdim() > kPersistMaxK)
    return false;
  // The register split (setmaxnreg) assumes the launch's per-thread registers.
  cudaFuncAttributes fa{};
  if (m.bits && (!m.d_qlayers || m.tp_world > 1)) return false;
  if (cudaFuncGetAttributes(&fa, persistent_kernel(n_rows, m.bits)) != cudaSuccess ||
      fa.numRegs != kPersistLaunchRegs)
    return false;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, persistent_kernel(n_rows, m.bits), kPersistThreads,
                                                    persistent_smem(n_rows, m.bits)) != cudaSuccess)
    return false;
  return per_sm >= 1;
}

void launch_decode_persistent(const Model &m, Session &s, int n_rows, int phase, cudaStream_t st) {
  const Dims &d = m.d;
  const PhaseRows pr = phase_rows(d, phase);
  if (m.tp_world > 1 && !s.tp_mapped) throw Error("RuntimeError", "persistent tensor-parallel decode needs mapped peers");
  PersistParams p;
  p.layers = m.d_layers;
  p.wmaps = static_cast<const CUtensorMap *>(m.d_wmaps);
  p.qlayers = m.d_qlayers;
  p.qhead = m.bits ? m.qhead[phase] : nullptr;
  if (m.bits && !p.qhead) throw Error("RuntimeError", "no quantized head image for this phase");
  p.n_layers = d.layers;
  p.H = d.hidden;
  p.QKV = d.qkv_rows();
  p.QD = m.full.qdim();
  p.F = m.full.ffn;
  p.HS = m.tp.h_rows;
  p.h0 = m.tp.h_row0;
  p.FL = d.ffn;
  p.f0 = m.tp.ffn_row0;
  p.vocab = d.vocab;
  p.eps = d.eps;
  p.embed = m.embed;
  p.final_norm = m.final_norm;
  // This rank's phase columns [c0, c1) of the head (all of them on one GPU): main rows
  // [c0, min(c1, n_main)) and, when n_main falls in the range, the extra row.
  const int width = pr.width(), slice = m.tp_world > 1 ? tp_head_slice(width, m.tp_world) : width;
  const int c0 = std::min(width, m.tp_rank * slice), c1 = std::min(width, c0 + slice);
  p.head = m.lm_head + size_t(pr.row0 + c0) * d.hidden;
  p.head_rows = std::max(0, std::min(c1, pr.n_main) - c0);
  if (p.head_rows > 0) encode_stage_map(&p.head_map, p.head, p.head_rows, d.hidden);
  p.extra_row = pr.extra >= 0 && c0 <= pr.n_main && pr.n_main < c1 ? pr.extra - pr.row0 - c0 : -1;
  p.x = s.x;
  p.qkv = s.qkv;
  p.attn = s.attn;
  p.mlp = s.mlp;
  p.logits = s.logits + c0;
  p.logit_stride = s.logit_stride;
  p.x_ll = s.x_ll;
  p.qkv_ll = s.qkv_ll;
  p.attn_ll = s.attn_ll;
  p.mlp_ll = s.mlp_ll;
  p.x_lls = d.hidden / 2;
  p.qkv_lls = d.qkv_rows() / 2;
  p.attn_lls = m.full.qdim() / 2;
  p.mlp_lls = m.full.ffn / 2;
  p.tp_world = m.tp_world;
  p.tp_ndst = m.tp_world > 1 ? m.tp_world - 1 : 0;
  for (int i = 0; i < kMaxTpWorld - 1; ++i) p.tp_dst[i] = i < p.tp_ndst ? s.tp_dst[i] : 0;
  DecodeAttnParams &a = p.ap;
  a.g.heads = d.heads;
  a.g.kv_heads = d.kv_heads;
  a.g.head_dim = d.head_dim;
  a.g.qdim = d.qdim();
  a.g.kvdim = d.kvdim();
  a.g.page_tokens = s.page_tokens;
  a.g.page_shift = 0;
  while ((1 << a.g.page_shift) < s.page_tokens) ++a.g.page_shift;
  if ((1 << a.g.page_shift) != s.page_tokens || s.page_tokens < kKvChunk)
    throw Error("RuntimeError", "persistent decode needs power-of-two pages of at least 64 positions");
  a.g.pages_per_row = s.pages_per_row;
  a.g.num_pages = s.num_pages;
  a.g.page_elems = s.kv_page_elems;
  a.g.eps = d.eps;
  a.g.scale = float(1.0 / std::sqrt(double(d.head_dim)));
  a.layer = 0;
  a.max_splits = decode_max_splits(m, s, n_rows);
  a.pool = s.kv;
  a.page_table = s.d_page_table;
  a.cur_pos = s.d_cur_pos;
  a.active = s.d_active;
  a.qkv = s.qkv;
  a.qn = a.kn = nullptr;
  a.cos_tab = m.rope_cos;
  a.sin_tab = m.rope_sin;
  a.part = s.attn_part;
  a.part_ll = s.part_ll;
  a.count = s.attn_count;
  a.out = s.attn + m.tp.q_row0;
  a.out_stride = m.full.qdim();
  a.out_ndst = 0;  // set in the kernel (peer offsets in shared memory)
  a.out_dst = nullptr;
  a.error = s.d_error;
  p.token = s.d_token;
  p.pos = s.d_pos;
  p.cur_pos = s.d_cur_pos;
  p.capacity = s.d_capacity;
  p.active = s.d_active;
  p.error = s.d_error;
  p.ctr = s.d_ctr;
  p.epoch = s.d_epoch;
  p.trace = s.d_trace;
  p.layer_dump = s.d_layer_dump;
  p.dump_stride = s.max_rows;
  p.inject_op = s.inject_op;
  p.ll_limit = s.inject_op > 0 ? (1ll << 16) : (1ll << 22);
  p.prefetch_stages = s.prefetch_stages;
  if (m.sm_count > kMaxPersistGrid) throw Error("RuntimeError", "persistent decode takes at most 256 SMs");
  attention_ranks(p, m.sm_count, m.bits ? kQ8Rows : 8);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m.sm_count);
  cfg.blockDim = dim3(kPersistThreads);
  cfg.dynamicSmemBytes = persistent_smem(n_rows, m.bits);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (m.bits == 8)
    YAR_CUDA(n_rows == 1 ? cudaLaunchKernelEx(&cfg, k_decode_persistent<1, 8>, p)
                         : cudaLaunchKernelEx(&cfg, k_decode_persistent<2, 8>, p));
  else if (m.bits == 4)
    YAR_CUDA(n_rows == 1 ? cudaLaunchKernelEx(&cfg, k_decode_persistent<1, 4>, p)
                         : cudaLaunchKernelEx(&cfg, k_decode_persistent<2, 4>, p));
  else
    YAR_CUDA(n_rows == 1 ? cudaLaunchKernelEx(&cfg, k_decode_persistent<1, 0>, p)
                         : cudaLaunchKernelEx(&cfg, k_decode_persistent<2, 0>, p));
}

}  // namespace yar
