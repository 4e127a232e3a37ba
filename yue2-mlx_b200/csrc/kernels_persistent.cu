// kernels_persistent.cu — the whole decode forward of one token (1 or 2 rows) as one
// persistent kernel: embedding, 28 x (QKV, attention, O, gate/up, down), LM head.
//
// Why: bs1 decode streams 2.95 GB of weights per token through ~143 dependent operations;
// as separate kernels every boundary costs a ramp and a tail (several us), far more than
// the bandwidth time of the small projections. Here each CTA's producer lane streams the
// CTA's weight rows for every task of the step, in order, through a 5-stage (160 KB)
// shared-memory ring, waiting only for ring space — never for activations — so HBM keeps
// streaming while the consumer warps wait at operation boundaries.
//
// Grid: one CTA per SM, co-resident by cooperative launch. Block: 8 consumer warps + 1
// producer warp. Operation boundaries are global counters: a CTA finishing its share
// fences its writes and adds 1; consumers of the next operation wait (bounded) until
// the counter reaches (epoch + 1) x contributions, where `epoch` counts completed steps
// (the last action of a step is CTA 0 advancing it), so counters never need a reset
// between steps. Inter-CTA data is read through L2 (ld.cg).
//
// The GEMV and attention code is the same device code as the standalone kernels
// (tma_ring.cuh, attn_decode.cuh): both paths produce identical logits.
//
// Failure: every wait is bounded and also gives up as soon as any CTA has recorded an
// error; a CTA that gave up keeps releasing ring stages and taking every barrier (so its
// producer finishes and no copy is left in flight) and keeps signalling counters (so
// other CTAs do not wait for it), without computing.
#include "attn_decode.cuh"
#include "tma_ring.cuh"

namespace yar {

constexpr int kPersistStages = 5;
constexpr int kPersistThreads = (kRingConsumers + 1) * 32;
constexpr int kPersistMaxK = 6144;
constexpr long long kCounterWaitLimit = 1ll << 22;  // polls of ~100 ns: under a second

struct PersistParams {
  const LayerWeights *layers;  // device array, one entry per layer
  int n_layers, H, QKV, QD, F, vocab;
  float eps;
  const bf16 *embed, *final_norm, *head;
  int head_rows, extra_row;  // phase rows [0, head_rows) of `head`, plus one extra row or -1
  bf16 *x, *qkv, *attn, *mlp, *logits;
  int logit_stride;
  DecodeAttnParams ap;
  int *token, *pos, *cur_pos, *capacity, *active, *error;
  int *ctr, *epoch;
  unsigned long long *trace;  // optional [cta][op][8] globaltimer stamps (ns), op = 5*layer + k
};

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int ld_acquire(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <int NB>
__global__ void __launch_bounds__(kPersistThreads, 1) k_decode_persistent(PersistParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  constexpr int NS = kPersistStages;
  using ASm = AttnSmem<128, 2>;
  // Layout: ring | act (GEMV activations) aliased with the attention teams' scratch (the
  // two are never live at once) | group partials.
  constexpr size_t kActBytes = size_t(NB) * kPersistMaxK * 2;
  constexpr size_t kUnion = kActBytes > 2 * sizeof(ASm) ? kActBytes : 2 * sizeof(ASm);
  bf16 *ring = reinterpret_cast<bf16 *>(smem_raw);
  bf16 *act = reinterpret_cast<bf16 *>(smem_raw + NS * kRingStageBytes);
  ASm *team_sm = reinterpret_cast<ASm *>(smem_raw + NS * kRingStageBytes);
  float *gred = reinterpret_cast<float *>(smem_raw + NS * kRingStageBytes + kUnion);
  __shared__ __align__(8) uint64_t full[NS], empty[NS];
  __shared__ float red[NB * kRingConsumers];
  __shared__ AttnRow<128> rowst[NB];
  __shared__ int s_epoch, s_bad;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nL = p.n_layers, H = p.H;
  auto task = [&](int l, int k) {
    const LayerWeights &w = p.layers[l];
    switch (k) {
      case 0: return GemvTask{w.qkv, p.QKV, H, p.x, H, w.ln1, p.eps, p.qkv, p.QKV, kEpiStore};
      case 1: return GemvTask{w.o, H, p.QD, p.attn, p.QD, nullptr, p.eps, p.x, H, kEpiResidual};
      case 2: return GemvTask{w.gu, 2 * p.F, H, p.x, H, w.ln2, p.eps, p.mlp, p.F, kEpiSwiGLU};
      default: return GemvTask{w.down, H, p.F, p.mlp, p.F, nullptr, p.eps, p.x, H, kEpiResidual};
    }
  };
  const GemvTask head{p.head, p.head_rows, H, p.x, H, p.final_norm, p.eps, p.logits, p.logit_stride, kEpiStore};

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRingConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_epoch = ld_acquire(p.epoch);
    s_bad = 0;
  }
  __syncthreads();
  const int epoch = s_epoch;
  const int all = int(gridDim.x);

  if (warp == kRingConsumers) {
    if (lane == 0) {
      long long it = 0;
      bool ok = true;
      int g0, g1;
      const int kop[4] = {0, 2, 3, 4};
      auto pstamp = [&](int o, int k) {
        if (p.trace) p.trace[(size_t(blockIdx.x) * (5 * nL + 1) + o) * 8 + k] = globaltimer();
      };
      for (int l = 0; l < nL && ok; ++l)
        for (int k = 0; k < 4 && ok; ++k) {
          const GemvTask t = task(l, k);
          task_groups(t.N, blockIdx.x, gridDim.x, g0, g1);
          pstamp(5 * l + kop[k], 4);
          ok = ring_produce<NS>(t, g0, g1, ring, full, empty, it, p.error);
          pstamp(5 * l + kop[k], 5);
        }
      if (ok) {
        task_groups(head.N, blockIdx.x, gridDim.x, g0, g1);
        pstamp(5 * nL, 4);
        ring_produce<NS>(head, g0, g1, ring, full, empty, it, p.error);
        pstamp(5 * nL, 5);
      }
      ring_drain<NS>(full, it);
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int ctid = threadIdx.x;
  bool bad = false;
  long long it = 0;
  auto stamp = [&](int o, int k) {
    if (p.trace && ctid == 0) p.trace[(size_t(blockIdx.x) * (5 * nL + 1) + o) * 8 + k] = globaltimer();
  };
  auto unify_bad = [&]() {
    if (bad) s_bad = 1;
    consumer_sync();
    bad = s_bad != 0;
  };
  // All consumer threads' writes are ordered before thread 0's release fence by the
  // barrier; one fence + one atomic publishes the CTA's share.
  auto signal = [&](int idx) {
    consumer_sync();
    if (ctid == 0) {
      __threadfence();
      atomicAdd(p.ctr + idx, 1);
    }
  };
  // Wait until counter idx reaches target; gives up on expiry or once any CTA failed.
  auto wait_for = [&](int idx, int target) {
    if (ctid == 0 && !s_bad) {
      long long i = 0;
      for (; i < kCounterWaitLimit; ++i) {
        if (ld_acquire(p.ctr + idx) >= target) break;
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
  const int c_embed = 0, c_head = 1 + 5 * nL;
  auto c_op = [&](int l, int k) { return 1 + 5 * l + k; };  // k: 0 qkv, 1 attn, 2 o, 3 gu, 4 down

  // Embedding of each active row's token and the position latch (CTA 0).
  if (blockIdx.x == 0) {
    for (int b = 0; b < NB; ++b) {
      if (!__ldcg(p.active + b)) continue;
      int tok = __ldcg(p.token + b);
      if (tok < 0 || tok >= p.vocab) {
        if (ctid == 0) atomicOr(p.error, 1);
        tok = 0;
      }
      const uint4 *src = reinterpret_cast<const uint4 *>(p.embed + size_t(tok) * H);
      uint4 *dst = reinterpret_cast<uint4 *>(p.x + size_t(b) * H);
      for (int c = ctid; c < H / 8; c += kRingConsumers * 32) dst[c] = src[c];
    }
    if (ctid == 0)
      for (int b = 0; b < NB; ++b) {
        if (!__ldcg(p.active + b)) continue;
        const int q = __ldcg(p.pos + b);
        p.cur_pos[b] = q;
        if (q >= __ldcg(p.capacity + b)) {
          atomicOr(p.error, 2);
          p.active[b] = 0;
        } else {
          p.pos[b] = q + 1;
        }
      }
    signal(c_embed);
  }
  wait_for(c_embed, epoch + 1);
  // This step's row state (activity, position, cos/sin, page table) for the attention units.
  for (int b = 0; b < NB; ++b) attn_row_load<128>(rowst[b], p.ap, b, ctid, kRingConsumers * 32);
  consumer_sync();

  const int team = warp / 4, ttid = ctid % kAttnThreads;
  const int n_units = NB * kvh_n * nsplit;
  for (int l = 0; l < nL; ++l) {
    int g0, g1;
    // Prefetch into L2 the cached K/V this CTA's attention units will read in this layer.
    for (int u = blockIdx.x * 2; u < n_units; u += 2 * gridDim.x)
      for (int tm = 0; tm < 2 && u + tm < n_units; ++tm) {
        const int uu = u + tm, row = uu / (kvh_n * nsplit), kvh = (uu / nsplit) % kvh_n, split = uu % nsplit;
        attn_prefetch_kv<128>(p.ap, rowst[row], row, l, kvh, split, ctid, kRingConsumers * 32);
      }
    // QKV (RMSNorm of x fused).
    {
      stamp(5 * l, 0);
      const GemvTask t = task(l, 0);
      task_groups(t.N, blockIdx.x, gridDim.x, g0, g1);
      ring_stage_act<NB>(t, act, red, ctid);
      stamp(5 * l, 1);
      ring_consume<NB, NS>(t, g0, g1, ring, act, full, empty, it, gred, p.error, bad, ctid);
      stamp(5 * l, 2);
      unify_bad();
      signal(c_op(l, 0));
      stamp(5 * l, 3);
    }
    // Attention: two 4-warp teams per CTA, units (row, kv head, split) round-robin.
    wait_for(c_op(l, 0), (epoch + 1) * all);
    stamp(5 * l + 1, 0);
    {
      DecodeAttnParams ap = p.ap;
      ap.layer = l;
      ap.qn = p.layers[l].qn;
      ap.kn = p.layers[l].kn;
      for (int u = blockIdx.x * 2 + team; u < n_units; u += 2 * gridDim.x) {
        const int row = u / (kvh_n * nsplit), kvh = (u / nsplit) % kvh_n, split = u % nsplit;
        bool merged = false;
        unsigned long long *st =
            (p.trace && team == 0) ? p.trace + (size_t(blockIdx.x) * (5 * nL + 1) + 5 * l + 1) * 8 : nullptr;
        if (!bad) merged = attn_unit<128, 2>(ap, team_sm[team], rowst[row], row, kvh, split, ttid, 2 + team, st);
        // An inactive row contributes its kv heads' counts without work (split 0 stands in).
        const bool count = merged || (split == 0 && (bad || !rowst[row].active));
        if (count) {
          team_sync(2 + team);
          if (ttid == 0) {
            __threadfence();
            atomicAdd(p.ctr + c_op(l, 1), 1);
          }
        }
      }
    }
    stamp(5 * l + 1, 2);
    // O (+ residual).
    wait_for(c_op(l, 1), (epoch + 1) * kvh_n * NB);
    {
      stamp(5 * l + 2, 0);
      const GemvTask t = task(l, 1);
      task_groups(t.N, blockIdx.x, gridDim.x, g0, g1);
      ring_stage_act<NB>(t, act, red, ctid);
      stamp(5 * l + 2, 1);
      ring_consume<NB, NS>(t, g0, g1, ring, act, full, empty, it, gred, p.error, bad, ctid);
      stamp(5 * l + 2, 2);
      unify_bad();
      signal(c_op(l, 2));
      stamp(5 * l + 2, 3);
    }
    // gate/up (RMSNorm of x fused, SwiGLU epilogue).
    wait_for(c_op(l, 2), (epoch + 1) * all);
    {
      stamp(5 * l + 3, 0);
      const GemvTask t = task(l, 2);
      task_groups(t.N, blockIdx.x, gridDim.x, g0, g1);
      ring_stage_act<NB>(t, act, red, ctid);
      stamp(5 * l + 3, 1);
      ring_consume<NB, NS>(t, g0, g1, ring, act, full, empty, it, gred, p.error, bad, ctid);
      stamp(5 * l + 3, 2);
      unify_bad();
      signal(c_op(l, 3));
      stamp(5 * l + 3, 3);
    }
    // down (+ residual).
    wait_for(c_op(l, 3), (epoch + 1) * all);
    {
      stamp(5 * l + 4, 0);
      const GemvTask t = task(l, 3);
      task_groups(t.N, blockIdx.x, gridDim.x, g0, g1);
      ring_stage_act<NB>(t, act, red, ctid);
      stamp(5 * l + 4, 1);
      ring_consume<NB, NS>(t, g0, g1, ring, act, full, empty, it, gred, p.error, bad, ctid);
      stamp(5 * l + 4, 2);
      unify_bad();
      signal(c_op(l, 4));
      stamp(5 * l + 4, 3);
    }
    wait_for(c_op(l, 4), (epoch + 1) * all);
  }
  // Final RMSNorm + phase rows of the LM head.
  {
    int g0, g1;
    stamp(5 * nL, 0);
    task_groups(head.N, blockIdx.x, gridDim.x, g0, g1);
    ring_stage_act<NB>(head, act, red, ctid);
    stamp(5 * nL, 1);
    ring_consume<NB, NS>(head, g0, g1, ring, act, full, empty, it, gred, p.error, bad, ctid);
    stamp(5 * nL, 2);
    if (p.extra_row >= 0 && blockIdx.x == gridDim.x - 1 && warp < NB && !bad) {
      // The ABC phase's extra row (ABC_END), from the normalized activations in `act`.
      const bf16 *wr = p.head + size_t(p.extra_row - 0) * H;
      float v = 0.f;
      for (int c = lane; c < H / 8; c += 32) {
        const uint4 wq = ldg16(wr + c * 8), av = *reinterpret_cast<const uint4 *>(act + warp * H + c * 8);
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
      if (lane == 0) p.logits[size_t(warp) * p.logit_stride + p.head_rows] = f2bf(v);
    }
    unify_bad();
    signal(c_head);
  }
  if (blockIdx.x == 0) {
    wait_for(c_head, (epoch + 1) * all);
    if (ctid == 0) {
      __threadfence();
      atomicExch(p.epoch, epoch + 1);
    }
  }
}

size_t persistent_smem(int NB) {
  const size_t act = size_t(NB) * kPersistMaxK * 2, teams = 2 * sizeof(AttnSmem<128, 2>);
  return size_t(kPersistStages) * kRingStageBytes + (act > teams ? act : teams) + size_t(ring_gred_floats(NB)) * 4;
}

void configure_persistent_kernels() {
  YAR_CUDA(cudaFuncSetAttribute(k_decode_persistent<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(persistent_smem(1))));
  YAR_CUDA(cudaFuncSetAttribute(k_decode_persistent<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(persistent_smem(2))));
}

// True when the persistent kernel handles this model and row count.
bool persistent_supported(const Model &m, int n_rows) {
  const Dims &d = m.d;
  if (n_rows < 1 || n_rows > 2) return false;
  if (d.head_dim != 128 || d.heads != 2 * d.kv_heads) return false;
  if (d.hidden % kRingPiece || d.qdim() % kRingPiece || d.ffn % kRingPiece || d.ffn > kPersistMaxK ||
      d.hidden > kPersistMaxK || d.qdim() > kPersistMaxK)
    return false;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, n_rows == 1 ? k_decode_persistent<1> : k_decode_persistent<2>,
                                                    kPersistThreads, persistent_smem(n_rows)) != cudaSuccess)
    return false;
  return per_sm >= 1;
}

void launch_decode_persistent(const Model &m, Session &s, int n_rows, int phase, cudaStream_t st) {
  const Dims &d = m.d;
  const PhaseRows pr = phase_rows(d, phase);
  PersistParams p;
  p.layers = m.d_layers;
  p.n_layers = d.layers;
  p.H = d.hidden;
  p.QKV = d.qkv_rows();
  p.QD = d.qdim();
  p.F = d.ffn;
  p.vocab = d.vocab;
  p.eps = d.eps;
  p.embed = m.embed;
  p.final_norm = m.final_norm;
  p.head = m.lm_head + size_t(pr.row0) * d.hidden;
  p.head_rows = pr.n_main;
  p.extra_row = pr.extra >= 0 ? pr.extra - pr.row0 : -1;
  p.x = s.x;
  p.qkv = s.qkv;
  p.attn = s.attn;
  p.mlp = s.mlp;
  p.logits = s.logits;
  p.logit_stride = s.logit_stride;
  DecodeAttnParams &a = p.ap;
  a.g.heads = d.heads;
  a.g.kv_heads = d.kv_heads;
  a.g.head_dim = d.head_dim;
  a.g.qdim = d.qdim();
  a.g.kvdim = d.kvdim();
  a.g.page_tokens = s.page_tokens;
  a.g.pages_per_row = s.pages_per_row;
  a.g.num_pages = s.num_pages;
  a.g.page_elems = s.kv_page_elems;
  a.g.eps = d.eps;
  a.g.scale = float(1.0 / std::sqrt(double(d.head_dim)));
  a.layer = 0;
  a.max_splits = s.max_splits;
  a.pool = s.kv;
  a.page_table = s.d_page_table;
  a.cur_pos = s.d_cur_pos;
  a.active = s.d_active;
  a.qkv = s.qkv;
  a.qn = a.kn = nullptr;
  a.cos_tab = m.rope_cos;
  a.sin_tab = m.rope_sin;
  a.part = s.attn_part;
  a.count = s.attn_count;
  a.out = s.attn;
  p.token = s.d_token;
  p.pos = s.d_pos;
  p.cur_pos = s.d_cur_pos;
  p.capacity = s.d_capacity;
  p.active = s.d_active;
  p.error = s.d_error;
  p.ctr = s.d_ctr;
  p.epoch = s.d_epoch;
  p.trace = s.d_trace;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m.sm_count);
  cfg.blockDim = dim3(kPersistThreads);
  cfg.dynamicSmemBytes = persistent_smem(n_rows);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (n_rows == 1)
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_decode_persistent<1>, p));
  else
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_decode_persistent<2>, p));
}

}  // namespace yar
