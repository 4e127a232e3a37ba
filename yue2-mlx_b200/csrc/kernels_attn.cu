// kernels_attn.cu — q/k RMSNorm + RoPE + paged KV append, split-KV GQA decode attention,
// and causal prefill attention, all with FP32 scores, softmax and P.V accumulation
// (native/src/ar.cpp:88-96, :276-291; oracle/port/lyra/ar.py:131-145 names this "FP32
// attention opmath, BF16 storage outside the operation").
//
// KV pool layout: [layer][page][k|v][kv_head][page_tokens][head_dim] BF16; a row's page
// table maps logical page i (positions i*P .. i*P+P-1) to a physical page. Physical slot
// = RoPE position (modeling_yue2.py:383-393: StaticKVCache writes slot pos).
#include "attn_decode.cuh"
#include "tma_ring.cuh"

namespace yar {

static AttnGeom geom(const Model &m, const Session &s) {
  AttnGeom g;
  g.heads = m.d.heads;
  g.kv_heads = m.d.kv_heads;
  g.head_dim = m.d.head_dim;
  g.qdim = m.d.qdim();
  g.kvdim = m.d.kvdim();
  g.page_tokens = s.page_tokens;
  g.page_shift = 0;
  while ((1 << g.page_shift) < s.page_tokens) ++g.page_shift;
  g.pages_per_row = s.pages_per_row;
  g.num_pages = s.num_pages;
  g.page_elems = s.kv_page_elems;
  g.eps = m.d.eps;
  g.scale = float(1.0 / std::sqrt(double(m.d.head_dim)));
  return g;
}

// ---------------------------------------------------------------------------------------
// Decode: grid (kv_head, split, row), 256 threads = one attention unit per CTA
// (attn_decode.cuh); each chunk's cached rows are brought into shared memory, then
// processed by the same code as the persistent kernel. With pages of at least 64
// positions a chunk's K rows and its V rows are each one contiguous block (a chunk never
// straddles a page): thread 0 moves them with two bulk copies on an mbarrier; smaller
// pages take 16-byte cp.async copies, row by row. Two chunk buffers (dynamic shared
// memory, [2][K | V][64][D]): chunk c + 1's copies are in flight while chunk c is
// computed, and the first chunk's while q and k are normalized and rotated.
template <int D>
__host__ __device__ constexpr size_t attn_decode_dyn_smem() { return size_t(2) * 2 * kKvChunk * D * sizeof(bf16); }

template <int D, int G>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(DecodeAttnParams p) {
  __shared__ AttnTeamSmem<D, G> sm;
  __shared__ AttnRow<D> rs;
  __shared__ __align__(8) uint64_t kv_full[2];
  extern __shared__ __align__(16) unsigned char attn_dyn[];
  bf16 *kvbuf = reinterpret_cast<bf16 *>(attn_dyn);
  const int kvh = blockIdx.x, split = blockIdx.y, row = blockIdx.z, tid = threadIdx.x;
  const bool bulk = p.g.page_tokens >= kKvChunk;
  float wv[D / 32];
  attn_load_norm_w<D, G>(p.qn, p.kn, wv, tid);
  if (tid == 0) {
    mbar_init(&kv_full[0], 1);
    mbar_init(&kv_full[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  pdl_launch_dependents();
  pdl_wait();
  attn_row_load<D>(rs, p, row, tid, kAttnThreads);
  __syncthreads();
  if (!rs.active) return;
  const int pos = rs.pos;
  const SplitPlan sp = split_plan(pos + 1, p.max_splits);
  if (split >= sp.n_splits) return;  // beyond the context: no work, no arrival
  const int c0 = split * sp.cps, c1 = min((split + 1) * sp.cps, sp.nchunks);
  // Chunk c's cached K and V rows (positions < pos: the new one is appended by attn_qk and
  // read from shared memory) into buffer `slot`, as one cp.async group.
  auto issue = [&](int c, int slot) {
    const int base = c * kKvChunk, n_main = min(kKvChunk, pos - base);
    bf16 *kb = kvbuf + size_t(slot) * 2 * kKvChunk * D, *vb = kb + kKvChunk * D;
    if (bulk) {
      if (tid == 0) {
        const unsigned bytes = unsigned(n_main) * D * 2;
        mbar_arrive_expect_tx(&kv_full[slot], 2 * bytes);
        if (bytes) {
          bulk_g2s(kb, kv_row_ptr<D>(p, rs, row, p.layer, 0, kvh, base), bytes, &kv_full[slot]);
          bulk_g2s(vb, kv_row_ptr<D>(p, rs, row, p.layer, 1, kvh, base), bytes, &kv_full[slot]);
        }
      }
      return;
    }
    for (int idx = tid; idx < n_main * (D / 8); idx += kAttnThreads) {
      const int r = idx / (D / 8), cc = idx % (D / 8);
      const bf16 *ks = kv_row_ptr<D>(p, rs, row, p.layer, 0, kvh, base + r) + cc * 8;
      const bf16 *vs = kv_row_ptr<D>(p, rs, row, p.layer, 1, kvh, base + r) + cc * 8;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(
                       __cvta_generic_to_shared(kb + r * D + cc * 8))),
                   "l"(ks)
                   : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(
                       __cvta_generic_to_shared(vb + r * D + cc * 8))),
                   "l"(vs)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  int issued = 0;  // chunks whose copies were issued (uniform across the CTA)
  if (c0 < c1) {
    issue(c0, 0);
    issued = 1;
  }
  attn_qk<D, G>(p, sm, rs, row, kvh, split == sp.n_splits - 1, wv, tid, 1);
  AttnWarpAcc<D, G> wacc;
  attn_warp_init(wacc);
  // A bulk wait that expires is latched CTA-wide (`bad`): no further copies are issued and
  // no chunk is computed; the unit still arrives (so the arrival count stays consistent)
  // and, before the CTA exits, waits (bounded) for every copy it issued.
  bool bad = false;
  int done = 0;  // chunks whose copies completed
  for (int c = c0; c < c1; ++c) {
    const int slot = (c - c0) & 1, base = c * kKvChunk, n_main = min(kKvChunk, pos - base);
    // The other buffer was last read by chunk c - 1, which every warp had finished at the
    // barrier ending that iteration: it is free for chunk c + 1.
    if (c + 1 < c1 && !bad) {
      issue(c + 1, slot ^ 1);
      ++issued;
    }
    if (bulk) {
      const bool failed = !bad && !mbar_wait(&kv_full[slot], unsigned((c - c0) >> 1) & 1u);
      if (__syncthreads_or(failed)) {
        if (!bad && tid == 0 && p.error) atomicOr(p.error, 8);
        bad = true;
      }
      if (bad) break;
      done = c - c0 + 1;
    } else if (c + 1 < c1) {
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    team_sync(1);
    const bf16 *kb = kvbuf + size_t(slot) * 2 * kKvChunk * D;
    attn_chunk<D, G>(sm.q_b, sm.knew, sm.vnew, kb, kb + kKvChunk * D, n_main, pos - base < kKvChunk, p.g.scale,
                     wacc, tid);
    team_sync(1);
  }
  if (bad)
    for (int i = done; i < issued; ++i) mbar_wait(&kv_full[i & 1], unsigned(i >> 1) & 1u);
  const AttnAcc<D> acc = attn_combine<D, G>(sm, wacc, tid, 1);
  attn_finish<D, G>(p, sm, acc, row, kvh, split, sp.n_splits, tid, 1);
}

void launch_attn_decode(const Model &m, Session &s, int layer, int n_rows, cudaStream_t st, int max_splits) {
  DecodeAttnParams p;
  p.g = geom(m, s);
  p.layer = layer;
  p.max_splits = max_splits > 0 && max_splits < s.max_splits ? max_splits : s.max_splits;
  p.pool = s.kv;
  p.page_table = s.d_page_table;
  p.cur_pos = s.d_cur_pos;
  p.active = s.d_active;
  p.qkv = s.qkv;
  p.qn = m.layers[layer].qn;
  p.kn = m.layers[layer].kn;
  p.cos_tab = m.rope_cos;
  p.sin_tab = m.rope_sin;
  p.part = s.attn_part;
  p.count = s.attn_count;
  // Under tensor parallelism this rank's heads sit at their place in the whole model's rows.
  p.out = s.attn + m.tp.q_row0;
  p.out_stride = m.full.qdim();
  p.out_ndst = 0;
  p.out_dst = nullptr;
  p.error = s.d_error;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m.d.kv_heads, p.max_splits, n_rows);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = m.d.head_dim == 128 ? attn_decode_dyn_smem<128>() : attn_decode_dyn_smem<64>();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int G = m.d.heads / m.d.kv_heads;
  if (m.d.head_dim == 128 && G == 2)
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<128, 2>, p));
  else if (m.d.head_dim == 128 && G == 1)
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<128, 1>, p));
  else if (m.d.head_dim == 64 && G == 2)
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<64, 2>, p));
  else if (m.d.head_dim == 64 && G == 1)
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<64, 1>, p));
  else
    throw Error("ValueError", "head_dim must be 64 or 128 and the GQA group 1 or 2");
}

// ---------------------------------------------------------------------------------------
// Prefill: q/k norm + RoPE for T tokens; k, v appended to the row's pages; q kept in
// pq [T][heads][D] (BF16). One CTA per token, one warp per head.
struct QkvPostParams {
  AttnGeom g;
  int layer, start, T;
  bf16 *pool;
  const int *ptab;
  const bf16 *qkv;  // [T][qdim + 2*kvdim]
  const bf16 *qn, *kn;
  const float *cos_tab, *sin_tab;
  bf16 *q_out;  // [T][heads][D]
};

template <int D>
__global__ void __launch_bounds__(256) k_qkv_post(QkvPostParams p) {
  __shared__ float buf[8][D];
  const AttnGeom &g = p.g;
  const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int pos = p.start + t;
  const bf16 *src = p.qkv + size_t(t) * (g.qdim + 2 * g.kvdim);
  const float *cosr = p.cos_tab + size_t(pos) * (D / 2);
  const float *sinr = p.sin_tab + size_t(pos) * (D / 2);
  const int nh = g.heads + 2 * g.kv_heads;
  for (int h = warp; h < nh; h += 8) {
    const bf16 *hs = src + h * D;
    if (h >= g.heads + g.kv_heads) {  // v: raw copy into the cache
      const int kvh = h - g.heads - g.kv_heads;
      bf16 *dst = kv_addr(p.pool, g, p.ptab, p.layer, 1, kvh, pos);
      for (int d = lane; d < D; d += 32) dst[d] = hs[d];
      continue;
    }
    float *v = buf[warp];
    for (int d = lane; d < D; d += 32) v[d] = bf2f(hs[d]);
    __syncwarp();
    const bool is_k = h >= g.heads;
    norm_rope_head<D>(v, is_k ? p.kn : p.qn, cosr, sinr, g.eps, lane);
    bf16 *dst = is_k ? kv_addr(p.pool, g, p.ptab, p.layer, 0, h - g.heads, pos)
                     : p.q_out + (size_t(t) * g.heads + h) * D;
    for (int d = lane; d < D; d += 32) dst[d] = f2bf(v[d]);
    __syncwarp();
  }
}

void launch_qkv_post_prefill(const Model &m, Session &s, int layer, int row, int start, int T,
                             cudaStream_t st) {
  QkvPostParams p;
  p.g = geom(m, s);
  p.layer = layer;
  p.start = start;
  p.T = T;
  p.pool = s.kv;
  p.ptab = s.d_page_table + size_t(row) * s.pages_per_row;
  p.qkv = s.pqkv;
  p.qn = m.layers[layer].qn;
  p.kn = m.layers[layer].kn;
  p.cos_tab = m.rope_cos;
  p.sin_tab = m.rope_sin;
  p.q_out = s.pq;
  if (m.d.head_dim == 128)
    k_qkv_post<128><<<T, 256, 0, st>>>(p);
  else
    k_qkv_post<64><<<T, 256, 0, st>>>(p);
  YAR_CUDA(cudaGetLastError());
}

// Causal prefill attention over the row's cache positions [0, start + T) for head_dim 64
// (head_dim 128 runs k_attn_prefill_tc in kernels_attn_tc.cu, or k_attn_prefill_mma below
// with session option 7 off): grid (ceil(T/64), heads), 256 threads,
// FP32 tiles of 64 queries x 64 keys in shared memory.
// Thread t owns queries 4*(t/16) .. +3 and, for scores, keys 4*(t%16) .. +3; for the
// output, dims (D/16)*(t%16) .. +D/16-1.
struct PrefillAttnParams {
  AttnGeom g;
  int layer, start, T;
  bf16 *pool;
  const int *ptab;
  const bf16 *q;  // [T][heads][D]
  bf16 *out;      // token t, head h at out[t * out_stride + h * D]
  int out_stride;
};

template <int D>
__global__ void __launch_bounds__(256) k_attn_prefill(PrefillAttnParams p) {
  constexpr int BQ = 64, BK = 64, DT = D / 16;
  extern __shared__ __align__(16) float sm[];
  float *qs = sm;              // [BQ][D+1]
  float *ks = qs + BQ * (D + 1);  // [BK][D+1]
  float *vs = ks + BK * (D + 1);  // [BK][D]
  float *ps = vs + BK * D;        // [BQ][BK+1]
  const AttnGeom &g = p.g;
  const int qt = blockIdx.x, h = blockIdx.y, kvh = h / (g.heads / g.kv_heads);
  const int t = threadIdx.x, qg = t / 16, kj = t % 16;
  const int q0 = qt * BQ;
  for (int i = t; i < BQ * D; i += 256) {
    const int r = i / D, d = i % D;
    qs[r * (D + 1) + d] = (q0 + r < p.T) ? bf2f(p.q[(size_t(q0 + r) * g.heads + h) * D + d]) : 0.f;
  }
  float m[4], l[4], o[4][DT];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < DT; ++j) o[i][j] = 0.f;
  }
  const int qlast = min(p.T, q0 + BQ) - 1;  // last query (local) in this tile
  const int kend = p.start + qlast + 1;     // keys visible to the last query
  for (int k0 = 0; k0 < kend; k0 += BK) {
    __syncthreads();
    for (int i = t; i < BK * D; i += 256) {
      const int r = i / D, d = i % D, kp = k0 + r;
      float kv = 0.f, vv = 0.f;
      if (kp < kend) {
        kv = bf2f(kv_addr(p.pool, g, p.ptab, p.layer, 0, kvh, kp)[d]);
        vv = bf2f(kv_addr(p.pool, g, p.ptab, p.layer, 1, kvh, kp)[d]);
      }
      ks[r * (D + 1) + d] = kv;
      vs[r * D + d] = vv;
    }
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
    for (int d = 0; d < D; ++d) {
      float qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = qs[(qg * 4 + i) * (D + 1) + d];
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = ks[(kj * 4 + j) * (D + 1) + d];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qpos = p.start + q0 + qg * 4 + i;
      float rmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kp = k0 + kj * 4 + j;
        s[i][j] = (kp <= qpos && kp < kend) ? s[i][j] * g.scale : -INFINITY;
        rmax = fmaxf(rmax, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xFFFFFFFFu, rmax, off));
      const float mn = fmaxf(m[i], rmax);
      float corr = 0.f, rsum = 0.f;
      if (mn != -INFINITY) {
        corr = expf(m[i] - mn);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float e = s[i][j] == -INFINITY ? 0.f : expf(s[i][j] - mn);
          ps[(qg * 4 + i) * (BK + 1) + kj * 4 + j] = e;
          rsum += e;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) ps[(qg * 4 + i) * (BK + 1) + kj * 4 + j] = 0.f;
        corr = 1.f;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rsum += __shfl_xor_sync(0xFFFFFFFFu, rsum, off);
      l[i] = l[i] * corr + rsum;
      m[i] = mn;
#pragma unroll
      for (int j = 0; j < DT; ++j) o[i][j] *= corr;
    }
    __syncwarp();
    __syncthreads();
    for (int j = 0; j < BK; ++j) {
      float vv[DT];
#pragma unroll
      for (int dd = 0; dd < DT; ++dd) vv[dd] = vs[j * D + kj * DT + dd];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float pv = ps[(qg * 4 + i) * (BK + 1) + j];
#pragma unroll
        for (int dd = 0; dd < DT; ++dd) o[i][dd] = fmaf(pv, vv[dd], o[i][dd]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = q0 + qg * 4 + i;
    if (qi >= p.T) continue;
    const float inv = 1.0f / l[i];
#pragma unroll
    for (int dd = 0; dd < DT; ++dd)
      p.out[size_t(qi) * p.out_stride + h * D + kj * DT + dd] = f2bf(o[i][dd] * inv);
  }
}

static size_t prefill_attn_smem(int D) { return (64 * (D + 1) * 2 + 64 * D + 64 * 65) * sizeof(float); }

// ---------------------------------------------------------------------------------------
// Causal prefill attention on tensor cores (head_dim 128): the same queries, keys, causal
// rule and FP32 softmax as k_attn_prefill, computed flash-attention style. Grid
// (ceil(T/64), heads), 4 warps; warp w owns queries 16w..16w+15 of the tile, held in
// registers as the A operand of mma.sync m16n8k16 (BF16 in, FP32 accumulate). Per tile of
// 64 keys (cp.async into rows padded to 272 bytes, two tiles in flight):
//   S = Q K^T (K rows as the B operand via ldmatrix), scaled and masked, folded into the
//   running row max / sum (quad shuffles) with exp rescaling of O;
//   O += P V with P taken from the S accumulators as the A operand, split into BF16 high
//   and low parts (two MMAs: P keeps ~16 mantissa bits, products within 2^-17 of FP32 P)
//   and V through ldmatrix.trans.
// Key rows past the last visible key are zeroed (their scores are masked; V must stay
// finite under P = 0).
constexpr int kPfPitch = 128 + 8;                        // BF16 elements per K/V row
constexpr int kPfTile = 64 * kPfPitch;                   // one K or V tile
constexpr size_t kPfSmem = size_t(2) * 2 * kPfTile * 2;  // two stages of K and V tiles

__device__ __forceinline__ void mma_bf16_16816(float *c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4_b16(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}
__device__ __forceinline__ void ldsm_x4_trans_b16(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3,
                                                  const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}
// (x, y) as a BF16 pair (x in the low half), and the pair of what that rounding left.
__device__ __forceinline__ void split_bf16_pair(float x, float y, uint32_t &hi, uint32_t &lo) {
  const uint32_t xh = __float_as_uint(rbf(x)), yh = __float_as_uint(rbf(y));
  hi = (xh >> 16) | (yh & 0xFFFF0000u);
  const uint32_t xl = __float_as_uint(rbf(x - __uint_as_float(xh))), yl = __float_as_uint(rbf(y - __uint_as_float(yh)));
  lo = (xl >> 16) | (yl & 0xFFFF0000u);
}

__global__ void __launch_bounds__(128) k_attn_prefill_mma(PrefillAttnParams p) {
  constexpr int D = 128, BQ = 64, BK = 64;
  extern __shared__ __align__(16) unsigned char pf_raw[];
  bf16 *tiles = reinterpret_cast<bf16 *>(pf_raw);  // [stage][K | V][64][kPfPitch]
  const AttnGeom &g = p.g;
  const int qt = blockIdx.x, h = blockIdx.y, kvh = h / (g.heads / g.kv_heads);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gr = lane >> 2, tq = lane & 3;
  const int q0 = qt * BQ;
  const int qlast = min(p.T, q0 + BQ) - 1;
  const int kend = p.start + qlast + 1;  // keys visible to the tile's last query
  const int ntiles = (kend + BK - 1) / BK;

  // K and V rows of key tile `kt` into stage `st` (one cp.async group).
  auto load_tile = [&](int kt, int st) {
    bf16 *kb = tiles + size_t(st) * 2 * kPfTile, *vb = kb + kPfTile;
    const int k0 = kt * BK, cc = tid & 15;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = (tid >> 4) + 8 * j, kp = k0 + r;
      bf16 *kd = kb + r * kPfPitch + cc * 8, *vd = vb + r * kPfPitch + cc * 8;
      if (kp < kend) {
        const bf16 *ks = kv_addr(p.pool, g, p.ptab, p.layer, 0, kvh, kp) + cc * 8;
        const bf16 *vs = ks + g.page_elems;  // the V block follows the K block of the page
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(
                         __cvta_generic_to_shared(kd))),
                     "l"(ks)
                     : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(
                         __cvta_generic_to_shared(vd))),
                     "l"(vs)
                     : "memory");
      } else {
        *reinterpret_cast<uint4 *>(kd) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4 *>(vd) = make_uint4(0, 0, 0, 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_tile(0, 0);

  // This warp's 16 queries as A fragments (rows gr and gr + 8), 8 k-tiles of 16 dims.
  uint32_t qa[8][4];
  {
    const int r0 = q0 + warp * 16 + gr, r1 = r0 + 8;
    const bf16 *q0p = p.q + (size_t(r0) * g.heads + h) * D, *q1p = p.q + (size_t(r1) * g.heads + h) * D;
#pragma unroll
    for (int kt = 0; kt < 8; ++kt) {
      const int d = kt * 16 + 2 * tq;
      qa[kt][0] = r0 < p.T ? *reinterpret_cast<const uint32_t *>(q0p + d) : 0u;
      qa[kt][1] = r1 < p.T ? *reinterpret_cast<const uint32_t *>(q1p + d) : 0u;
      qa[kt][2] = r0 < p.T ? *reinterpret_cast<const uint32_t *>(q0p + d + 8) : 0u;
      qa[kt][3] = r1 < p.T ? *reinterpret_cast<const uint32_t *>(q1p + d + 8) : 0u;
    }
  }
  const int qpos0 = p.start + q0 + warp * 16 + gr, qpos1 = qpos0 + 8;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float oa[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) oa[n][0] = oa[n][1] = oa[n][2] = oa[n][3] = 0.f;

  for (int kt = 0; kt < ntiles; ++kt) {
    const int st = kt & 1;
    // The other stage was last read before the previous tile's closing barrier.
    if (kt + 1 < ntiles) {
      load_tile(kt + 1, st ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const bf16 *kb = tiles + size_t(st) * 2 * kPfTile, *vb = kb + kPfTile;
    const int k0 = kt * BK;
    // S = Q K^T: 8 n-tiles of 8 keys.
    float sa[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      sa[n][0] = sa[n][1] = sa[n][2] = sa[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // 32 dims per ldmatrix.x4
        uint32_t b0, b1, b2, b3;
        ldsm_x4_b16(b0, b1, b2, b3, kb + (n * 8 + (lane & 7)) * kPfPitch + kk * 32 + (lane >> 3) * 8);
        mma_bf16_16816(sa[n], qa[2 * kk][0], qa[2 * kk][1], qa[2 * kk][2], qa[2 * kk][3], b0, b1);
        mma_bf16_16816(sa[n], qa[2 * kk + 1][0], qa[2 * kk + 1][1], qa[2 * kk + 1][2], qa[2 * kk + 1][3], b2, b3);
      }
    }
    // Scale, mask, and fold into the running max / sum of rows gr (0, 1) and gr + 8 (2, 3).
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int kp = k0 + n * 8 + 2 * tq;
      sa[n][0] = kp <= qpos0 ? sa[n][0] * g.scale : -INFINITY;
      sa[n][1] = kp + 1 <= qpos0 ? sa[n][1] * g.scale : -INFINITY;
      sa[n][2] = kp <= qpos1 ? sa[n][2] * g.scale : -INFINITY;
      sa[n][3] = kp + 1 <= qpos1 ? sa[n][3] * g.scale : -INFINITY;
      mx0 = fmaxf(mx0, fmaxf(sa[n][0], sa[n][1]));
      mx1 = fmaxf(mx1, fmaxf(sa[n][2], sa[n][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = mn0 == -INFINITY ? 1.f : expf(m0 - mn0), c1 = mn1 == -INFINITY ? 1.f : expf(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      sa[n][0] = sa[n][0] == -INFINITY ? 0.f : expf(sa[n][0] - mn0);
      sa[n][1] = sa[n][1] == -INFINITY ? 0.f : expf(sa[n][1] - mn0);
      sa[n][2] = sa[n][2] == -INFINITY ? 0.f : expf(sa[n][2] - mn1);
      sa[n][3] = sa[n][3] == -INFINITY ? 0.f : expf(sa[n][3] - mn1);
      ps0 += sa[n][0] + sa[n][1];
      ps1 += sa[n][2] + sa[n][3];
    }
    l0 = l0 * c0 + ps0;
    l1 = l1 * c1 + ps1;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      oa[n][0] *= c0;
      oa[n][1] *= c0;
      oa[n][2] *= c1;
      oa[n][3] *= c1;
    }
    // O += P V: 4 k-tiles of 16 keys, 16 n-tiles of 8 dims (pairs via ldmatrix.x4.trans).
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t h0, l0b, h1, l1b, h2, l2b, h3, l3b;
      split_bf16_pair(sa[2 * kk][0], sa[2 * kk][1], h0, l0b);
      split_bf16_pair(sa[2 * kk][2], sa[2 * kk][3], h1, l1b);
      split_bf16_pair(sa[2 * kk + 1][0], sa[2 * kk + 1][1], h2, l2b);
      split_bf16_pair(sa[2 * kk + 1][2], sa[2 * kk + 1][3], h3, l3b);
      const int vrow = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans_b16(b0, b1, b2, b3, vb + vrow * kPfPitch + np * 16 + (lane >> 4) * 8);
        mma_bf16_16816(oa[2 * np], h0, h1, h2, h3, b0, b1);
        mma_bf16_16816(oa[2 * np], l0b, l1b, l2b, l3b, b0, b1);
        mma_bf16_16816(oa[2 * np + 1], h0, h1, h2, h3, b2, b3);
        mma_bf16_16816(oa[2 * np + 1], l0b, l1b, l2b, l3b, b2, b3);
      }
    }
    __syncthreads();  // every warp is done with this stage before it is refilled
  }
  // Row sums across the quad, then the BF16 outputs.
  l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 1);
  l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 2);
  l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 1);
  l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 2);
  const int r0 = q0 + warp * 16 + gr, r1 = r0 + 8;
  const float i0 = 1.0f / l0, i1 = 1.0f / l1;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int d = n * 8 + 2 * tq;
    if (r0 < p.T) {
      bf16 *o = p.out + size_t(r0) * p.out_stride + h * D + d;
      o[0] = f2bf(oa[n][0] * i0);
      o[1] = f2bf(oa[n][1] * i0);
    }
    if (r1 < p.T) {
      bf16 *o = p.out + size_t(r1) * p.out_stride + h * D + d;
      o[0] = f2bf(oa[n][2] * i1);
      o[1] = f2bf(oa[n][3] * i1);
    }
  }
}

void configure_attn_kernels() {
  YAR_CUDA(cudaFuncSetAttribute(k_attn_decode<128, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(attn_decode_dyn_smem<128>())));
  YAR_CUDA(cudaFuncSetAttribute(k_attn_decode<128, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(attn_decode_dyn_smem<128>())));
  YAR_CUDA(cudaFuncSetAttribute(k_attn_decode<64, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(attn_decode_dyn_smem<64>())));
  YAR_CUDA(cudaFuncSetAttribute(k_attn_decode<64, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(attn_decode_dyn_smem<64>())));
  YAR_CUDA(cudaFuncSetAttribute(k_attn_prefill_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kPfSmem)));
  YAR_CUDA(cudaFuncSetAttribute(k_attn_prefill<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(prefill_attn_smem(64))));
}

// kernels_attn_tc.cu: the tcgen05 kernel for head_dim 128; false when it does not apply.
bool launch_attn_prefill_tc(const Model &m, Session &s, const AttnGeom &g, int layer, int row, int start, int T,
                            cudaStream_t st);

void launch_attn_prefill(const Model &m, Session &s, int layer, int row, int start, int T,
                         cudaStream_t st) {
  PrefillAttnParams p;
  p.g = geom(m, s);
  p.layer = layer;
  p.start = start;
  p.T = T;
  p.pool = s.kv;
  p.ptab = s.d_page_table + size_t(row) * s.pages_per_row;
  p.q = s.pq;
  p.out = s.pattn + m.tp.q_row0;
  p.out_stride = m.full.qdim();
  const int D = m.d.head_dim;
  if (D == 128 && s.prefill_attn_tc && launch_attn_prefill_tc(m, s, p.g, layer, row, start, T, st)) return;
  dim3 grid((T + 63) / 64, m.d.heads);
  if (D == 128)
    k_attn_prefill_mma<<<grid, 128, kPfSmem, st>>>(p);
  else
    k_attn_prefill<64><<<grid, 256, prefill_attn_smem(D), st>>>(p);
  YAR_CUDA(cudaGetLastError());
}

}  // namespace yar
