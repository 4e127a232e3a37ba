// attn_decode.cuh — the split-KV GQA decode attention, shared by the standalone kernel
// (k_attn_decode) and the persistent decode kernel, so both produce the same bits.
//
// The cached positions of a row are cut into chunks of 64 (one chunk never straddles a
// page of >= 64 positions, so its K rows and its V rows are each one contiguous 16 KB
// block for head_dim 128). A split is a run of consecutive chunks; a unit = (row, kv head,
// split) is processed by 256 threads (8 warps):
//   1. q-norm + RoPE of the group's G q heads; the unit holding the new position also
//      norms and ropes the new k and appends k, v to the paged cache;
//   2. per chunk (rows staged in shared memory): each warp takes eight of the 64 positions
//      — FP32 scores (4 lanes per position), its running max / exp-sum / output rescaled by
//      exp(m_old - m_new), P.V over its rows — with no barrier among the warps; the warps'
//      states are combined once at the end of the unit;
//   3. a partial (max, sum, o[D]) per q head; the last of the row's splits to arrive merges
//      them into the BF16 head outputs (native/src/ar.cpp:88-96, :276-291;
//      oracle/port/lyra/ar.py:131-145).
#pragma once
#include "common.cuh"
#include "tma_ring.cuh"

namespace yar {

struct AttnGeom {
  int heads, kv_heads, head_dim, qdim, kvdim, page_tokens, page_shift, pages_per_row, num_pages;
  size_t page_elems;  // kv_heads * P * D
  float eps, scale;
};

// Address of (layer, kv, kv_head, position) for a row's page table.
__device__ __forceinline__ bf16 *kv_addr(bf16 *pool, const AttnGeom &g, const int *ptab, int layer,
                                         int kv, int head, int pos) {
  const int page = ptab[pos >> g.page_shift], slot = pos & (g.page_tokens - 1);
  const size_t blk = (size_t(layer) * g.num_pages + page) * 2 + kv;
  return pool + blk * g.page_elems + (size_t(head) * g.page_tokens + slot) * g.head_dim;
}

// Per-head RMSNorm (modeling_yue2.py:185) then half-split RoPE with BF16 cos/sin and a
// rounding after every product and sum (modeling_yue2.py:152-156). `v` holds the raw
// BF16 head values (as floats) in shared memory; `warp` threads cooperate on one head.
template <int D>
__device__ __forceinline__ void norm_rope_head(float *v, const bf16 *w, const float *cosr, const float *sinr,
                               float eps, int lane) {
  float ss = 0.f;
  for (int d = lane; d < D; d += 32) ss += v[d] * v[d];
  ss = warp_sum(ss);
  const float scale = rms_scale_bf16(ss, D, eps);
  float nv[D / 32];
#pragma unroll
  for (int i = 0; i < D / 32; ++i) {
    const int d = lane + 32 * i;
    nv[i] = rbf(rbf(v[d] * scale) * bf2f(w[d]));
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < D / 32; ++i) v[lane + 32 * i] = nv[i];
  __syncwarp();
  constexpr int H = D / 2;
  float out[D / 32];
#pragma unroll
  for (int i = 0; i < D / 32; ++i) {
    const int d = lane + 32 * i;
    if (d < H) {
      const float c = cosr[d], s = sinr[d];
      out[i] = rbf(rbf(v[d] * c) - rbf(v[d + H] * s));
    } else {
      const float c = cosr[d - H], s = sinr[d - H];
      out[i] = rbf(rbf(v[d] * c) + rbf(v[d - H] * s));
    }
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < D / 32; ++i) v[lane + 32 * i] = out[i];
  __syncwarp();
}

constexpr int kAttnThreads = 256;  // one unit at a time on all 8 warps

struct DecodeAttnParams {
  AttnGeom g;
  int layer, max_splits;
  bf16 *pool;
  const int *page_table;
  const int *cur_pos;
  const int *active;
  const bf16 *qkv;  // [rows][qdim + 2*kvdim] raw projections
  const bf16 *qn, *kn;
  const float *cos_tab, *sin_tab;
  float *part;   // [rows][heads][max_splits][D + 2]
  int *count;    // [rows][kv_heads]
  bf16 *out;     // row r, head h at out[r * out_stride + h * D]
  int out_stride;
  int out_ndst;  // tensor parallelism: also stored at out + out_dst[i] bytes (peer copies)
  const long long *out_dst;
  int *error;  // device error word: expired waits of the standalone kernel (may be null)
  // Flagged transport (the persistent kernel; null: plain buffers): raw projections read
  // from flagged words [rows][qkv_ll_stride] once they carry qkv_flag, head outputs
  // written as flagged words [rows][out_ll_stride] with out_flag.
  const uint2 *qkv_ll = nullptr;
  int qkv_ll_stride = 0;
  uint32_t qkv_flag = 0;
  uint2 *out_ll = nullptr;
  int out_ll_stride = 0;
  uint32_t out_flag = 0;
  long long ll_limit = 1ll << 22;  // polls of a flagged wait before it gives up
  // Split partials as flagged words (FP32 value + flag), [rows][heads][max_splits][D + 2]
  // (m, l, o[D]), merged by a dedicated merge job (attn_merge_ll) instead of the last
  // split to arrive; null: plain partials in `part` and arrival counters.
  uint2 *part_ll = nullptr;
  uint32_t part_flag = 0;
};

constexpr int kKvChunk = 64;  // positions per KV chunk

// The split plan of a row whose context holds L positions (the new one included): split s
// covers chunks [s * cps, min((s + 1) * cps, nchunks)); the last split holds the new position.
struct SplitPlan {
  int nchunks, cps, n_splits;
};
__host__ __device__ __forceinline__ SplitPlan split_plan(int L, int max_splits) {
  SplitPlan r;
  r.nchunks = (L + kKvChunk - 1) / kKvChunk;
  r.cps = (r.nchunks + max_splits - 1) / max_splits;
  r.n_splits = (r.nchunks + r.cps - 1) / r.cps;
  return r;
}

// Shared memory of one team.
template <int D, int G>
struct __align__(16) AttnTeamSmem {
  bf16 q_b[G][D];              // normed, roped q (BF16-exact values)
  bf16 knew[D], vnew[D];       // the new position's k (normed, roped) and v, as cached
  float wml[kAttnThreads / 32][G][2];  // per-warp (max, exp-sum) at the unit's end
  float wc[kAttnThreads / 32][G];      // per-warp weight exp(m_w - M) in the combine (-1: no positions)
  float pvp[kAttnThreads / 32][G * D];  // per-warp unnormalized outputs at the unit's end
  int last_flag;
};

// Per-step state of one row, staged in shared memory once: activity, the position being
// decoded, its RoPE cos/sin, and the page table.
template <int D>
struct AttnRow {
  static constexpr int kMaxPages = 128;
  int active, pos;
  float cosr[D / 2], sinr[D / 2];
  int ptab[kMaxPages];
};

// Fill `rs` for `row` with `nthreads` threads starting at thread `tid`; the caller
// synchronizes afterwards. Tables longer than kMaxPages stay in global memory.
// `active` and `pos` as the caller computed them for this step.
template <int D>
__device__ void attn_row_load_at(AttnRow<D> &rs, const DecodeAttnParams &p, int row, int active, int pos, int tid,
                                 int nthreads) {
  if (tid == 0) {
    rs.active = active;
    rs.pos = pos;
  }
  for (int i = tid; i < D / 2; i += nthreads) {
    rs.cosr[i] = p.cos_tab[size_t(pos) * (D / 2) + i];
    rs.sinr[i] = p.sin_tab[size_t(pos) * (D / 2) + i];
  }
  const int n = p.g.pages_per_row < AttnRow<D>::kMaxPages ? p.g.pages_per_row : AttnRow<D>::kMaxPages;
  for (int i = tid; i < n; i += nthreads) rs.ptab[i] = p.page_table[size_t(row) * p.g.pages_per_row + i];
}
// The row's activity and latched position from p.active / p.cur_pos.
template <int D>
__device__ void attn_row_load(AttnRow<D> &rs, const DecodeAttnParams &p, int row, int tid, int nthreads) {
  attn_row_load_at<D>(rs, p, row, __ldcg(p.active + row), __ldcg(p.cur_pos + row), tid, nthreads);
}

template <int D>
__device__ __forceinline__ bf16 *kv_row_ptr(const DecodeAttnParams &p, const AttnRow<D> &rs, int row, int layer,
                                           int kv, int kvh, int q) {
  const AttnGeom &g = p.g;
  const int lp = q >> g.page_shift;
  const int page = lp < AttnRow<D>::kMaxPages ? rs.ptab[lp] : p.page_table[size_t(row) * g.pages_per_row + lp];
  const size_t blk = (size_t(layer) * g.num_pages + page) * 2 + kv;
  return p.pool + blk * g.page_elems + (size_t(kvh) * g.page_tokens + (q & (g.page_tokens - 1))) * D;
}

// lo += a.lo * b.lo and hi += a.hi * b.hi for BF16 pairs a, b, FP32 accumulators: the
// mixed-precision FMA takes the BF16 halves directly (their conversion to FP32 is exact,
// so each result is fmaf of the converted values, rounded once) instead of unpacking
// both operands with shifts and masks first.
__device__ __forceinline__ void fma_bf16x2(float &lo, float &hi, uint32_t a, uint32_t b) {
  asm("{\n .reg .b16 al, ah, bl, bh;\n mov.b32 {al, ah}, %2;\n mov.b32 {bl, bh}, %3;\n"
      " fma.rn.f32.bf16 %0, al, bl, %0;\n fma.rn.f32.bf16 %1, ah, bh, %1;\n}"
      : "+f"(lo), "+f"(hi)
      : "r"(a), "r"(b));
}

__device__ __forceinline__ void team_sync(int bar_id) {
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "n"(kAttnThreads) : "memory");
}

__device__ __forceinline__ void attn_stamp(unsigned long long *st, int k, int tid) {
  if (st && tid == 0) st[k] = (unsigned long long)clock64();
}

// q/k RMSNorm (modeling_yue2.py:185) then half-split RoPE (:152-156) of one head held
// in registers, lane l owning dims l, l+32, ...: the RoPE pairs (d, d + D/2) are in the
// same lane. BF16 rounding after every product and sum, as upstream.
template <int D>
__device__ __forceinline__ void norm_rope_regs(float (&v)[D / 32], const float (&w)[D / 32], const float *cosr,
                                               const float *sinr, float eps, int lane) {
  constexpr int NPL = D / 32, HALF = NPL / 2;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NPL; ++i) ss += v[i] * v[i];
  ss = warp_sum(ss);
  const float scale = rms_scale_bf16(ss, D, eps);
  float nv[NPL];
#pragma unroll
  for (int i = 0; i < NPL; ++i) nv[i] = rbf(rbf(v[i] * scale) * w[i]);
#pragma unroll
  for (int i = 0; i < HALF; ++i) {
    const int d = lane + 32 * i;
    const float c = cosr[d], sn = sinr[d];
    v[i] = rbf(rbf(nv[i] * c) - rbf(nv[i + HALF] * sn));
    v[i + HALF] = rbf(rbf(nv[i + HALF] * c) + rbf(nv[i] * sn));
  }
}

// Warps 0..G-1 load the q-norm weight and warp G the k-norm weight (a layer constant:
// callers issue this before waiting for the projections).
template <int D, int G>
__device__ __forceinline__ void attn_load_norm_w(const bf16 *qn, const bf16 *kn, float (&wv)[D / 32], int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  if (warp <= G) {
    const bf16 *w = warp == G ? kn : qn;
#pragma unroll
    for (int i = 0; i < D / 32; ++i) wv[i] = bf2f(w[lane + 32 * i]);
  }
}

// Step 1 of a unit: q heads into sm.q_s; when `holds_new`, the new k/v into sm.knew/vnew
// and appended to the cache at the row's position.
// With flagged input (p.qkv_ll) the projections are polled until they carry p.qkv_flag;
// returns false on every team thread when such a wait gave up (code 64 recorded).
// Bounded poll of the flagged words holding elements a + 32 i and, when b >= 0, b + 32 i
// (i < N) until all carry `flag`: every pass issues all 2N loads before checking any.
template <int N>
__device__ __forceinline__ bool ll_wait_lane_words(const uint2 *words, int a, int b, uint32_t flag,
                                                   uint32_t (&da)[N], uint32_t (&db)[N], const int *error,
                                                   long long limit) {
  for (long long it = 0;; ++it) {
    // Every load of the pass is issued before any flag is compared.
    uint2 wa[N], wb[N];
#pragma unroll
    for (int i = 0; i < N; ++i) wa[i] = ll_load1(words + ((a + 32 * i) >> 1));
    if (b >= 0) {
#pragma unroll
      for (int i = 0; i < N; ++i) wb[i] = ll_load1(words + ((b + 32 * i) >> 1));
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) wb[i] = make_uint2(0u, flag);
    }
    uint32_t ok = 1u;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      da[i] = wa[i].x;
      db[i] = wb[i].x;
      ok &= uint32_t(wa[i].y == flag) & uint32_t(wb[i].y == flag);
    }
    if (ok) return true;
    if (it >= limit) return false;
    if ((it & 255) == 255 && error && ll_error_word(error) != 0) return false;
    if (it >= 8) __nanosleep(32);
  }
}

template <int D, int G>
__device__ bool attn_qk(const DecodeAttnParams &p, AttnTeamSmem<D, G> &sm, const AttnRow<D> &rs, int row, int kvh,
                        bool holds_new, const float (&wv)[D / 32], int tid, int bar_id) {
  static_assert(G < kAttnThreads / 32, "one warp per q head plus one for the new k");
  constexpr int NPL = D / 32;
  const AttnGeom &g = p.g;
  const int warp = tid >> 5, lane = tid & 31;
  bool ok = true;
  if (warp < G || (warp == G && holds_new)) {
    const bool is_k = warp == G;
    const int rw = g.qdim + 2 * g.kvdim;
    const int e0 = is_k ? g.qdim + kvh * D : (kvh * G + warp) * D, ev = g.qdim + g.kvdim + kvh * D;
    // Elements e0 + lane + 32 i (and, for the k warp, the v elements ev + lane + 32 i) of the
    // row's projections: plain, or half (e & 1) of flagged word e / 2, all of a lane's
    // words polled together (one round trip once they are written).
    float hv[NPL], vv[NPL];
    if (!p.qkv_ll) {
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        hv[i] = bf2f(__ldcg(p.qkv + size_t(row) * rw + e0 + lane + 32 * i));
        vv[i] = is_k ? bf2f(__ldcg(p.qkv + size_t(row) * rw + ev + lane + 32 * i)) : 0.f;
      }
    } else {
      const uint2 *words = p.qkv_ll + size_t(row) * p.qkv_ll_stride;
      uint32_t wq[NPL], wv2[NPL];
      ok = ll_wait_lane_words<NPL>(words, e0 + lane, is_k ? ev + lane : -1, p.qkv_flag, wq, wv2, p.error,
                                   p.ll_limit);
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        const int e = e0 + lane + 32 * i;  // 32 i is even: every element of a lane has e's parity
        hv[i] = (e & 1) ? bf_hi(wq[i]) : bf_lo(wq[i]);
        vv[i] = (e & 1) ? bf_hi(wv2[i]) : bf_lo(wv2[i]);
      }
    }
    norm_rope_regs<D>(hv, wv, rs.cosr, rs.sinr, g.eps, lane);
    if (!is_k) {
#pragma unroll
      for (int i = 0; i < NPL; ++i) sm.q_b[warp][lane + 32 * i] = f2bf(hv[i]);
    } else {
      bf16 *kd = kv_row_ptr<D>(p, rs, row, p.layer, 0, kvh, rs.pos);
      bf16 *vd = kv_row_ptr<D>(p, rs, row, p.layer, 1, kvh, rs.pos);
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        const bf16 kb = f2bf(hv[i]), vb = f2bf(vv[i]);
        kd[lane + 32 * i] = kb;
        vd[lane + 32 * i] = vb;
        sm.knew[lane + 32 * i] = kb;
        sm.vnew[lane + 32 * i] = vb;
      }
    }
  }
  if (!p.qkv_ll) {
    team_sync(bar_id);
    return true;
  }
  int all_ok;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.s32 %0, 1, 0, q;\n}"
      : "=r"(all_ok)
      : "r"(int(ok)), "r"(bar_id), "n"(kAttnThreads)
      : "memory");
  if (!all_ok && tid == 0 && p.error) atomicOr(p.error, 64);
  return all_ok != 0;
}

// The final state of one unit for thread tid < G x D: output tid (q head tid / D, dim
// tid % D) as the running max, exp-sum and unnormalized output.
template <int D>
struct AttnAcc {
  float m, l, o;
};

// Chunk streaming: warp w owns positions [8w, 8w + 8) of every 64-position chunk and keeps
// its own online-softmax state, so a chunk needs no barrier among the warps. Lane l works
// on position p = l / 4 of the warp's eight for scores (part l % 4 of the D dims, reduced
// by two shuffles), and on dims [l * D/32, +D/32) for P.V; the warps' states are combined
// once per unit (attn_combine).
template <int D, int G>
struct AttnWarpAcc {
  float m[G], l[G];     // running max and exp-sum of the warp's positions (same on every lane)
  float o[G][D / 32];   // this lane's output dims, unnormalized
};
template <int D, int G>
__device__ __forceinline__ void attn_warp_init(AttnWarpAcc<D, G> &a) {
#pragma unroll
  for (int h = 0; h < G; ++h) {
    a.m[h] = -INFINITY;
    a.l[h] = 0.f;
#pragma unroll
    for (int k = 0; k < D / 32; ++k) a.o[h][k] = 0.f;
  }
}

// 16-byte chunk j of the part (D/4 dims) that lane `lane` reads of a K row, in a rotated
// order: the eight lanes of one shared-memory phase (two positions x four parts) then hit
// eight distinct bank groups (rows are D x 2 bytes, a multiple of 128).
template <int D>
__device__ __forceinline__ int attn_kchunk(int lane, int j) {
  constexpr int CPP = D / 32;  // 16-byte chunks per part
  const int p = lane >> 2, part = lane & 3;
  const int rot = CPP == 4 ? 2 * (p & 1) + (part >> 1) : (p & 1);
  return part * CPP + ((j + rot) & (CPP - 1));
}

// One chunk for this warp: positions [8w, 8w + 8) of rows [0, n_main) of Ks/Vs (shared
// memory, row pitch D) and, when `extra`, the new position (knew/vnew) as row n_main.
// FP32 scores (mixed-precision BF16 FMAs), the warp's running max/sum/output rescaled by
// exp(m_old - m_new); only this warp's rows are read.
// q comes from shared memory (q_b, after attn_qk) chunk by chunk in the same rotated order
// as the K loads (conflict-free too), which keeps 32 registers free in the caller.
template <int D, int G>
__device__ __forceinline__ void attn_chunk(const bf16 (&q_b)[G][D], const bf16 *knew, const bf16 *vnew,
                                           const bf16 *Ks, const bf16 *Vs, int n_main, bool extra, float scale,
                                           AttnWarpAcc<D, G> &acc, int tid) {
  constexpr int CPP = D / 32, DL = D / 32;
  const int lane = tid & 31, warp = tid >> 5;
  const int n = n_main + (extra ? 1 : 0);
  const int i = warp * 8 + (lane >> 2);
  const bool valid = i < n;
  float sc[G];
  {
    float lo[G], hi[G];
#pragma unroll
    for (int h = 0; h < G; ++h) lo[h] = hi[h] = 0.f;
    if (valid) {
      const bf16 *kr = i < n_main ? Ks + size_t(i) * D : knew;
#pragma unroll
      for (int j = 0; j < CPP; ++j) {
        const int c = attn_kchunk<D>(lane, j);
        const uint4 k8 = *reinterpret_cast<const uint4 *>(kr + c * 8);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const uint4 q8 = *reinterpret_cast<const uint4 *>(&q_b[h][c * 8]);
          fma_bf16x2(lo[h], hi[h], q8.x, k8.x);
          fma_bf16x2(lo[h], hi[h], q8.y, k8.y);
          fma_bf16x2(lo[h], hi[h], q8.z, k8.z);
          fma_bf16x2(lo[h], hi[h], q8.w, k8.w);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float d = lo[h] + hi[h];
      d += __shfl_xor_sync(0xFFFFFFFFu, d, 1);
      d += __shfl_xor_sync(0xFFFFFFFFu, d, 2);
      sc[h] = valid ? d * scale : -INFINITY;
    }
  }
  float pv[G], alpha[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float mc = sc[h];
    mc = fmaxf(mc, __shfl_xor_sync(0xFFFFFFFFu, mc, 4));
    mc = fmaxf(mc, __shfl_xor_sync(0xFFFFFFFFu, mc, 8));
    mc = fmaxf(mc, __shfl_xor_sync(0xFFFFFFFFu, mc, 16));
    const float mn = fmaxf(acc.m[h], mc);
    // mn is -inf only while the warp has seen no position at all (then nothing changes).
    alpha[h] = mn == -INFINITY ? 1.f : expf(acc.m[h] - mn);
    pv[h] = valid ? expf(sc[h] - mn) : 0.f;
    float ps = pv[h];
    ps += __shfl_xor_sync(0xFFFFFFFFu, ps, 4);
    ps += __shfl_xor_sync(0xFFFFFFFFu, ps, 8);
    ps += __shfl_xor_sync(0xFFFFFFFFu, ps, 16);
    acc.l[h] = acc.l[h] * alpha[h] + ps;
    acc.m[h] = mn;
#pragma unroll
    for (int k = 0; k < DL; ++k) acc.o[h][k] *= alpha[h];
  }
  const int nw = min(8, n - warp * 8);  // the warp's valid rows (uniform across the warp)
#pragma unroll
  for (int pp = 0; pp < 8; ++pp) {
    float w[G];
#pragma unroll
    for (int h = 0; h < G; ++h) w[h] = __shfl_sync(0xFFFFFFFFu, pv[h], pp * 4);
    if (pp < nw) {
      const int r = warp * 8 + pp;
      const bf16 *vr = (r < n_main ? Vs + size_t(r) * D : vnew) + lane * DL;
      float v[DL];
      if constexpr (DL == 4) {
        const uint2 v4 = *reinterpret_cast<const uint2 *>(vr);
        v[0] = bf_lo(v4.x), v[1] = bf_hi(v4.x), v[2] = bf_lo(v4.y), v[3] = bf_hi(v4.y);
      } else {
        const uint32_t v2 = *reinterpret_cast<const uint32_t *>(vr);
        v[0] = bf_lo(v2), v[1] = bf_hi(v2);
      }
#pragma unroll
      for (int h = 0; h < G; ++h)
#pragma unroll
        for (int k = 0; k < DL; ++k) acc.o[h][k] = fmaf(w[h], v[k], acc.o[h][k]);
    }
  }
}

// Combine the eight warps' states (in warp order) into the unit's (max, sum, output) for
// thread tid < G x D. Ends with a barrier; sm.pvp is the exchange space.
template <int D, int G>
__device__ __forceinline__ AttnAcc<D> attn_combine(AttnTeamSmem<D, G> &sm, const AttnWarpAcc<D, G> &acc, int tid,
                                                   int bar_id) {
  constexpr int DL = D / 32, NW = kAttnThreads / 32;
  static_assert(sizeof(sm.pvp) >= sizeof(float) * NW * G * D, "combine space");
  const int lane = tid & 31, warp = tid >> 5;
  float *wo = &sm.pvp[0][0];  // [warp][G][D]
#pragma unroll
  for (int h = 0; h < G; ++h) {
#pragma unroll
    for (int k = 0; k < DL; ++k) wo[(warp * G + h) * D + lane * DL + k] = acc.o[h][k];
    if (lane == 0) {
      sm.wml[warp][h][0] = acc.m[h];
      sm.wml[warp][h][1] = acc.l[h];
    }
  }
  team_sync(bar_id);
  // The weight exp(m_w - M) of warp w's state for head h, computed once (thread h x NW + w)
  // instead of by each of the head's D threads.
  if (tid < G * NW) {
    const int h = tid / NW, w = tid % NW;
    float M = -INFINITY;
#pragma unroll
    for (int v = 0; v < NW; ++v) M = fmaxf(M, sm.wml[v][h][0]);
    const float mw = sm.wml[w][h][0];
    sm.wc[w][h] = (M == -INFINITY || mw == -INFINITY) ? -1.f : expf(mw - M);
  }
  team_sync(bar_id);
  AttnAcc<D> r{-INFINITY, 0.f, 0.f};
  if (tid < G * D) {
    const int h = tid / D, d = tid % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sm.wml[w][h][0]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float c = sm.wc[w][h];
        if (c < 0.f) continue;
        L += sm.wml[w][h][1] * c;
        O += wo[(w * G + h) * D + d] * c;
      }
    }
    r.m = M, r.l = L, r.o = O;
  }
  team_sync(bar_id);
  return r;
}

constexpr int kMergeBatch = 16;  // splits whose partials one merge round trip reads

// Fold a batch of split partials (m, l, o; m = -inf: absent) into the running (M, L, O) of
// one output, in split order: rescale the running state to the batch's max, then add each
// split's exp-weighted l and o. Every merge path uses this, so their bits agree.
template <int MB>
__device__ __forceinline__ void merge_fold(float &M, float &Ls, float &O, const float (&mv)[MB], const float (&lv)[MB],
                                           const float (&ov)[MB]) {
  float Mb = M;
#pragma unroll
  for (int j = 0; j < MB; ++j) Mb = fmaxf(Mb, mv[j]);
  if (Mb == -INFINITY) return;
  const float r = M == -INFINITY ? 0.f : expf(M - Mb);
  Ls *= r;
  O *= r;
#pragma unroll
  for (int j = 0; j < MB; ++j) {
    if (mv[j] == -INFINITY) continue;
    const float c = expf(mv[j] - Mb);
    Ls += lv[j] * c;
    O += ov[j] * c;
  }
  M = Mb;
}

// Store the BF16 output v of head (kvh * G + hd), dim d of `row` (thread t < G x D owns
// t = hd * D + d; whole warps take part: adjacent dims pair up in one flagged word).
template <int D, int G>
__device__ __forceinline__ void attn_out_store(const DecodeAttnParams &p, int row, int kvh, int hd, int d, bf16 v) {
  if (p.out_ll) {
    const bf16 v1 =
        __ushort_as_bfloat16((unsigned short)__shfl_down_sync(0xFFFFFFFFu, (unsigned)__bfloat16_as_ushort(v), 1));
    if ((d & 1) == 0)
      ll_store_all(p.out_ll + size_t(row) * p.out_ll_stride + (((kvh * G + hd) * D + d) >> 1), pack_bf16x2(v, v1),
                   p.out_flag, p.out_ndst, p.out_dst);
  } else {
    bf16 *o = p.out + size_t(row) * p.out_stride + (kvh * G + hd) * D + d;
    *o = v;
    for (int i = 0; i < p.out_ndst; ++i) *reinterpret_cast<bf16 *>(reinterpret_cast<char *>(o) + p.out_dst[i]) = v;
  }
}

// Merge the n_active split partials of the G heads of (row, kv_head) into the BF16 head
// outputs. Thread t < G x D owns output t (head t / D, dim t % D) and reads that dim plus
// (m, l) of up to kMergeBatch splits in one round trip; batches fold into the running
// (M, L, O) in split order (merge_fold). The merging unit resets the arrival counter.
template <int D, int G>
__device__ void attn_merge(const DecodeAttnParams &p, const float *part_base, int kvh, int row, int n_active,
                           int tid) {
  constexpr int MB = kMergeBatch;
  if (tid < G * D) {
    const int hd = tid / D, d = tid % D;
    const float *pr0 = part_base + size_t(kvh * G + hd) * p.max_splits * (D + 2);
    float M = -INFINITY, Ls = 0.f, O = 0.f;
    for (int s0 = 0; s0 < n_active; s0 += MB) {
      float mv[MB], lv[MB], ov[MB];
#pragma unroll
      for (int j = 0; j < MB; ++j) {
        mv[j] = -INFINITY;
        lv[j] = ov[j] = 0.f;
        if (s0 + j < n_active) {
          const float *pr = pr0 + size_t(s0 + j) * (D + 2);
          mv[j] = __ldcg(pr);
          lv[j] = __ldcg(pr + 1);
          ov[j] = __ldcg(pr + 2 + d);
        }
      }
      merge_fold<MB>(M, Ls, O, mv, lv, ov);
    }
    attn_out_store<D, G>(p, row, kvh, hd, d, f2bf(O * (1.0f / Ls)));
  }
  if (tid == 0) p.count[row * p.g.kv_heads + kvh] = 0;
}

// Flagged partials (p.part_ll): this unit's combined state as words of its split's slot.
template <int D, int G>
__device__ __forceinline__ void attn_partial_ll(const DecodeAttnParams &p, const AttnAcc<D> &acc, int row, int kvh,
                                                int split, int tid) {
  if (tid < G * D) {
    const int hd = tid / D, d = tid % D;
    uint2 *pr = p.part_ll + ((size_t(row) * p.g.heads + kvh * G + hd) * p.max_splits + split) * (D + 2);
    ll_store(pr + 2 + d, __float_as_uint(acc.o), p.part_flag);
    if (d == 0) {
      ll_store(pr, __float_as_uint(acc.m), p.part_flag);
      ll_store(pr + 1, __float_as_uint(acc.l), p.part_flag);
    }
  }
}

// A row whose context is one split: its unit's state is the head output (the merge of a
// single partial computes the same bits: exp(0) = 1).
template <int D, int G>
__device__ __forceinline__ void attn_single_out(const DecodeAttnParams &p, const AttnAcc<D> &acc, int row, int kvh,
                                                int tid) {
  if (tid < G * D) {
    float M = -INFINITY, Ls = 0.f, O = 0.f;
    const float mv[1] = {acc.m}, lv[1] = {acc.l}, ov[1] = {acc.o};
    merge_fold<1>(M, Ls, O, mv, lv, ov);
    attn_out_store<D, G>(p, row, kvh, tid / D, tid % D, f2bf(O * (1.0f / Ls)));
  }
}

// Merge job of (row, kv_head) over flagged partials: every batch of kMergeBatch splits is
// polled (bounded; each pass issues all its loads first, and a warp leaves the poll when
// all its lanes' words carry p.part_flag), then folded as attn_merge does. Lane L loads
// (m, l) of split s0 + L % kMergeBatch and every lane the o of its own dim for each split;
// (m, l) reach the other lanes by shuffles. False (nothing stored, error 64 recorded)
// when a wait gave up. `st` (tracing, optional): SM clocks when the first batch was
// complete (slot 3), when all were folded (slot 4) and when the outputs were stored (slot 5).
template <int D, int G>
__device__ bool attn_merge_ll(const DecodeAttnParams &p, int row, int kvh, int n_splits, int tid,
                              unsigned long long *st = nullptr) {
  constexpr int MB = kMergeBatch;
  static_assert(MB <= 32 && G * D % 32 == 0, "one (m, l) per lane; whole warps");
  bool ok = true;
  if (tid < G * D) {
    const int hd = tid / D, d = tid % D, lane = tid & 31;
    const uint2 *pr0 = p.part_ll + (size_t(row) * p.g.heads + kvh * G + hd) * p.max_splits * (D + 2);
    float M = -INFINITY, Ls = 0.f, O = 0.f;
    for (int s0 = 0; s0 < n_splits && ok; s0 += MB) {
      uint2 wm, wl, wo[MB];
      for (long long it = 0;; ++it) {
        const uint2 *prm = pr0 + size_t(min(s0 + lane % MB, n_splits - 1)) * (D + 2);  // past the end: a repeat
        wm = ll_load1(prm);
        wl = ll_load1(prm + 1);
#pragma unroll
        for (int j = 0; j < MB; ++j) wo[j] = ll_load1(pr0 + size_t(min(s0 + j, n_splits - 1)) * (D + 2) + 2 + d);
        uint32_t mine = uint32_t(wm.y == p.part_flag) & uint32_t(wl.y == p.part_flag);
#pragma unroll
        for (int j = 0; j < MB; ++j) mine &= uint32_t(wo[j].y == p.part_flag);
        if (__all_sync(0xFFFFFFFFu, mine != 0u)) break;
        if (it >= p.ll_limit ||
            ((it & 255) == 255 && p.error && __any_sync(0xFFFFFFFFu, ll_error_word(p.error) != 0))) {
          ok = false;
          break;
        }
        if (it >= 8) __nanosleep(32);
      }
      if (s0 == 0) attn_stamp(st, 3, tid);
      if (!ok) break;
      // merge_fold's arithmetic with each split's weight computed once, on its lane, and
      // shuffled (the same expf of the same operands, folded in the same order, so the
      // bits equal merge_fold's): the batch max by a butterfly (max is exact in any order),
      // the rescale of the running state, then split by split in order.
      const int jl = lane % MB;
      const float m_l = s0 + jl < n_splits ? __uint_as_float(wm.x) : -INFINITY;
      float Mb = fmaxf(M, m_l);
#pragma unroll
      for (int off = 1; off < MB; off <<= 1) Mb = fmaxf(Mb, __shfl_xor_sync(0xFFFFFFFFu, Mb, off));
      if (Mb != -INFINITY) {
        const float r = M == -INFINITY ? 0.f : expf(M - Mb);
        Ls *= r;
        O *= r;
        const float c_l = m_l == -INFINITY ? -1.f : expf(m_l - Mb);  // -1: no split (skipped)
        const float l_l = __uint_as_float(wl.x);
#pragma unroll
        for (int j = 0; j < MB; ++j) {
          const float c = __shfl_sync(0xFFFFFFFFu, c_l, j), l = __shfl_sync(0xFFFFFFFFu, l_l, j);
          if (c < 0.f) continue;
          Ls += l * c;
          O += __uint_as_float(wo[j].x) * c;
        }
        M = Mb;
      }
    }
    attn_stamp(st, 4, tid);
    // The pairing store needs the whole warp (ok is warp-uniform here).
    if (ok) attn_out_store<D, G>(p, row, kvh, hd, d, f2bf(O * (1.0f / Ls)));
    attn_stamp(st, 5, tid);
  }
  if (!ok && tid % 32 == 0 && p.error) atomicOr(p.error, 64);
  return ok;
}

// Flagged output of an inactive row: the G heads of kv head `kvh` as zero words with the
// step's flag, so the consumers of every row's words never wait on a row without work.
template <int D, int G>
__device__ void attn_write_inactive(const DecodeAttnParams &p, int row, int kvh, int tid) {
  for (int w = tid; w < G * D / 2; w += kAttnThreads)
    ll_store_all(p.out_ll + size_t(row) * p.out_ll_stride + ((kvh * G * D) >> 1) + w, 0u, p.out_flag, p.out_ndst,
                 p.out_dst);
}

// Step 3: store this unit's partial, count its arrival, and merge when it is the last of
// the row's n_splits units for this kv head. Returns true when it merged.
template <int D, int G>
__device__ bool attn_finish(const DecodeAttnParams &p, AttnTeamSmem<D, G> &sm, const AttnAcc<D> &acc, int row,
                            int kvh, int split, int n_splits, int tid, int bar_id) {
  const int hd = tid / D, d = tid % D;
  float *part_base = p.part + (size_t(row) * p.g.heads) * p.max_splits * (D + 2);
  if (tid < G * D) {
    float *pr = part_base + (size_t(kvh * G + hd) * p.max_splits + split) * (D + 2);
    pr[2 + d] = acc.o;
    if (d == 0) {
      pr[0] = acc.m;
      pr[1] = acc.l;
    }
  }
  // The team barrier orders the team's partial before thread 0's acq_rel add, which also
  // makes the other units' partials visible to the last arriver (then shared by a barrier).
  team_sync(bar_id);
  if (tid == 0) {
    int prev;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                 : "=r"(prev)
                 : "l"(p.count + row * p.g.kv_heads + kvh)
                 : "memory");
    sm.last_flag = prev == n_splits - 1;
  }
  team_sync(bar_id);
  if (!sm.last_flag) return false;
  attn_merge<D, G>(p, part_base, kvh, row, n_splits, tid);
  return true;
}

}  // namespace yar
