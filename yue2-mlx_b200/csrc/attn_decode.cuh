// attn_decode.cuh — the split-KV GQA decode attention, shared by the standalone kernel
// (k_attn_decode) and the persistent decode kernel, so both produce the same bits.
//
// The cached positions of a row are cut into chunks of 64 (one chunk never straddles a
// page of >= 64 positions, so its K rows and its V rows are each one contiguous 16 KB
// block for head_dim 128). A split is a run of consecutive chunks; a unit = (row, kv head,
// split) is processed by 256 threads (8 warps):
//   1. q-norm + RoPE of the group's G q heads; the unit holding the new position also
//      norms and ropes the new k and appends k, v to the paged cache;
//   2. per chunk (rows staged in shared memory): FP32 scores with 2-4 threads per (head,
//      position), the chunk's max and exp-sum, P.V with one output dim per thread (or a
//      fixed split of the positions when G x D < 256), folded into the running (max, sum,
//      o) with exp rescaling;
//   3. a partial (max, sum, o[D]) per q head; the last of the row's splits to arrive merges
//      them into the BF16 head outputs (native/src/ar.cpp:88-96, :276-291;
//      oracle/port/lyra/ar.py:131-145).
#pragma once
#include "common.cuh"

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
  float p_s[G][kKvChunk];      // exp(score - chunk max)
  float red[2][kAttnThreads / 32];
  float pvp[kAttnThreads / G / (D / 8)][G * D];  // P.V partials per position phase
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
template <int D>
__device__ void attn_row_load(AttnRow<D> &rs, const DecodeAttnParams &p, int row, int tid, int nthreads) {
  const int pos = __ldcg(p.cur_pos + row);
  if (tid == 0) {
    rs.active = __ldcg(p.active + row);
    rs.pos = pos;
  }
  for (int i = tid; i < D / 2; i += nthreads) {
    rs.cosr[i] = p.cos_tab[size_t(pos) * (D / 2) + i];
    rs.sinr[i] = p.sin_tab[size_t(pos) * (D / 2) + i];
  }
  const int n = p.g.pages_per_row < AttnRow<D>::kMaxPages ? p.g.pages_per_row : AttnRow<D>::kMaxPages;
  for (int i = tid; i < n; i += nthreads) rs.ptab[i] = p.page_table[size_t(row) * p.g.pages_per_row + i];
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
template <int D, int G>
__device__ void attn_qk(const DecodeAttnParams &p, AttnTeamSmem<D, G> &sm, const AttnRow<D> &rs, int row, int kvh,
                        bool holds_new, const float (&wv)[D / 32], int tid, int bar_id) {
  static_assert(G < kAttnThreads / 32, "one warp per q head plus one for the new k");
  constexpr int NPL = D / 32;
  const AttnGeom &g = p.g;
  const int warp = tid >> 5, lane = tid & 31;
  if (warp < G || (warp == G && holds_new)) {
    const bool is_k = warp == G;
    const bf16 *qkv = p.qkv + size_t(row) * (g.qdim + 2 * g.kvdim);
    const bf16 *src = is_k ? qkv + g.qdim + kvh * D : qkv + (kvh * G + warp) * D;
    float hv[NPL], vv[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      hv[i] = bf2f(__ldcg(src + lane + 32 * i));
      if (is_k) vv[i] = bf2f(__ldcg(qkv + g.qdim + g.kvdim + kvh * D + lane + 32 * i));
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
  team_sync(bar_id);
}

// Running state of one thread: output tid (q head tid / D, dim tid % D) when tid < G x D.
template <int D>
struct AttnAcc {
  float m, l, o;
};
template <int D>
__device__ __forceinline__ void attn_acc_init(AttnAcc<D> &a) {
  a.m = -INFINITY;
  a.l = 0.f;
  a.o = 0.f;
}

// Step 2, one chunk: rows [0, n_main) of Ks/Vs (shared memory, row pitch D) and, when
// `extra`, the new position (sm.knew/vnew) as row n_main. Ends with a barrier.
//   Scores: the threads of head hd (256 / G of them) form 4-thread groups; part p of a
//   group holds its quarter of q in registers (in the rotated order below) and dots it
//   with that quarter of rows ps, ps + slots, ... (16-byte K loads in an order rotated by
//   row and part, so a quarter-warp never hits one bank group twice); the 4 parts are
//   added by shuffles.
//   P.V: thread (head hd, dim group dg of 8 dims, phase q) sums p_r * V[r][8 dg .. +7]
//   over the rows r = q (mod phases) with 16-byte V loads; the phases are added in order
//   through shared memory, one output per thread.
template <int D, int G>
__device__ void attn_chunk(AttnTeamSmem<D, G> &sm, const bf16 *Ks, const bf16 *Vs, int n_main, bool extra, float scale,
                           AttnAcc<D> &acc, int tid, int bar_id) {
  constexpr int NC = D / 8;                  // 16-byte chunks per row
  constexpr int THD = kAttnThreads / G;      // threads per head
  constexpr int CP = NC / 4;                 // chunks per part
  constexpr int SLOTS = THD / 4;             // position slots per head
  constexpr int PPT = kKvChunk / SLOTS;      // positions per thread
  constexpr int WPH = THD / 32;              // warps per head
  constexpr int NPH = THD / NC;              // P.V position phases
  static_assert(CP >= 1 && (CP & (CP - 1)) == 0 && PPT >= 1 && NPH >= 1, "unsupported attention shape");
  const int lane = tid & 31, warp = tid >> 5;
  const int hd = tid / THD, u = tid % THD, part = u % 4, ps = u / 4;
  const int n = n_main + (extra ? 1 : 0);
  // This part's q chunks in the rotated order of the K loads (the rotation depends on the
  // lane only), BF16 pairs.
  uint4 qr[CP];
#pragma unroll
  for (int j = 0; j < CP; ++j) {
    const int cj = (j + ps * (CP > 1 ? CP / 2 : 1) + (part >> 1)) & (CP - 1);
    qr[j] = *reinterpret_cast<const uint4 *>(&sm.q_b[hd][(part * CP + cj) * 8]);
  }
  float sc[PPT];
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    const int i = ps + k * SLOTS;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    if (i < n) {
      const bf16 *kr = i < n_main ? Ks + size_t(i) * D : sm.knew;
#pragma unroll
      for (int j = 0; j < CP; ++j) {
        const int cj = (j + ps * (CP > 1 ? CP / 2 : 1) + (part >> 1)) & (CP - 1);
        const uint4 k8 = *reinterpret_cast<const uint4 *>(kr + (part * CP + cj) * 8);
        const uint4 q8 = qr[j];
        fma_bf16x2(a0, a1, q8.x, k8.x);
        fma_bf16x2(a2, a3, q8.y, k8.y);
        fma_bf16x2(a0, a1, q8.z, k8.z);
        fma_bf16x2(a2, a3, q8.w, k8.w);
      }
    }
    float dot = (a0 + a1) + (a2 + a3);
    dot += __shfl_xor_sync(0xFFFFFFFFu, dot, 1);
    dot += __shfl_xor_sync(0xFFFFFFFFu, dot, 2);
    sc[k] = i < n ? dot * scale : -INFINITY;
  }
  float mx = sc[0];
#pragma unroll
  for (int k = 1; k < PPT; ++k) mx = fmaxf(mx, sc[k]);
  mx = warp_max(mx);
  if (lane == 0) sm.red[0][warp] = mx;
  team_sync(bar_id);
  float mc = -INFINITY;
#pragma unroll
  for (int w = 0; w < WPH; ++w) mc = fmaxf(mc, sm.red[0][hd * WPH + w]);
  float pt = 0.f;
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    const int i = ps + k * SLOTS;
    const float pe = i < n ? expf(sc[k] - mc) : 0.f;
    if (part == 0) sm.p_s[hd][i] = pe;
    pt += pe;
  }
  const float psum = warp_sum(part == 0 ? pt : 0.f);
  if (lane == 0) sm.red[1][warp] = psum;
  team_sync(bar_id);
  // P.V partials.
  {
    const int dg = u % NC, q = u / NC;
    float o8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = q; r < n; r += NPH) {
      const float pr = sm.p_s[hd][r];
      const uint4 v8 = *reinterpret_cast<const uint4 *>((r < n_main ? Vs + size_t(r) * D : sm.vnew) + dg * 8);
      o8[0] = fmaf(pr, bf_lo(v8.x), o8[0]);
      o8[1] = fmaf(pr, bf_hi(v8.x), o8[1]);
      o8[2] = fmaf(pr, bf_lo(v8.y), o8[2]);
      o8[3] = fmaf(pr, bf_hi(v8.y), o8[3]);
      o8[4] = fmaf(pr, bf_lo(v8.z), o8[4]);
      o8[5] = fmaf(pr, bf_hi(v8.z), o8[5]);
      o8[6] = fmaf(pr, bf_lo(v8.w), o8[6]);
      o8[7] = fmaf(pr, bf_hi(v8.w), o8[7]);
    }
    float *dst = &sm.pvp[q][hd * D + dg * 8];
    *reinterpret_cast<float4 *>(dst) = make_float4(o8[0], o8[1], o8[2], o8[3]);
    *reinterpret_cast<float4 *>(dst + 4) = make_float4(o8[4], o8[5], o8[6], o8[7]);
  }
  team_sync(bar_id);
  if (tid < G * D) {
    const int oh = tid / D;
    float oc = 0.f;
#pragma unroll
    for (int q = 0; q < NPH; ++q) oc += sm.pvp[q][tid];
    float lcv = 0.f, mcv = -INFINITY;
#pragma unroll
    for (int w = 0; w < WPH; ++w) {
      lcv += sm.red[1][oh * WPH + w];
      mcv = fmaxf(mcv, sm.red[0][oh * WPH + w]);
    }
    const float mn = fmaxf(acc.m, mcv);
    const float ca = expf(acc.m - mn), cb = expf(mcv - mn);
    acc.l = acc.l * ca + lcv * cb;
    acc.o = acc.o * ca + oc * cb;
    acc.m = mn;
  }
  team_sync(bar_id);
}

// Merge the n_active split partials of the G heads of (row, kv_head) into the BF16 head
// outputs. Thread t < G x D owns output t (head t / D, dim t % D) and reads that dim plus
// (m, l) of up to 8 splits in one round trip; batches fold into the running (M, L, O)
// with exp rescaling, in split order. The merging unit resets the arrival counter.
template <int D, int G>
__device__ void attn_merge(const DecodeAttnParams &p, const float *part_base, int kvh, int row, int n_active,
                           int tid) {
  constexpr int MB = 8;
  if (tid < G * D) {
    const int hd = tid / D, d = tid % D;
    const float *pr0 = part_base + size_t(kvh * G + hd) * p.max_splits * (D + 2);
    float M = -INFINITY, Ls = 0.f, O = 0.f;
    for (int s0 = 0; s0 < n_active; s0 += MB) {
      float mv[MB], lv[MB], ov[MB];
#pragma unroll
      for (int j = 0; j < MB; ++j) {
        mv[j] = -INFINITY;
        if (s0 + j < n_active) {
          const float *pr = pr0 + size_t(s0 + j) * (D + 2);
          mv[j] = __ldcg(pr);
          lv[j] = __ldcg(pr + 1);
          ov[j] = __ldcg(pr + 2 + d);
        }
      }
      float Mb = M;
#pragma unroll
      for (int j = 0; j < MB; ++j) Mb = fmaxf(Mb, mv[j]);
      if (Mb == -INFINITY) continue;
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
    bf16 *o = p.out + size_t(row) * p.out_stride + (kvh * G + hd) * D + d;
    const bf16 v = f2bf(O * (1.0f / Ls));
    *o = v;
    for (int i = 0; i < p.out_ndst; ++i) *reinterpret_cast<bf16 *>(reinterpret_cast<char *>(o) + p.out_dst[i]) = v;
  }
  if (tid == 0) p.count[row * p.g.kv_heads + kvh] = 0;
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
