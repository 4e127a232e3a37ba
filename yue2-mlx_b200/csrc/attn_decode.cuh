// attn_decode.cuh — the split-KV GQA decode attention unit, shared by the standalone
// kernel (k_attn_decode) and the persistent decode kernel, so both produce the same bits.
//
// A unit = (row, kv head, split) processed by a team of 128 threads (4 warps): q-norm +
// RoPE of the group's q heads, the new k (norm + RoPE) and v appended to the paged cache
// by the unit whose range holds the new position, FP32 scores/softmax/P.V over the
// split's positions, a partial (max, sum, o[D]) per q head, and — for the last unit of
// (row, kv head) to arrive — the merge of all splits into the BF16 head outputs
// (native/src/ar.cpp:88-96, :276-291; oracle/port/lyra/ar.py:131-145).
#pragma once
#include "common.cuh"

namespace yar {

struct AttnGeom {
  int heads, kv_heads, head_dim, qdim, kvdim, page_tokens, pages_per_row, num_pages;
  size_t page_elems;  // kv_heads * P * D
  float eps, scale;
};

// Address of (layer, kv, kv_head, position) for a row's page table.
__device__ __forceinline__ bf16 *kv_addr(bf16 *pool, const AttnGeom &g, const int *ptab, int layer,
                                         int kv, int head, int pos) {
  const int page = ptab[pos / g.page_tokens], slot = pos % g.page_tokens;
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

template <int D>
__device__ __forceinline__ void norm_rope_head_s(float *v, const float *w, const float *cosr, const float *sinr, float eps,
                                 int lane) {
  float ss = 0.f;
  for (int d = lane; d < D; d += 32) ss += v[d] * v[d];
  ss = warp_sum(ss);
  const float scale = rms_scale_bf16(ss, D, eps);
  float nv[D / 32];
#pragma unroll
  for (int i = 0; i < D / 32; ++i) {
    const int d = lane + 32 * i;
    nv[i] = rbf(rbf(v[d] * scale) * w[d]);
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
    if (d < H)
      out[i] = rbf(rbf(v[d] * cosr[d]) - rbf(v[d + H] * sinr[d]));
    else
      out[i] = rbf(rbf(v[d] * cosr[d - H]) + rbf(v[d - H] * sinr[d - H]));
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < D / 32; ++i) v[lane + 32 * i] = out[i];
  __syncwarp();
}

constexpr int kAttnThreads = 128;

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
  bf16 *out;     // [rows][qdim]
};

template <int D, int G>
struct AttnSmem {
  static constexpr int NW = kAttnThreads / 32, LPP = D / 8, PPW = 32 / LPP, MS = 64;
  float q_s[G][D];
  float knew[D], vnew[D];
  float m_s[NW][PPW][G], l_s[NW][PPW][G];
  float o_s[NW * PPW][G][D];
  float wsplit[G][MS];
  float inv_l[G];
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

// The split geometry every unit of a row computes identically.
struct SplitRange {
  int chunk, n_active, p0, p1;
};
__device__ __forceinline__ SplitRange split_range(int L, int max_splits, int split) {
  SplitRange r;
  r.chunk = (L + max_splits - 1) / max_splits;
  r.chunk = max(64, (r.chunk + 15) & ~15);
  r.n_active = (L + r.chunk - 1) / r.chunk;
  r.p0 = split * r.chunk;
  r.p1 = min(L, r.p0 + r.chunk);
  return r;
}

template <int D>
__device__ __forceinline__ bf16 *kv_row_ptr(const DecodeAttnParams &p, const AttnRow<D> &rs, int row, int layer,
                                           int kv, int kvh, int q) {
  const AttnGeom &g = p.g;
  const int lp = q / g.page_tokens;
  const int page = lp < AttnRow<D>::kMaxPages ? rs.ptab[lp] : p.page_table[size_t(row) * g.pages_per_row + lp];
  const size_t blk = (size_t(layer) * g.num_pages + page) * 2 + kv;
  return p.pool + blk * g.page_elems + (size_t(kvh) * g.page_tokens + q % g.page_tokens) * D;
}

// Ask L2 to fetch the cached K/V lines a unit will read (positions before the new one),
// so the unit's loads hit L2 instead of queueing behind the weight stream.
template <int D>
__device__ void attn_prefetch_kv(const DecodeAttnParams &p, const AttnRow<D> &rs, int row, int layer, int kvh,
                                 int split, int tid, int nthreads) {
  if (!rs.active) return;
  const SplitRange r = split_range(rs.pos + 1, p.max_splits, split);
  if (split >= r.n_active) return;
  const int pend = min(r.p1, rs.pos);
  constexpr int LINES = D * 2 / 128;  // 128-byte lines per position and tensor
  for (int i = tid; i < (pend - r.p0) * 2 * LINES; i += nthreads) {
    const int q = r.p0 + i / (2 * LINES), kv = (i / LINES) & 1, ln = i % LINES;
    const char *a = reinterpret_cast<const char *>(kv_row_ptr<D>(p, rs, row, layer, kv, kvh, q)) + ln * 128;
    asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
  }
}

__device__ __forceinline__ void team_sync(int bar_id) {
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "n"(kAttnThreads) : "memory");
}

// Merge the n_active split partials of the G heads of (row, kv_head): per-split weights
// exp(m_s - M) are formed once in shared memory, then every output dim sums its splits
// with independent (pipelined) L2 loads. The last unit to arrive resets the counter.
template <int D, int G>
__device__ void attn_merge(const DecodeAttnParams &p, AttnSmem<D, G> &sm, const float *part_base, int kvh, int row,
                           int n_active, int tid, int bar_id) {
  constexpr int MS = AttnSmem<D, G>::MS;
  const int lane = tid & 31, warp = tid >> 5;
  for (int h = warp; h < G; h += kAttnThreads / 32) {
    const float *pr0 = part_base + size_t(kvh * G + h) * p.max_splits * (D + 2);
    float mv[MS / 32], lv[MS / 32];
    float M = -INFINITY;
#pragma unroll
    for (int i = 0; i < MS / 32; ++i) {
      const int s = lane + 32 * i;
      mv[i] = s < n_active ? __ldcg(pr0 + s * (D + 2)) : -INFINITY;
      lv[i] = s < n_active ? __ldcg(pr0 + s * (D + 2) + 1) : 0.f;
      M = fmaxf(M, mv[i]);
    }
    M = warp_max(M);
    float Ls = 0.f;
#pragma unroll
    for (int i = 0; i < MS / 32; ++i) {
      const float c = mv[i] == -INFINITY ? 0.f : expf(mv[i] - M);
      sm.wsplit[h][lane + 32 * i] = c;
      Ls += lv[i] * c;
    }
    Ls = warp_sum(Ls);
    if (lane == 0) sm.inv_l[h] = 1.0f / Ls;
  }
  team_sync(bar_id);
  for (int idx = tid; idx < G * D; idx += kAttnThreads) {
    const int h = idx / D, d = idx % D;
    const float *pr0 = part_base + size_t(kvh * G + h) * p.max_splits * (D + 2) + 2 + d;
    float O = 0.f;
#pragma unroll 8
    for (int s = 0; s < n_active; ++s) O += __ldcg(pr0 + s * (D + 2)) * sm.wsplit[h][s];
    p.out[size_t(row) * p.g.qdim + (kvh * G + h) * D + d] = f2bf(O * sm.inv_l[h]);
  }
  if (tid == 0) p.count[row * p.g.kv_heads + kvh] = 0;
}

// q/k RMSNorm (modeling_yue2.py:185) then half-split RoPE (:152-156) of one head held
// in registers, lane l owning dims l, l+32, ...: the RoPE pairs (d, d + D/2) are in the
// same lane. Same arithmetic and order as norm_rope_head_s.
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

__device__ __forceinline__ void attn_stamp(unsigned long long *st, int k, int tid) {
  if (st && tid == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    st[k] = t;
  }
}

// One unit. Returns true when this unit merged (row, kvh) (its outputs are written).
// Dependent memory round trips: (1) the first K/V round (L2 hits when prefetched)
// together with the raw q/k/v and the q/k norm weights; (2) partial + arrival count;
// (3) for the last of the n_active units, the split partials for the merge.
// `st` (optional) receives globaltimer stamps at the unit's checkpoints (slots 3..6).
template <int D, int G>
__device__ bool attn_unit(const DecodeAttnParams &p, AttnSmem<D, G> &sm, const AttnRow<D> &rs, int row, int kvh,
                          int split, int tid, int bar_id, unsigned long long *st = nullptr) {
  using S = AttnSmem<D, G>;
  constexpr int LPP = S::LPP, PPW = S::PPW, NW = S::NW, NPL = D / 32;
  static_assert(G < NW, "one warp per q head plus one for the new k");
  constexpr int UN = 8;  // positions per lane group per round
  const AttnGeom &g = p.g;
  const int lane = tid & 31, warp = tid >> 5;
  const int grp = lane / LPP, sub = lane % LPP;

  if (!rs.active) return false;
  const int pos = rs.pos;
  const SplitRange sr = split_range(pos + 1, p.max_splits, split);
  const int n_active = sr.n_active;
  if (split >= n_active) return false;  // beyond the context: no work, no arrival
  const int p0 = sr.p0, p1 = sr.p1;
  const bool holds_new = p0 <= pos && pos < p1;
  float *part_base = p.part + (size_t(row) * g.heads) * p.max_splits * (D + 2);
  auto kv_ptr = [&](int kv, int q) { return kv_row_ptr<D>(p, rs, row, p.layer, kv, kvh, q); };
  // (1) First K/V round, raw q (and new k, v) and the norm weights.
  const int pend = holds_new ? pos : p1;
  uint4 kr[UN], vr[UN];
  int pp[UN];
  auto load_round = [&](int base) {
#pragma unroll
    for (int u = 0; u < UN; ++u) {
      const int q = base + u * NW * PPW + grp;
      pp[u] = q < pend ? q : -1;
      if (pp[u] >= 0) {
        kr[u] = ldg16(kv_ptr(0, q) + sub * 8);
        vr[u] = ldg16(kv_ptr(1, q) + sub * 8);
      } else {
        kr[u] = make_uint4(0, 0, 0, 0);
        vr[u] = kr[u];
      }
    }
  };
  int base = p0 + warp * PPW;
  load_round(base);
  const bf16 *qkv = p.qkv + size_t(row) * (g.qdim + 2 * g.kvdim);
  const int my_head = warp;  // warps 0..G-1: q heads; warp G: the new k (when held)
  const bool does_head = my_head < G || (my_head == G && holds_new);
  if (does_head) {
    const bool is_k = my_head == G;
    const bf16 *src = is_k ? qkv + g.qdim + kvh * D : qkv + (kvh * G + my_head) * D;
    const bf16 *wn = is_k ? p.kn : p.qn;
    float hv[NPL], vv[NPL], wv[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      hv[i] = bf2f(__ldcg(src + lane + 32 * i));
      wv[i] = bf2f(wn[lane + 32 * i]);
      if (is_k) vv[i] = bf2f(__ldcg(qkv + g.qdim + g.kvdim + kvh * D + lane + 32 * i));
    }
    norm_rope_regs<D>(hv, wv, rs.cosr, rs.sinr, g.eps, lane);
    float *dst = is_k ? sm.knew : sm.q_s[my_head];
#pragma unroll
    for (int i = 0; i < NPL; ++i) dst[lane + 32 * i] = hv[i];
    if (is_k) {
      bf16 *kd = kv_ptr(0, pos), *vd = kv_ptr(1, pos);
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        sm.vnew[lane + 32 * i] = vv[i];
        kd[lane + 32 * i] = f2bf(hv[i]);
        vd[lane + 32 * i] = f2bf(vv[i]);
      }
    }
  }
  team_sync(bar_id);
  attn_stamp(st, 3, tid);

  // Per-lane state: its group's running max/sum per q head and 8 output dims.
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[h][j] = 0.f;
  }
  float qreg[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int j = 0; j < 8; ++j) qreg[h][j] = sm.q_s[h][sub * 8 + j];

  auto consume = [&](int ppos, const float *kf, const float *vf) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float sc = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) sc = fmaf(qreg[h][j], kf[j], sc);
#pragma unroll
      for (int o = LPP / 2; o > 0; o >>= 1) sc += __shfl_xor_sync(0xFFFFFFFFu, sc, o);
      if (ppos < 0) continue;  // lane group without a position this step
      sc *= g.scale;
      const float mn = fmaxf(m[h], sc);
      const float corr = expf(m[h] - mn), e = expf(sc - mn);
      l[h] = l[h] * corr + e;
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[h][j] = acc[h][j] * corr + e * vf[j];
      m[h] = mn;
    }
  };

  // Cached positions (pos itself, when held here, comes from shared memory).
  while (base < pend) {
#pragma unroll
    for (int u = 0; u < UN; ++u) {
      const float kf[8] = {bf_lo(kr[u].x), bf_hi(kr[u].x), bf_lo(kr[u].y), bf_hi(kr[u].y),
                           bf_lo(kr[u].z), bf_hi(kr[u].z), bf_lo(kr[u].w), bf_hi(kr[u].w)};
      const float vf[8] = {bf_lo(vr[u].x), bf_hi(vr[u].x), bf_lo(vr[u].y), bf_hi(vr[u].y),
                           bf_lo(vr[u].z), bf_hi(vr[u].z), bf_lo(vr[u].w), bf_hi(vr[u].w)};
      consume(pp[u], kf, vf);
    }
    base += NW * PPW * UN;
    if (base < pend) load_round(base);
  }
  if (holds_new && warp == 0) {
    // The new position, processed by lane group 0 of warp 0 (other groups pass -1).
    float kf[8], vf[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      kf[j] = rbf(sm.knew[sub * 8 + j]);
      vf[j] = rbf(sm.vnew[sub * 8 + j]);
    }
    consume(grp == 0 ? pos : -1, kf, vf);
  }

  attn_stamp(st, 4, tid);
  // Merge lane groups and warps of this unit.
  const int slot = warp * PPW + grp;
#pragma unroll
  for (int h = 0; h < G; ++h) {
    if (sub == 0) {
      sm.m_s[warp][grp][h] = m[h];
      sm.l_s[warp][grp][h] = l[h];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) sm.o_s[slot][h][sub * 8 + j] = acc[h][j];
  }
  team_sync(bar_id);
  for (int idx = tid; idx < G * D; idx += kAttnThreads) {
    const int h = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w)
      for (int q = 0; q < PPW; ++q) M = fmaxf(M, sm.m_s[w][q][h]);
    float Ls = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < NW; ++w)
        for (int q = 0; q < PPW; ++q) {
          const float mv = sm.m_s[w][q][h];
          if (mv == -INFINITY) continue;
          const float c = expf(mv - M);
          Ls += sm.l_s[w][q][h] * c;
          O += sm.o_s[w * PPW + q][h][d] * c;
        }
    }
    float *pr = part_base + (size_t(kvh * G + h) * p.max_splits + split) * (D + 2);
    pr[2 + d] = O;
    if (d == 0) {
      pr[0] = M;
      pr[1] = Ls;
    }
  }
  // (3) Arrival: one release fence after the team barrier covers the team's partial.
  team_sync(bar_id);
  if (tid == 0) {
    __threadfence();
    const int prev = atomicAdd(p.count + row * g.kv_heads + kvh, 1);
    sm.last_flag = prev == n_active - 1;
  }
  team_sync(bar_id);
  attn_stamp(st, 5, tid);
  if (!sm.last_flag) return false;
  __threadfence();
  // (4) The last of the n_active units merges them.
  attn_merge<D, G>(p, sm, part_base, kvh, row, n_active, tid, bar_id);
  attn_stamp(st, 6, tid);
  return true;
}

}  // namespace yar
