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
  static constexpr int NW = kAttnThreads / 32, LPP = D / 8, PPW = 32 / LPP, kMaxPages = 128, MS = 64;
  float q_s[G][D];
  float knew[D], vnew[D];
  float m_s[NW][PPW][G], l_s[NW][PPW][G];
  float o_s[NW * PPW][G][D];
  float qn_s[D], kn_s[D];
  int ptab_s[kMaxPages];
  float wsplit[G][MS];
  float inv_l[G];
  int last_flag;
};

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

// One unit. Returns true when this unit merged (row, kvh) (its outputs are written).
template <int D, int G>
__device__ bool attn_unit(const DecodeAttnParams &p, AttnSmem<D, G> &sm, int row, int kvh, int split, int nsplit,
                          int tid, int bar_id) {
  using S = AttnSmem<D, G>;
  constexpr int LPP = S::LPP, PPW = S::PPW, NW = S::NW;
  constexpr int UN = 8;  // positions per lane group per round
  const AttnGeom &g = p.g;
  const int lane = tid & 31, warp = tid >> 5;
  const int grp = lane / LPP, sub = lane % LPP;

  if (!__ldcg(p.active + row)) return false;
  const int *ptab_g = p.page_table + size_t(row) * g.pages_per_row;
  const bool ptab_in_smem = g.pages_per_row <= S::kMaxPages;
  if (ptab_in_smem)
    for (int i = tid; i < g.pages_per_row; i += kAttnThreads) sm.ptab_s[i] = ptab_g[i];
  for (int d = tid; d < D; d += kAttnThreads) {
    sm.qn_s[d] = bf2f(p.qn[d]);
    sm.kn_s[d] = bf2f(p.kn[d]);
  }
  const int pos = __ldcg(p.cur_pos + row);
  const int L = pos + 1;
  int chunk = (L + nsplit - 1) / nsplit;
  chunk = max(64, (chunk + 15) & ~15);
  const int n_active = (L + chunk - 1) / chunk;
  const int p0 = split * chunk, p1 = min(L, p0 + chunk);
  const bool holds_new = p0 <= pos && pos < p1;
  float *part_base = p.part + (size_t(row) * g.heads) * p.max_splits * (D + 2);
  if (split >= n_active) {
    // Beyond the context: nothing to read, and the merge never looks at this split.
    // Only take part in the arrival count.
    team_sync(bar_id);
    if (tid == 0) {
      __threadfence();
      const int prev = atomicAdd(p.count + row * g.kv_heads + kvh, 1);
      sm.last_flag = prev == nsplit - 1;
    }
    team_sync(bar_id);
    if (!sm.last_flag) return false;
    __threadfence();
    attn_merge<D, G>(p, sm, part_base, kvh, row, n_active, tid, bar_id);
    return true;
  }
  team_sync(bar_id);  // page table and norm weights staged
  const int *ptab = ptab_in_smem ? sm.ptab_s : ptab_g;
  auto kv_ptr = [&](int kv, int q) {
    const int page = ptab[q / g.page_tokens], slot = q % g.page_tokens;
    const size_t blk = (size_t(p.layer) * g.num_pages + page) * 2 + kv;
    return p.pool + blk * g.page_elems + (size_t(kvh) * g.page_tokens + slot) * D;
  };
  // Issue the first round of K/V loads now; q-norm and RoPE run while they are in flight.
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
  const float *cosr = p.cos_tab + size_t(pos) * (D / 2);
  const float *sinr = p.sin_tab + size_t(pos) * (D / 2);
  for (int h = warp; h < G + (holds_new ? 1 : 0); h += NW) {
    const bool is_k = h == G;
    const bf16 *src = is_k ? qkv + g.qdim + kvh * D : qkv + (kvh * G + h) * D;
    float *dst = is_k ? sm.knew : sm.q_s[h];
    for (int d = lane; d < D; d += 32) dst[d] = bf2f(__ldcg(src + d));
    __syncwarp();
    norm_rope_head_s<D>(dst, is_k ? sm.kn_s : sm.qn_s, cosr, sinr, g.eps, lane);
  }
  if (holds_new)
    for (int d = tid; d < D; d += kAttnThreads) sm.vnew[d] = bf2f(__ldcg(qkv + g.qdim + g.kvdim + kvh * D + d));
  team_sync(bar_id);
  if (holds_new) {
    bf16 *kd = kv_ptr(0, pos);
    bf16 *vd = kv_ptr(1, pos);
    for (int d = tid; d < D; d += kAttnThreads) {
      kd[d] = f2bf(sm.knew[d]);
      vd[d] = f2bf(sm.vnew[d]);
    }
  }

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
  __threadfence();
  team_sync(bar_id);
  if (tid == 0) {
    const int prev = atomicAdd(p.count + row * g.kv_heads + kvh, 1);
    sm.last_flag = prev == nsplit - 1;
  }
  team_sync(bar_id);
  if (!sm.last_flag) return false;
  __threadfence();
  attn_merge<D, G>(p, sm, part_base, kvh, row, n_active, tid, bar_id);
  return true;
}

}  // namespace yar
