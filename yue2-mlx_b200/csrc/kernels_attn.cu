// kernels_attn.cu — q/k RMSNorm + RoPE + paged KV append, split-KV GQA decode attention,
// and causal prefill attention, all with FP32 scores, softmax and P.V accumulation
// (native/src/ar.cpp:88-96, :276-291; oracle/port/lyra/ar.py:131-145 names this "FP32
// attention opmath, BF16 storage outside the operation").
//
// KV pool layout: [layer][page][k|v][kv_head][page_tokens][head_dim] BF16; a row's page
// table maps logical page i (positions i*P .. i*P+P-1) to a physical page. Physical slot
// = RoPE position (modeling_yue2.py:383-393: StaticKVCache writes slot pos).
#include "common.cuh"

namespace yar {

struct AttnGeom {
  int heads, kv_heads, head_dim, qdim, kvdim, page_tokens, pages_per_row, num_pages;
  size_t page_elems;  // kv_heads * P * D
  float eps, scale;
};

static AttnGeom geom(const Model &m, const Session &s) {
  AttnGeom g;
  g.heads = m.d.heads;
  g.kv_heads = m.d.kv_heads;
  g.head_dim = m.d.head_dim;
  g.qdim = m.d.qdim();
  g.kvdim = m.d.kvdim();
  g.page_tokens = s.page_tokens;
  g.pages_per_row = s.pages_per_row;
  g.num_pages = s.num_pages;
  g.page_elems = s.kv_page_elems;
  g.eps = m.d.eps;
  g.scale = float(1.0 / std::sqrt(double(m.d.head_dim)));
  return g;
}

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
__device__ void norm_rope_head(float *v, const bf16 *w, const float *cosr, const float *sinr,
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
__device__ void norm_rope_head_s(float *v, const float *w, const float *cosr, const float *sinr, float eps,
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

// ---------------------------------------------------------------------------------------
// Decode: grid (kv_head, split, row), 128 threads. Each CTA applies q-norm + RoPE to the
// group's q heads, handles positions [split*chunk, min(L, (split+1)*chunk)), and the CTA
// whose range holds the new position also normalizes/rotates the new k and appends k, v.
// Partial (max, sum, o[D]) per q head go to scratch; the last CTA of each (row, kv_head)
// to finish merges the splits and writes the BF16 head outputs.
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

// Merge the n_active split partials of the G heads of (row, kv_head): per-split weights
// exp(m_s - M) are formed once in shared memory, then every output dim sums its splits
// with independent (pipelined) L2 loads. The last CTA to arrive resets the counter.
template <int D, int G>
__device__ void attn_merge(const DecodeAttnParams &p, const float *part_base, int kvh, int row, int n_active) {
  constexpr int MS = 64;  // >= max_splits
  __shared__ float wsplit[G][MS];
  __shared__ float inv_l[G];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
      wsplit[h][lane + 32 * i] = c;
      Ls += lv[i] * c;
    }
    Ls = warp_sum(Ls);
    if (lane == 0) inv_l[h] = 1.0f / Ls;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += kAttnThreads) {
    const int h = idx / D, d = idx % D;
    const float *pr0 = part_base + size_t(kvh * G + h) * p.max_splits * (D + 2) + 2 + d;
    float O = 0.f;
#pragma unroll 8
    for (int s = 0; s < n_active; ++s) O += __ldcg(pr0 + s * (D + 2)) * wsplit[h][s];
    p.out[size_t(row) * p.g.qdim + (kvh * G + h) * D + d] = f2bf(O * inv_l[h]);
  }
  if (threadIdx.x == 0) p.count[row * p.g.kv_heads + kvh] = 0;
}

template <int D, int G>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(DecodeAttnParams p) {
  constexpr int LPP = D / 8;      // lanes per position (8 dims each)
  constexpr int PPW = 32 / LPP;   // positions per warp step
  constexpr int NW = kAttnThreads / 32;
  constexpr int UN = 8;           // positions per lane group per round
  constexpr int kMaxPages = 128;  // page-table entries staged in shared memory
  const AttnGeom &g = p.g;
  const int kvh = blockIdx.x, split = blockIdx.y, row = blockIdx.z;
  const int nsplit = gridDim.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane / LPP, sub = lane % LPP;

  __shared__ float q_s[G][D];
  __shared__ float knew[D], vnew[D];
  __shared__ float m_s[NW][PPW][G], l_s[NW][PPW][G];
  __shared__ float o_s[NW * PPW][G][D];
  __shared__ float qn_s[D], kn_s[D];
  __shared__ int ptab_s[kMaxPages];
  __shared__ int last_flag;

  pdl_launch_dependents();
  // Before the wait: data no earlier kernel of this step writes (page table, norm weights).
  const int *ptab_g = p.page_table + size_t(row) * g.pages_per_row;
  const bool ptab_in_smem = g.pages_per_row <= kMaxPages;
  if (ptab_in_smem)
    for (int i = threadIdx.x; i < g.pages_per_row; i += kAttnThreads) ptab_s[i] = ptab_g[i];
  for (int d = threadIdx.x; d < D; d += kAttnThreads) {
    qn_s[d] = bf2f(p.qn[d]);
    kn_s[d] = bf2f(p.kn[d]);
  }
  pdl_wait();
  if (!p.active[row]) return;
  const int pos = p.cur_pos[row];
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
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const int prev = atomicAdd(p.count + row * g.kv_heads + kvh, 1);
      last_flag = prev == nsplit - 1;
    }
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    attn_merge<D, G>(p, part_base, kvh, row, n_active);
    return;
  }
  __syncthreads();  // page table and norm weights staged
  const int *ptab = ptab_in_smem ? ptab_s : ptab_g;
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
    float *dst = is_k ? knew : q_s[h];
    for (int d = lane; d < D; d += 32) dst[d] = bf2f(src[d]);
    __syncwarp();
    norm_rope_head_s<D>(dst, is_k ? kn_s : qn_s, cosr, sinr, g.eps, lane);
  }
  if (holds_new)
    for (int d = threadIdx.x; d < D; d += kAttnThreads) vnew[d] = bf2f(qkv[g.qdim + g.kvdim + kvh * D + d]);
  __syncthreads();
  if (holds_new) {
    bf16 *kd = kv_ptr(0, pos);
    bf16 *vd = kv_ptr(1, pos);
    for (int d = threadIdx.x; d < D; d += kAttnThreads) {
      kd[d] = f2bf(knew[d]);
      vd[d] = f2bf(vnew[d]);
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
    for (int j = 0; j < 8; ++j) qreg[h][j] = q_s[h][sub * 8 + j];

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
      kf[j] = rbf(knew[sub * 8 + j]);
      vf[j] = rbf(vnew[sub * 8 + j]);
    }
    consume(grp == 0 ? pos : -1, kf, vf);
  }

  // Merge lane groups and warps of this CTA.
  const int slot = warp * PPW + grp;
#pragma unroll
  for (int h = 0; h < G; ++h) {
    if (sub == 0) {
      m_s[warp][grp][h] = m[h];
      l_s[warp][grp][h] = l[h];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) o_s[slot][h][sub * 8 + j] = acc[h][j];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += kAttnThreads) {
    const int h = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w)
      for (int q = 0; q < PPW; ++q) M = fmaxf(M, m_s[w][q][h]);
    float Ls = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < NW; ++w)
        for (int q = 0; q < PPW; ++q) {
          const float mv = m_s[w][q][h];
          if (mv == -INFINITY) continue;
          const float c = expf(mv - M);
          Ls += l_s[w][q][h] * c;
          O += o_s[w * PPW + q][h][d] * c;
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
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(p.count + row * g.kv_heads + kvh, 1);
    last_flag = prev == nsplit - 1;
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  attn_merge<D, G>(p, part_base, kvh, row, n_active);
}

void launch_attn_decode(const Model &m, Session &s, int layer, int n_rows, cudaStream_t st) {
  DecodeAttnParams p;
  p.g = geom(m, s);
  p.layer = layer;
  p.max_splits = s.max_splits;
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
  p.out = s.attn;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m.d.kv_heads, s.max_splits, n_rows);
  cfg.blockDim = dim3(kAttnThreads);
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
  else if (m.d.head_dim == 128 && G == 4)
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<128, 4>, p));
  else if (m.d.head_dim == 64 && G == 2)
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<64, 2>, p));
  else if (m.d.head_dim == 64 && G == 1)
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<64, 1>, p));
  else if (m.d.head_dim == 64 && G == 4)
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<64, 4>, p));
  else
    throw Error("ValueError", "head_dim must be 64 or 128 and the GQA group 1, 2 or 4");
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

// Causal prefill attention over the row's cache positions [0, start + T): grid
// (ceil(T/64), heads), 256 threads, FP32 tiles of 64 queries x 64 keys in shared memory.
// Thread t owns queries 4*(t/16) .. +3 and, for scores, keys 4*(t%16) .. +3; for the
// output, dims (D/16)*(t%16) .. +D/16-1.
struct PrefillAttnParams {
  AttnGeom g;
  int layer, start, T;
  bf16 *pool;
  const int *ptab;
  const bf16 *q;  // [T][heads][D]
  bf16 *out;      // [T][qdim]
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
      p.out[size_t(qi) * g.qdim + h * D + kj * DT + dd] = f2bf(o[i][dd] * inv);
  }
}

static size_t prefill_attn_smem(int D) { return (64 * (D + 1) * 2 + 64 * D + 64 * 65) * sizeof(float); }

void configure_attn_kernels() {
  YAR_CUDA(cudaFuncSetAttribute(k_attn_prefill<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(prefill_attn_smem(128))));
  YAR_CUDA(cudaFuncSetAttribute(k_attn_prefill<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(prefill_attn_smem(64))));
}

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
  p.out = s.pattn;
  const int D = m.d.head_dim;
  const size_t smem = prefill_attn_smem(D);
  dim3 grid((T + 63) / 64, m.d.heads);
  if (D == 128)
    k_attn_prefill<128><<<grid, 256, smem, st>>>(p);
  else
    k_attn_prefill<64><<<grid, 256, smem, st>>>(p);
  YAR_CUDA(cudaGetLastError());
}

}  // namespace yar
