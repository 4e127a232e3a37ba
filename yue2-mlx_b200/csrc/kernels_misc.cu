// kernels_misc.cu — embedding gathers, per-step position bookkeeping and the prefill
// RMSNorm (modeling_yue2.py:131-132, :432; native/src/ar.cpp:259).
#include "common.cuh"

namespace yar {

// First kernel of a decode step: x[row] = embed[token[row]]; the row's position for this
// step is latched into cur_pos and pos advances (only for active rows that have room; a
// full row is deactivated and flagged instead of writing past its capacity).
__global__ void __launch_bounds__(256) k_embed_rows(const bf16 *embed, const int *token, int *pos,
                                                    int *cur_pos, const int *capacity, int *active,
                                                    int *error, int H, int vocab, bf16 *x) {
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x;
  if (!active[row]) return;
  int tok = token[row];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) atomicOr(error, 1);
    tok = 0;
  }
  const bf16 *src = embed + size_t(tok) * H;
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x)
    reinterpret_cast<uint4 *>(x + size_t(row) * H)[c] = reinterpret_cast<const uint4 *>(src)[c];
  __syncthreads();
  if (threadIdx.x == 0) {
    const int p = pos[row];
    cur_pos[row] = p;
    if (p >= capacity[row]) {
      atomicOr(error, 2);
      active[row] = 0;
    } else {
      pos[row] = p + 1;
    }
  }
}

void launch_embed_rows(const Model &m, Session &s, int n_rows, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_rows);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  YAR_CUDA(cudaLaunchKernelEx(&cfg, k_embed_rows, m.embed, (const int *)s.d_token, s.d_pos, s.d_cur_pos,
                              (const int *)s.d_capacity, s.d_active, s.d_error, m.d.hidden, m.d.vocab,
                              s.x));
}

__global__ void k_embed_tokens(const bf16 *embed, const int *ids, int H, bf16 *x) {
  const int t = blockIdx.x;
  const bf16 *src = embed + size_t(ids[t]) * H;
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x)
    reinterpret_cast<uint4 *>(x + size_t(t) * H)[c] = reinterpret_cast<const uint4 *>(src)[c];
}

void launch_embed_tokens(const bf16 *embed, const int *ids, int T, int H, bf16 *x, cudaStream_t st) {
  k_embed_tokens<<<T, 256, 0, st>>>(embed, ids, H, x);
  YAR_CUDA(cudaGetLastError());
}

// out[t] = bf16(bf16(x[t] * bf16(rsqrt(mean(x[t]^2) + eps))) * w), one CTA per row.
__global__ void __launch_bounds__(256) k_rmsnorm_rows(const bf16 *x, const bf16 *w, int H, float eps,
                                                      bf16 *out) {
  __shared__ float red[8];
  pdl_launch_dependents();
  pdl_wait();  // programmatic launch: x comes from the preceding kernel
  const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bf16 *xr = x + size_t(t) * H;
  float ss = 0.f;
  for (int k = threadIdx.x; k < H; k += 256) {
    const float v = bf2f(xr[k]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float scale = rms_scale_bf16(tot, H, eps);
  for (int k = threadIdx.x; k < H; k += 256)
    out[size_t(t) * H + k] = f2bf(rbf(bf2f(xr[k]) * scale) * bf2f(w[k]));
}

void launch_rmsnorm_rows(const bf16 *x, const bf16 *w, int T, int H, float eps, bf16 *out,
                         cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(T);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  YAR_CUDA(cudaLaunchKernelEx(&cfg, k_rmsnorm_rows, x, w, H, eps, out));
}

}  // namespace yar
