// kernels_tp.cu — the two element-wise steps around the tensor-parallel exchanges.
//
//   k_residual_f32   x[r][i] = bf16(x[r][i] + bf16(sum[r][i])): the all-reduced FP32 sum
//                    of O (or down) rounded once and added to the BF16 residual, the same
//                    rounding points as the single-GPU residual epilogue
//                    (native/src/ar.cpp:292-298).
//   k_gather_logits  the all-gathered head slices, laid out [rank][row][slice], into the
//                    [row][logit_stride] logits rows the sampler reads.
#include "common.cuh"

namespace yar {

__global__ void __launch_bounds__(256) k_residual_f32(bf16 *x, const float *sum, int n) {
  const int i = (blockIdx.x * 256 + threadIdx.x) * 4;
  if (i >= n) return;
  const float4 s = *reinterpret_cast<const float4 *>(sum + i);
  uint2 *xp = reinterpret_cast<uint2 *>(x + i);
  const uint2 old = *xp;
  const float a = bf_lo(old.x) + rbf(s.x), b = bf_hi(old.x) + rbf(s.y);
  const float c = bf_lo(old.y) + rbf(s.z), d = bf_hi(old.y) + rbf(s.w);
  *xp = make_uint2((__float_as_uint(rbf(a)) >> 16) | (__float_as_uint(rbf(b)) & 0xFFFF0000u),
                   (__float_as_uint(rbf(c)) >> 16) | (__float_as_uint(rbf(d)) & 0xFFFF0000u));
}

void launch_residual_f32(bf16 *x, const float *sum, int n_rows, int H, cudaStream_t st) {
  if (H % 4) throw Error("ValueError", "residual width must be a multiple of 4");
  const int n = n_rows * H;
  k_residual_f32<<<(n / 4 + 255) / 256, 256, 0, st>>>(x, sum, n);
  YAR_CUDA(cudaGetLastError());
}

__global__ void __launch_bounds__(256) k_gather_logits(const bf16 *recv, int n_rows, int slice, int width,
                                                       bf16 *logits, int logit_stride) {
  const int row = blockIdx.y;
  for (int j = blockIdx.x * 256 + threadIdx.x; j < width; j += gridDim.x * 256) {
    const int rank = j / slice, col = j - rank * slice;
    logits[size_t(row) * logit_stride + j] = recv[(size_t(rank) * n_rows + row) * slice + col];
  }
}

void launch_gather_logits(const bf16 *recv, int n_rows, int slice, int width, bf16 *logits, int logit_stride,
                          cudaStream_t st) {
  const int blocks = (width + 255) / 256 < 148 ? (width + 255) / 256 : 148;
  k_gather_logits<<<dim3(blocks, n_rows), 256, 0, st>>>(recv, n_rows, slice, width, logits, logit_stride);
  YAR_CUDA(cudaGetLastError());
}

}  // namespace yar
