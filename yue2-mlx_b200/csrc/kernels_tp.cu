// kernels_tp.cu — the layout steps around the tensor-parallel all-gathers.
//
// Each rank computes a block of columns of an activation ([rows][stride], block k at
// columns [k*n, k*n + n)); the all-gather moves whole contiguous buffers, laid out
// [rank][rows][n]. k_tp_pack copies this rank's block out of the activation rows;
// k_tp_unpack writes every rank's block back into them (for the LM head, the phase
// columns of the logits rows the sampler reads). With one row the blocks are contiguous
// already and the engine gathers in place, without either kernel.
#include "common.cuh"

namespace yar {

__global__ void __launch_bounds__(256) k_tp_pack(const bf16 *buf, int stride, int col0, int n, int n_rows,
                                                 bf16 *send) {
  const int r = blockIdx.y;
  for (int j = blockIdx.x * 256 + threadIdx.x; j < n; j += gridDim.x * 256)
    send[size_t(r) * n + j] = buf[size_t(r) * stride + col0 + j];
}

__global__ void __launch_bounds__(256) k_tp_unpack(const bf16 *recv, int n_rows, int n, int width, bf16 *buf,
                                                   int stride) {
  const int r = blockIdx.y;
  for (int c = blockIdx.x * 256 + threadIdx.x; c < width; c += gridDim.x * 256) {
    const int k = c / n, j = c - k * n;
    buf[size_t(r) * stride + c] = recv[(size_t(k) * n_rows + r) * n + j];
  }
}

static int blocks_for(int n) { return (n + 255) / 256 < 148 ? (n + 255) / 256 : 148; }

void launch_tp_pack(const bf16 *buf, int stride, int col0, int n, int n_rows, bf16 *send, cudaStream_t st) {
  k_tp_pack<<<dim3(blocks_for(n), n_rows), 256, 0, st>>>(buf, stride, col0, n, n_rows, send);
  YAR_CUDA(cudaGetLastError());
}

void launch_tp_unpack(const bf16 *recv, int world, int n_rows, int n, int width, bf16 *buf, int stride,
                      cudaStream_t st) {
  if (width > world * n) throw Error("ValueError", "unpack width exceeds the gathered blocks");
  k_tp_unpack<<<dim3(blocks_for(width), n_rows), 256, 0, st>>>(recv, n_rows, n, width, buf, stride);
  YAR_CUDA(cudaGetLastError());
}

}  // namespace yar
