// kernels_quant.cu — load-time kernels of the `8bit` precision (affine, group 64: per
// 64-column group w = scale * q + bias; ar.cpp:20-29 and :305-311 run these weights
// through mlx quantized_matmul). The raw form is the converted artifact's: q as bytes
// [rows][K] (the U32 words' little-endian bytes, element 4i + j in bits 8j..8j+7 of word
// i), BF16 scale and bias bits [rows][K / 64].
//   k_q8_dequant: the BF16 weights scale * q + bias (one FP32 fma, rounded once) that
//                 prefill and the batched / per-operation decode paths read;
//   k_q8_image:   the stage image the persistent decode kernel streams (the layout the
//                 8-bit ring consumer reads: 16-row units, K / 2048 stages of
//                 kQ8StageBytes each, see tma_ring.cuh).
#include "engine.h"
#include "tma_ring.cuh"

namespace yar {

__global__ void k_q8_dequant(const uint8_t *__restrict__ q, const uint16_t *__restrict__ s,
                             const uint16_t *__restrict__ b, long long rows, int K, bf16 *__restrict__ out) {
  const long long chunks = rows * (K / 8);
  for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c < chunks;
       c += (long long)gridDim.x * blockDim.x) {
    const long long row = c / (K / 8);
    const int k = int(c % (K / 8)) * 8;
    const uint2 qv = *reinterpret_cast<const uint2 *>(q + row * K + k);
    const float sc = __uint_as_float(uint32_t(s[row * (K / 64) + k / 64]) << 16);
    const float bi = __uint_as_float(uint32_t(b[row * (K / 64) + k / 64]) << 16);
    const uint32_t w[2] = {qv.x, qv.y};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t word = w[i >> 1], sh = (i & 1) * 16;
      const float lo = __fmaf_rn(sc, float((word >> sh) & 0xFFu), bi);
      const float hi = __fmaf_rn(sc, float((word >> (sh + 8)) & 0xFFu), bi);
      o[i] = pack_bf16x2(__float2bfloat16_rn(lo), __float2bfloat16_rn(hi));
    }
    *reinterpret_cast<uint4 *>(out + row * K + k) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// One item per 16-byte weight chunk (2048 per stage) and per scale/bias word (512 per
// stage) of the image of rows [0, rows).
__global__ void k_q8_image(const uint8_t *__restrict__ q, const uint16_t *__restrict__ s,
                           const uint16_t *__restrict__ b, int rows, int K, unsigned char *__restrict__ img) {
  constexpr int kItems = kQ8QBytes / 16 + kQ8StageBytes / 4 - kQ8QBytes / 4;  // 2048 + 512
  const int KS = K / kRingPiece;
  const long long stages = (long long)((rows + kQ8Rows - 1) / kQ8Rows) * KS;
  for (long long it = blockIdx.x * (long long)blockDim.x + threadIdx.x; it < stages * kItems;
       it += (long long)gridDim.x * blockDim.x) {
    const long long stage = it / kItems;
    const int i = int(it % kItems), u = int(stage / KS), ks = int(stage % KS);
    unsigned char *st = img + stage * kQ8StageBytes;
    if (i < kQ8QBytes / 16) {
      // Chunk ((w * 4 + j) * 2 + h) * 32 + lane: for k-tiles 2h, 2h + 1 the words (row g,
      // kt), (row g + 8, kt), each the bytes of columns 16 kt + {2t, 2t+1, 2t+8, 2t+9} of
      // the group's 64.
      const int lane = i & 31, h = (i >> 5) & 1, j = (i >> 6) & 3, w = i >> 8;
      const int g = lane >> 2, t = lane & 3;
      uint32_t words[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int kt = 2 * h + (m >> 1), row = u * kQ8Rows + g + 8 * (m & 1);
        const int col = ks * kRingPiece + w * 256 + j * 64 + kt * 16 + 2 * t;
        uint32_t v = 0;
        if (row < rows) {
          const uint8_t *r = q + (long long)row * K + col;
          v = uint32_t(r[0]) | (uint32_t(r[1]) << 8) | (uint32_t(r[8]) << 16) | (uint32_t(r[9]) << 24);
        }
        words[m] = v;
      }
      *reinterpret_cast<uint4 *>(st + i * 16) = make_uint4(words[0], words[1], words[2], words[3]);
    } else {
      // Word 16 G + 2 (r % 8) + r / 8: scale (low) and bias (high) of unit row r, group G.
      const int wi = i - kQ8QBytes / 16, G = wi >> 4, r = ((wi & 15) >> 1) + 8 * (wi & 1);
      const int row = u * kQ8Rows + r, gi = ks * (kRingPiece / 64) + G;
      uint32_t v = 0;
      if (row < rows) v = uint32_t(s[(long long)row * (K / 64) + gi]) | (uint32_t(b[(long long)row * (K / 64) + gi]) << 16);
      *reinterpret_cast<uint32_t *>(st + kQ8QBytes + wi * 4) = v;
    }
  }
}

size_t q8_image_bytes(int rows, int K) {
  return size_t((rows + kQ8Rows - 1) / kQ8Rows) * size_t(K / kRingPiece) * kQ8StageBytes;
}

void launch_q8_dequant(const uint8_t *q, const uint16_t *s, const uint16_t *b, long long rows, int K, bf16 *out,
                       cudaStream_t st) {
  if (rows <= 0) return;
  k_q8_dequant<<<1184, 256, 0, st>>>(q, s, b, rows, K, out);
  YAR_CUDA(cudaGetLastError());
}

void launch_q8_image(const uint8_t *q, const uint16_t *s, const uint16_t *b, int rows, int K, unsigned char *img,
                     cudaStream_t st) {
  if (rows <= 0) return;
  if (K % kRingPiece) throw Error("ValueError", "8-bit stage images need K a multiple of 2048");
  k_q8_image<<<1184, 256, 0, st>>>(q, s, b, rows, K, img);
  YAR_CUDA(cudaGetLastError());
}

}  // namespace yar
