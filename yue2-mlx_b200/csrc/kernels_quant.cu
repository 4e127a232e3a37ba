// kernels_quant.cu — load-time kernels of the `8bit` and `4bit` precisions (affine, group
// 64: per 64-column group w = scale * q + bias; ar.cpp:20-29 and :305-311 run these weights
// through mlx quantized_matmul). The raw form is the converted artifact's: the U32 words'
// little-endian bytes [rows][K * bits / 8] (element (32 / bits) i + j in bits (bits j)..
// of word i), BF16 scale and bias bits [rows][K / 64].
//   k_q_dequant: the BF16 weights scale * q + bias (one FP32 fma, rounded once) that
//                prefill and the batched / per-operation decode paths read;
//   k_q_image:   the stage image the persistent decode kernel streams (the layout the
//                quantized ring consumer reads: 16-row units, K / 2048 stages of
//                kQ8StageBytes or kQ4StageBytes each, see tma_ring.cuh).
#include "engine.h"
#include "tma_ring.cuh"

namespace yar {

// Element k of a raw row: a byte (8 bits) or nibble k & 1 of byte k / 2 (4 bits: element
// 8i + j in bits 4j.. of word i, so the low nibble of each byte comes first).
template <int BITS>
__device__ __forceinline__ uint32_t raw_q(const uint8_t *row, int k) {
  if (BITS == 8) return row[k];
  return (row[k >> 1] >> ((k & 1) * 4)) & 0xFu;
}

template <int BITS>
__global__ void k_q_dequant(const uint8_t *__restrict__ q, const uint16_t *__restrict__ s,
                            const uint16_t *__restrict__ b, long long rows, int K, bf16 *__restrict__ out) {
  const long long chunks = rows * (K / 8);
  for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c < chunks;
       c += (long long)gridDim.x * blockDim.x) {
    const long long row = c / (K / 8);
    const int k = int(c % (K / 8)) * 8;
    const uint8_t *qr = q + row * (K * BITS / 8);
    const float sc = __uint_as_float(uint32_t(s[row * (K / 64) + k / 64]) << 16);
    const float bi = __uint_as_float(uint32_t(b[row * (K / 64) + k / 64]) << 16);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = __fmaf_rn(sc, float(raw_q<BITS>(qr, k + 2 * i)), bi);
      const float hi = __fmaf_rn(sc, float(raw_q<BITS>(qr, k + 2 * i + 1)), bi);
      o[i] = pack_bf16x2(__float2bfloat16_rn(lo), __float2bfloat16_rn(hi));
    }
    *reinterpret_cast<uint4 *>(out + row * K + k) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// One item per 16-byte weight chunk (kQ8QBytes or kQ4QBytes / 16 per stage) and per
// scale/bias word (512 per stage) of the image of rows [0, rows).
template <int BITS>
__global__ void k_q_image(const uint8_t *__restrict__ q, const uint16_t *__restrict__ s,
                          const uint16_t *__restrict__ b, int rows, int K, unsigned char *__restrict__ img) {
  constexpr int kQB = BITS == 8 ? kQ8QBytes : kQ4QBytes, kStage = q_stage_bytes<BITS>();
  constexpr int kChunks = kQB / 16, kItems = kChunks + (kStage - kQB) / 4;
  const int KS = K / kRingPiece;
  const long long stages = (long long)((rows + kQ8Rows - 1) / kQ8Rows) * KS;
  for (long long it = blockIdx.x * (long long)blockDim.x + threadIdx.x; it < stages * kItems;
       it += (long long)gridDim.x * blockDim.x) {
    const long long stage = it / kItems;
    const int i = int(it % kItems), u = int(stage / KS), ks = int(stage % KS);
    unsigned char *st = img + stage * kStage;
    auto at = [&](int row, int col) -> uint32_t {
      return row < rows ? raw_q<BITS>(q + (long long)row * (K * BITS / 8), col) : 0u;
    };
    if (i < kChunks) {
      uint32_t words[4];
      if (BITS == 8) {
        // Chunk ((w * 4 + j) * 2 + h) * 32 + lane: for k-tiles 2h, 2h + 1 the words (row g,
        // kt), (row g + 8, kt), each the bytes of columns 16 kt + {2t, 2t+1, 2t+8, 2t+9} of
        // the group's 64.
        const int lane = i & 31, h = (i >> 5) & 1, j = (i >> 6) & 3, w = i >> 8;
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int kt = 2 * h + (m >> 1), row = u * kQ8Rows + g + 8 * (m & 1);
          const int col = ks * kRingPiece + w * 256 + j * 64 + kt * 16 + 2 * t;
          words[m] = at(row, col) | (at(row, col + 1) << 8) | (at(row, col + 8) << 16) | (at(row, col + 9) << 24);
        }
      } else {
        // Chunk (w * 4 + j) * 32 + lane: word kt holds fragment s (rows g + 8 (s & 1),
        // columns 16 kt + 2t + 8 (s >> 1) and + 1) in nibbles s and 4 + s.
        const int lane = i & 31, j = (i >> 5) & 3, w = i >> 7;
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int kt = 0; kt < 4; ++kt) {
          uint32_t v = 0;
#pragma unroll
          for (int sf = 0; sf < 4; ++sf) {
            const int row = u * kQ8Rows + g + 8 * (sf & 1);
            const int col = ks * kRingPiece + w * 256 + j * 64 + kt * 16 + 2 * t + 8 * (sf >> 1);
            v |= (at(row, col) << (4 * sf)) | (at(row, col + 1) << (16 + 4 * sf));
          }
          words[kt] = v;
        }
      }
      *reinterpret_cast<uint4 *>(st + i * 16) = make_uint4(words[0], words[1], words[2], words[3]);
    } else {
      // Word 16 G + 2 (r % 8) + r / 8: scale (low) and bias (high) of unit row r, group G.
      const int wi = i - kChunks, G = wi >> 4, r = ((wi & 15) >> 1) + 8 * (wi & 1);
      const int row = u * kQ8Rows + r, gi = ks * (kRingPiece / 64) + G;
      uint32_t v = 0;
      if (row < rows) v = uint32_t(s[(long long)row * (K / 64) + gi]) | (uint32_t(b[(long long)row * (K / 64) + gi]) << 16);
      *reinterpret_cast<uint32_t *>(st + kQB + wi * 4) = v;
    }
  }
}

size_t q_image_bytes(int rows, int K, int bits) {
  return size_t((rows + kQ8Rows - 1) / kQ8Rows) * size_t(K / kRingPiece) *
         size_t(bits == 8 ? kQ8StageBytes : kQ4StageBytes);
}

void launch_q_dequant(const uint8_t *q, const uint16_t *s, const uint16_t *b, long long rows, int K, int bits,
                      bf16 *out, cudaStream_t st) {
  if (rows <= 0) return;
  if (bits == 8)
    k_q_dequant<8><<<1184, 256, 0, st>>>(q, s, b, rows, K, out);
  else
    k_q_dequant<4><<<1184, 256, 0, st>>>(q, s, b, rows, K, out);
  YAR_CUDA(cudaGetLastError());
}

void launch_q_image(const uint8_t *q, const uint16_t *s, const uint16_t *b, int rows, int K, int bits,
                    unsigned char *img, cudaStream_t st) {
  if (rows <= 0) return;
  if (K % kRingPiece) throw Error("ValueError", "quantized stage images need K a multiple of 2048");
  if (bits == 8)
    k_q_image<8><<<1184, 256, 0, st>>>(q, s, b, rows, K, img);
  else
    k_q_image<4><<<1184, 256, 0, st>>>(q, s, b, rows, K, img);
  YAR_CUDA(cudaGetLastError());
}

}  // namespace yar
