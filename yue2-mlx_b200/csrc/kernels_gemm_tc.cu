// kernels_gemm_tc.cu — the prefill linears on the 5th-generation tensor cores.
//
// C[M][N] (+)= A[M][K] . W[N][K]^T with A the chunk's token activations and W a weight
// matrix, both row-major ("K-major") BF16; FP32 accumulation in tensor memory. One CTA per
// 128 x 128 output tile, 128 threads:
//   * lane 0 of warp 0 streams 64-wide K slices of the A and W tiles with TMA
//     (cp.async.bulk.tensor, SWIZZLE_128B) into a 6-stage shared-memory ring;
//   * lane 0 of warp 1 issues tcgen05.mma (kind::f16, BF16 x BF16 -> FP32, M = N = 128,
//     K = 16 per instruction) on each slice and releases the slice with tcgen05.commit;
//   * after the last slice all four warps read their 32 TMEM lanes (= tile rows) with
//     tcgen05.ld and apply the epilogue of the mma.sync GEMM (store, residual add, SwiGLU
//     of interleaved gate/up rows) with the same BF16 rounding points.
// Rows past M are zero-filled by TMA and not stored. Every wait is bounded: on expiry the
// CTA records an error, still drains its copies and MMAs, frees its tensor memory and
// exits; the host reads the error word after the prefill.
#include <cuda.h>

#include "common.cuh"

namespace yar {

constexpr int kTcBM = 128, kTcBN = 128, kTcBK = 64, kTcStages = 6, kTcThreads = 128;
constexpr int kTcTileA = kTcBM * kTcBK * 2;  // 16 KB
constexpr int kTcTileB = kTcBN * kTcBK * 2;  // 16 KB
constexpr int kTcSmem = kTcStages * (kTcTileA + kTcTileB) + 1024;  // + alignment slack
constexpr long long kTcWaitLimit = 1ll << 24;

// Instruction descriptor, kind::f16: FP32 accumulator (bits 4-5 = 1), A and B BF16 (bits
// 7-9 and 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kTcIdesc =
    (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kTcBN >> 3) << 17) | (uint32_t(kTcBM >> 4) << 24);

struct TcParams {
  bf16 *C;
  int M, N, K, ldc;
  int *error;
  float *ws;   // split-K: FP32 partials [splits][M][N] instead of the epilogue (null: none)
  int kb_per;  // 64-wide K slices per CTA (blockIdx.z picks the CTA's range)
};

__device__ __forceinline__ uint32_t tc_smem(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ bool tc_wait(uint64_t *bar, unsigned parity) {
  for (long long i = 0; i < kTcWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(tc_smem(bar)), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}
// Shared-memory matrix descriptor of a K-major tile written by TMA with 128-byte swizzle:
// rows of 128 bytes (64 BF16), 8-row swizzle atoms 1024 bytes apart (stride byte offset),
// descriptor version 1, layout type 2 (SWIZZLE_128B). The tile base is 1024-aligned; the
// k-th 16-element step of the MMA starts 32 bytes further (start address + 2).
__device__ __forceinline__ uint64_t tc_desc(const void *tile) {
  return (uint64_t(tc_smem(tile) >> 4) & 0x3FFFull) | (1ull << 16) | (uint64_t(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, TcParams p) {
  extern __shared__ unsigned char tc_raw[];
  unsigned char *base = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *sa = base, *sb = base + kTcStages * kTcTileA;
  __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], done;
  __shared__ uint32_t tmem_slot;
  __shared__ int s_fail;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kTcBN, m0 = blockIdx.y * kTcBM, KB = p.kb_per, kb0 = blockIdx.z * p.kb_per;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_smem(&full[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_smem(&empty[s])));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_smem(&done)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_fail = 0;
  }
  if (warp == 0) {  // 128 FP32 accumulator columns x 128 lanes
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_smem(&tmem_slot)),
                 "r"(kTcBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;

  // Lane 0 of warp 0 produces and lane 0 of warp 1 issues the MMAs; the other lanes of
  // those warps wait for their lane 0 at __syncwarp (parked, not spinning on `done`, which
  // would take the warp's issue slots from the one lane doing the work).
  pdl_launch_dependents();
  if (warp == 0) {
    if (lane == 0) {
      // Producer: TMA loads of the A and W slices. The first stages' weight slices are
      // requested before waiting for the kernel that writes A (programmatic launch: the
      // weights are constants); their A slices, and everything after, once it is done.
      auto load_a = [&](int kb, int s) {
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
            "[%2];" ::"r"(tc_smem(sa + s * kTcTileA)),
            "l"(&tma_a), "r"(tc_smem(&full[s])), "r"((kb0 + kb) * kTcBK), "r"(m0)
            : "memory");
      };
      auto load_b = [&](int kb, int s) {
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
            "[%2];" ::"r"(tc_smem(sb + s * kTcTileB)),
            "l"(&tma_b), "r"(tc_smem(&full[s])), "r"((kb0 + kb) * kTcBK), "r"(n0)
            : "memory");
      };
      const int pre = KB < kTcStages ? KB : kTcStages;
      for (int kb = 0; kb < pre; ++kb) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_smem(&full[kb])),
                     "r"(kTcTileA + kTcTileB)
                     : "memory");
        load_b(kb, kb);
      }
      pdl_wait();
      for (int kb = 0; kb < pre; ++kb) load_a(kb, kb);
      int issued = pre;
      for (int kb = pre; kb < KB; ++kb) {
        const int s = kb % kTcStages;
        if (!tc_wait(&empty[s], unsigned((kb / kTcStages) - 1) & 1u)) {
          atomicOr(p.error, 64);
          s_fail = 1;
          break;
        }
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_smem(&full[s])),
                     "r"(kTcTileA + kTcTileB)
                     : "memory");
        load_a(kb, s);
        load_b(kb, s);
        issued = kb + 1;
      }
      // Never leave with a copy in flight: wait (bounded) for the last stages issued.
      for (int kb = issued > kTcStages ? issued - kTcStages : 0; kb < issued; ++kb)
        tc_wait(&full[kb % kTcStages], unsigned(kb / kTcStages) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer.
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % kTcStages;
        if (!tc_wait(&full[s], unsigned(kb / kTcStages) & 1u)) {
          atomicOr(p.error, 64);
          s_fail = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t da = tc_desc(sa + s * kTcTileA), db = tc_desc(sb + s * kTcTileB);
  #pragma unroll
        for (int k = 0; k < kTcBK / 16; ++k) {
          const uint32_t acc = (kb | k) != 0;
          asm volatile(
              "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
              " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(tmem),
              "l"(da + 2 * k), "l"(db + 2 * k), "r"(kTcIdesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
              : "memory");
        }
        // The slice's smem is free once these MMAs have read it.
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         tc_smem(&empty[s]))
                     : "memory");
      }
      // Completes when every MMA issued above has finished (also after a failure).
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       tc_smem(&done))
                   : "memory");
    }
    __syncwarp();
  }
  // Epilogue: warp w owns TMEM lanes (tile rows) 32w..32w+31. (Every thread has waited for
  // the predecessor kernel before touching C.)
  pdl_wait();
  if (!tc_wait(&done, 0u)) {
    if (lane == 0) atomicOr(p.error, 64);
    s_fail = 1;
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (!s_fail) {
    const int row = m0 + warp * 32 + lane;
    for (int c = 0; c < kTcBN; c += 32) {
      uint32_t v[32];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
          "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
            "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
            "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
            "=r"(v[30]), "=r"(v[31])
          : "r"(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c)));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (row >= p.M) continue;
      const int col = n0 + c;
      if (p.ws) {  // split-K partial: FP32 values, the epilogue runs after the reduction
        uint4 *dst = reinterpret_cast<uint4 *>(p.ws + (size_t(blockIdx.z) * p.M + row) * p.N + col);
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[q] = make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        continue;
      }
      if (EPI == kEpiSwiGLU) {
        uint32_t o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float r2[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float gate = rbf(__uint_as_float(v[4 * j + 2 * h])), up = rbf(__uint_as_float(v[4 * j + 2 * h + 1]));
            r2[h] = rbf(silu_f32(gate)) * up;
          }
          o[j] = (__float_as_uint(rbf(r2[0])) >> 16) | (__float_as_uint(rbf(r2[1])) & 0xFFFF0000u);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(p.C + size_t(row) * p.ldc + (col >> 1));
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
      } else {
        uint4 *dst = reinterpret_cast<uint4 *>(p.C + size_t(row) * p.ldc + col);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t o[4];
          uint4 old = make_uint4(0, 0, 0, 0);
          if (EPI == kEpiResidual) old = dst[q];
          const uint32_t ow[4] = {old.x, old.y, old.z, old.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float lo = __uint_as_float(v[8 * q + 2 * j]), hi = __uint_as_float(v[8 * q + 2 * j + 1]);
            if (EPI == kEpiResidual) {
              lo = bf_lo(ow[j]) + rbf(lo);
              hi = bf_hi(ow[j]) + rbf(hi);
            }
            o[j] = (__float_as_uint(rbf(lo)) >> 16) | (__float_as_uint(rbf(hi)) & 0xFFFF0000u);
          }
          dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcBN));
}

// Split-K: out = epilogue(sum over splits of the FP32 partials, in split order). One thread
// per 8 consecutive columns of a row.
template <int EPI>
__global__ void __launch_bounds__(256) k_splitk_reduce(const float *ws, int splits, int M, int N, bf16 *C, int ldc) {
  pdl_launch_dependents();
  pdl_wait();
  const long long idx = blockIdx.x * 256ll + threadIdx.x, groups = N / 8;
  if (idx >= (long long)M * groups) return;
  const int row = int(idx / groups), col = int(idx % groups) * 8;
  float v[8];
  for (int s = 0; s < splits; ++s) {
    const float4 *src = reinterpret_cast<const float4 *>(ws + (size_t(s) * M + row) * N + col);
    const float4 a = src[0], b = src[1];
    const float w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = s == 0 ? w[j] : v[j] + w[j];
  }
  if (EPI == kEpiSwiGLU) {
    uint32_t o[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float r2[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float gate = rbf(v[4 * j + 2 * h]), up = rbf(v[4 * j + 2 * h + 1]);
        r2[h] = rbf(silu_f32(gate)) * up;
      }
      o[j] = (__float_as_uint(rbf(r2[0])) >> 16) | (__float_as_uint(rbf(r2[1])) & 0xFFFF0000u);
    }
    *reinterpret_cast<uint2 *>(C + size_t(row) * ldc + (col >> 1)) = make_uint2(o[0], o[1]);
  } else {
    uint4 *dst = reinterpret_cast<uint4 *>(C + size_t(row) * ldc + col);
    uint4 old = make_uint4(0, 0, 0, 0);
    if (EPI == kEpiResidual) old = *dst;
    const uint32_t ow[4] = {old.x, old.y, old.z, old.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float lo = v[2 * j], hi = v[2 * j + 1];
      if (EPI == kEpiResidual) {
        lo = bf_lo(ow[j]) + rbf(lo);
        hi = bf_hi(ow[j]) + rbf(hi);
      }
      o[j] = (__float_as_uint(rbf(lo)) >> 16) | (__float_as_uint(rbf(hi)) & 0xFFFF0000u);
    }
    *dst = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ------------------------------------------------------------------------------- host
namespace {
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiled encode_fn() {
  static EncodeTiled fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}
// Row-major [rows][K] BF16, boxes of 64 (K) x box_rows, 128-byte swizzle, zero fill past the end.
CUtensorMap kmajor_map(const bf16 *ptr, int rows, int K, int box_rows) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(K) * 2};
  const cuuint32_t box[2] = {cuuint32_t(kTcBK), cuuint32_t(box_rows)};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<bf16 *>(ptr), dims, strides, box,
                                 es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error("RuntimeError", "cuTensorMapEncodeTiled failed");
  return m;
}
}  // namespace

// The decode GEMVs' stage map (tma_ring.cuh): W [N][K] row-major BF16 viewed as {64
// columns, N rows, K/64 column blocks} with byte strides {2K, 128}; a {64, 8, 32} box is
// one 32 KB stage (8 rows x 2048 columns), written to shared memory with the 128-byte
// swizzle; rows past N are zero-filled.
void encode_stage_map(CUtensorMap *map, const bf16 *W, int N, int K) {
  if (N < 1 || K < 2048 || K % 2048 != 0 || (reinterpret_cast<uintptr_t>(W) & 15) != 0)
    throw Error("RuntimeError", "stage map: W must be 16-byte aligned with K a multiple of 2048");
  const EncodeTiled fn = encode_fn();
  if (!fn) throw Error("RuntimeError", "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[3] = {64, cuuint64_t(N), cuuint64_t(K / 64)};
  const cuuint64_t strides[2] = {cuuint64_t(K) * 2, 128};
  const cuuint32_t box[3] = {64, 8, 32};
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<bf16 *>(W), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error("RuntimeError", "cuTensorMapEncodeTiled failed for a stage map");
}

bool encode_rows128_map(CUtensorMap *map, const bf16 *base, uint64_t rows) {
  const EncodeTiled fn = encode_fn();
  if (!fn || rows == 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  const cuuint64_t dims[2] = {128, cuuint64_t(rows)};
  const cuuint64_t strides[1] = {256};
  const cuuint32_t box[2] = {64, 64};
  const cuuint32_t es[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<bf16 *>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void configure_gemm_tc_kernels() {
  YAR_CUDA(cudaFuncSetAttribute(k_gemm_tc<kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem));
  YAR_CUDA(cudaFuncSetAttribute(k_gemm_tc<kEpiResidual>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem));
  YAR_CUDA(cudaFuncSetAttribute(k_gemm_tc<kEpiSwiGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem));
}

// True when the tensor-core path takes this shape (otherwise the mma.sync GEMM runs).
bool gemm_tc_supported(const bf16 *A, int M, int K, const bf16 *W, int N, const bf16 *C, int ldc) {
  auto al16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  return encode_fn() != nullptr && M >= 1 && K % kTcBK == 0 && N % kTcBN == 0 && ldc % 8 == 0 && al16(A) &&
         al16(W) && al16(C);
}

void launch_gemm_tc(const bf16 *A, int M, int K, const bf16 *W, int N, bf16 *C, int ldc, int epilogue, int *error,
                    float *ws, size_t ws_floats, cudaStream_t st, int split_n) {
  const CUtensorMap ma = kmajor_map(A, M, K, kTcBM), mb = kmajor_map(W, N, K, kTcBN);
  // Split K across CTAs while the tile grid leaves SMs idle (small M: batched decode).
  const int NS = split_n > 0 ? split_n : N;
  if (split_n > 0 && NS < N) throw Error("ValueError", "split_n below N");
  const int tiles = (NS / kTcBN) * ((M + kTcBM - 1) / kTcBM), KB = K / kTcBK;
  int splits = 1;
  while (ws && split_n >= 0 && splits < 8 && tiles * splits < 120 && KB % (splits * 2) == 0 &&
         size_t(splits * 2) * M * NS <= ws_floats)
    splits *= 2;
  TcParams p{C, M, N, K, ldc, error, splits > 1 ? ws : nullptr, KB / splits};
  // Programmatic launches: each kernel may start while its predecessor finishes and waits
  // (griddepcontrol.wait) before reading its outputs or writing anything.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(N / kTcBN, (M + kTcBM - 1) / kTcBM, splits);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kTcSmem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (epilogue == kEpiSwiGLU)
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_tc<kEpiSwiGLU>, ma, mb, p));
  else if (epilogue == kEpiResidual)
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_tc<kEpiResidual>, ma, mb, p));
  else
    YAR_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_tc<kEpiStore>, ma, mb, p));
  if (splits > 1) {
    const long long threads = (long long)M * (N / 8);
    cfg.gridDim = dim3(unsigned((threads + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    if (epilogue == kEpiSwiGLU)
      YAR_CUDA(cudaLaunchKernelEx(&cfg, k_splitk_reduce<kEpiSwiGLU>, (const float *)ws, splits, M, N, C, ldc));
    else if (epilogue == kEpiResidual)
      YAR_CUDA(cudaLaunchKernelEx(&cfg, k_splitk_reduce<kEpiResidual>, (const float *)ws, splits, M, N, C, ldc));
    else
      YAR_CUDA(cudaLaunchKernelEx(&cfg, k_splitk_reduce<kEpiStore>, (const float *)ws, splits, M, N, C, ldc));
  }
}

}  // namespace yar
