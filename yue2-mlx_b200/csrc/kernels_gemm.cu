// kernels_gemm.cu — prefill linears C[M][N] = A[M][K] * W[N][K]^T (BF16 in, FP32
// accumulation, one BF16 rounding), with the same epilogues as the decode GEMVs
// (store / residual add / SwiGLU on interleaved gate-up columns). Reference op:
// model_ops::linear on [1, T, *] activations (native/src/ar.cpp:20-28, :266-298).
//
// Tiles of 128x128x32 through a 3-stage cp.async ring, eight warps of 64x32, warp-level
// m16n8k16 tensor-core MMAs fed by ldmatrix. Ragged M, N and K are zero-filled by the
// copies and masked in the epilogue.
#include "common.cuh"

namespace yar {

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3, PAD = 8, LDS = BK + PAD;

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool pred) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3,
                                            const void *p) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(s));
}
__device__ __forceinline__ void mma_bf16(float *c, const uint32_t *a, const uint32_t *b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

template <int EPI>
__global__ void __launch_bounds__(256) k_gemm(const bf16 *__restrict__ A, int M, int K,
                                              const bf16 *__restrict__ W, int N, bf16 *C, int ldc) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  bf16 *As = reinterpret_cast<bf16 *>(smem_raw);      // [STAGES][BM][LDS]
  bf16 *Bs = As + STAGES * BM * LDS;                  // [STAGES][BN][LDS]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp >> 2, wn = warp & 3;            // 2 x 4 warps of 64 x 32
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int KT = (K + BK - 1) / BK;

  auto load = [&](int stage, int kt) {
    const int k0 = kt * BK;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = tid + i * 256;  // 512 16-byte chunks per operand tile
      const int r = c >> 2, kc = (c & 3) * 8;
      const bool ka = k0 + kc < K;
      const int ar = m0 + r, br = n0 + r;
      cp_async16(As + (stage * BM + r) * LDS + kc, A + size_t(min(ar, M - 1)) * K + (ka ? k0 + kc : 0),
                 ka && ar < M);
      cp_async16(Bs + (stage * BN + r) * LDS + kc, W + size_t(min(br, N - 1)) * K + (ka ? k0 + kc : 0),
                 ka && br < N);
    }
  };

  float acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < KT) load(s, s);
    cp_async_commit();
  }
  for (int kt = 0; kt < KT; ++kt) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    if (kt + STAGES - 1 < KT) load((kt + STAGES - 1) % STAGES, kt + STAGES - 1);
    cp_async_commit();
    const int st = kt % STAGES;
    const bf16 *as = As + st * BM * LDS, *bs = Bs + st * BN * LDS;
#pragma unroll
    for (int ks = 0; ks < BK; ks += 16) {
      uint32_t af[4][4], bfr[4][2];
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        const int r = wm * 64 + mt * 16 + (lane & 15), c = ks + (lane >> 4) * 8;
        ldmatrix_x4(af[mt][0], af[mt][1], af[mt][2], af[mt][3], as + r * LDS + c);
      }
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int r = wn * 32 + np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks + ((lane >> 3) & 1) * 8;
        ldmatrix_x4(bfr[2 * np][0], bfr[2 * np][1], bfr[2 * np + 1][0], bfr[2 * np + 1][1],
                    bs + r * LDS + c);
      }
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma_bf16(acc[mt][nt], af[mt], bfr[nt]);
    }
  }
  cp_async_wait<0>();

#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = m0 + wm * 64 + mt * 16 + (lane >> 2) + half * 8;
      if (r >= M) continue;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int c = n0 + wn * 32 + nt * 8 + (lane & 3) * 2;
        if (c >= N) continue;
        const float v0 = acc[mt][nt][half * 2], v1 = acc[mt][nt][half * 2 + 1];
        if (EPI == kEpiSwiGLU) {
          const float gate = rbf(v0), up = rbf(v1);
          C[size_t(r) * ldc + (c >> 1)] = f2bf(rbf(silu_f32(gate)) * up);
        } else if (EPI == kEpiResidual) {
          bf16 *o = C + size_t(r) * ldc + c;
          o[0] = f2bf(bf2f(o[0]) + rbf(v0));
          o[1] = f2bf(bf2f(o[1]) + rbf(v1));
        } else {
          bf16 *o = C + size_t(r) * ldc + c;
          o[0] = f2bf(v0);
          o[1] = f2bf(v1);
        }
      }
    }
}

template <int EPI>
static void gemm_launch(const bf16 *A, int M, int K, const bf16 *W, int N, bf16 *C, int ldc,
                        cudaStream_t st) {
  const size_t smem = size_t(STAGES) * (BM + BN) * LDS * sizeof(bf16);
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  k_gemm<EPI><<<grid, 256, smem, st>>>(A, M, K, W, N, C, ldc);
  YAR_CUDA(cudaGetLastError());
}

void configure_gemm_kernels() {
  const int smem = int(size_t(STAGES) * (BM + BN) * LDS * sizeof(bf16));
  YAR_CUDA(cudaFuncSetAttribute(k_gemm<kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  YAR_CUDA(cudaFuncSetAttribute(k_gemm<kEpiResidual>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  YAR_CUDA(cudaFuncSetAttribute(k_gemm<kEpiSwiGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
}

void launch_gemm(const bf16 *A, int M, int K, const bf16 *W, int N, bf16 *C, int ldc, int epilogue,
                 cudaStream_t st) {
  if (K % 8 != 0 || N % 2 != 0) throw Error("ValueError", "GEMM needs K % 8 == 0 and even N");
  if (epilogue == kEpiSwiGLU) return gemm_launch<kEpiSwiGLU>(A, M, K, W, N, C, ldc, st);
  if (epilogue == kEpiResidual) return gemm_launch<kEpiResidual>(A, M, K, W, N, C, ldc, st);
  return gemm_launch<kEpiStore>(A, M, K, W, N, C, ldc, st);
}

}  // namespace yar
