// kernels_gemv_tma.cu — decode GEMV with the weight stream staged through shared memory
// by bulk asynchronous copies (cp.async.bulk, the TMA engine's linear mode) and mbarriers.
//
// Same operator and fusions as kernels_gemv.cu (RMSNorm prologue; store / residual /
// SwiGLU epilogue; reference ops native/src/ar.cpp:20-51, :266-298), for K a multiple of
// 2048 and one or two activation rows (bs1 and a CFG pair).
//
// One CTA per SM: 8 consumer warps + 1 producer warp. The CTA owns a contiguous range of
// 8-row groups; a group is streamed as K/2048 stages, each 8 row pieces of 2048 BF16
// (4 KB, contiguous in the row-major matrix) = 32 KB. A 3-stage ring keeps 96 KB per SM in
// flight without holding registers. The producer starts copying before
// griddepcontrol.wait (weights do not depend on the previous kernel), so a kernel's first
// 96 KB per SM arrive while its predecessor finishes; 96 KB of stages + the activations
// leave room for the next kernel's CTA on the same SM.
//
// Every mbarrier wait is bounded; on expiry the kernel records an error code and stops
// issuing work, and the producer drains the copies it issued before exiting.
#include "common.cuh"

namespace yar {

constexpr int kTmaConsumers = 8;
constexpr int kTmaThreads = (kTmaConsumers + 1) * 32;
constexpr int kTmaStages = 3;
constexpr int kTmaPiece = 2048;                      // BF16 elements per row piece
constexpr int kTmaStageBytes = 8 * kTmaPiece * 2;    // 32 KB
constexpr long long kWaitLimit = 1ll << 26;          // ~seconds of try_wait polling

struct TmaGemvParams {
  const bf16 *W;
  int N, K;
  const bf16 *in;
  int in_stride;
  const bf16 *norm_w;
  float eps;
  bf16 *out;
  int out_stride;
  int *error;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded wait for the barrier phase with the given parity; false on expiry.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity) {
  const uint32_t a = smem_u32(bar);
  for (long long i = 0; i < kWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kTmaConsumers * 32) : "memory");
}

template <int NB, int EPI>
__global__ void __launch_bounds__(kTmaThreads, 1) k_gemv_tma(TmaGemvParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16 *stage = reinterpret_cast<bf16 *>(smem_raw);                               // [S][8][2048]
  bf16 *act = reinterpret_cast<bf16 *>(smem_raw + kTmaStages * kTmaStageBytes);  // [NB][K]
  __shared__ __align__(8) uint64_t full[kTmaStages], empty[kTmaStages];
  __shared__ float red[NB][kTmaConsumers];
  __shared__ float rowres[NB][8];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int K = p.K, KS = K / kTmaPiece;  // stages per 8-row group
  const int groups = (p.N + 7) / 8;
  const int g0 = int((long long)blockIdx.x * groups / gridDim.x);
  const int g1 = int((long long)(blockIdx.x + 1) * groups / gridDim.x);
  const int nst = (g1 - g0) * KS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTmaStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTmaConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kTmaConsumers) {
    // Producer: one lane issues every copy; the weights are ready before the wait.
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nst; ++i) {
        const int s = i % kTmaStages;
        if (i >= kTmaStages && !mbar_wait(&empty[s], ((i / kTmaStages) - 1) & 1)) {
          atomicOr(p.error, 4);
          break;
        }
        const int g = g0 + i / KS, ks = i % KS;
        const int r0 = g * 8, nrows = min(8, p.N - r0);
        mbar_arrive_expect_tx(&full[s], unsigned(nrows) * kTmaPiece * 2);
        for (int r = 0; r < nrows; ++r)
          bulk_g2s(stage + (size_t(s) * 8 + r) * kTmaPiece, p.W + size_t(r0 + r) * K + size_t(ks) * kTmaPiece,
                   kTmaPiece * 2, &full[s]);
        issued = i + 1;
      }
      // Never leave with copies in flight: wait (bounded) for the last stages issued.
      for (int i = max(0, issued - kTmaStages); i < issued; ++i) mbar_wait(&full[i % kTmaStages], (i / kTmaStages) & 1);
    }
    pdl_wait();
    return;
  }

  // Consumers: stage the (optionally normalized) activation rows.
  pdl_wait();
  const int ctid = threadIdx.x;  // 0 .. 255
  if (p.norm_w) {
    for (int b = 0; b < NB; ++b) {
      const bf16 *x = p.in + size_t(b) * p.in_stride;
      float ss = 0.f;
      for (int k = ctid * 8; k < K; k += kTmaConsumers * 32 * 8) {
        const uint4 v = ldg16(x + k);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = bf_lo(w4[j]), c = bf_hi(w4[j]);
          ss += a * a + c * c;
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) red[b][warp] = ss;
    }
    consumer_sync();
    for (int b = 0; b < NB; ++b) {
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < kTmaConsumers; ++i) tot += red[b][i];
      const float scale = rms_scale_bf16(tot, K, p.eps);
      const bf16 *x = p.in + size_t(b) * p.in_stride;
      for (int k = ctid * 8; k < K; k += kTmaConsumers * 32 * 8) {
        const uint4 v = ldg16(x + k), wn = ldg16(p.norm_w + k);
        const uint32_t xv[4] = {v.x, v.y, v.z, v.w}, wv[4] = {wn.x, wn.y, wn.z, wn.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float lo = rbf(rbf(bf_lo(xv[j]) * scale) * bf_lo(wv[j]));
          const float hi = rbf(rbf(bf_hi(xv[j]) * scale) * bf_hi(wv[j]));
          o[j] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xFFFF0000u);
        }
        *reinterpret_cast<uint4 *>(act + b * K + k) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  } else {
    for (int b = 0; b < NB; ++b) {
      const bf16 *x = p.in + size_t(b) * p.in_stride;
      for (int c = ctid; c < K / 8; c += kTmaConsumers * 32)
        *reinterpret_cast<uint4 *>(act + b * K + c * 8) = ldg16(x + c * 8);
    }
  }
  consumer_sync();

  float acc[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.f;
  // After a wait expires this warp stops waiting and computing but still takes part in
  // every consumer barrier, so no warp is left waiting on it.
  bool bad = false;
  for (int i = 0; i < nst; ++i) {
    const int s = i % kTmaStages;
    if (!bad && !mbar_wait(&full[s], (i / kTmaStages) & 1)) {
      if (lane == 0) atomicOr(p.error, 8);
      bad = true;
    }
    const int g = g0 + i / KS, ks = i % KS;
    const int row = g * 8 + warp;
    if (!bad && row < p.N) {
      const bf16 *wr = stage + (size_t(s) * 8 + warp) * kTmaPiece;
      const bf16 *ar = act + size_t(ks) * kTmaPiece;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int c = lane + 32 * t;
        const uint4 wq = *reinterpret_cast<const uint4 *>(wr + c * 8);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const uint4 av = *reinterpret_cast<const uint4 *>(ar + size_t(b) * K + c * 8);
          float v = acc[b];
          v = fmaf(bf_lo(wq.x), bf_lo(av.x), v);
          v = fmaf(bf_hi(wq.x), bf_hi(av.x), v);
          v = fmaf(bf_lo(wq.y), bf_lo(av.y), v);
          v = fmaf(bf_hi(wq.y), bf_hi(av.y), v);
          v = fmaf(bf_lo(wq.z), bf_lo(av.z), v);
          v = fmaf(bf_hi(wq.z), bf_hi(av.z), v);
          v = fmaf(bf_lo(wq.w), bf_lo(av.w), v);
          v = fmaf(bf_hi(wq.w), bf_hi(av.w), v);
          acc[b] = v;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (ks != KS - 1) continue;
    // End of an 8-row group: reduce each warp's row, then the epilogue for the group.
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const float v = warp_sum(acc[b]);
      if (lane == 0) rowres[b][warp] = v;
      acc[b] = 0.f;
    }
    consumer_sync();
    const int r0 = g * 8;
    if (EPI == kEpiSwiGLU) {
      if (ctid < 4 * NB) {
        const int b = ctid / 4, j = ctid % 4;  // pair j of the group: rows 2j (gate), 2j+1 (up)
        if (r0 + 2 * j + 1 < p.N) {
          const float gate = rbf(rowres[b][2 * j]), up = rbf(rowres[b][2 * j + 1]);
          p.out[size_t(b) * p.out_stride + (r0 >> 1) + j] = f2bf(rbf(silu_f32(gate)) * up);
        }
      }
    } else if (ctid < 8 * NB) {
      const int b = ctid / 8, r = ctid % 8;
      if (r0 + r < p.N) {
        bf16 *o = p.out + size_t(b) * p.out_stride + r0 + r;
        if (EPI == kEpiResidual)
          *o = f2bf(bf2f(*o) + rbf(rowres[b][r]));
        else
          *o = f2bf(rowres[b][r]);
      }
    }
    consumer_sync();
  }
}

size_t gemv_tma_smem(int NB, int K) { return size_t(kTmaStages) * kTmaStageBytes + size_t(NB) * K * 2; }

template <int NB, int EPI>
static void tma_launch(const TmaGemvParams &p, int sm_count, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count);
  cfg.blockDim = dim3(kTmaThreads);
  cfg.dynamicSmemBytes = gemv_tma_smem(NB, p.K);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  YAR_CUDA(cudaLaunchKernelEx(&cfg, k_gemv_tma<NB, EPI>, p));
}

void configure_gemv_tma_kernels() {
  const int bytes = int(gemv_tma_smem(2, 6144));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv_tma<1, kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv_tma<1, kEpiResidual>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv_tma<1, kEpiSwiGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv_tma<2, kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv_tma<2, kEpiResidual>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv_tma<2, kEpiSwiGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

// Returns false when the shape is not handled here (the caller uses another kernel).
bool launch_gemv_tma(const bf16 *W, int N, int K, const bf16 *in, int in_stride, const bf16 *norm_w, float eps,
                     bf16 *out, int out_stride, int epilogue, int n_rows, int *error, int sm_count,
                     cudaStream_t st) {
  if (K % kTmaPiece != 0 || n_rows < 1 || n_rows > 2) return false;
  if ((reinterpret_cast<uintptr_t>(W) & 15) != 0) return false;
  if (epilogue == kEpiSwiGLU && (N % 2) != 0) return false;
  TmaGemvParams p{W, N, K, in, in_stride, norm_w, eps, out, out_stride, error};
  if (n_rows == 1) {
    if (epilogue == kEpiSwiGLU) tma_launch<1, kEpiSwiGLU>(p, sm_count, st);
    else if (epilogue == kEpiResidual) tma_launch<1, kEpiResidual>(p, sm_count, st);
    else tma_launch<1, kEpiStore>(p, sm_count, st);
  } else {
    if (epilogue == kEpiSwiGLU) tma_launch<2, kEpiSwiGLU>(p, sm_count, st);
    else if (epilogue == kEpiResidual) tma_launch<2, kEpiResidual>(p, sm_count, st);
    else tma_launch<2, kEpiStore>(p, sm_count, st);
  }
  return true;
}

}  // namespace yar
