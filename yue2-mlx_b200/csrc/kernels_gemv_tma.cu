// kernels_gemv_tma.cu — decode GEMV with the weight stream staged through shared memory
// by TMA tensor copies (one 32 KB stage per copy, tma_ring.cuh) and mbarriers.
//
// Same operator and fusions as kernels_gemv.cu (RMSNorm prologue; store / residual /
// SwiGLU epilogue; reference ops native/src/ar.cpp:20-51, :266-298), for K a multiple of
// 2048 and one or two activation rows (bs1 and a CFG pair).
//
// One CTA per SM: 8 consumer warps + 1 producer warp. The CTA owns a contiguous range of
// 8-row groups; a group is streamed as K/2048 stages of 8 rows x 2048 BF16 = 32 KB. A
// 3-stage ring keeps 96 KB per SM in flight without holding registers. The producer starts
// copying before griddepcontrol.wait (weights do not depend on the previous kernel), so a
// kernel's first 96 KB per SM arrive while its predecessor finishes; 96 KB of stages + the
// activations leave room for the next kernel's CTA on the same SM.
//
// Every mbarrier wait is bounded; on expiry the kernel records an error code and stops
// issuing work, and the producer drains the copies it issued before exiting.
#include "tma_ring.cuh"

namespace yar {

constexpr int kTmaThreads = (kRingConsumers + 1) * 32;
constexpr int kTmaStages = 3;

struct TmaGemvParams {
  CUtensorMap wmap;  // the weight's stage map (encode_stage_map)
  GemvTask t;
  int *error;
};

template <int NB, int EPI>
__global__ void __launch_bounds__(kTmaThreads, 1) k_gemv_tma(const __grid_constant__ TmaGemvParams p) {
  // 1024-byte alignment: the stages are 128-byte-swizzled tensor copies.
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  bf16 *ring = reinterpret_cast<bf16 *>(smem_raw);                                  // [S][8 x 2048]
  bf16 *act = reinterpret_cast<bf16 *>(smem_raw + kTmaStages * kRingStageBytes);  // [NB][K]
  __shared__ __align__(8) uint64_t full[kTmaStages], empty[kTmaStages];
  __shared__ float red[NB * kRingConsumers];
  GemvTask t = p.t;
  t.wmap = &p.wmap;
  float *gred = reinterpret_cast<float *>(smem_raw + kTmaStages * kRingStageBytes + size_t(NB) * t.K * 2);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if ((smem_u32(ring) & 1023) != 0) {  // never copy into a misaligned ring
    if (threadIdx.x == 0) atomicOr(p.error, 1);
    return;
  }
  int g0, g1;
  task_groups(t.N, blockIdx.x, gridDim.x, g0, g1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTmaStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRingConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kRingConsumers) {
    // Producer: the weights do not depend on the previous kernel, so copying starts
    // before the wait.
    if (lane == 0) {
      long long it = 0;
      ring_produce<kTmaStages>(t, g0, g1, ring, full, empty, it, p.error);
      ring_drain<kTmaStages>(full, it);
    }
    pdl_wait();
    return;
  }
  pdl_wait();
  ring_stage_act<NB>(t, act, red, threadIdx.x);
  long long it = 0;
  bool bad = false, dead = false;
  ring_consume<NB, kTmaStages>(t, g0, g1, ring, act, full, empty, it, gred, p.error, bad, dead, threadIdx.x);
}

size_t gemv_tma_smem(int NB, int K) {
  return size_t(kTmaStages) * kRingStageBytes + size_t(NB) * K * 2 + size_t(ring_gred_floats(NB)) * 4;
}

template <int NB, int EPI>
static void tma_launch(const TmaGemvParams &p, int sm_count, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count);
  cfg.blockDim = dim3(kTmaThreads);
  cfg.dynamicSmemBytes = gemv_tma_smem(NB, p.t.K);
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
  if (K % kRingPiece != 0 || K > kStageMaxK || n_rows < 1 || n_rows > 2) return false;
  if ((reinterpret_cast<uintptr_t>(W) & 15) != 0) return false;
  if (epilogue == kEpiSwiGLU && (N % 2) != 0) return false;
  TmaGemvParams p{};
  p.t = GemvTask{W, N, K, in, in_stride, norm_w, eps, out, out_stride, epilogue};
  p.error = error;
  encode_stage_map(&p.wmap, W, N, K);
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
