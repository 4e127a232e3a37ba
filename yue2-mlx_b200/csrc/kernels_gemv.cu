// kernels_gemv.cu — decode GEMVs y[b] = W x[b] for up to 8 rows, BF16 weights streamed
// once from HBM, FP32 accumulation, one BF16 rounding of each output.
//
// Reference ops: model_ops::linear (native/src/ar.cpp:20-28) for q/k/v, o_proj, the MLP
// projections and the LM head, with these fusions:
//   prologue  optional RMSNorm of the input rows (ar.cpp:30-35, modeling_yue2.py:131-132),
//             recomputed by every CTA from the BF16 residual (2 * K bytes per row, L2 hits);
//   epilogue  store; residual add x += bf16(Wx) (ar.cpp:292-298); SwiGLU on interleaved
//             gate/up rows, out[j] = bf16(bf16(silu_f32(g_j)) * u_j) (ar.cpp:36-51).
//
// Layout: W is row-major [N][K]; each lane reads 16-byte chunks c = lane, lane+32, ... of a
// row, so every warp load instruction covers 512 contiguous bytes. A warp owns RW
// consecutive rows at a time (RW = 2 keeps a gate/up pair in one warp). Loads of a
// row-group are issued back to back (U chunks per row) before any math so each lane has
// U*RW 16-byte requests in flight.
#include "common.cuh"

namespace yar {

struct GemvParams {
  const bf16 *W;
  int N, K;
  const bf16 *in;
  int in_stride;
  const bf16 *norm_w;
  float eps;
  bf16 *out;
  int out_stride;
};

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;

template <int NB, int RW, int EPI>
__global__ void __launch_bounds__(kGemvThreads) k_gemv(GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  bf16 *act = reinterpret_cast<bf16 *>(smem_raw);  // [NB][K]
  __shared__ float red[NB][kGemvWarps];

  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int K = p.K, nchunk = K >> 3;
  const int groups = (p.N + RW - 1) / RW;
  const int gw = blockIdx.x * kGemvWarps + warp, tw = gridDim.x * kGemvWarps;
  constexpr int U = 4;

  // Issue the first row-group's weight loads before waiting on the producer of x.
  uint4 wpre[RW][U];
  int g0 = gw;
  const bool have0 = g0 < groups;
  if (have0) {
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      const int row = min(g0 * RW + r, p.N - 1);
      const bf16 *wr = p.W + size_t(row) * K;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = lane + 32 * u;
        wpre[r][u] = c < nchunk ? ldg_stream(wr + c * 8) : make_uint4(0, 0, 0, 0);
      }
    }
  }
  pdl_wait();

  // Stage the (optionally normalized) input rows in shared memory.
  if (p.norm_w) {
    for (int b = 0; b < NB; ++b) {
      const bf16 *x = p.in + size_t(b) * p.in_stride;
      float ss = 0.f;
      for (int k = threadIdx.x * 8; k < K; k += kGemvThreads * 8) {
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
    __syncthreads();
    for (int b = 0; b < NB; ++b) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) tot += red[b][w];
      const float scale = rms_scale_bf16(tot, K, p.eps);
      const bf16 *x = p.in + size_t(b) * p.in_stride;
      for (int k = threadIdx.x; k < K; k += kGemvThreads)
        act[b * K + k] = f2bf(rbf(bf2f(x[k]) * scale) * bf2f(p.norm_w[k]));
    }
  } else {
    for (int b = 0; b < NB; ++b) {
      const bf16 *x = p.in + size_t(b) * p.in_stride;
      for (int c = threadIdx.x; c < nchunk; c += kGemvThreads)
        *reinterpret_cast<uint4 *>(act + b * K + c * 8) = ldg16(x + c * 8);
    }
  }
  __syncthreads();

  for (int g = g0; g < groups; g += tw) {
    float acc[RW][NB];
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[r][b] = 0.f;
    const bf16 *wrow[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) wrow[r] = p.W + size_t(min(g * RW + r, p.N - 1)) * K;

    for (int c0 = 0; c0 < nchunk; c0 += 32 * U) {
      uint4 wv[RW][U];
      if (g == g0 && c0 == 0) {
#pragma unroll
        for (int r = 0; r < RW; ++r)
#pragma unroll
          for (int u = 0; u < U; ++u) wv[r][u] = wpre[r][u];
      } else {
#pragma unroll
        for (int r = 0; r < RW; ++r)
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int c = c0 + lane + 32 * u;
            wv[r][u] = c < nchunk ? ldg_stream(wrow[r] + c * 8) : make_uint4(0, 0, 0, 0);
          }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + lane + 32 * u;
        if (c < nchunk) {
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            const uint4 av = *reinterpret_cast<const uint4 *>(act + b * K + c * 8);
            const float a[8] = {bf_lo(av.x), bf_hi(av.x), bf_lo(av.y), bf_hi(av.y),
                                bf_lo(av.z), bf_hi(av.z), bf_lo(av.w), bf_hi(av.w)};
#pragma unroll
            for (int r = 0; r < RW; ++r) {
              const uint4 w = wv[r][u];
              float s = acc[r][b];
              s = fmaf(bf_lo(w.x), a[0], s);
              s = fmaf(bf_hi(w.x), a[1], s);
              s = fmaf(bf_lo(w.y), a[2], s);
              s = fmaf(bf_hi(w.y), a[3], s);
              s = fmaf(bf_lo(w.z), a[4], s);
              s = fmaf(bf_hi(w.z), a[5], s);
              s = fmaf(bf_lo(w.w), a[6], s);
              s = fmaf(bf_hi(w.w), a[7], s);
              acc[r][b] = s;
            }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[r][b] = warp_sum(acc[r][b]);

    if (EPI == kEpiSwiGLU) {
      // RW == 2: row 2j is gate j, row 2j+1 is up j.
      if (lane < NB && g * 2 + 1 < p.N) {
        const int b = lane;
        float gv = 0.f, uv = 0.f;
#pragma unroll
        for (int bb = 0; bb < NB; ++bb)
          if (bb == b) {
            gv = acc[0][bb];
            uv = acc[1][bb];
          }
        const float gate = rbf(gv), up = rbf(uv);
        p.out[size_t(b) * p.out_stride + g] = f2bf(rbf(silu_f32(gate)) * up);
      }
    } else {
      if (lane < NB * RW) {
        const int b = lane % NB, r = lane / NB;
        const int row = g * RW + r;
        float v = 0.f;
#pragma unroll
        for (int rr = 0; rr < RW; ++rr)
#pragma unroll
          for (int bb = 0; bb < NB; ++bb)
            if (rr == r && bb == b) v = acc[rr][bb];
        if (row < p.N) {
          bf16 *o = p.out + size_t(b) * p.out_stride + row;
          if (EPI == kEpiResidual)
            *o = f2bf(bf2f(*o) + rbf(v));
          else
            *o = f2bf(v);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// Streaming GEMV for the pinned shapes (K = 256 * SPR * 8: 2048 or 6144). One CTA per SM
// (256 threads, <= 128 registers: half the register file, so the next kernel of the
// programmatic-launch chain can become resident and start its own loads). Each warp owns
// a contiguous range of units (one row, or one gate/up row pair) and streams them as
// "slices" — 8 chunks of 16 bytes per lane, 4 KB per warp — through a two-slice register
// ring: 16 loads of 16 bytes in flight per lane. The first two slices are requested before
// griddepcontrol.wait, so they overlap the producer kernel's tail.
template <int NB, int RW, int EPI, int SPR>
__global__ void __launch_bounds__(kGemvThreads, 1) k_gemv_stream(GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  bf16 *act = reinterpret_cast<bf16 *>(smem_raw);  // [NB][K]
  __shared__ float red[NB][kGemvWarps];
  constexpr int K = SPR * 8 * 256;
  constexpr int CPL = SPR * 8;  // chunks per lane per row
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long units = p.N / RW;
  const long long W = (long long)gridDim.x * kGemvWarps, w = (long long)blockIdx.x * kGemvWarps + warp;
  const int u0 = int(w * units / W), u1 = int((w + 1) * units / W);
  const int total = (u1 - u0) * RW * SPR;  // slices of this warp

  auto slice_ptr = [&](int sl) {
    const int row = u0 * RW + sl / SPR;   // units are RW consecutive rows
    const int j0 = (sl % SPR) * 8;        // first chunk index (per lane) of the slice
    return p.W + size_t(row) * K + size_t(lane + 32 * j0) * 8;
  };
  auto load_slice = [&](uint4 *b, int sl) {
    const bf16 *q = slice_ptr(sl);
#pragma unroll
    for (int t = 0; t < 8; ++t) b[t] = ldg_stream(q + t * 256);
  };
  uint4 buf0[8], buf1[8];
  if (total > 0) load_slice(buf0, 0);
  if (total > 1) load_slice(buf1, 1);
  pdl_wait();

  if (p.norm_w) {
    for (int b = 0; b < NB; ++b) {
      const bf16 *x = p.in + size_t(b) * p.in_stride;
      float ss = 0.f;
      for (int k = threadIdx.x * 8; k < K; k += kGemvThreads * 8) {
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
    __syncthreads();
    for (int b = 0; b < NB; ++b) {
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < kGemvWarps; ++i) tot += red[b][i];
      const float scale = rms_scale_bf16(tot, K, p.eps);
      const bf16 *x = p.in + size_t(b) * p.in_stride;
      for (int k = threadIdx.x * 8; k < K; k += kGemvThreads * 8) {
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
      for (int c = threadIdx.x; c < K / 8; c += kGemvThreads)
        *reinterpret_cast<uint4 *>(act + b * K + c * 8) = ldg16(x + c * 8);
    }
  }
  __syncthreads();

  float acc[NB], res0[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = res0[b] = 0.f;

  // Consume one slice: FMAs into acc; at the end of a row reduce across the warp, and at
  // the end of a unit apply the epilogue.
  auto consume = [&](const uint4 *bv, int sl) {
    const int j0 = (sl % SPR) * 8;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int c = lane + 32 * (j0 + t);
      const uint4 wq = bv[t];
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const uint4 av = *reinterpret_cast<const uint4 *>(act + b * K + c * 8);
        float s = acc[b];
        s = fmaf(bf_lo(wq.x), bf_lo(av.x), s);
        s = fmaf(bf_hi(wq.x), bf_hi(av.x), s);
        s = fmaf(bf_lo(wq.y), bf_lo(av.y), s);
        s = fmaf(bf_hi(wq.y), bf_hi(av.y), s);
        s = fmaf(bf_lo(wq.z), bf_lo(av.z), s);
        s = fmaf(bf_hi(wq.z), bf_hi(av.z), s);
        s = fmaf(bf_lo(wq.w), bf_lo(av.w), s);
        s = fmaf(bf_hi(wq.w), bf_hi(av.w), s);
        acc[b] = s;
      }
    }
    if (sl % SPR != SPR - 1) return;  // row continues
    const int rr = (sl / SPR) % RW;   // row within the unit
    const int unit = u0 + sl / (SPR * RW);
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = warp_sum(acc[b]);
    if (RW == 2 && rr == 0) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        res0[b] = acc[b];
        acc[b] = 0.f;
      }
      return;
    }
    if (lane < NB) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b != lane) continue;
        if (EPI == kEpiSwiGLU) {
          const float gate = rbf(res0[b]), up = rbf(acc[b]);
          p.out[size_t(b) * p.out_stride + unit] = f2bf(rbf(silu_f32(gate)) * up);
        } else {
          bf16 *o = p.out + size_t(b) * p.out_stride + unit;
          if (EPI == kEpiResidual)
            *o = f2bf(bf2f(*o) + rbf(acc[b]));
          else
            *o = f2bf(acc[b]);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
  };

  for (int sl = 0; sl < total; sl += 2) {
    consume(buf0, sl);
    if (sl + 2 < total) load_slice(buf0, sl + 2);
    if (sl + 1 < total) {
      consume(buf1, sl + 1);
      if (sl + 3 < total) load_slice(buf1, sl + 3);
    }
  }
}

template <int NB, int RW, int EPI, int SPR>
static void gemv_stream_launch(const GemvParams &p, int sm_count, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = size_t(NB) * p.K * sizeof(bf16);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  YAR_CUDA(cudaLaunchKernelEx(&cfg, k_gemv_stream<NB, RW, EPI, SPR>, p));
}

template <int NB, int SPR>
static void gemv_stream_dispatch(const GemvParams &p, int epi, int sm_count, cudaStream_t st) {
  if (epi == kEpiSwiGLU) return gemv_stream_launch<NB, 2, kEpiSwiGLU, SPR>(p, sm_count, st);
  if (epi == kEpiResidual) return gemv_stream_launch<NB, 1, kEpiResidual, SPR>(p, sm_count, st);
  return gemv_stream_launch<NB, 1, kEpiStore, SPR>(p, sm_count, st);
}

template <int NB, int SPR>
static void gemv_stream_configure() {
  const int bytes = 200 * 1024;
  YAR_CUDA(cudaFuncSetAttribute(k_gemv_stream<NB, 2, kEpiSwiGLU, SPR>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv_stream<NB, 1, kEpiResidual, SPR>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv_stream<NB, 1, kEpiStore, SPR>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

template <int NB, int RW, int EPI>
static void gemv_launch(const GemvParams &p, int sm_count, cudaStream_t st) {
  const int groups = (p.N + RW - 1) / RW;
  int grid = (groups + kGemvWarps - 1) / kGemvWarps;
  grid = grid < 2 * sm_count ? grid : 2 * sm_count;
  const size_t smem = size_t(NB) * p.K * sizeof(bf16);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  YAR_CUDA(cudaLaunchKernelEx(&cfg, k_gemv<NB, RW, EPI>, p));
}

template <int NB>
static void gemv_configure_nb() {
  const int bytes = 200 * 1024;
  YAR_CUDA(cudaFuncSetAttribute(k_gemv<NB, 2, kEpiSwiGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv<NB, 1, kEpiResidual>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv<NB, 2, kEpiResidual>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv<NB, 1, kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  YAR_CUDA(cudaFuncSetAttribute(k_gemv<NB, 2, kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  if constexpr (NB <= 2) {
    gemv_stream_configure<NB, 1>();
    gemv_stream_configure<NB, 3>();
  }
}

// Kernel attributes cannot be set while a stream is being captured; the loader calls this
// once per device before any launch.
void configure_gemv_kernels() {
  gemv_configure_nb<1>();
  gemv_configure_nb<2>();
  gemv_configure_nb<3>();
  gemv_configure_nb<4>();
  gemv_configure_nb<5>();
  gemv_configure_nb<6>();
  gemv_configure_nb<7>();
  gemv_configure_nb<8>();
}

template <int NB>
static void gemv_dispatch_epi(const GemvParams &p, int epi, int sm_count, cudaStream_t st) {
  // One or two rows (bs1, a CFG pair): the streaming kernel; more rows keep the
  // register-lighter kernel below (the streaming kernel would spill).
  if constexpr (NB <= 2) {
    if (p.K == 2048) return gemv_stream_dispatch<NB, 1>(p, epi, sm_count, st);
    if (p.K == 6144) return gemv_stream_dispatch<NB, 3>(p, epi, sm_count, st);
  }
  if (epi == kEpiSwiGLU) return gemv_launch<NB, 2, kEpiSwiGLU>(p, sm_count, st);
  // Two rows per warp when there are enough rows to fill the machine, else one.
  const bool wide = p.N / 2 >= 2 * sm_count * kGemvWarps;
  if (epi == kEpiResidual)
    return wide ? gemv_launch<NB, 2, kEpiResidual>(p, sm_count, st)
                : gemv_launch<NB, 1, kEpiResidual>(p, sm_count, st);
  return wide ? gemv_launch<NB, 2, kEpiStore>(p, sm_count, st)
              : gemv_launch<NB, 1, kEpiStore>(p, sm_count, st);
}

bool launch_gemv_tma(const bf16 *W, int N, int K, const bf16 *in, int in_stride, const bf16 *norm_w, float eps,
                     bf16 *out, int out_stride, int epilogue, int n_rows, int *error, int sm_count,
                     cudaStream_t st);

void launch_gemv(const bf16 *W, int N, int K, const bf16 *in, int in_stride, const bf16 *norm_w,
                 float eps, bf16 *out, int out_stride, int epilogue, int n_rows,
                 int *error, int sm_count, cudaStream_t st) {
  if (K % 8 != 0) throw Error("ValueError", "GEMV inner dimension must be a multiple of 8");
  if (error && launch_gemv_tma(W, N, K, in, in_stride, norm_w, eps, out, out_stride, epilogue, n_rows, error,
                               sm_count, st))
    return;
  // Rows beyond 8 are processed in groups of up to 8 (the weights are re-streamed).
  for (int r0 = 0; r0 < n_rows; r0 += 8) {
    const int nb = n_rows - r0 < 8 ? n_rows - r0 : 8;
    GemvParams p{W, N, K, in + size_t(r0) * in_stride, in_stride, norm_w, eps,
                 out + size_t(r0) * out_stride, out_stride};
    switch (nb) {
      case 1: gemv_dispatch_epi<1>(p, epilogue, sm_count, st); break;
      case 2: gemv_dispatch_epi<2>(p, epilogue, sm_count, st); break;
      case 3: gemv_dispatch_epi<3>(p, epilogue, sm_count, st); break;
      case 4: gemv_dispatch_epi<4>(p, epilogue, sm_count, st); break;
      case 5: gemv_dispatch_epi<5>(p, epilogue, sm_count, st); break;
      case 6: gemv_dispatch_epi<6>(p, epilogue, sm_count, st); break;
      case 7: gemv_dispatch_epi<7>(p, epilogue, sm_count, st); break;
      default: gemv_dispatch_epi<8>(p, epilogue, sm_count, st); break;
    }
  }
}

}  // namespace yar
