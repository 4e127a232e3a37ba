// tma_ring.cuh — the shared-memory weight ring of the decode GEMVs: bulk asynchronous
// copies (cp.async.bulk, the TMA engine's linear mode) into 32 KB stages tracked by
// mbarriers, one producer lane and eight consumer warps. Used by the standalone GEMV
// kernel and by the persistent decode kernel, which therefore compute identical bits.
//
// A GEMV task y = W x (W row-major [N][K], K a multiple of 2048) is cut into 8-row groups;
// a CTA owns groups [g0, g1) and streams each group as K/2048 stages of 8 row pieces of
// 2048 BF16 (4 KB each, contiguous). Consumer warp w computes row 8g + w; lanes read the
// piece lane-contiguously (16-byte chunks c = lane + 32t), so shared-memory reads are
// conflict-free. Every wait is bounded.
#pragma once
#include "common.cuh"

namespace yar {

constexpr int kRingConsumers = 8;
constexpr int kRingPiece = 2048;                    // BF16 elements per row piece
constexpr int kRingStageBytes = 8 * kRingPiece * 2;  // 32 KB
constexpr long long kRingWaitLimit = 1ll << 22;      // try_wait polls before giving up (seconds)

struct GemvTask {
  const bf16 *W;
  int N, K;
  const bf16 *in;  // activation rows (read through L2: other CTAs may have written them)
  int in_stride;
  const bf16 *norm_w;  // RMSNorm weight, or null
  float eps;
  bf16 *out;
  int out_stride;
  int epi;  // kEpiStore / kEpiResidual / kEpiSwiGLU
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
// Bounded wait for the phase with the given parity to complete; false on expiry.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity) {
  const uint32_t a = smem_u32(bar);
  for (long long i = 0; i < kRingWaitLimit; ++i) {
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
// Barrier 1 among the 256 consumer threads (the producer warp never joins it).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kRingConsumers * 32) : "memory");
}

__device__ __forceinline__ void task_groups(int N, int cta, int ctas, int &g0, int &g1) {
  const int groups = (N + 7) / 8;
  g0 = int((long long)cta * groups / ctas);
  g1 = int((long long)(cta + 1) * groups / ctas);
}

// Producer: issue this CTA's stages of one task, continuing the ring sequence `it`.
// Returns false (and stops) when a wait for a free stage expires.
template <int NS>
__device__ bool ring_produce(const GemvTask &t, int g0, int g1, bf16 *ring, uint64_t *full, uint64_t *empty,
                             long long &it, int *error) {
  const int KS = t.K / kRingPiece;
  for (int g = g0; g < g1; ++g)
    for (int ks = 0; ks < KS; ++ks, ++it) {
      const int s = int(it % NS);
      if (it >= NS && !mbar_wait(&empty[s], unsigned((it / NS) - 1) & 1u)) {
        atomicOr(error, 4);
        return false;
      }
      const int r0 = g * 8, nrows = min(8, t.N - r0);
      mbar_arrive_expect_tx(&full[s], unsigned(nrows) * kRingPiece * 2);
      for (int r = 0; r < nrows; ++r)
        bulk_g2s(ring + (size_t(s) * 8 + r) * kRingPiece, t.W + size_t(r0 + r) * t.K + size_t(ks) * kRingPiece,
                 kRingPiece * 2, &full[s]);
    }
  return true;
}

// Producer epilogue: never leave with copies in flight — wait (bounded) for the last NS
// stages issued to land.
template <int NS>
__device__ void ring_drain(uint64_t *full, long long issued) {
  for (long long i = issued > NS ? issued - NS : 0; i < issued; ++i) mbar_wait(&full[i % NS], unsigned(i / NS) & 1u);
}

// Consumers: the task's activation rows into `act` ([NB][K] BF16), RMSNorm applied when the
// task has a norm weight (modeling_yue2.py:131-132). `red` holds NB x 8 floats.
template <int NB>
__device__ void ring_stage_act(const GemvTask &t, bf16 *act, float *red, int ctid) {
  const int lane = ctid & 31, warp = ctid >> 5, K = t.K;
  if (t.norm_w) {
    for (int b = 0; b < NB; ++b) {
      const bf16 *x = t.in + size_t(b) * t.in_stride;
      float ss = 0.f;
      for (int k = ctid * 8; k < K; k += kRingConsumers * 32 * 8) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(x + k));
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = bf_lo(w4[j]), c = bf_hi(w4[j]);
          ss += a * a + c * c;
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) red[b * kRingConsumers + warp] = ss;
    }
    consumer_sync();
    for (int b = 0; b < NB; ++b) {
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < kRingConsumers; ++i) tot += red[b * kRingConsumers + i];
      const float scale = rms_scale_bf16(tot, K, t.eps);
      const bf16 *x = t.in + size_t(b) * t.in_stride;
      for (int k = ctid * 8; k < K; k += kRingConsumers * 32 * 8) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(x + k));
        const uint4 wn = ldg16(t.norm_w + k);
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
      const bf16 *x = t.in + size_t(b) * t.in_stride;
      for (int c = ctid; c < K / 8; c += kRingConsumers * 32)
        *reinterpret_cast<uint4 *>(act + b * K + c * 8) = __ldcg(reinterpret_cast<const uint4 *>(x + c * 8));
    }
  }
  consumer_sync();
}

// Consumers: consume the task's stages (continuing `it`), apply the epilogue per 8-row
// group. After a wait expires (`bad`), stages are still released and barriers still
// taken, without computing. `rowres` holds NB x 8 floats.
template <int NB, int NS>
__device__ void ring_consume(const GemvTask &t, int g0, int g1, const bf16 *ring, const bf16 *act, uint64_t *full,
                             uint64_t *empty, long long &it, float *rowres, int *error, bool &bad, int ctid) {
  const int lane = ctid & 31, warp = ctid >> 5, K = t.K, KS = K / kRingPiece;
  float acc[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.f;
  for (int g = g0; g < g1; ++g) {
    for (int ks = 0; ks < KS; ++ks, ++it) {
      const int s = int(it % NS);
      if (!bad && !mbar_wait(&full[s], unsigned(it / NS) & 1u)) {
        if (lane == 0) atomicOr(error, 8);
        bad = true;
      }
      const int row = g * 8 + warp;
      if (!bad && row < t.N) {
        const bf16 *wr = ring + (size_t(s) * 8 + warp) * kRingPiece;
        const bf16 *ar = act + size_t(ks) * kRingPiece;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int c = lane + 32 * q;
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
    }
    // End of an 8-row group: reduce each warp's row, then the group's epilogue.
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const float v = warp_sum(acc[b]);
      if (lane == 0) rowres[b * 8 + warp] = v;
      acc[b] = 0.f;
    }
    consumer_sync();
    const int r0 = g * 8;
    if (!bad) {
      if (t.epi == kEpiSwiGLU) {
        if (ctid < 4 * NB) {
          const int b = ctid / 4, j = ctid % 4;  // pair j of the group: rows 2j (gate), 2j+1 (up)
          if (r0 + 2 * j + 1 < t.N) {
            const float gate = rbf(rowres[b * 8 + 2 * j]), up = rbf(rowres[b * 8 + 2 * j + 1]);
            t.out[size_t(b) * t.out_stride + (r0 >> 1) + j] = f2bf(rbf(silu_f32(gate)) * up);
          }
        }
      } else if (ctid < 8 * NB) {
        const int b = ctid / 8, r = ctid % 8;
        if (r0 + r < t.N) {
          bf16 *o = t.out + size_t(b) * t.out_stride + r0 + r;
          if (t.epi == kEpiResidual)
            *o = f2bf(bf2f(__ldcg(o)) + rbf(rowres[b * 8 + r]));
          else
            *o = f2bf(rowres[b * 8 + r]);
        }
      }
    }
    consumer_sync();
  }
}

}  // namespace yar
