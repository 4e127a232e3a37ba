// kernels_attn_tc.cu — causal prefill attention (head_dim 128) on the 5th-generation tensor
// cores: tcgen05.mma with both products accumulating in tensor memory, K/V tiles brought
// by TMA straight from the paged KV cache, the tensor pipe working on one tile while the
// softmax threads work on the next.
//
// The same queries, keys, causal rule and FP32 softmax as k_attn_prefill_mma (modeling_yue2
// .py:174-213: scale head_dim^-0.5 in FP32, FP32 softmax, FP32 P.V): one CTA per 128 queries
// of one query head. Warps 0..3 are the softmax threads, thread t owning query row t (=
// TMEM lane t); lane 0 of warp 4 issues every copy and MMA. Per tile j of 64 keys (both in
// one KV page: pages hold a multiple of 64 positions):
//   * the issue lane has TMA load the tile's K and V rows ({64, 64} boxes, 128-byte swizzle,
//     two per matrix) into one of four stages, up to four tiles ahead;
//   * it issues S_j = Q K_j^T (M = 128 queries, N = 64 keys, K = 128 dims: 8 tcgen05.mma
//     kind::f16, BF16 in, FP32 out) into one of two 64-column TMEM buffers, two tiles ahead
//     of the softmax, and commits it;
//   * thread t reads its 64 scores (tcgen05.ld), masks them (tiles on the diagonal only),
//     scales them into log2 units, and writes P = 2^(s - m) as BF16 high and low parts (P keeps ~16 significant bits)
//     into one of two pairs of swizzled 128 x 64 operand tiles. m is the row's running
//     maximum, raised only when a tile's maximum exceeds it by more than 8 (so P <= 256);
//     when it is raised the thread rescales its sum l and, once the previous P.V has
//     landed, its row of O in tensor memory by 2^(m_old - m_new). O / l is the same
//     quotient whichever m the terms share;
//   * the issue lane then adds P_hi V + P_lo V (M = 128, N = 128 dims, K = 64 keys; V read
//     in place as an MN-major operand) into O in TMEM columns 128..255.
// O / l is finally stored as BF16 for query rows below T. Keys past the last visible one
// are masked out of S, and their V rows in the last tile are zeroed, so that P = 0 meets a
// finite V. Every wait is bounded: on expiry the CTA records an error word, issues nothing
// more, waits (bounded) for what it issued, frees its tensor memory and exits.
#include <cuda.h>

#include "attn_decode.cuh"
#include "common.cuh"

namespace yar {

namespace {
constexpr int kAtBQ = 128, kAtBK = 64, kAtD = 128, kAtStages = 4;
constexpr int kAtSoftmax = 128, kAtThreads = kAtSoftmax + 32;  // softmax warps + the issue warp
constexpr int kAtSlice = 128 * 128;  // 128 rows x 128 bytes: one 64-wide K slice of 128 rows
constexpr int kAtKV = kAtBK * 128;   // 64 rows x 128 bytes: one 64-dim slice of a K or V tile
constexpr int kAtStage = 4 * kAtKV;  // K (two slices) + V (two slices): 32 KB
constexpr int kAtOffQ = 0;           // Q: two slices (dims 0..63, 64..127)
constexpr int kAtOffKV = 2 * kAtSlice;
constexpr int kAtOffP = kAtOffKV + kAtStages * kAtStage;  // two buffers of (P high, P low)
constexpr int kAtSmem = kAtOffP + 4 * kAtSlice + 1024;   // + alignment slack: 230,400 bytes
constexpr long long kAtWaitLimit = 1ll << 24;
constexpr float kAtRescale = 8.f;  // raise m when a tile's max exceeds it by more (log2 units)
// Instruction descriptors, kind::f16: FP32 accumulator, BF16 A and B, A K-major, N >> 3 at
// bit 17, M >> 4 at bit 24; S reads B (K) K-major, P.V reads B (V) MN-major (bit 16).
constexpr uint32_t kAtIdescS = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kAtBK >> 3) << 17) |
                               (uint32_t(kAtBQ >> 4) << 24);
constexpr uint32_t kAtIdescO = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | (uint32_t(kAtD >> 3) << 17) |
                               (uint32_t(kAtBQ >> 4) << 24);
constexpr uint32_t kAtColsO = 128, kAtTmemCols = 256;  // S buffers at columns 0 and 64

__device__ __forceinline__ uint32_t at_smem(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ bool at_wait(uint64_t *bar, unsigned parity) {
  for (long long i = 0; i < kAtWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(at_smem(bar)), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}
__device__ __forceinline__ void at_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(at_smem(bar)) : "memory");
}
// Matrix descriptor of a K-major operand tile in the 128-byte-swizzled layout (rows of 128
// bytes, 8-row atoms 1024 bytes apart); the k-th 16-element step starts 32 bytes further.
__device__ __forceinline__ uint64_t at_desc(const void *tile) {
  return (uint64_t(at_smem(tile) >> 4) & 0x3FFFull) | (1ull << 16) | (uint64_t(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}
// Matrix descriptor of an MN-major operand in the same swizzled layout: each 128-byte row
// holds 64 consecutive MN elements of one k, 8-row groups along k lie 1024 bytes apart
// (stride byte offset) and the next 64 MN elements one 8 KB slice further (leading byte
// offset). A 16-step along k starts two groups (2048 bytes) further.
__device__ __forceinline__ uint64_t at_desc_mn(const void *tile) {
  return (uint64_t(at_smem(tile) >> 4) & 0x3FFFull) | (uint64_t(kAtKV >> 4) << 16) | (uint64_t(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}
// 2^x by the PTX approximate base-2 exponential (relative error below 2^-22; 2^-inf = 0).
__device__ __forceinline__ float at_ex2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Byte offset of 16-byte chunk c (elements 8c..8c+7) of row r in that layout.
__device__ __forceinline__ int at_sw(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }
__device__ __forceinline__ void at_mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void at_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(at_smem(bar))
               : "memory");
}
// 32 consecutive FP32 columns of this warp's 32 TMEM lanes (thread = lane); the wait is in
// the same statement, so no use of the values can be scheduled before it.
__device__ __forceinline__ void at_ld32(uint32_t addr, float *v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      "\n tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 64 consecutive columns: two loads in flight, one wait.
__device__ __forceinline__ void at_ld64(uint32_t addr, float *v) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];"
      "\n "
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, "
      "%44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, "
      "[%65];"
      "\n tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(addr), "r"(addr + 32)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
// Store 32 FP32 columns of this warp's lanes and wait for the store.
__device__ __forceinline__ void at_st32(uint32_t addr, const float *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      "\n tcgen05.wait::st.sync.aligned;"
      ::"r"(addr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
}  // namespace

struct PrefillTcParams {
  AttnGeom g;
  int layer, start, T;
  const int *ptab;  // the row's page table
  const bf16 *q;    // [T][heads][D]
  bf16 *out;        // token t, head h at out[t * out_stride + h * D]
  int out_stride;
  int *error;
};

__global__ void __launch_bounds__(kAtThreads, 1)
    k_attn_prefill_tc(const __grid_constant__ CUtensorMap kv_map, PrefillTcParams p) {
  extern __shared__ unsigned char at_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(at_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t kv_full[kAtStages], s_done[2], p_ready[2], o_done[2], drain;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int s_fail;
  const AttnGeom &g = p.g;
  const int t = threadIdx.x, warp = t >> 5;
  const int h = blockIdx.y, kvh = h / (g.heads / g.kv_heads), q0 = blockIdx.x * kAtBQ;
  const int kend = p.start + min(p.T, q0 + kAtBQ);  // keys visible to the tile's last query
  const int ntiles = (kend + kAtBK - 1) / kAtBK;

  if (t == 0) {
    for (int s = 0; s < kAtStages; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(at_smem(&kv_full[s])));
    for (int b = 0; b < 2; ++b) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(at_smem(&s_done[b])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(at_smem(&p_ready[b])), "r"(kAtSoftmax));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(at_smem(&o_done[b])));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(at_smem(&drain)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_fail = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(at_smem(&tmem_slot)),
                 "r"(kAtTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  // Q rows into the two swizzled slices (row t = query q0 + t; zeros past T).
  if (t < kAtSoftmax) {
    const bf16 *qr = p.q + (size_t(q0 + t) * g.heads + h) * kAtD;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint4 v = q0 + t < p.T ? *reinterpret_cast<const uint4 *>(qr + c * 8) : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4 *>(sm + kAtOffQ + (c >> 3) * kAtSlice + at_sw(t, c & 7)) = v;
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  auto stage = [&](int j) { return sm + kAtOffKV + (j % kAtStages) * kAtStage; };
  auto pbuf = [&](int j) { return sm + kAtOffP + (j & 1) * 2 * kAtSlice; };

  if (warp == kAtSoftmax / 32) {
    // ---- the issue lane: copies and MMAs -------------------------------------------------
    if ((t & 31) == 0) {
      // Key row of position kp in the pool seen as [rows][128] (K: kv = 0, V: kv = 1).
      auto pool_row = [&](int kv, int kp) -> int {
        const int page = p.ptab[kp >> g.page_shift], slot = kp & (g.page_tokens - 1);
        return int(((size_t(p.layer) * g.num_pages + page) * 2 + kv) * (size_t(g.kv_heads) * g.page_tokens) +
                   size_t(kvh) * g.page_tokens + slot);
      };
      int loaded = 0;  // tiles whose copies have been issued
      auto issue_tile = [&](int j) {
        unsigned char *st = stage(j);
        uint64_t *bar = &kv_full[j % kAtStages];
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(at_smem(bar)), "r"(kAtStage)
                     : "memory");
        for (int kv = 0; kv < 2; ++kv) {
          const int y = pool_row(kv, j * kAtBK);
          for (int x = 0; x < 2; ++x)
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
                "%4}], [%2];" ::"r"(at_smem(st + (2 * kv + x) * kAtKV)),
                "l"(&kv_map), "r"(at_smem(bar)), "r"(x * 64), "r"(y)
                : "memory");
        }
        loaded = j + 1;
      };
      // S_j = Q K_j^T into TMEM columns 64 (j & 1).., once tile j has landed.
      auto issue_s = [&](int j) -> bool {
        if (!at_wait(&kv_full[j % kAtStages], unsigned(j / kAtStages) & 1u)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const unsigned char *st = stage(j);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t a = at_desc(sm + kAtOffQ + (ks >> 2) * kAtSlice) + 2 * (ks & 3);
          const uint64_t b = at_desc(st + (ks >> 2) * kAtKV) + 2 * (ks & 3);
          at_mma(tmem + uint32_t(j & 1) * kAtBK, a, b, kAtIdescS, uint32_t(ks != 0));
        }
        at_commit(&s_done[j & 1]);
        return true;
      };
      for (int i = 0; i < min(kAtStages, ntiles); ++i) issue_tile(i);
      bool fail = !issue_s(0) || (ntiles > 1 && !issue_s(1));
      for (int j = 0; j < ntiles && !fail; ++j) {
        // P_j written (and, for the last tile, V's rows past kend zeroed) by all 128 threads.
        if (s_fail || !at_wait(&p_ready[j & 1], unsigned(j >> 1) & 1u)) {
          fail = true;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const unsigned char *st = stage(j), *pb = pbuf(j);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t a = at_desc(pb + (ks >> 2) * kAtSlice) + 2 * (ks & 3);
          const uint64_t b = at_desc_mn(st + 2 * kAtKV) + uint64_t(ks & 3) * (2048 >> 4);
          at_mma(tmem + kAtColsO, a, b, kAtIdescO, uint32_t(j > 0 || ks > 0));
        }
        at_commit(&o_done[j & 1]);
        if (j + 2 < ntiles && !issue_s(j + 2)) {
          fail = true;
          break;
        }
        if (j + kAtStages < ntiles) {  // P.V_j has read stage j: refill it
          if (!at_wait(&o_done[j & 1], unsigned(j >> 1) & 1u)) {
            fail = true;
            break;
          }
          issue_tile(j + kAtStages);
        }
      }
      if (fail) {
        // Issue nothing more; wait (bounded) for the copies and MMAs already issued.
        s_fail = 1;
        for (int i = loaded > kAtStages ? loaded - kAtStages : 0; i < loaded; ++i)
          at_wait(&kv_full[i % kAtStages], unsigned(i / kAtStages) & 1u);
        at_commit(&drain);  // arrives once every MMA this lane issued has completed
        at_wait(&drain, 0u);
        if (p.error) atomicOr(p.error, 64);
      }
    }
  } else {
    // ---- softmax threads: thread t owns query row t ----------------------------------------
    const int qpos = p.start + q0 + t;
    const float sl2 = g.scale * 1.4426950408889634f;  // scale * log2(e): scores in log2 units
    const uint32_t lanes = tmem + (uint32_t(warp * 32) << 16);
    float m = -INFINITY, l = 0.f;
    bool fail = false;
    for (int j = 0; j < ntiles; ++j) {
      bool ok = at_wait(&s_done[j & 1], unsigned(j >> 1) & 1u) &&
                at_wait(&kv_full[j % kAtStages], unsigned(j / kAtStages) & 1u);
      if (__any_sync(0xFFFFFFFFu, !ok || s_fail != 0)) {  // s_fail: the issue lane gave up
        fail = true;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float s[kAtBK];
      at_ld64(lanes + uint32_t(j & 1) * kAtBK, s);
      // The causal mask, on tiles reaching past the CTA's first query only (CTA-uniform).
      if ((j + 1) * kAtBK - 1 > p.start + q0) {
#pragma unroll
        for (int k = 0; k < kAtBK; ++k) s[k] = j * kAtBK + k <= qpos ? s[k] : -INFINITY;
      }
      // Row maximum of the raw scores in eight independent chains; the scale is positive,
      // so max(s) * sl2 is the maximum of the rounded scaled scores.
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = s[i];
#pragma unroll
      for (int k = 8; k < kAtBK; ++k) mx8[k & 7] = fmaxf(mx8[k & 7], s[k]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) *
                       sl2;
      const bool raise = mx > m + kAtRescale;  // false while both are -inf
      if (__any_sync(0xFFFFFFFFu, raise)) {
        const float mn = raise ? mx : m;
        const float c = raise ? exp2f(m - mn) : 1.f;  // 0 when m was -inf
        l *= c;
        m = mn;
        if (j > 0) {  // rescale O once P.V_{j-1} has landed (nothing later is issued yet)
          ok = at_wait(&o_done[(j - 1) & 1], unsigned((j - 1) >> 1) & 1u);
          if (__any_sync(0xFFFFFFFFu, !ok)) {
            fail = true;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
          for (int cb = 0; cb < kAtD; cb += 32) {
            float v[32];
            at_ld32(lanes + kAtColsO + cb, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= c;
            at_st32(lanes + kAtColsO + cb, v);
          }
        }
      }
      // P = 2^(s * sl2 - m) (one rounding before the exponential), summed in eight chains.
      const float nm = m == -INFINITY ? 0.f : -m;
      float ps8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) ps8[i] = 0.f;
#pragma unroll
      for (int k = 0; k < kAtBK; ++k) {
        s[k] = at_ex2(fmaf(s[k], sl2, nm));  // masked: 2^-inf = 0
        ps8[k & 7] += s[k];
      }
      l += ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
      // P buffer j & 1 was last read by P.V_{j-2}.
      if (j >= 2) {
        ok = at_wait(&o_done[j & 1], unsigned((j - 2) >> 1) & 1u);
        if (__any_sync(0xFFFFFFFFu, !ok)) {
          fail = true;
          break;
        }
      }
      unsigned char *ph = pbuf(j), *pl = ph + kAtSlice;
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = s[cc * 8 + 2 * e], y = s[cc * 8 + 2 * e + 1];
          const __nv_bfloat162 hi = __floats2bfloat162_rn(x, y);
          hw[e] = *reinterpret_cast<const uint32_t *>(&hi);
          const __nv_bfloat162 lo =
              __floats2bfloat162_rn(x - __uint_as_float(hw[e] << 16), y - __uint_as_float(hw[e] & 0xFFFF0000u));
          lw[e] = *reinterpret_cast<const uint32_t *>(&lo);
        }
        *reinterpret_cast<uint4 *>(ph + at_sw(t, cc)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4 *>(pl + at_sw(t, cc)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
      // The last tile's V rows at or past kend: zeros (their P is 0; the rows may hold any bits).
      const int r0 = kend - j * kAtBK;
      if (r0 < kAtBK) {
        unsigned char *v = stage(j) + 2 * kAtKV;
        const int per = (kAtBK - r0) * 8;  // 16-byte chunks per slice
        for (int i = t; i < 2 * per; i += kAtSoftmax)
          *reinterpret_cast<uint4 *>(v + (i / per) * kAtKV + (r0 + (i % per) / 8) * 128 + (i % 8) * 16) =
              make_uint4(0, 0, 0, 0);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      at_arrive(&p_ready[j & 1]);
    }
    if (!fail) {
      const bool ok = at_wait(&o_done[(ntiles - 1) & 1], unsigned((ntiles - 1) >> 1) & 1u);
      fail = __any_sync(0xFFFFFFFFu, !ok);
    }
    if (fail) {
      s_fail = 1;
      if ((t & 31) == 0 && p.error) atomicOr(p.error, 64);
    } else {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const float inv = 1.0f / l;
      bf16 *dst = p.out + size_t(q0 + t) * p.out_stride + h * kAtD;
#pragma unroll
      for (int cb = 0; cb < kAtD; cb += 32) {
        float v[32];
        at_ld32(lanes + kAtColsO + cb, v);
        if (q0 + t < p.T) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_bfloat162 o2 = __floats2bfloat162_rn(v[c * 8 + 2 * e] * inv, v[c * 8 + 2 * e + 1] * inv);
              w[e] = *reinterpret_cast<const uint32_t *>(&o2);
            }
            *reinterpret_cast<uint4 *>(dst + cb + c * 8) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAtTmemCols));
}

void configure_attn_tc_kernels() {
  YAR_CUDA(cudaFuncSetAttribute(k_attn_prefill_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kAtSmem));
}

bool launch_attn_prefill_tc(const Model &m, Session &s, const AttnGeom &g, int layer, int row, int start, int T,
                            cudaStream_t st) {
  if (g.head_dim != kAtD || g.page_tokens % kAtBK != 0) return false;
  const uint64_t rows = uint64_t(m.d.layers) * s.num_pages * 2 * s.kv_page_elems / kAtD;
  if (rows >= (uint64_t(1) << 31)) return false;
  CUtensorMap map;
  if (!encode_rows128_map(&map, s.kv, rows)) return false;
  PrefillTcParams p;
  p.g = g;
  p.layer = layer;
  p.start = start;
  p.T = T;
  p.ptab = s.d_page_table + size_t(row) * s.pages_per_row;
  p.q = s.pq;
  p.out = s.pattn + m.tp.q_row0;
  p.out_stride = m.full.qdim();
  p.error = s.d_error;
  dim3 grid((T + kAtBQ - 1) / kAtBQ, m.d.heads);
  k_attn_prefill_tc<<<grid, kAtThreads, kAtSmem, st>>>(map, p);
  YAR_CUDA(cudaGetLastError());
  return true;
}

}  // namespace yar
