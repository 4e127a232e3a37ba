// tma_ring.cuh — the shared-memory weight ring of the decode GEMVs: one TMA tensor copy
// (cp.async.bulk.tensor) per 32 KB stage, tracked by mbarriers, one producer lane and eight
// consumer warps. Used by the standalone GEMV kernel and by the persistent decode kernel,
// which therefore compute identical bits.
//
// A GEMV task y = W x (W row-major [N][K], K a multiple of 2048) is cut into 8-row groups;
// a CTA owns groups [g0, g1) and streams each group as K/2048 stages of 8 rows x 2048
// columns. A stage arrives through the matrix's stage map: a 3-D view of W as {64 columns,
// N rows, K/64 column blocks} with strides {2K, 128} bytes and a {64, 8, 32} box under the
// 128-byte swizzle, so one copy moves the whole 32 KB and shared memory receives 32 blocks
// of 8 rows x 128 bytes in which row r's 16-byte chunk c sits at chunk c ^ r. The eight
// rows of an ldmatrix 8x8 matrix (one chunk of rows 0..7) then fall in eight different
// bank groups, and rows past N arrive zero-filled. (Eight 4 KB linear copies into padded
// rows take about 1.45x the time per stage: the copy engine works per request.)
// Every wait is bounded.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace yar {

constexpr int kRingConsumers = 8;
constexpr int kRingPiece = 2048;                       // columns of a stage
constexpr int kRingStageElems = 8 * kRingPiece;        // 8 rows x 2048 BF16
constexpr int kRingStageBytes = kRingStageElems * 2;   // 32 KB (the tensor copy's transaction bytes)
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
  // Tensor parallelism: every output value is also stored at out + dst[i] bytes for
  // i < n_dst — the same place in each peer rank's mapped copy of the buffer.
  int n_dst;
  const long long *dst;
  // Flagged transport (the persistent kernel): activations read from flagged words `in_ll`
  // (row stride in words) once they carry `in_flag`, outputs written as flagged words to
  // `out_ll` with `out_flag` (and to the peers' copies); a residual epilogue reads the old
  // residual words, which carry `res_flag`. Null: plain BF16 buffers (`in`, `out`).
  const uint2 *in_ll = nullptr;
  int in_ll_stride = 0;
  uint32_t in_flag = 0;
  uint2 *out_ll = nullptr;
  int out_ll_stride = 0;
  uint32_t out_flag = 0, res_flag = 0;
  long long ll_limit = 1ll << 22;  // polls of a flagged wait before it gives up
  // Flagged residual epilogue: the old residual words of this CTA's output columns
  // [res_lo, res_lo + kResKeepCols) in shared memory (row b at word b * kResKeepCols / 2),
  // read instead of polling the residual words in global memory. Null: poll.
  const uint32_t *res_smem = nullptr;
  int res_lo = 0;
  // The stage map of W (encode_stage_map), for producers that copy through it
  // (ring_produce); a kernel-parameter or global-memory address.
  const CUtensorMap *wmap = nullptr;
  // Gathered input (plain loads, when in_ll is null): row b read from in_row[b] (null:
  // zeros) instead of in + b * in_stride; the persistent kernel's first QKV reads each
  // row's token embedding this way.
  bool in_gather = false;
  const bf16 *in_row[2] = {nullptr, nullptr};
  // Per-warp staging (flagged input, no RMSNorm): ring_consume itself makes each consumer
  // warp poll and stage only its own k-range of every row, so a warp starts as soon as its
  // inputs are written (no staging barrier across the CTA); no ring_stage_act call.
  bool stage_per_warp = false;
  // Affine 8-bit weights (ring_consume_q8): W's stage image (q8_stage_image), and shared
  // memory for each 64-column group of the staged rows ([rows][K / 64]): the FP32 sum of
  // its values and the power-of-two factor of its FP16 copy. With `sumx` set the staging
  // fills both and leaves the rows in `act` as FP16 (q8_stage_chunk).
  const unsigned char *qimg = nullptr;
  float *sumx = nullptr, *qfac = nullptr, *qneg = nullptr;
};

// Host: W's stage map ({64, N, K/64} view, {64, 8, 32} box, 128-byte swizzle) into `map`.
void encode_stage_map(CUtensorMap *map, const bf16 *W, int N, int K);
constexpr int kResKeepCols = 64;  // residual columns per row a CTA can keep in shared memory

// ---------------------------------------------------------------------------------------
// Flagged words: two BF16 values (low half = the even element) and a 32-bit flag in one
// 8-byte word, written with one 8-byte store. A reader that sees the expected flag in a
// word sees that word's data (the store is single-copy atomic at 8 bytes), so a consumer
// waits by polling the data itself: no fence, no counter, no second load. The flag names
// the step and the operation that wrote the word, so words of earlier steps never match.
constexpr long long kLlWaitLimit = 1ll << 22;  // polls before giving up (about a second)

__device__ __forceinline__ void ll_store(uint2 *p, uint32_t data, uint32_t flag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(data), "r"(flag) : "memory");
}
// Store one flagged word locally and into each peer's mapped copy (byte offsets dst[i]).
__device__ __forceinline__ void ll_store_all(uint2 *p, uint32_t data, uint32_t flag, int n_dst,
                                             const long long *dst) {
  ll_store(p, data, flag);
  for (int i = 0; i < n_dst; ++i) ll_store(reinterpret_cast<uint2 *>(reinterpret_cast<char *>(p) + dst[i]), data, flag);
}
__device__ __forceinline__ uint4 ll_load2(const uint2 *p) {  // words p[0], p[1] (16-byte aligned)
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ uint2 ll_load1(const uint2 *p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ll_error_word(const int *p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Wait (bounded) for 2*NQ consecutive words at p (16-byte aligned) to carry `flag` and
// return their data halves; false when the limit passed or another CTA recorded an error.
template <int NQ>
__device__ __forceinline__ bool ll_wait(const uint2 *p, uint32_t flag, uint32_t (&data)[2 * NQ], const int *error,
                                        long long limit = kLlWaitLimit) {
  for (long long i = 0;; ++i) {
    uint4 v[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) v[q] = ll_load2(p + 2 * q);  // every load issued before any check
    uint32_t ok = 1u;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      data[2 * q] = v[q].x;
      data[2 * q + 1] = v[q].z;
      ok &= uint32_t(v[q].y == flag) & uint32_t(v[q].w == flag);
    }
    if (ok) return true;
    if (i >= limit) return false;
    if ((i & 255) == 255 && error && ll_error_word(error) != 0) return false;
    if (i >= 8) __nanosleep(32);
  }
}
__device__ __forceinline__ bool ll_wait1(const uint2 *p, uint32_t flag, uint32_t &data, const int *error,
                                         long long limit = kLlWaitLimit) {
  for (long long i = 0;; ++i) {
    const uint2 v = ll_load1(p);
    data = v.x;
    if (v.y == flag) return true;
    if (i >= limit) return false;
    if ((i & 255) == 255 && error && ll_error_word(error) != 0) return false;
    if (i >= 8) __nanosleep(32);
  }
}
__device__ __forceinline__ uint32_t pack_bf16x2(bf16 lo, bf16 hi) {
  return uint32_t(__bfloat16_as_ushort(lo)) | (uint32_t(__bfloat16_as_ushort(hi)) << 16);
}

// Store v at o and at its copies in the peers' mapped buffers.
__device__ __forceinline__ void store_all(bf16 *o, bf16 v, int n_dst, const long long *dst) {
  *o = v;
  for (int i = 0; i < n_dst; ++i) *reinterpret_cast<bf16 *>(reinterpret_cast<char *>(o) + dst[i]) = v;
}

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
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
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
// The same copy with an L2 eviction-priority policy (createpolicy).
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, unsigned bytes, uint64_t *bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// Stage (rows [row0, row0 + 8), columns [2048 ks, 2048 ks + 2048)) of a matrix through its
// stage map into `dst` (1024-byte aligned), completing kRingStageBytes on `bar`.
__device__ __forceinline__ void stage_load(bf16 *dst, const CUtensorMap *map, int row0, int ks, uint64_t *bar,
                                           uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(0), "r"(row0), "r"(ks * (kRingPiece / 64)), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// The same stage pulled into L2 only.
__device__ __forceinline__ void stage_prefetch(const CUtensorMap *map, int row0, int ks) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(map), "r"(0), "r"(row0),
               "r"(ks * (kRingPiece / 64))
               : "memory");
}
// Offset (elements) in a swizzled stage of the 16-byte chunk C (columns 8C..8C+7) of row r.
__device__ __forceinline__ int stage_chunk(int C, int r) { return (C >> 3) * 512 + r * 64 + (((C & 7) ^ r) << 3); }
// Weights are read once per token and 3 GB pass through L2 between two reads of the same
// row, so they are marked evict-first: L2 keeps the KV cache and the activations instead.
__device__ __forceinline__ uint64_t weight_stream_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// Barrier 1 among the 256 consumer threads (the producer warp never joins it).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kRingConsumers * 32) : "memory");
}

// CTA `cta`'s groups [g0, g1) of an N-row task (groups of `urows` rows: 8 for BF16 stages,
// 16 for 8-bit ones): contiguous ranges of floor or ceil of groups / ctas, the ceil ranges
// at the CTAs whose position (cta + rot) % ctas the even split gives them. `rot` lets
// consecutive operations put their extra groups on different CTAs (which group a CTA
// computes does not change the group's arithmetic).
__device__ __forceinline__ void task_groups(int N, int cta, int ctas, int &g0, int &g1, int rot = 0, int urows = 8) {
  const int groups = (N + urows - 1) / urows;
  const int pos = (cta + rot) % ctas;
  g0 = int((long long)pos * groups / ctas);
  g1 = int((long long)(pos + 1) * groups / ctas);
}

// Producer: issue this CTA's stages of one task (one stage-map copy each), continuing the
// ring sequence `it`. Returns false (and stops) when a wait for a free stage expires.
template <int NS>
__device__ bool ring_produce(const GemvTask &t, int g0, int g1, bf16 *ring, uint64_t *full, uint64_t *empty,
                             long long &it, int *error) {
  const int KS = t.K / kRingPiece;
  const uint64_t pol = weight_stream_policy();
  for (int g = g0; g < g1; ++g)
    for (int ks = 0; ks < KS; ++ks, ++it) {
      const int s = int(it % NS);
      if (it >= NS && !mbar_wait(&empty[s], unsigned((it / NS) - 1) & 1u)) {
        atomicOr(error, 4);
        return false;
      }
      mbar_arrive_expect_tx(&full[s], unsigned(kRingStageBytes));
      stage_load(ring + size_t(s) * kRingStageElems, t.wmap, g * 8, ks, &full[s], pol);
    }
  return true;
}

// Producer epilogue: never leave with copies in flight — wait (bounded) for the last NS
// stages issued to land.
template <int NS>
__device__ void ring_drain(uint64_t *full, long long issued) {
  for (long long i = issued > NS ? issued - NS : 0; i < issued; ++i) mbar_wait(&full[i % NS], unsigned(i / NS) & 1u);
}

// `red` (ring_stage_act) holds NB x 8 floats.
// Activation rows are kept in shared memory in MMA-fragment order: within every block of
// 32 elements (16 two-element words), word w sits at position (w % 4) * 4 + w / 4, so the
// four words a lane needs for two k-tiles (w = q, q + 4, q + 8, q + 12) are one 16-byte
// load. A 16-byte chunk of 8 consecutive elements (words w0..w0+3, w0 % 4 == 0) scatters to
// positions w0 / 4, + 4, + 8, + 12.
__device__ __forceinline__ void act_store_chunk(bf16 *row, int k, uint4 v) {
  uint32_t *blk = reinterpret_cast<uint32_t *>(row + (k & ~31));
  const int w0 = (k & 31) >> 1;
  blk[w0 >> 2] = v.x;
  blk[4 + (w0 >> 2)] = v.y;
  blk[8 + (w0 >> 2)] = v.z;
  blk[12 + (w0 >> 2)] = v.w;
}
__device__ __forceinline__ uint4 act_load_chunk(const bf16 *row, int k) {
  const uint32_t *blk = reinterpret_cast<const uint32_t *>(row + (k & ~31));
  const int w0 = (k & 31) >> 1;
  return make_uint4(blk[w0 >> 2], blk[4 + (w0 >> 2)], blk[8 + (w0 >> 2)], blk[12 + (w0 >> 2)]);
}

// The task's RMSNorm weight chunks of this thread (a layer constant: callers may load it
// before waiting for the activations).
__device__ __forceinline__ void ring_norm_w_load(const GemvTask &t, uint4 (&wn)[4], int ctid) {
  constexpr int T = kRingConsumers * 32;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int k = (ctid + j * T) * 8;
    if (t.norm_w && k < t.K) wn[j] = ldg16(t.norm_w + k);
  }
}

// 8-bit tasks: the statistics of a staged 16-byte chunk of row `row` (columns k..k+7) and
// its rewrite to FP16. A 64-column group's 8 chunks sit at 8 consecutive lanes (lanes
// 8m..8m+7, k = 64 G + 8 (lane & 7)); every lane of the warp takes part. The lanes add the
// chunk's BF16 values in FP32 (sum(x): the bias term) and take their largest magnitude m;
// lane 8m stores the sum at sums[G], the group's factor f = 2^e at facs[G] (e >= 0 the least
// with m / f < 2^15) and -1024 sum / f at negs[G] (the weights enter the MMAs offset by 1024:
// this starts a group's accumulator at minus that offset's share). Each lane then rewrites
// its chunk as the FP16 values x / f:
// exact (a power-of-two scale of a BF16 value, whose 8-bit significand FP16's 11 bits
// hold), except below 2^-14 f where FP16 is subnormal and rounds to a multiple of 2^-24 f.
__device__ __forceinline__ void q8_stage_chunk(bf16 *row, float *sums, float *facs, float *negs, int k, int lane) {
  const uint4 x = act_load_chunk(row, k);
  const uint32_t w4[4] = {x.x, x.y, x.z, x.w};
  float s = 0.f, m = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float lo = bf_lo(w4[q]), hi = bf_hi(w4[q]);
    s = (s + lo) + hi;
    m = fmaxf(m, fmaxf(fabsf(lo), fabsf(hi)));
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  }
  // m < 2^(ex - 126) for biased exponent ex: e = ex - 141 puts m / 2^e below 2^15.
  const int e = max(0, ((__float_as_int(m) >> 23) & 0xFF) - 141);
  const float inv = __int_as_float((127 - e) << 23);
  uint32_t h[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __half2 v = __floats2half2_rn(bf_lo(w4[q]) * inv, bf_hi(w4[q]) * inv);
    h[q] = *reinterpret_cast<const uint32_t *>(&v);
  }
  act_store_chunk(row, k, make_uint4(h[0], h[1], h[2], h[3]));
  if ((lane & 7) == 0) {
    sums[k >> 6] = s;
    facs[k >> 6] = __int_as_float((127 + e) << 23);
    negs[k >> 6] = -1024.f * s * inv;  // exact scalings of s by powers of two
  }
}

// Chunks of 8 activations a consumer thread stages per row: chunk ctid + j x 256 for
// j < MC (the kernel's bound, at most kStageChunks), so K <= MC x 2048.
constexpr int kStageChunks = 4;
constexpr int kStageMaxK = kStageChunks * kRingConsumers * 32 * 8;

// Consumers: the task's activation rows into `act` ([NB][K] BF16, fragment order), RMSNorm
// applied when the task has a norm weight (modeling_yue2.py:131-132). Flagged input is
// polled in passes: every pass issues the loads of all of this thread's chunks of every row
// (before checking any, so the wait costs one round trip once the words are written), then
// stores them raw to `act` and checks their flags; the pass that sees every flag holds the
// data. RMSNorm then reduces the sum of squares of that pass and rescales `act` in place.
// `error` (flagged input only): the device error word — an expired wait records code 64
// there and returns false on every consumer thread (the staged rows are then meaningless).
// `keep` (optional): the raw input chunks of columns [keep_lo, keep_hi) (multiples of 8,
// at most kResKeepCols apart) are also stored there, row b at keep + b * kResKeepCols / 8:
// the residual a later epilogue of this CTA adds. K <= MC x 2048.
template <int NB, int MC = kStageChunks>
__device__ bool ring_stage_act(const GemvTask &t, bf16 *act, float *red, int ctid, const uint4 (*wn_pre)[4] = nullptr,
                               int *error = nullptr, uint4 *keep = nullptr, int keep_lo = 0, int keep_hi = 0) {
  static_assert(MC >= 1 && MC <= kStageChunks, "chunks per thread");
  constexpr int T = kRingConsumers * 32;
  const int lane = ctid & 31, warp = ctid >> 5, K = t.K;
  float ss[NB];
  bool ok = true;
  // Rows polled per pass: all of them while their chunks fit 4 per thread (the words in
  // flight stay in registers), else one row after another (their words are written by the
  // same epilogues, so the later rows cost about one more round trip).
  constexpr int RP = NB * MC <= 4 ? NB : 1;
#pragma unroll
  for (int b0 = 0; b0 < NB && ok; b0 += RP) {
  for (long long it = 0;; ++it) {
    // Every load of the pass is issued before any flag is compared (a comparison between
    // two loads would make the second wait for the first's round trip); then each chunk is
    // stored raw to `act` (and `keep`), and its squares are summed.
    uint4 wa[RP][MC], wc[RP][MC];
#pragma unroll
    for (int r = 0; r < RP; ++r)
#pragma unroll
      for (int j = 0; j < MC; ++j) {
        const int b = b0 + r, k = (ctid + j * T) * 8;
        if (k >= K) continue;
        if (t.in_ll) {
          const uint2 *p = t.in_ll + size_t(b) * t.in_ll_stride + (k >> 1);
          wa[r][j] = ll_load2(p);
          wc[r][j] = ll_load2(p + 2);
        } else {
          const bf16 *row = t.in_gather ? t.in_row[b] : t.in + size_t(b) * t.in_stride;
          const uint4 x = row ? __ldcg(reinterpret_cast<const uint4 *>(row + k)) : make_uint4(0u, 0u, 0u, 0u);
          wa[r][j] = make_uint4(x.x, 0u, x.y, 0u);
          wc[r][j] = make_uint4(x.z, 0u, x.w, 0u);
        }
      }
    uint32_t flags_ok = 1u;
#pragma unroll
    for (int r = 0; r < RP; ++r) {
      const int b = b0 + r;
      ss[b] = 0.f;
#pragma unroll
      for (int j = 0; j < MC; ++j) {
        const int k = (ctid + j * T) * 8;
        if (k >= K) continue;
        const uint4 a = wa[r][j], c = wc[r][j];
        flags_ok &= uint32_t(a.y == t.in_flag) & uint32_t(a.w == t.in_flag) & uint32_t(c.y == t.in_flag) &
                    uint32_t(c.w == t.in_flag);
        const uint4 x = make_uint4(a.x, a.z, c.x, c.z);
        act_store_chunk(act + b * K, k, x);
        if (keep && k >= keep_lo && k < keep_hi) keep[b * (kResKeepCols / 8) + ((k - keep_lo) >> 3)] = x;
        if (t.norm_w) {
          const uint32_t w4[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float lo = bf_lo(w4[q]), hi = bf_hi(w4[q]);
            ss[b] += lo * lo + hi * hi;
          }
        }
      }
    }
    if (!t.in_ll || flags_ok) break;
    if (it >= t.ll_limit || ((it & 255) == 255 && error && ll_error_word(error) != 0)) {
      ok = false;
      break;
    }
    if (it >= 8) __nanosleep(32);
  }
  }
  if (t.norm_w) {
    uint4 wn[4];
    if (wn_pre) {
#pragma unroll
      for (int j = 0; j < 4; ++j) wn[j] = (*wn_pre)[j];
    } else {
      ring_norm_w_load(t, wn, ctid);
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const float s = warp_sum(ss[b]);
      if (lane == 0) red[b * kRingConsumers + warp] = s;
    }
    consumer_sync();
    for (int b = 0; b < NB; ++b) {
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < kRingConsumers; ++i) tot += red[b * kRingConsumers + i];
      const float scale = rms_scale_bf16(tot, K, t.eps);
#pragma unroll
      for (int j = 0; j < MC; ++j) {
        const int k = (ctid + j * T) * 8;
        if (k >= K) continue;
        const uint4 x = act_load_chunk(act + b * K, k);  // this thread's own raw chunk
        const uint32_t xq[4] = {x.x, x.y, x.z, x.w};
        const uint32_t wq[4] = {wn[j].x, wn[j].y, wn[j].z, wn[j].w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float lo = rbf(rbf(bf_lo(xq[q]) * scale) * bf_lo(wq[q]));
          const float hi = rbf(rbf(bf_hi(xq[q]) * scale) * bf_hi(wq[q]));
          o[q] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xFFFF0000u);
        }
        act_store_chunk(act + b * K, k, make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
  }
  if (t.sumx) {
    const int KG = K / 64;
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int j = 0; j < MC; ++j) {
        const int k = (ctid + j * T) * 8;
        if (k >= K) continue;  // warp-uniform: K is a multiple of 2048
        q8_stage_chunk(act + b * K, t.sumx + b * KG, t.qfac + b * KG, t.qneg + b * KG, k, lane);
      }
  }
  if (!t.in_ll) {
    consumer_sync();
    return true;
  }
  // The barrier also agrees on the outcome of every thread's waits.
  int all_ok;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.and.pred q, 1, %2, p;\n selp.s32 %0, 1, 0, q;\n}"
      : "=r"(all_ok)
      : "r"(int(ok)), "n"(kRingConsumers * 32)
      : "memory");
  if (!all_ok && ctid == 0 && error) atomicOr(error, 64);
  return all_ok != 0;
}

// Per-warp flagged staging (a task without RMSNorm): warp `warp` polls only its own
// k-range of every row — chunk (ks, lane) = columns ks * 2048 + 256 warp + 8 lane, +8 for
// ks < K / 2048 <= MC — issuing every load of a pass before comparing any, and stores it
// to `act` in fragment order (ring_consume reads exactly this range). Rows are polled
// together while their chunks fit 4 per lane, else one after another. The warp leaves a
// poll together (its lanes vote); false when the wait gave up.
template <int NB, int MC>
__device__ bool ll_stage_warp(const GemvTask &t, bf16 *act, int lane, int warp, const int *error) {
  constexpr int RP = NB * MC <= 4 ? NB : 1;
  const int KS = t.K / kRingPiece;
#pragma unroll
  for (int b0 = 0; b0 < NB; b0 += RP) {
    for (long long it = 0;; ++it) {
      uint4 wa[RP][MC], wc[RP][MC];
#pragma unroll
      for (int r = 0; r < RP; ++r)
#pragma unroll
        for (int ks = 0; ks < MC; ++ks) {
          if (ks >= KS) continue;
          const int k = ks * kRingPiece + warp * 256 + lane * 8;
          const uint2 *p = t.in_ll + size_t(b0 + r) * t.in_ll_stride + (k >> 1);
          wa[r][ks] = ll_load2(p);
          wc[r][ks] = ll_load2(p + 2);
        }
      uint32_t ok = 1u;
#pragma unroll
      for (int r = 0; r < RP; ++r)
#pragma unroll
        for (int ks = 0; ks < MC; ++ks) {
          if (ks >= KS) continue;
          const int k = ks * kRingPiece + warp * 256 + lane * 8;
          const uint4 a = wa[r][ks], c = wc[r][ks];
          ok &= uint32_t(a.y == t.in_flag) & uint32_t(a.w == t.in_flag) & uint32_t(c.y == t.in_flag) &
                uint32_t(c.w == t.in_flag);
          act_store_chunk(act + size_t(b0 + r) * t.K, k, make_uint4(a.x, a.z, c.x, c.z));
        }
      if (__all_sync(0xFFFFFFFFu, ok != 0u)) break;
      if (it >= t.ll_limit ||
          ((it & 255) == 255 && error && __any_sync(0xFFFFFFFFu, ll_error_word(error) != 0)))
        return false;
      if (it >= 8) __nanosleep(32);
    }
  }
  if (t.sumx) {  // this warp's groups only: the warp's own consumer reads them
    const int KG = t.K / 64;
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int ks = 0; ks < MC; ++ks) {
        if (ks >= KS) continue;
        const int k = ks * kRingPiece + warp * 256 + lane * 8;
        q8_stage_chunk(act + size_t(b) * t.K, t.sumx + b * KG, t.qfac + b * KG, t.qneg + b * KG, k, lane);
      }
  }
  return true;
}

// True on every consumer thread when `v` is true on any (barrier 1, the 256 consumers).
__device__ __forceinline__ bool consumer_any(bool v) {
  int r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.s32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"(int(v)), "n"(kRingConsumers * 32)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void ldsm_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_16816(float *c, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  // A rows 8..15 are zero (a1 = a3 = 0): rows 0..NB-1 carry the activation rows.
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

constexpr int kRingMaxGroups = 12;  // 8-row groups whose partial sums wait for one epilogue (gate/up: 10-11 per CTA)

// Bytes of the group-partials buffer ring_consume needs.
__host__ __device__ constexpr int ring_gred_floats(int NB) { return kRingMaxGroups * kRingConsumers * NB * 8; }

// The epilogue of 8-row groups [gb, ge) of a task: the 8 warps' partial sums of each output
// (gred, group gb first) are added in warp order and stored (flagged words or plain BF16),
// with the task's epilogue applied. Every consumer thread takes part.
template <int NB>
__device__ __forceinline__ void ring_epilogue(const GemvTask &t, int gb, int ge, const float *gred, int *error,
                                              int ctid) {
  if (t.out_ll) {
    // Flagged epilogue: one thread per pair of adjacent outputs, one flagged word each.
    const bool swiglu = t.epi == kEpiSwiGLU;
    const int per_group = NB * (swiglu ? 2 : 4);
    for (int u = ctid; u < (ge - gb) * per_group; u += kRingConsumers * 32) {
      const int gi = u / per_group, rem = u % per_group;
      const float *src = gred + size_t(gi) * kRingConsumers * NB * 8;
      const int r0 = (gb + gi) * 8;
      float v[2];
      int col;
      const int b = swiglu ? rem / 2 : rem / 4, j = swiglu ? rem % 2 : rem % 4;
      if (swiglu) {
        if (r0 + 4 * j + 3 >= t.N) continue;
#pragma unroll
        for (int e = 0; e < 2; ++e) {  // outputs 2j + e of the group: rows 2(2j + e) (gate), +1 (up)
          const int rg = 2 * (2 * j + e);
          float gs = 0.f, us = 0.f;
#pragma unroll
          for (int w = 0; w < kRingConsumers; ++w) {
            gs += src[w * NB * 8 + b * 8 + rg];
            us += src[w * NB * 8 + b * 8 + rg + 1];
          }
          v[e] = rbf(silu_f32(rbf(gs))) * rbf(us);
        }
        col = (r0 >> 1) + 2 * j;
      } else {
        if (r0 + 2 * j + 1 >= t.N) continue;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float a = 0.f;
#pragma unroll
          for (int w = 0; w < kRingConsumers; ++w) a += src[w * NB * 8 + b * 8 + 2 * j + e];
          v[e] = a;
        }
        col = r0 + 2 * j;
      }
      uint2 *o = t.out_ll + size_t(b) * t.out_ll_stride + (col >> 1);
      bf16 lo, hi;
      if (t.epi == kEpiResidual) {
        uint32_t old = 0;
        if (t.res_smem) {
          old = t.res_smem[b * (kResKeepCols / 2) + ((col - t.res_lo) >> 1)];
        } else if (!ll_wait1(o, t.res_flag, old, error, t.ll_limit)) {
          atomicOr(error, 64);
          continue;
        }
        lo = f2bf(bf_lo(old) + rbf(v[0]));
        hi = f2bf(bf_hi(old) + rbf(v[1]));
      } else {
        lo = f2bf(v[0]);
        hi = f2bf(v[1]);
      }
      ll_store_all(o, pack_bf16x2(lo, hi), t.out_flag, t.n_dst, t.dst);
    }
  } else {
    const bool swiglu = t.epi == kEpiSwiGLU;
    const int per_group = NB * (swiglu ? 4 : 8);
    for (int u = ctid; u < (ge - gb) * per_group; u += kRingConsumers * 32) {
      const int gi = u / per_group, rem = u % per_group;
      const float *src = gred + size_t(gi) * kRingConsumers * NB * 8;
      const int r0 = (gb + gi) * 8;
      if (swiglu) {
        const int b = rem / 4, j = rem % 4;  // pair j of the group: rows 2j (gate), 2j+1 (up)
        if (r0 + 2 * j + 1 >= t.N) continue;
        float gs = 0.f, us = 0.f;
#pragma unroll
        for (int w = 0; w < kRingConsumers; ++w) {
          gs += src[w * NB * 8 + b * 8 + 2 * j];
          us += src[w * NB * 8 + b * 8 + 2 * j + 1];
        }
        const float gate = rbf(gs), up = rbf(us);
        store_all(t.out + size_t(b) * t.out_stride + (r0 >> 1) + j, f2bf(rbf(silu_f32(gate)) * up), t.n_dst, t.dst);
      } else {
        const int b = rem / 8, r = rem % 8;
        if (r0 + r >= t.N) continue;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kRingConsumers; ++w) v += src[w * NB * 8 + b * 8 + r];
        bf16 *o = t.out + size_t(b) * t.out_stride + r0 + r;
        if (t.epi == kEpiResidual)
          store_all(o, f2bf(bf2f(__ldcg(o)) + rbf(v)), t.n_dst, t.dst);
        else
          store_all(o, f2bf(v), t.n_dst, t.dst);
      }
    }
  }
}

// Consumers: consume the task's stages (continuing `it`) and apply the epilogue. Each
// stage is 8 weight rows x 2048 (swizzled, see the top of this file); warp w owns the k
// range [256w, 256w+256) of every stage and runs tensor-core MMAs with the 8 weight rows
// as the B operand (n = 8, read by ldmatrix straight from the ring) and the activation rows
// as rows 0..NB-1 of A,
// accumulating in FP32 across the stages of a group. Warps park their per-group partial
// sums in `gred`; one barrier per up to kRingMaxGroups groups, then the 8 partials of
// each output are added in warp order and the epilogue is applied. After a failure
// elsewhere (`bad`) stages are still waited for and released and barriers still taken,
// without computing; once a ring wait itself expired (`dead`: the producer is presumed
// stuck, a copy may still be landing) no stage is waited for or released any more.
// A task with `stage_per_warp` is staged here, warp by warp (ll_stage_warp, K <= MC x 2048);
// the batch barrier then also agrees on `bad`.
template <int NB, int NS, int MC = kStageChunks>
__device__ void ring_consume(const GemvTask &t, int g0, int g1, const bf16 *ring, bf16 *act, uint64_t *full,
                             uint64_t *empty, long long &it, float *gred, int *error, bool &bad, bool &dead,
                             int ctid) {
  static_assert(NB >= 1 && NB <= 8, "activation rows must fit the MMA's first 8 rows");
  const int lane = ctid & 31, warp = ctid >> 5, K = t.K, KS = K / kRingPiece;
  if (t.stage_per_warp && !bad && !ll_stage_warp<NB, MC>(t, act, lane, warp, error)) {
    if (lane == 0 && error) atomicOr(error, 64);
    bad = true;
  }
  __syncwarp();
  const int grow = lane >> 2, gcol = (lane & 3) * 2;  // fragment row / column pair of this lane
  // ldmatrix x4 addresses: lane l gives row l & 7 of matrix l >> 3, the 16-byte chunk
  // k0 / 8 + (l >> 3) of the stage (matrices k, k+8, k+16, k+24 of rows 0..7).
  const int lrow = lane & 7, lmat = lane >> 3;
  // Ring position of `it`, kept incrementally.
  int s = int(it % NS);
  unsigned phase = unsigned(it / NS) & 1u;
  for (int gb = g0; gb < g1; gb += kRingMaxGroups) {
    const int ge = min(g1, gb + kRingMaxGroups);
    for (int g = gb; g < ge; ++g) {
      // Two independent accumulator chains (even / odd k-tile pairs) halve the MMAs that
      // serialize on one accumulator; they are added at the end.
      float c2[2][4] = {};
      for (int ks = 0; ks < KS; ++ks) {
        bool landed = false;
        if (!dead) {
          landed = mbar_wait(&full[s], phase);
          if (!landed) {
            if (lane == 0) atomicOr(error, 8);
            dead = bad = true;
          }
        }
        if (!bad) {
          const bf16 *wst = ring + size_t(s) * kRingStageElems;
          const bf16 *ar = act + size_t(ks) * kRingPiece;
#pragma unroll
          for (int kt = 0; kt < 16; kt += 2) {
            const int k0 = warp * 256 + kt * 16;  // two k-tiles of 16: [k0, k0 + 32)
            uint32_t b0, b1, b2, b3;
            ldsm_x4(b0, b1, b2, b3, wst + stage_chunk((k0 >> 3) + lmat, lrow));
            uint4 a4 = make_uint4(0, 0, 0, 0);  // (a0, a2) of k-tile kt, then of kt + 1
            if (grow < NB) a4 = *reinterpret_cast<const uint4 *>(ar + size_t(grow) * K + k0 + gcol * 4);
            const uint32_t a0 = a4.x, a2 = a4.y, a0n = a4.z, a2n = a4.w;
            mma_16816(c2[0], a0, a2, b0, b1);
            mma_16816(c2[1], a0n, a2n, b2, b3);
          }
        }
        __syncwarp();
        if (lane == 0 && landed) mbar_arrive(&empty[s]);
        ++it;
        if (++s == NS) {
          s = 0;
          phase ^= 1u;
        }
      }
      float c[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) c[q] = c2[0][q] + c2[1][q];
      // c[0], c[1] of lane (b, j): activation row b's partial dot with weight rows
      // 2j, 2j+1 over this warp's k range.
      if (grow < NB) {
        float *dst = gred + (size_t(g - gb) * kRingConsumers + warp) * NB * 8 + grow * 8 + gcol;
        dst[0] = c[0];
        dst[1] = c[1];
      }
    }
    bad = consumer_any(bad);  // the batch barrier; a warp's own staging may have failed
    if (!bad) ring_epilogue<NB>(t, gb, ge, gred, error, ctid);
    if (ge < g1) consumer_sync();  // the next batch reuses gred
  }
}

// ---------------------------------------------------------------------------------------
// Affine 8-bit weights (the `8bit` precision: per 64-column group w = scale * q + bias,
// q in [0, 255], BF16 scale and bias; mlx quantized_matmul as ar.cpp:20-29 calls it).
// A stage is 16 weight rows x 2048 columns of one matrix's image (q8_stage_image writes
// it): kQ8QBytes of weights followed by 512 scale/bias words, one bulk copy. The weights
// are laid out for the MMA's A operand (16 rows: the whole stage in one m16n8k16 per
// k-tile, the weights as exact FP16 integers; the activation rows, staged as FP16, are the
// B operand's columns): warp w's 64-column group j
// is 2 x 32 lanes x 16 bytes at ((w * 4 + j) * 2 + h) * 512 + lane * 16, lane (g = lane / 4,
// t = lane % 4) holding, for k-tiles kt = 2h and 2h + 1, the words (row g, kt), (row g + 8,
// kt) of bytes at columns 16 kt + {2t, 2t + 1, 2t + 8, 2t + 9} of the group. Scale/bias
// word (G, i) — BF16 scale low, BF16 bias high — of the stage's group G = 4w + j sits at
// kQ8QBytes + (16 G + 2 (r % 8) + r / 8) x 4 for unit row r. Rows past N are zero.
constexpr int kQ8Rows = 16;
constexpr int kQ8QBytes = kQ8Rows * kRingPiece;                         // 32 KB of 8-bit weights
constexpr int kQ8StageBytes = kQ8QBytes + kQ8Rows * (kRingPiece / 64) * 4;  // + scale/bias words: 34,816
// 4-bit weights (the `4bit` precision) use the same units and scale/bias words with half
// the weight bytes: lane (g, t)'s 16 bytes of warp w's group j sit at ((w * 4 + j) * 32 +
// lane) * 16, one word per k-tile kt holding the eight nibbles of its A fragments — a0
// (row g, columns 2t, 2t + 1), a1 (row g + 8, same columns), a2 (row g, 2t + 8, 2t + 9),
// a3 (row g + 8, same) — fragment s's even column in bits 4s..4s+3 and its odd column in
// bits 16 + 4s..16 + 4s + 3.
constexpr int kQ4QBytes = kQ8Rows * kRingPiece / 2;                     // 16 KB of 4-bit weights
constexpr int kQ4StageBytes = kQ4QBytes + kQ8Rows * (kRingPiece / 64) * 4;  // 18,432
template <int BITS>
__host__ __device__ constexpr int q_stage_bytes() {
  return BITS == 8 ? kQ8StageBytes : kQ4StageBytes;
}

// Two 8-bit weights (the bytes of w that selector `sel` picks) as an FP16 pair offset by
// 1024: each byte q placed under the exponent byte 0x64 is the FP16 value 1024 + q (ulp 1 in
// [1024, 2048)). The offset is not subtracted per weight: a group's accumulator starts at
// -1024 sum(x) instead (q8_stage_chunk's negs).
__device__ __forceinline__ uint32_t q8_f16x2(uint32_t w, uint32_t sel) { return __byte_perm(w, 0x64646464u, sel); }
// Two 4-bit weights as an FP16 pair offset by 1024: the nibbles at bits 0..3 and 16..19 of
// w under exponent 0x64 are 1024 + n; with mask 0x00F000F0 (bits 4..7, 20..23) they are
// 1024 + 16 n, exact as well (ulp 1 below 2048), so two fragments per word need no shift.
__device__ __forceinline__ uint32_t q4_f16x2(uint32_t w, uint32_t mask) { return (w & mask) | 0x64006400u; }
// m16n8k16, FP16 operands, FP32 accumulators (no side effects: the compiler may schedule
// it among independent work).
__device__ __forceinline__ void mma_f16_16816(float *c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// One k-tile of a stage: the words (row g, kt) = wg and (row g + 8, kt) = wg8 hold bytes of
// columns {2t, 2t + 1, 2t + 8, 2t + 9}: A fragments a0 / a2 from wg, a1 / a3 from wg8.
__device__ __forceinline__ void q8_mma_tile(float *c, uint32_t wg, uint32_t wg8, uint32_t b0, uint32_t b1) {
  mma_f16_16816(c, q8_f16x2(wg, 0x4140u), q8_f16x2(wg8, 0x4140u), q8_f16x2(wg, 0x4342u), q8_f16x2(wg8, 0x4342u), b0,
                b1);
}
// The same k-tile from one 4-bit word (fragments a0..a3 at nibble offsets 0, 4, 8, 12). Rows
// g + 8 (a1, a3: the upper nibble of each byte pair) enter as 1024 + 16 q, so their sums
// come out as 16 sum(x q) on top of the offset: the caller scales them by 1/16.
__device__ __forceinline__ void q4_mma_tile(float *c, uint32_t w, uint32_t b0, uint32_t b1) {
  const uint32_t w8 = w >> 8;
  mma_f16_16816(c, q4_f16x2(w, 0x000F000Fu), q4_f16x2(w, 0x00F000F0u), q4_f16x2(w8, 0x000F000Fu),
                q4_f16x2(w8, 0x00F000F0u), b0, b1);
}

// Consumers of a quantized task (BITS 8 or 4): 16-row units [u0, u1), each K / 2048 stages
// (continuing `it`; 8-bit stages fill a kQ8StageBytes slot, 4-bit ones kQ4StageBytes of it).
// The staging left the activation rows as FP16 with a power-of-two factor f per 64-column
// group (q8_stage_chunk). Warp w runs its 256 columns of every stage: per 64-column group,
// four MMAs (16 weight rows as FP16 integers offset by 1024 x the activation rows) in two
// independent chains, the first started at -1024 sum(x / f), give sum(x q) / f per row, and
// the group adds (scale f) * that + bias * sum(x) in FP32 — the affine dequantization of
// every weight folded into two FMAs per output. Partial sums go to gred as ring_consume's,
// two 8-row groups per unit, and the same epilogue follows (ring_epilogue). Failure
// handling is ring_consume's.
template <int NB, int NS, int MC = kStageChunks, int BITS = 8>
__device__ void ring_consume_q8(const GemvTask &t, int u0, int u1, const unsigned char *ring, bf16 *act,
                                uint64_t *full, uint64_t *empty, long long &it, float *gred, int *error, bool &bad,
                                bool &dead, int ctid) {
  static_assert(NB >= 1 && NB <= 2, "8-bit stages take one or two activation rows");
  const int lane = ctid & 31, warp = ctid >> 5, K = t.K, KS = K / kRingPiece, KG = K / 64;
  if (t.stage_per_warp && !bad && !ll_stage_warp<NB, MC>(t, act, lane, warp, error)) {
    if (lane == 0 && error) atomicOr(error, 64);
    bad = true;
  }
  __syncwarp();
  const int g = lane >> 2, tq = lane & 3;  // A row g (and g + 8); B/C column pair 2 tq, 2 tq + 1
  int s = int(it % NS);
  unsigned phase = unsigned(it / NS) & 1u;
  constexpr int kUnits = kRingMaxGroups / 2;  // units whose partial sums wait for one epilogue
  const int G8 = (t.N + 7) / 8;
  for (int ub = u0; ub < u1; ub += kUnits) {
    const int ue = min(u1, ub + kUnits);
    for (int u = ub; u < ue; ++u) {
      // acc: (row g, activation row 2 tq), (g, 2 tq + 1), (g + 8, 2 tq), (g + 8, 2 tq + 1)
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int ks = 0; ks < KS; ++ks) {
        bool landed = false;
        if (!dead) {
          landed = mbar_wait(&full[s], phase);
          if (!landed) {
            if (lane == 0) atomicOr(error, 8);
            dead = bad = true;
          }
        }
        if (!bad) {
          const unsigned char *st = ring + size_t(s) * kQ8StageBytes;  // slots of kQ8StageBytes
          constexpr int kQB = BITS == 8 ? kQ8QBytes : kQ4QBytes;
          const bf16 *ar = act + size_t(ks) * kRingPiece;
          // Group sums and factors of activation rows 2 tq, 2 tq + 1 for the warp's 4 groups.
          float4 sx[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
          float4 fx[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
          float4 nx[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
#pragma unroll
          for (int e = 0; e < 2; ++e)
            if (2 * tq + e < NB) {
              const int o = (2 * tq + e) * KG + ks * 32 + warp * 4;
              sx[e] = *reinterpret_cast<const float4 *>(t.sumx + o);
              fx[e] = *reinterpret_cast<const float4 *>(t.qfac + o);
              nx[e] = *reinterpret_cast<const float4 *>(t.qneg + o);
            }
          const float sx0[4] = {sx[0].x, sx[0].y, sx[0].z, sx[0].w}, sx1[4] = {sx[1].x, sx[1].y, sx[1].z, sx[1].w};
          const float fx0[4] = {fx[0].x, fx[0].y, fx[0].z, fx[0].w}, fx1[4] = {fx[1].x, fx[1].y, fx[1].z, fx[1].w};
          const float nx0[4] = {nx[0].x, nx[0].y, nx[0].z, nx[0].w}, nx1[4] = {nx[1].x, nx[1].y, nx[1].z, nx[1].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int k0 = warp * 256 + j * 64;
            uint4 x01 = make_uint4(0, 0, 0, 0), x23 = make_uint4(0, 0, 0, 0);  // B: k-tiles 0, 1 / 2, 3
            if (g < NB) {
              x01 = *reinterpret_cast<const uint4 *>(ar + size_t(g) * K + k0 + tq * 8);
              x23 = *reinterpret_cast<const uint4 *>(ar + size_t(g) * K + k0 + 32 + tq * 8);
            }
            // c0 starts at the offset's share (-1024 sum(x / f) per activation row), c1 at 0.
            float c0[4] = {nx0[j], nx1[j], nx0[j], nx1[j]}, c1[4] = {0.f, 0.f, 0.f, 0.f};
            if constexpr (BITS == 8) {
              const uint4 *qp = reinterpret_cast<const uint4 *>(st + ((warp * 4 + j) * 64 + lane) * 16);
              const uint4 q01 = qp[0], q23 = qp[32];
              q8_mma_tile(c0, q01.x, q01.y, x01.x, x01.y);
              q8_mma_tile(c1, q23.x, q23.y, x23.x, x23.y);
              q8_mma_tile(c0, q01.z, q01.w, x01.z, x01.w);
              q8_mma_tile(c1, q23.z, q23.w, x23.z, x23.w);
            } else {
              const uint4 qv = *reinterpret_cast<const uint4 *>(st + ((warp * 4 + j) * 32 + lane) * 16);
              q4_mma_tile(c0, qv.x, x01.x, x01.y);
              q4_mma_tile(c1, qv.z, x23.x, x23.y);
              q4_mma_tile(c0, qv.y, x01.z, x01.w);
              q4_mma_tile(c1, qv.w, x23.z, x23.w);
            }
            const uint2 sb = *reinterpret_cast<const uint2 *>(st + kQB + ((warp * 4 + j) * 16 + 2 * g) * 4);
            // 4 bits: rows g + 8 came out as 16 sum(x q) (q4_mma_tile); 1/16 is exact.
            const float s_g = bf_lo(sb.x), b_g = bf_hi(sb.x), b_g8 = bf_hi(sb.y);
            const float s_g8 = BITS == 8 ? bf_lo(sb.y) : bf_lo(sb.y) * 0.0625f;
            acc[0] = fmaf(s_g * fx0[j], c0[0] + c1[0], fmaf(b_g, sx0[j], acc[0]));
            acc[1] = fmaf(s_g * fx1[j], c0[1] + c1[1], fmaf(b_g, sx1[j], acc[1]));
            acc[2] = fmaf(s_g8 * fx0[j], c0[2] + c1[2], fmaf(b_g8, sx0[j], acc[2]));
            acc[3] = fmaf(s_g8 * fx1[j], c0[3] + c1[3], fmaf(b_g8, sx1[j], acc[3]));
          }
        }
        __syncwarp();
        if (lane == 0 && landed) mbar_arrive(&empty[s]);
        ++it;
        if (++s == NS) {
          s = 0;
          phase ^= 1u;
        }
      }
      if (tq == 0) {  // columns 0, 1: the activation rows
        float *d0 = gred + (size_t(2 * (u - ub)) * kRingConsumers + warp) * NB * 8;
        float *d1 = d0 + size_t(kRingConsumers) * NB * 8;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          d0[b * 8 + g] = acc[b];
          d1[b * 8 + g] = acc[2 + b];
        }
      }
    }
    bad = consumer_any(bad);  // the batch barrier; a warp's own staging may have failed
    if (!bad) ring_epilogue<NB>(t, 2 * ub, min(2 * ue, G8), gred, error, ctid);
    if (ue < u1) consumer_sync();  // the next batch reuses gred
  }
}

}  // namespace yar
