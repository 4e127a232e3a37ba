// kernels_sampler.cu — one sampler step per request on phase-local BF16 logits.
//
// Filter chain = upstream distribution (vendor/yue/src/yue2/sampling.py:16-53) on the
// phase rows (native/src/sampling.cpp:38-99), after the CFG mix (sampling.cpp:100-115):
//   s = f32(bf16(u + bf16(bf16(c - u) * f32(scale))))          (CFG, when two rows)
//   s[end] = -inf while step < min_tokens
//   s[t] = s < 0 ? s * alpha[n] : s / alpha[n] for the n-times-repeated ids of the window
//   greedy: first argmax                       (temperature == 0)
//   s /= f32(T); s < kth-largest(s) -> -inf    (top-k by value, ties kept)
//   shifted nucleus over survivors sorted by (score desc, index asc)
// Draw: u = Philox uniform(seed, step); e_i = yexp(s_i - s_0); first survivor whose
// sequential FP32 running sum of e exceeds u * sum(e). All of it is exact-FP32 code
// (exact_math.cuh), so the CPU restatement reproduces the token bit for bit.
#include "common.cuh"

namespace yar {

constexpr int kSampThreads = 1024;
// Phase widths up to this many columns keep the FP32 score row in shared memory (the
// semantic phase's 32,769 do); wider rows (ABC) work in the global scratch row.
constexpr int kSampSmemScores = 36864;
// Dynamic shared memory: the score row, then the radix histograms (32 warps x 256 bins).
constexpr size_t kSampSmemBytes = kSampSmemScores * sizeof(float) + 32 * 256 * sizeof(int);

struct SamplerParams {
  RequestState *req;
  const bf16 *logits;
  int logit_stride;
  float *scores;      // [requests][logit_stride] scratch
  int *token;         // [rows]
  int *active;        // [rows]
  int32_t *out_tokens;
  int out_cap;
  int write_scores;   // also leave the filtered FP32 scores in `scores` (tests)
  int32_t *picked;    // optional [requests] local token of this step
  unsigned long long *trace;  // optional: SM-clock stamps of request 0's phases (16 slots)
};

__device__ __forceinline__ int native_to_local(int tok, int phase, int width) {
  if (phase == kPhaseAbc) {
    if (tok >= 0 && tok < kEOD) return tok;
    return tok == kAbcEnd ? kEOD : -1;
  }
  if (phase == kPhaseSemantic) {
    if (tok == kMusicEnd) return 0;
    if (tok >= kCodecOffset && tok < kCodecOffset + kCodecSize) return tok - kMusicEnd;
    return -1;
  }
  return (tok >= 0 && tok < width) ? tok : -1;
}
__device__ __forceinline__ int local_to_native(int loc, int phase) {
  if (phase == kPhaseAbc) return loc < kEOD ? loc : kAbcEnd;
  if (phase == kPhaseSemantic) return kMusicEnd + loc;
  return loc;
}

__global__ void __launch_bounds__(kSampThreads) k_sampler(SamplerParams p) {
  __shared__ uint64_t cand[kCandCap];
  __shared__ int list_n, kth_cnt;
  __shared__ float ev[kCandCap];
  __shared__ int tot[256];
  __shared__ float pv[kCandCap];
  __shared__ int ncand, sel_bin, kth_rem, result, tie_total;
  __shared__ float red_v[32];
  __shared__ int red_i[32];
  __shared__ uint32_t prefix_s;

  pdl_launch_dependents();
  pdl_wait();
  // Phase stamps (tracing only): 0 start, 1 CFG mix, 2 penalty, 3 temperature, 4-6 radix
  // passes, 7 candidates, 8 sort, 9 exp, 10 nucleus + draw, 11 done; 12/13 globaltimer ns
  // at start / end.
  auto stamp = [&](int k) {
    if (p.trace && blockIdx.x == 0 && threadIdx.x == 0) p.trace[k] = (unsigned long long)clock64();
  };
  unsigned long long t_start = 0;
  auto stamp_ns = [&](int k) {
    if (p.trace && blockIdx.x == 0 && threadIdx.x == 0) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      p.trace[k] = t;
      if (k == 12) t_start = t;
    }
  };
  stamp_ns(12);
  stamp(0);
  RequestState &st = p.req[blockIdx.x];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (st.done || st.step >= st.max_tokens) return;
  const int n = st.width, step = st.step;
  const bf16 *lc = p.logits + size_t(st.row_c) * p.logit_stride;
  const bf16 *lu = st.row_u >= 0 ? p.logits + size_t(st.row_u) * p.logit_stride : nullptr;
  extern __shared__ float s_row[];
  int *hist = reinterpret_cast<int *>(s_row + kSampSmemScores);  // [32 warps][256 bins]
  const bool in_smem = n <= kSampSmemScores;
  float *s = in_smem ? s_row : p.scores + size_t(blockIdx.x) * p.logit_stride;

  // CFG mix and FP32 upcast (independent loads, several in flight per thread).
  const float scale = st.cfg_scale;
  auto mix = [&](int i) {
    float v = bf2f(lc[i]);
    if (lu) {
      const float u = bf2f(lu[i]);
      const float delta = round_bf16(f_sub(v, u));
      const float scaled = round_bf16(f_mul(delta, scale));
      v = round_bf16(f_add(u, scaled));
    }
    s[i] = v;
  };
  const bool vec = (reinterpret_cast<uintptr_t>(lc) & 15) == 0 && (!lu || (reinterpret_cast<uintptr_t>(lu) & 15) == 0);
  const bool s_vec = (reinterpret_cast<uintptr_t>(s) & 15) == 0;
  if (vec) {
    // 16-byte loads: 8 logits per load, every load of a thread in flight at once.
    const int nv = n / 8;
    for (int c = tid; c < nv; c += kSampThreads) {
      const uint4 cq = *reinterpret_cast<const uint4 *>(lc + size_t(c) * 8);
      const uint4 uq = lu ? *reinterpret_cast<const uint4 *>(lu + size_t(c) * 8) : cq;
      const uint32_t cw[4] = {cq.x, cq.y, cq.z, cq.w}, uw[4] = {uq.x, uq.y, uq.z, uq.w};
      float v8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = (e & 1) ? bf_hi(cw[e >> 1]) : bf_lo(cw[e >> 1]);
        if (lu) {
          const float u = (e & 1) ? bf_hi(uw[e >> 1]) : bf_lo(uw[e >> 1]);
          const float delta = round_bf16(f_sub(v, u));
          const float scaled = round_bf16(f_mul(delta, scale));
          v = round_bf16(f_add(u, scaled));
        }
        v8[e] = v;
      }
      // Two 16-byte stores when the score row allows them (eight 4-byte stores 32 bytes
      // apart per lane conflict 8 ways in shared memory).
      if (s_vec) {
        *reinterpret_cast<float4 *>(s + c * 8) = make_float4(v8[0], v8[1], v8[2], v8[3]);
        *reinterpret_cast<float4 *>(s + c * 8 + 4) = make_float4(v8[4], v8[5], v8[6], v8[7]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) s[c * 8 + e] = v8[e];
      }
    }
    for (int i = nv * 8 + tid; i < n; i += kSampThreads) mix(i);
  } else {
    constexpr int U = 8;
    int i = tid;
    for (; i + (U - 1) * kSampThreads < n; i += U * kSampThreads) {
      bf16 c[U], uu[U];
#pragma unroll
      for (int j = 0; j < U; ++j) {
        c[j] = lc[i + j * kSampThreads];
        uu[j] = lu ? lu[i + j * kSampThreads] : c[j];
      }
#pragma unroll
      for (int j = 0; j < U; ++j) {
        float v = bf2f(c[j]);
        if (lu) {
          const float u = bf2f(uu[j]);
          const float delta = round_bf16(f_sub(v, u));
          const float scaled = round_bf16(f_mul(delta, scale));
          v = round_bf16(f_add(u, scaled));
        }
        s[i + j * kSampThreads] = v;
      }
    }
    for (; i < n; i += kSampThreads) mix(i);
  }
  __syncthreads();
  stamp(1);
  if (tid == 0 && step < st.min_tokens && st.end_local >= 0) s[st.end_local] = -INFINITY;
  __syncthreads();
  // Window penalty: thread t < W owns history entry t; the first occurrence of each id
  // applies alpha[count of that id in the window].
  if (st.penalty_on && st.n_out > 0) {
    const int W = min(st.window, st.n_out);
    __shared__ int loc_s[kMaxPenaltyWindow];
    if (tid < W) loc_s[tid] = native_to_local(st.hist[(st.n_out - W + tid) % kHistCap], st.phase, n);
    __syncthreads();
    if (tid < W) {
      const int me = loc_s[tid];
      bool first = me >= 0;
      int count = 0;
      for (int j = 0; j < W; ++j) {
        if (loc_s[j] == me) {
          ++count;
          if (j < tid) first = false;
        }
      }
      if (first) {
        const float a = st.alpha[count], v = s[me];
        const float r = v < 0.f ? f_mul(v, a) : f_div(v, a);
        s[me] = st.legacy ? round_bf16(r) : r;  // legacy_off: BF16 scores
      }
    }
    __syncthreads();
  }

  stamp(2);
  int local = -1;
  if (st.temperature == 0.f) {
    // Greedy: first index of the maximum.
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int i = tid; i < n; i += kSampThreads) {
      const float v = s[i];
      if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      red_v[warp] = bv;
      red_i[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      float v = red_v[0];
      int i0 = red_i[0];
      for (int w = 1; w < kSampThreads / 32; ++w)
        if (red_v[w] > v || (red_v[w] == v && red_i[w] < i0)) {
          v = red_v[w];
          i0 = red_i[w];
        }
      result = i0 < n ? i0 : 0;
    }
    __syncthreads();
    local = result;
  } else {
    if (st.temperature != 1.f) {
      if (st.legacy)
        for (int i = tid; i < n; i += kSampThreads) s[i] = round_bf16(f_div(s[i], st.temperature));
      else
        for (int i = tid; i < n; i += kSampThreads) s[i] = f_div(s[i], st.temperature);
      __syncthreads();
    }
    stamp(3);
    // k-th largest value: radix select on order-preserving keys, four 8-bit digits from
    // the top. Each warp counts into its own 256-bin histogram with shared-memory atomics,
    // so warps never contend when the logits crowd a few bins; the 32 histograms are
    // summed per bin and warp 0 finds the bin holding the k-th key by a scan from the top.
    const int k = min(st.top_k, n);
    uint32_t pre = 0;
    int rem = k;
    int *wh = hist + warp * 256;
    // Once the rows sharing the found prefix fit the list (their count is the selected
    // bin's), only they can hold the k-th key: their indices are listed (in `cand`, idle
    // until the candidates are gathered) and the remaining passes count the list instead of
    // every row.
    int *list = reinterpret_cast<int *>(cand);
    constexpr int kListCap = kCandCap * 2;
    int m = n;
    bool listed = false;
    if (tid == 0) kth_cnt = n;  // (set by every pass; read after its barriers)
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int b = lane; b < 256; b += 32) wh[b] = 0;
      __syncwarp();
      const uint32_t hmask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int base = warp * 32; base < m; base += kSampThreads) {
        const int j = base + lane;
        uint32_t bin = 0xFFFFFFFFu;
        if (j < m) {
          const uint32_t key = f32_order_key(s[listed ? list[j] : j]);
          if ((key & hmask) == (pre & hmask)) bin = (key >> shift) & 255u;
        }
        if (bin != 0xFFFFFFFFu) atomicAdd(&wh[bin], 1);
      }
      __syncthreads();
      if (tid < 256) {
        int c = 0;
#pragma unroll 8
        for (int w = 0; w < kSampThreads / 32; ++w) c += hist[w * 256 + tid];
        tot[tid] = c;
      }
      __syncthreads();
      if (warp == 0) {
        // Lane l owns bins 255 - 8l - j (j < 8), counted from the top.
        int cnt[8], mine = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          cnt[j] = tot[255 - 8 * lane - j];
          mine += cnt[j];
        }
        int incl = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += y;
        }
        const int before = incl - mine;
        if (before < rem && before + mine >= rem) {
          int acc = before, b = 255 - 8 * lane;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            b = 255 - 8 * lane - j;
            if (acc + cnt[j] >= rem) break;
            acc += cnt[j];
          }
          kth_rem = rem - acc;
          kth_cnt = tot[b];
          prefix_s = pre | (uint32_t(b) << shift);
        }
      }
      __syncthreads();
      pre = prefix_s;
      rem = kth_rem;
      if (!listed && pass < 3 && kth_cnt <= kListCap) {
        if (tid == 0) list_n = 0;
        __syncthreads();
        // One shared-memory atomic per warp and round (the matching lanes' slots follow from
        // the ballot), not one per row: the list only feeds the later passes' counts, so
        // the order of its entries does not matter.
        for (int base = 0; base < n; base += kSampThreads) {
          const int i = base + tid;
          const bool hit = i < n && (f32_order_key(s[i]) >> shift) == (pre >> shift);
          const unsigned m = __ballot_sync(0xFFFFFFFFu, hit);
          int first = 0;
          if (lane == 0 && m) first = atomicAdd(&list_n, __popc(m));
          first = __shfl_sync(0xFFFFFFFFu, first, 0);
          if (hit) list[first + __popc(m & ((1u << lane) - 1u))] = i;
        }
        __syncthreads();
        listed = true;
        m = list_n;
      }
      stamp(4 + (pass < 2 ? pass : 2));
    }
    const float thr = f32_from_order_key(prefix_s);
    // Survivors in (score desc, index asc) order are the rows strictly above the k-th
    // value (at most k-1 of them, sorted here) followed by every row equal to it (a tie
    // group of any size, already in index order, walked implicitly). When the k-th value
    // is -inf the tie group is empty: only finite rows survive.
    const bool ties_live = thr > -INFINITY;
    const int chunk = (n + kSampThreads - 1) / kSampThreads;
    const int c0 = min(n, tid * chunk), c1 = min(n, c0 + chunk);
    if (tid == 0) ncand = 0;
    __syncthreads();
    int my_ties = 0;
    for (int i = c0; i < c1; ++i) {
      const float v = s[i];
      if (v > thr) {
        const int slot = atomicAdd(&ncand, 1);
        if (slot < kCandCap) cand[slot] = (uint64_t(~f32_order_key(v)) << 32) | uint32_t(i);
      } else if (v == thr && ties_live) {
        ++my_ties;
      } else if (p.write_scores) {
        s[i] = -INFINITY;
      }
    }
    // Exclusive scan of the per-thread tie counts (tie rank = index order).
    int incl = my_ties;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) red_i[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = red_i[lane];
      int wi = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, wi, o);
        if (lane >= o) wi += y;
      }
      red_i[lane] = wi - w;  // exclusive warp offsets
      if (lane == 31) tie_total = wi;
    }
    __syncthreads();
    const int tie_before = red_i[warp] + incl - my_ties;
    const int na = ncand, nt = tie_total;
    stamp(7);
    if (na > kCandCap || na + nt == 0) {
      if (tid == 0) {
        st.error = na + nt == 0 ? 2 : 1;
        result = -1;
      }
      __syncthreads();
      local = -1;
    } else {
      int np2 = 1;
      while (np2 < na) np2 <<= 1;
      if (np2 <= 64) {
        // Bitonic sort of up to 64 keys in warp 0's registers (element lane + 32 h).
        if (warp == 0) {
          uint64_t e[2] = {lane < na ? cand[lane] : ~0ull, lane + 32 < na ? cand[lane + 32] : ~0ull};
          for (int size = 2; size <= 64; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
              if (stride == 32) {
                const uint64_t lo = e[0] < e[1] ? e[0] : e[1], hi = e[0] < e[1] ? e[1] : e[0];
                e[0] = lo;
                e[1] = hi;
              } else {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const int i = lane + 32 * h;
                  const uint64_t y = __shfl_xor_sync(0xFFFFFFFFu, e[h], stride);
                  const bool up = (i & size) == 0, lower = (i & stride) == 0;
                  const uint64_t mn = e[h] < y ? e[h] : y, mx = e[h] < y ? y : e[h];
                  e[h] = lower == up ? mn : mx;
                }
              }
            }
          if (lane < na) cand[lane] = e[0];
          if (lane + 32 < na) cand[lane + 32] = e[1];
        }
        __syncthreads();
      } else {
      for (int i = na + tid; i < np2; i += kSampThreads) cand[i] = ~0ull;
      __syncthreads();
      // Bitonic sort, ascending keys = (score desc, index asc).
      for (int size = 2; size <= np2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          for (int i = tid; i < np2; i += kSampThreads) {
            const int j = i ^ stride;
            if (j > i) {
              const bool up = (i & size) == 0;
              const uint64_t a = cand[i], b = cand[j];
              if ((a > b) == up) {
                cand[i] = b;
                cand[j] = a;
              }
            }
          }
          __syncthreads();
        }
      }
      }
      stamp(8);
      const float s0 = na > 0 ? s[uint32_t(cand[0])] : thr;
      for (int i = tid; i < na; i += kSampThreads) ev[i] = yexp(f_sub(s[uint32_t(cand[i])], s0));
      __syncthreads();
      stamp(9);
      // Nucleus: the normalizer is a sequential FP32 sum (thread 0); the divisions
      // p_i = e_i / total are independent (all threads); the running sum is sequential.
      const float et = yexp(f_sub(thr, s0));
      if (st.top_p < 1.f) {
        if (tid == 0) {
          float total = 0.f;
          for (int i = 0; i < na; ++i) total = f_add(total, ev[i]);
          for (int j = 0; j < nt; ++j) total = f_add(total, et);
          red_v[0] = total;
        }
        __syncthreads();
        const float total = red_v[0];
        for (int i = tid; i < na; i += kSampThreads) pv[i] = st.legacy ? round_bf16(f_div(ev[i], total)) : f_div(ev[i], total);
        __syncthreads();
      }
      if (tid == 0) {
        int keep_ties = nt;
        if (st.top_p < 1.f) {
          const float total = red_v[0];
          // Row i is removed when the mass before it exceeds top_p (from row 1 on). The
          // legacy_off path (BF16 scores) rounds p, the running sum and the preceding mass
          // to BF16, compares with bf16(top_p) and keeps the first three rows
          // (vendor/yue/src/yue2/sampling.py:46-50).
          const bool lg = st.legacy != 0;
          const float top_p = lg ? round_bf16(st.top_p) : st.top_p;
          const int keep_min = lg ? 3 : 1;
          auto preceding = [&](float c, float p) { return lg ? round_bf16(f_sub(round_bf16(c), p)) : f_sub(c, p); };
          float c = 0.f;
          for (int i = 0; i < na; ++i) {
            const float pi = pv[i];
            c = f_add(c, pi);
            if (i >= keep_min && preceding(c, pi) > top_p) ev[i] = -1.f;  // removed
          }
          // Within the tie group p is constant and the preceding mass never decreases, so
          // the kept ties are a prefix of the group.
          const float pt = lg ? round_bf16(f_div(et, total)) : f_div(et, total);
          keep_ties = 0;
          for (int j = 0; j < nt; ++j) {
            c = f_add(c, pt);
            if (na + j >= keep_min && preceding(c, pt) > top_p) break;
            ++keep_ties;
          }
        }
        const float u = step_uniform((uint64_t(st.seed_hi) << 32) | st.seed_lo, uint32_t(step), st.stream);
        float total = 0.f;
        for (int i = 0; i < na; ++i)
          if (ev[i] >= 0.f) total = f_add(total, ev[i]);
        for (int j = 0; j < keep_ties; ++j) total = f_add(total, et);
        const float target = f_mul(u, total);
        float acc = 0.f;
        int pick = -1, last = -1;  // >= 0: candidate slot; <= -2: tie rank -(pick+2)
        for (int i = 0; i < na && pick == -1; ++i) {
          if (ev[i] < 0.f) continue;
          last = i;
          acc = f_add(acc, ev[i]);
          if (target < acc) pick = i;
        }
        for (int j = 0; j < keep_ties && pick == -1; ++j) {
          last = -(j + 2);
          acc = f_add(acc, et);
          if (target < acc) pick = -(j + 2);
        }
        if (pick == -1) pick = last;
        sel_bin = pick;
        kth_rem = keep_ties;
        result = pick >= 0 ? int(uint32_t(cand[pick])) : -1;
      }
      __syncthreads();
      const int pick = sel_bin, keep_ties = kth_rem;
      if (pick <= -2) {
        // The chosen tie has rank -(pick+2) in index order: the thread whose chunk holds
        // that rank finds it.
        const int rank = -(pick + 2);
        if (rank >= tie_before && rank < tie_before + my_ties) {
          int r = tie_before;
          for (int i = c0; i < c1; ++i)
            if (s[i] == thr) {
              if (r == rank) result = i;
              ++r;
            }
        }
      }
      if (p.write_scores) {
        for (int i = tid; i < na; i += kSampThreads)
          if (ev[i] < 0.f) s[uint32_t(cand[i])] = -INFINITY;
        __syncthreads();
        if (keep_ties < nt) {
          int r = tie_before;
          for (int i = c0; i < c1; ++i)
            if (s[i] == thr) {
              if (r >= keep_ties) s[i] = -INFINITY;
              ++r;
            }
        }
      }
      __syncthreads();
      stamp(10);
      local = result;
    }
  }
  __syncthreads();
  stamp(11);
  if (in_smem && p.write_scores) {
    float *g = p.scores + size_t(blockIdx.x) * p.logit_stride;
    for (int i = tid; i < n; i += kSampThreads) g[i] = s[i];
  }
  if (tid == 0) {
    if (p.picked) p.picked[blockIdx.x] = local;
    if (local < 0) {
      st.done = 1;
      p.active[st.row_c] = 0;
      if (st.row_u >= 0) p.active[st.row_u] = 0;
      return;
    }
    const int native = local_to_native(local, st.phase);
    st.step = step + 1;
    if (local == st.end_local) {
      st.done = 1;
    } else {
      if (p.out_tokens && st.n_out < p.out_cap) p.out_tokens[size_t(blockIdx.x) * p.out_cap + st.n_out] = native;
      st.hist[st.n_out % kHistCap] = native;
      st.n_out += 1;
    }
    p.token[st.row_c] = native;
    if (st.row_u >= 0) p.token[st.row_u] = native;
    if (st.done || st.step >= st.max_tokens) {
      // The reference forwards no token after the end token or the last step.
      p.active[st.row_c] = 0;
      if (st.row_u >= 0) p.active[st.row_u] = 0;
    }
    stamp_ns(13);
    // Step log (tracing only): request 0's start and end ns for step `step` (64-step ring).
    if (p.trace && blockIdx.x == 0) {
      p.trace[16 + (step & 63) * 4] = t_start;
      p.trace[16 + (step & 63) * 4 + 1] = p.trace[13];
    }
  }
}

static void launch_sampler_impl(RequestState *req, const bf16 *logits, int logit_stride, float *scores, int *token,
                                int *active, int32_t *out_tokens, int out_cap, int write_scores, int32_t *picked,
                                int n_requests, cudaStream_t st, unsigned long long *trace);

void launch_sampler_ex(RequestState *req, const bf16 *logits, int logit_stride, float *scores, int *token,
                       int *active, int32_t *out_tokens, int out_cap, int write_scores, int32_t *picked,
                       int n_requests, cudaStream_t st) {
  launch_sampler_impl(req, logits, logit_stride, scores, token, active, out_tokens, out_cap, write_scores, picked,
                      n_requests, st, nullptr);
}

static void launch_sampler_impl(RequestState *req, const bf16 *logits, int logit_stride, float *scores, int *token,
                                int *active, int32_t *out_tokens, int out_cap, int write_scores, int32_t *picked,
                                int n_requests, cudaStream_t st, unsigned long long *trace) {
  SamplerParams p{req, logits, logit_stride, scores, token, active, out_tokens, out_cap, write_scores, picked, trace};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_requests);
  cfg.blockDim = dim3(kSampThreads);
  cfg.dynamicSmemBytes = kSampSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  YAR_CUDA(cudaLaunchKernelEx(&cfg, k_sampler, p));
}

void configure_sampler_kernels() {
  YAR_CUDA(cudaFuncSetAttribute(k_sampler, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSampSmemBytes)));
}

void launch_sampler(const Model &m, Session &s, int n_requests, cudaStream_t st) {
  // With tracing on, the sampler's phase stamps follow the persistent kernel's timeline.
  unsigned long long *trace =
      s.d_trace ? s.d_trace + size_t(m.sm_count) * (5 * m.d.layers + 1) * 8 : nullptr;
  launch_sampler_impl(s.d_req, s.logits, s.logit_stride, s.d_scores, s.d_token, s.d_active, s.d_out_tokens,
                      s.out_cap, 0, nullptr, n_requests, st, trace);
}

}  // namespace yar
