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
  __shared__ float ev[kCandCap];
  __shared__ int hist[4096];
  __shared__ int ncand, sel_bin, kth_rem, result, tie_total;
  __shared__ float red_v[32];
  __shared__ int red_i[32];
  __shared__ uint32_t prefix_s;

  pdl_launch_dependents();
  pdl_wait();
  RequestState &st = p.req[blockIdx.x];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (st.done || st.step >= st.max_tokens) return;
  const int n = st.width, step = st.step;
  const bf16 *lc = p.logits + size_t(st.row_c) * p.logit_stride;
  const bf16 *lu = st.row_u >= 0 ? p.logits + size_t(st.row_u) * p.logit_stride : nullptr;
  extern __shared__ float s_row[];
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
  {
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
        s[me] = v < 0.f ? f_mul(v, a) : f_div(v, a);
      }
    }
    __syncthreads();
  }

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
      for (int i = tid; i < n; i += kSampThreads) s[i] = f_div(s[i], st.temperature);
      __syncthreads();
    }
    // k-th largest value: radix select on order-preserving keys, digits of 12, 12 and 8
    // bits from the top; histogram updates are aggregated per warp (lanes with the same
    // bin add once) and the bin holding the k-th key is found by a block-wide scan.
    const int k = min(st.top_k, n);
    if (tid == 0) {
      prefix_s = 0;
      kth_rem = k;
    }
    __syncthreads();
    const int shifts[3] = {20, 8, 0}, widths[3] = {12, 12, 8};
    for (int pass = 0; pass < 3; ++pass) {
      const int shift = shifts[pass], nb = 1 << widths[pass];
      for (int b = tid; b < nb; b += kSampThreads) hist[b] = 0;
      __syncthreads();
      const uint32_t pre = prefix_s;
      const uint32_t hmask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + widths[pass]));
      for (int base = warp * 32; base < n; base += kSampThreads) {
        const int i = base + lane;
        uint32_t bin = 0xFFFFFFFFu;
        if (i < n) {
          const uint32_t key = f32_order_key(s[i]);
          if ((key & hmask) == (pre & hmask)) bin = (key >> shift) & uint32_t(nb - 1);
        }
        const unsigned peers = __match_any_sync(0xFFFFFFFFu, bin);
        if (bin != 0xFFFFFFFFu && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
      }
      __syncthreads();
      // Counts from the top bin down: thread t owns bins [nb-1-per*(t+1)+1, nb-1-per*t].
      const int per = (nb + kSampThreads - 1) / kSampThreads;
      const int hi = nb - 1 - per * tid;
      int mine = 0;
      for (int j = 0; j < per; ++j)
        if (hi - j >= 0) mine += hist[hi - j];
      int incl = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane == 31) red_i[warp] = incl;
      __syncthreads();
      if (warp == 0) {
        const int w = red_i[lane];
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xFFFFFFFFu, wi, o);
          if (lane >= o) wi += y;
        }
        red_i[lane] = wi - w;
      }
      __syncthreads();
      const int before = red_i[warp] + incl - mine;  // keys in bins above this thread's bins
      const int rem = kth_rem;
      __syncthreads();
      if (before < rem && before + mine >= rem) {
        int acc = before, b = hi;
        for (int j = 0; j < per && hi - j >= 0; ++j) {
          b = hi - j;
          if (acc + hist[b] >= rem) break;
          acc += hist[b];
        }
        kth_rem = rem - acc;
        prefix_s = pre | (uint32_t(b) << shift);
      }
      __syncthreads();
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
      const float s0 = na > 0 ? s[uint32_t(cand[0])] : thr;
      for (int i = tid; i < na; i += kSampThreads) ev[i] = yexp(f_sub(s[uint32_t(cand[i])], s0));
      __syncthreads();
      if (tid == 0) {
        const float et = yexp(f_sub(thr, s0));
        int keep_ties = nt;
        if (st.top_p < 1.f) {
          float total = 0.f;
          for (int i = 0; i < na; ++i) total = f_add(total, ev[i]);
          for (int j = 0; j < nt; ++j) total = f_add(total, et);
          float c = 0.f;
          for (int i = 0; i < na; ++i) {
            const float pi = f_div(ev[i], total);
            c = f_add(c, pi);
            if (i >= 1 && f_sub(c, pi) > st.top_p) ev[i] = -1.f;  // removed
          }
          // Within the tie group p is constant and c - p never decreases, so the kept
          // ties are a prefix of the group.
          const float pt = f_div(et, total);
          keep_ties = 0;
          for (int j = 0; j < nt; ++j) {
            c = f_add(c, pt);
            if (na + j >= 1 && f_sub(c, pt) > st.top_p) break;
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
      local = result;
    }
  }
  __syncthreads();
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
  }
}

void launch_sampler_ex(RequestState *req, const bf16 *logits, int logit_stride, float *scores, int *token,
                       int *active, int32_t *out_tokens, int out_cap, int write_scores, int32_t *picked,
                       int n_requests, cudaStream_t st) {
  SamplerParams p{req, logits, logit_stride, scores, token, active, out_tokens, out_cap, write_scores, picked};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_requests);
  cfg.blockDim = dim3(kSampThreads);
  cfg.dynamicSmemBytes = kSampSmemScores * sizeof(float);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  YAR_CUDA(cudaLaunchKernelEx(&cfg, k_sampler, p));
}

void configure_sampler_kernels() {
  YAR_CUDA(cudaFuncSetAttribute(k_sampler, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kSampSmemScores * sizeof(float))));
}

void launch_sampler(const Model &m, Session &s, int n_requests, cudaStream_t st) {
  (void)m;
  launch_sampler_ex(s.d_req, s.logits, s.logit_stride, s.d_scores, s.d_token, s.d_active, s.d_out_tokens,
                    s.out_cap, 0, nullptr, n_requests, st);
}

}  // namespace yar
