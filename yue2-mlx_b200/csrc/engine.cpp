// engine.cpp — sessions (paged KV cache, activations, sampler state), chunked prefill,
// the decode step (captured once as a CUDA graph and replayed per token) and the
// generate_tokens loop (native/src/sampling.cpp:185-288; upstream sampling.py:57-154).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <sstream>

#include "engine.h"
#include "exact_math.cuh"
#include "nlohmann/json.hpp"
#include "yue2ar.h"

namespace yar {

void launch_sampler_ex(RequestState *req, const bf16 *logits, int logit_stride, float *scores, int *token,
                       int *active, int32_t *out_tokens, int out_cap, int write_scores, int32_t *picked,
                       int n_requests, cudaStream_t st);

static double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

template <typename T>
static T *dmalloc(size_t n) {
  T *p = nullptr;
  YAR_CUDA(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
  return p;
}

Session *create_session(Model *m, int max_rows, int max_ctx, int page_tokens) {
  if (max_rows < 1 || max_rows > 256) throw Error("ValueError", "max_rows must be in [1, 256]");
  if (max_ctx < 1 || max_ctx > m->d.context)
    throw Error("ValueError", "KV cache capacity must be in [1, " + std::to_string(m->d.context) + "]");
  if (page_tokens == 0) page_tokens = 256;
  if (page_tokens < 16 || page_tokens > 4096 || (page_tokens & (page_tokens - 1)))
    throw Error("ValueError", "page_tokens must be a power of two in [16, 4096]");
  YAR_CUDA(cudaSetDevice(m->device));
  auto *s = new Session();
  try {
    const Dims &d = m->d;
    s->m = m;
    s->max_rows = max_rows;
    s->max_ctx = max_ctx;
    s->page_tokens = page_tokens;
    s->pages_per_row = (max_ctx + page_tokens - 1) / page_tokens;
    s->num_pages = s->pages_per_row * max_rows;
    s->kv_page_elems = size_t(d.kv_heads) * page_tokens * d.head_dim;
    YAR_CUDA(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
    s->kv = dmalloc<bf16>(size_t(d.layers) * s->num_pages * 2 * s->kv_page_elems);
    s->row_pages.assign(max_rows, {});
    for (int p = s->num_pages - 1; p >= 0; --p) s->free_pages.push_back(p);
    s->d_page_table = dmalloc<int>(size_t(max_rows) * s->pages_per_row);
    YAR_CUDA(cudaMemset(s->d_page_table, 0, size_t(max_rows) * s->pages_per_row * sizeof(int)));
    s->d_pos = dmalloc<int>(max_rows);
    s->d_cur_pos = dmalloc<int>(max_rows);
    s->d_capacity = dmalloc<int>(max_rows);
    s->d_token = dmalloc<int>(max_rows);
    s->d_active = dmalloc<int>(max_rows);
    s->d_error = dmalloc<int>(1);
    for (int *p : {s->d_pos, s->d_cur_pos, s->d_capacity, s->d_token, s->d_active})
      YAR_CUDA(cudaMemset(p, 0, max_rows * sizeof(int)));
    YAR_CUDA(cudaMemset(s->d_error, 0, sizeof(int)));
    s->capacity.assign(max_rows, 0);
    s->pos.assign(max_rows, 0);
    s->qkv = dmalloc<bf16>(size_t(max_rows) * d.qkv_rows());
    int widest = d.vocab;
    if (d.vocab == 184704) widest = std::max(phase_rows(d, kPhaseAbc).width(), phase_rows(d, kPhaseSemantic).width());
    s->logit_stride = (widest + 7) & ~7;
    // The exchange region: residual rows, attention and FFN activations (at the whole
    // model's width: under tensor parallelism each rank writes its block and the exchange
    // fills in the others), logits rows and the persistent kernel's counters.
    const Dims &f = m->full;
    s->n_ctr = 2 + 5 * d.layers;
    {
      size_t off = 0;
      auto take = [&](size_t bytes) {
        const size_t o = off;
        off = (off + bytes + 255) & ~size_t(255);
        return o;
      };
      const size_t ox = take(size_t(max_rows) * d.hidden * 2), oa = take(size_t(max_rows) * f.qdim() * 2),
                   om = take(size_t(max_rows) * f.ffn * 2), ol = take(size_t(max_rows) * s->logit_stride * 2),
                   oc = take(size_t(s->n_ctr) * 4);
      // Flagged words: 8 bytes per two values, for the persistent kernel's 1 or 2 rows.
      const size_t llr = size_t(std::min(max_rows, 2));
      const size_t oxl = take(llr * d.hidden * 4), oql = take(llr * d.qkv_rows() * 4), oal = take(llr * f.qdim() * 4),
                   oml = take(llr * f.ffn * 4),
                   opl = take(llr * d.heads * kSessionMaxSplits * (d.head_dim + 2) * sizeof(uint2));
      s->xregion = dmalloc<char>(off);
      s->xregion_bytes = off;
      YAR_CUDA(cudaMemset(s->xregion, 0, off));
      s->x = reinterpret_cast<bf16 *>(s->xregion + ox);
      s->attn = reinterpret_cast<bf16 *>(s->xregion + oa);
      s->mlp = reinterpret_cast<bf16 *>(s->xregion + om);
      s->logits = reinterpret_cast<bf16 *>(s->xregion + ol);
      s->d_ctr = reinterpret_cast<int *>(s->xregion + oc);
      s->x_ll = reinterpret_cast<uint2 *>(s->xregion + oxl);
      s->qkv_ll = reinterpret_cast<uint2 *>(s->xregion + oql);
      s->attn_ll = reinterpret_cast<uint2 *>(s->xregion + oal);
      s->mlp_ll = reinterpret_cast<uint2 *>(s->xregion + oml);
      s->part_ll = reinterpret_cast<uint2 *>(s->xregion + opl);
      s->ll_bytes = off - oxl;
    }
    s->max_splits = kSessionMaxSplits;
    s->attn_part = dmalloc<float>(size_t(max_rows) * d.heads * s->max_splits * (d.head_dim + 2));
    s->attn_count = dmalloc<int>(size_t(max_rows) * d.kv_heads);
    YAR_CUDA(cudaMemset(s->attn_count, 0, size_t(max_rows) * d.kv_heads * sizeof(int)));
    const int T = s->prefill_chunk;
    s->px = dmalloc<bf16>(size_t(T) * d.hidden);
    s->ph = dmalloc<bf16>(size_t(T) * d.hidden);
    s->pqkv = dmalloc<bf16>(size_t(T) * d.qkv_rows());
    s->pq = dmalloc<bf16>(size_t(T) * d.qdim());
    s->pattn = dmalloc<bf16>(size_t(T) * f.qdim());
    s->pmlp = dmalloc<bf16>(size_t(T) * f.ffn);
    s->pids = dmalloc<int>(T);
    s->max_requests = max_rows;
    s->d_req = dmalloc<RequestState>(max_rows);
    YAR_CUDA(cudaMemset(s->d_req, 0, max_rows * sizeof(RequestState)));
    s->out_cap = max_ctx;
    s->d_out_tokens = dmalloc<int32_t>(size_t(max_rows) * s->out_cap);
    s->d_scores = dmalloc<float>(size_t(max_rows) * s->logit_stride);
    YAR_CUDA(cudaMallocHost(&s->h_pinned, 1 << 20));
    s->gemm_ws_floats = size_t(4) << 20;
    s->gemm_ws = dmalloc<float>(s->gemm_ws_floats);
    if (m->tp_world > 1) {
      const size_t block = std::max({size_t(std::max(T, max_rows)) * std::max({d.qdim(), d.ffn, m->tp.h_rows}),
                                     size_t(max_rows) * tp_head_slice(widest, m->tp_world)});
      s->tp_send = dmalloc<bf16>(block);
      s->tp_recv = dmalloc<bf16>(size_t(m->tp_world) * block);
    }
    s->d_epoch = dmalloc<int>(1);
    YAR_CUDA(cudaMemset(s->d_epoch, 0, sizeof(int)));
    YAR_CUDA(cudaDeviceSynchronize());
    // Collective under tensor parallelism: map the peers' exchange regions (their counters
    // are zero already: each rank zeroed its region before this exchange).
    if (m->tp_world > 1)
      s->tp_mapped = tp_map_peers(*m, s->xregion, s->xregion_bytes, s->tp_peer_regions, s->tp_dst, s->stream);
  } catch (...) {
    delete s;
    throw;
  }
  return s;
}

void free_session(Session *s) {
  if (!s) return;
  cudaSetDevice(s->m->device);
  cudaStreamSynchronize(s->stream);
  for (auto &g : s->graphs) cudaGraphExecDestroy(g.exec);
  tp_unmap_peers(s->tp_peer_regions);
  for (void *p : std::initializer_list<void *>{s->kv, s->d_page_table, s->d_pos, s->d_cur_pos, s->d_capacity,
                                               s->d_token, s->d_active, s->d_error, s->xregion, s->qkv,
                                               s->attn_part, s->attn_count, s->px, s->ph, s->pqkv, s->pq,
                                               s->pattn, s->pmlp, s->pids, s->d_req, s->d_out_tokens,
                                               s->d_scores, s->d_epoch, s->d_trace, s->gemm_ws, s->tp_send,
                                               s->tp_recv, s->d_layer_dump})
    if (p) cudaFree(p);
  if (s->h_pinned) cudaFreeHost(s->h_pinned);
  if (s->stream) cudaStreamDestroy(s->stream);
  delete s;
}

static void check_row(const Session &s, int row) {
  if (row < 0 || row >= s.max_rows) throw Error("ValueError", "row outside the session");
}

void row_reset(Session &s, int row, int capacity) {
  check_row(s, row);
  if (capacity < 1 || capacity > s.max_ctx)
    throw Error("ValueError", "KV cache capacity must be in [1, " + std::to_string(s.max_ctx) + "]");
  YAR_CUDA(cudaStreamSynchronize(s.stream));
  for (int p : s.row_pages[row]) s.free_pages.push_back(p);
  s.row_pages[row].clear();
  const int need = (capacity + s.page_tokens - 1) / s.page_tokens;
  if (int(s.free_pages.size()) < need) throw Error("ValueError", "KV page pool exhausted; generation was not shortened");
  std::vector<int> table(s.pages_per_row, 0);
  for (int i = 0; i < need; ++i) {
    table[i] = s.free_pages.back();
    s.row_pages[row].push_back(table[i]);
    s.free_pages.pop_back();
  }
  YAR_CUDA(cudaMemcpyAsync(s.d_page_table + size_t(row) * s.pages_per_row, table.data(),
                           table.size() * sizeof(int), cudaMemcpyHostToDevice, s.stream));
  const int zero = 0;
  YAR_CUDA(cudaMemcpyAsync(s.d_pos + row, &zero, sizeof(int), cudaMemcpyHostToDevice, s.stream));
  YAR_CUDA(cudaMemcpyAsync(s.d_capacity + row, &capacity, sizeof(int), cudaMemcpyHostToDevice, s.stream));
  YAR_CUDA(cudaMemcpyAsync(s.d_active + row, &zero, sizeof(int), cudaMemcpyHostToDevice, s.stream));
  YAR_CUDA(cudaStreamSynchronize(s.stream));
  s.capacity[row] = capacity;
  s.pos[row] = 0;
}

// Phase columns [c0, c1) of the LM head for `n_rows` input rows into out ([n_rows][stride],
// column c at out[c - c0]). `normed`: `in` holds the final-normed rows and the main rows
// go through the GEMM (an even number of them) with the GEMV for an odd last one; else
// the GEMVs apply the final RMSNorm themselves. Each column's value depends only on its
// weight row, so any column range gives the bits of the whole projection.
static void project_cols(const Model &m, Session &s, const bf16 *in, int in_stride, bool normed, int n_rows,
                         int phase, int c0, int c1, bf16 *out, int stride) {
  const PhaseRows pr = phase_rows(m.d, phase);
  const int H = m.d.hidden;
  cudaStream_t st = s.stream;
  const bf16 *norm_w = normed ? nullptr : m.final_norm;
  const int main_end = std::min(c1, pr.n_main);
  const bf16 *head = m.lm_head + size_t(pr.row0) * H;
  if (main_end > c0) {
    if (normed) {
      // Even rows as GEMMs: the whole 128-column blocks (aligned to absolute phase columns;
      // tensor-parallel ranges start on such a block) on tcgen05, never split along K, and
      // the last partial block on mma.sync — so a column's kernel, hence its bits, does not
      // depend on which range (rank) holds it.
      const int n_even = pr.n_main & ~1, g_end = std::min(main_end, n_even);
      int t0 = (c0 + 127) / 128 * 128, t1 = g_end / 128 * 128;
      if (t1 <= t0 || !gemm_tc_supported(in, n_rows, H, head + size_t(t0) * H, t1 - t0, out + (t0 - c0), stride))
        t0 = t1 = g_end;
      if (t0 > c0) launch_gemm(in, n_rows, H, head + size_t(c0) * H, t0 - c0, out, stride, kEpiStore, st);
      if (t1 > t0)
        launch_gemm_tc(in, n_rows, H, head + size_t(t0) * H, t1 - t0, out + (t0 - c0), stride, kEpiStore, s.d_error,
                       nullptr, 0, st, -1);
      if (g_end > t1) launch_gemm(in, n_rows, H, head + size_t(t1) * H, g_end - t1, out + (t1 - c0), stride, kEpiStore, st);
      if (n_even < main_end)
        launch_gemv(head + size_t(n_even) * H, 1, H, in, in_stride, nullptr, m.d.eps, out + (n_even - c0), stride,
                    kEpiStore, n_rows, s.d_error, m.sm_count, st);
    } else {
      launch_gemv(head + size_t(c0) * H, main_end - c0, H, in, in_stride, norm_w, m.d.eps, out, stride, kEpiStore,
                  n_rows, s.d_error, m.sm_count, st);
    }
  }
  if (pr.extra >= 0 && c0 <= pr.n_main && pr.n_main < c1)
    launch_gemv(m.lm_head + size_t(pr.extra) * H, 1, H, in, in_stride, norm_w, m.d.eps, out + (pr.n_main - c0),
                stride, kEpiStore, n_rows, s.d_error, m.sm_count, st);
}

// LM head over the phase columns for `n_rows` input rows into logits rows (stride
// logit_stride). Under tensor parallelism rank r projects columns [r*slice, (r+1)*slice)
// into its send block, the blocks are all-gathered and laid out as whole logits rows on
// every rank.
static void project(const Model &m, Session &s, const bf16 *in, int in_stride, bool normed, int n_rows, int phase,
                    bf16 *out) {
  const int width = phase_rows(m.d, phase).width();
  if (m.tp_world == 1) return project_cols(m, s, in, in_stride, normed, n_rows, phase, 0, width, out, s.logit_stride);
  const int slice = tp_head_slice(width, m.tp_world);
  const int a = std::min(width, m.tp_rank * slice), b = std::min(width, a + slice);
  project_cols(m, s, in, in_stride, normed, n_rows, phase, a, b, s.tp_send, slice);
  tp_allgather_bf16(m, s.tp_send, s.tp_recv, size_t(n_rows) * slice, s.stream);
  launch_tp_unpack(s.tp_recv, m.tp_world, n_rows, slice, width, out, s.logit_stride, s.stream);
}

// Under tensor parallelism: every rank's block of columns [k*n, k*n + n) of the activation
// rows buf ([n_rows][stride]) into every rank's buf. One row whose blocks tile it is
// gathered in place; otherwise through the pack / all-gather / unpack steps.
static void tp_gather(const Model &m, Session &s, bf16 *buf, int n_rows, int stride, int n) {
  if (m.tp_world == 1) return;
  const int W = m.tp_world;
  if (n_rows == 1 && stride == W * n) {
    tp_allgather_bf16(m, buf + size_t(m.tp_rank) * n, buf, size_t(n), s.stream);
    return;
  }
  launch_tp_pack(buf, stride, m.tp_rank * n, n, n_rows, s.tp_send, s.stream);
  tp_allgather_bf16(m, s.tp_send, s.tp_recv, size_t(n_rows) * n, s.stream);
  launch_tp_unpack(s.tp_recv, W, n_rows, n, W * n, buf, stride, s.stream);
}

// The shapes of one layer's linears on this rank (the whole layer on one GPU): hidden
// width, query width of the model / of this rank, FFN width of the model / of this rank,
// and this rank's block of hidden rows of O and down.
struct LayerShape {
  int H, Qf, Ql, Ff, Fl, Hs, h0;
};
static LayerShape layer_shape(const Model &m) {
  return {m.d.hidden, m.full.qdim(), m.d.qdim(), m.full.ffn, m.d.ffn, m.tp.h_rows, m.tp.h_row0};
}

void row_prefill(Session &s, int row, const int32_t *ids, int n, int phase, int chunk,
                 int (*cancel)(void *), void *cancel_ctx) {
  check_row(s, row);
  const Model &m = *s.m;
  const Dims &d = m.d;
  if (n < 1) throw Error("ValueError", "AR prefix must contain at least one token");
  for (int i = 0; i < n; ++i)
    if (ids[i] < 0 || ids[i] >= d.vocab)
      throw Error("ValueError", "Token IDs must be in [0, " + std::to_string(d.vocab) + ")");
  phase_rows(d, phase);
  if (chunk <= 0) chunk = 1024;
  chunk = std::min(chunk, s.prefill_chunk);
  const int start0 = s.pos[row];
  if (start0 + n > s.capacity[row]) throw Error("ValueError", "KV cache capacity exceeded; generation was not shortened");
  cudaStream_t st = s.stream;
  YAR_CUDA(cudaMemsetAsync(s.d_error, 0, sizeof(int), st));
  const int H = d.hidden, QKV = d.qkv_rows();
  // Linears on the tcgen05 tensor-core GEMM where the shape allows (K % 64, N % 128);
  // otherwise the mma.sync GEMM.
  // Linears are split by output rows under tensor parallelism: the K split follows the
  // whole model's N (tp_world x this rank's).
  auto gemm = [&](const bf16 *A, int M, int K, const bf16 *W, int N, bf16 *C, int ldc, int epi) {
    if (gemm_tc_supported(A, M, K, W, N, C, ldc))
      launch_gemm_tc(A, M, K, W, N, C, ldc, epi, s.d_error, s.gemm_ws, s.gemm_ws_floats, st, N * m.tp_world);
    else
      launch_gemm(A, M, K, W, N, C, ldc, epi, st);
  };
  const LayerShape ls = layer_shape(m);
  for (int c0 = 0; c0 < n; c0 += chunk) {
    if (cancel && cancel(cancel_ctx)) throw Error("InterruptedError", "Cancelled during prefill");
    const int T = std::min(chunk, n - c0), start = start0 + c0;
    YAR_CUDA(cudaMemcpyAsync(s.pids, ids + c0, T * sizeof(int), cudaMemcpyHostToDevice, st));
    launch_embed_tokens(m.embed, s.pids, T, H, s.px, st);
    for (int l = 0; l < d.layers; ++l) {
      const LayerWeights &w = m.layers[l];
      launch_rmsnorm_rows(s.px, w.ln1, T, H, d.eps, s.ph, st);
      gemm(s.ph, T, H, w.qkv, QKV, s.pqkv, QKV, kEpiStore);
      launch_qkv_post_prefill(m, s, l, row, start, T, st);
      launch_attn_prefill(m, s, l, row, start, T, st);
      tp_gather(m, s, s.pattn, T, ls.Qf, ls.Ql);
      gemm(s.pattn, T, ls.Qf, w.o, ls.Hs, s.px + ls.h0, H, kEpiResidual);
      tp_gather(m, s, s.px, T, H, ls.Hs);
      launch_rmsnorm_rows(s.px, w.ln2, T, H, d.eps, s.ph, st);
      gemm(s.ph, T, H, w.gu, 2 * ls.Fl, s.pmlp + size_t(m.tp_rank) * ls.Fl, ls.Ff, kEpiSwiGLU);
      tp_gather(m, s, s.pmlp, T, ls.Ff, ls.Fl);
      gemm(s.pmlp, T, ls.Ff, w.down, ls.Hs, s.px + ls.h0, H, kEpiResidual);
      tp_gather(m, s, s.px, T, H, ls.Hs);
    }
    if (c0 + T == n)
      project(m, s, s.px + size_t(T - 1) * H, H, false, 1, phase, s.logits + size_t(row) * s.logit_stride);
    YAR_CUDA(cudaStreamSynchronize(st));
  }
  int err = 0;
  YAR_CUDA(cudaMemcpy(&err, s.d_error, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) throw Error("RuntimeError", "device error flags " + std::to_string(err));
  s.pos[row] = start0 + n;
  YAR_CUDA(cudaMemcpyAsync(s.d_pos + row, &s.pos[row], sizeof(int), cudaMemcpyHostToDevice, st));
  YAR_CUDA(cudaStreamSynchronize(st));
}

// One decode forward of rows [0, n_rows): embed -> 28 x (QKV, attention, O, gate/up, down)
// -> LM head. Inactive rows are skipped by the embed/attention kernels.
static bool use_persistent(Session &s, int n_rows) {
  // The persistent kernel streams each 64-position KV chunk as one contiguous copy, so a
  // chunk must not straddle pages. Under tensor parallelism it needs the peers' exchange
  // regions mapped (otherwise the per-operation path exchanges through NCCL).
  if (!s.use_persistent || n_rows < 1 || n_rows > 2 || s.page_tokens < 64) return false;
  if (s.m->tp_world > 1 && !s.tp_mapped) return false;
  if (s.persistent_ok[n_rows] < 0) s.persistent_ok[n_rows] = persistent_supported(*s.m, n_rows) ? 1 : 0;
  return s.persistent_ok[n_rows] == 1;
}

// Zero the persistent kernel's operation counters and step epoch (and the split-KV
// arrival counts) before a sequence of decode steps.
//
// Under tensor parallelism peers add to this rank's counters, and a peer may already be in
// its next step's first exchange while this rank is still on the host: the counters and the
// epoch are never zeroed then (targets grow with the epoch), except every 2^20 steps, when
// all ranks stop at a barrier, zero them, and meet again before any of them goes on.
static void reset_step_sync(Session &s) {
  // The flagged words restart with the epoch: their flags (step, operation) must not match
  // anything written before the reset.
  if (s.m->tp_world == 1 || !s.tp_mapped) {
    YAR_CUDA(cudaMemsetAsync(s.d_ctr, 0, s.n_ctr * sizeof(int), s.stream));
    YAR_CUDA(cudaMemsetAsync(s.d_epoch, 0, sizeof(int), s.stream));
    YAR_CUDA(cudaMemsetAsync(s.x_ll, 0, s.ll_bytes, s.stream));
  } else if (s.tp_epoch_steps >= (1ll << 20)) {
    tp_barrier(*s.m, s.tp_send, s.stream);
    YAR_CUDA(cudaMemsetAsync(s.d_ctr, 0, s.n_ctr * sizeof(int), s.stream));
    YAR_CUDA(cudaMemsetAsync(s.d_epoch, 0, sizeof(int), s.stream));
    YAR_CUDA(cudaMemsetAsync(s.x_ll, 0, s.ll_bytes, s.stream));
    tp_barrier(*s.m, s.tp_send, s.stream);
    s.tp_epoch_steps = 0;
  }
  YAR_CUDA(cudaMemsetAsync(s.attn_count, 0, size_t(s.max_rows) * s.m->d.kv_heads * sizeof(int), s.stream));
}

// Hidden-state record (session option): the residual rows into slot `slot` of the record
// (0 = embedding, l + 1 = after layer l).
static void dump_hidden(Session &s, int slot, int n_rows) {
  if (!s.d_layer_dump) return;
  const size_t H = size_t(s.m->d.hidden);
  YAR_CUDA(cudaMemcpyAsync(s.d_layer_dump + size_t(slot) * s.max_rows * H, s.x, size_t(n_rows) * H * sizeof(bf16),
                           cudaMemcpyDeviceToDevice, s.stream));
}

// Batches of at least this many rows run the decode linears as tcgen05 GEMMs: the weights
// are read once per step for all rows instead of once per 8 rows.
constexpr int kBatchedRows = 16;

// One decode forward of many rows: RMSNorm rows -> tcgen05 GEMM (QKV, O + residual,
// gate/up + SwiGLU, down + residual), the split-KV decode attention per row, and the
// phase head as a GEMM over the normalized rows.
static void decode_forward_batched(Session &s, int n_rows, int phase) {
  const Model &m = *s.m;
  const Dims &d = m.d;
  cudaStream_t st = s.stream;
  const int H = d.hidden;
  auto gemm = [&](const bf16 *A, int K, const bf16 *W, int N, bf16 *C, int ldc, int epi) {
    if (gemm_tc_supported(A, n_rows, K, W, N, C, ldc))
      launch_gemm_tc(A, n_rows, K, W, N, C, ldc, epi, s.d_error, s.gemm_ws, s.gemm_ws_floats, st, N * m.tp_world);
    else
      launch_gemm(A, n_rows, K, W, N, C, ldc, epi, st);
  };
  // About two waves of attention CTAs (5 resident per SM): fewer, longer splits per row
  // than the one-row path, so each CTA streams several chunks. (Counted with the whole
  // model's KV heads, so tensor-parallel ranks split each head's positions the same way.)
  const int kvh = m.full.kv_heads;
  const int splits = std::max(1, (2 * 5 * m.sm_count + n_rows * kvh - 1) / (n_rows * kvh));
  const LayerShape ls = layer_shape(m);
  launch_embed_rows(m, s, n_rows, st);
  dump_hidden(s, 0, n_rows);
  for (int l = 0; l < d.layers; ++l) {
    const LayerWeights &w = m.layers[l];
    launch_rmsnorm_rows(s.x, w.ln1, n_rows, H, d.eps, s.ph, st);
    gemm(s.ph, H, w.qkv, d.qkv_rows(), s.qkv, d.qkv_rows(), kEpiStore);
    launch_attn_decode(m, s, l, n_rows, st, splits);
    tp_gather(m, s, s.attn, n_rows, ls.Qf, ls.Ql);
    gemm(s.attn, ls.Qf, w.o, ls.Hs, s.x + ls.h0, H, kEpiResidual);
    tp_gather(m, s, s.x, n_rows, H, ls.Hs);
    launch_rmsnorm_rows(s.x, w.ln2, n_rows, H, d.eps, s.ph, st);
    gemm(s.ph, H, w.gu, 2 * ls.Fl, s.mlp + size_t(m.tp_rank) * ls.Fl, ls.Ff, kEpiSwiGLU);
    tp_gather(m, s, s.mlp, n_rows, ls.Ff, ls.Fl);
    gemm(s.mlp, ls.Ff, w.down, ls.Hs, s.x + ls.h0, H, kEpiResidual);
    tp_gather(m, s, s.x, n_rows, H, ls.Hs);
    dump_hidden(s, l + 1, n_rows);
  }
  // Head: GEMM over the normalized rows (odd last phase row and ABC extra row as GEMVs).
  launch_rmsnorm_rows(s.x, m.final_norm, n_rows, H, d.eps, s.ph, st);
  project(m, s, s.ph, H, true, n_rows, phase, s.logits);
}

static void decode_forward(Session &s, int n_rows, int phase) {
  const Model &m = *s.m;
  const Dims &d = m.d;
  cudaStream_t st = s.stream;
  if (use_persistent(s, n_rows)) {
    launch_decode_persistent(m, s, n_rows, phase, st);
    return;
  }
  if (n_rows >= kBatchedRows && n_rows <= s.prefill_chunk) {
    decode_forward_batched(s, n_rows, phase);
    return;
  }
  const LayerShape ls = layer_shape(m);
  const int H = d.hidden;
  launch_embed_rows(m, s, n_rows, st);
  dump_hidden(s, 0, n_rows);
  for (int l = 0; l < d.layers; ++l) {
    const LayerWeights &w = m.layers[l];
    launch_gemv(w.qkv, d.qkv_rows(), H, s.x, H, w.ln1, d.eps, s.qkv, d.qkv_rows(), kEpiStore, n_rows, s.d_error,
                m.sm_count, st);
    launch_attn_decode(m, s, l, n_rows, st, decode_max_splits(m, s, n_rows));
    tp_gather(m, s, s.attn, n_rows, ls.Qf, ls.Ql);
    launch_gemv(w.o, ls.Hs, ls.Qf, s.attn, ls.Qf, nullptr, d.eps, s.x + ls.h0, H, kEpiResidual, n_rows, s.d_error,
                m.sm_count, st);
    tp_gather(m, s, s.x, n_rows, H, ls.Hs);
    launch_gemv(w.gu, 2 * ls.Fl, H, s.x, H, w.ln2, d.eps, s.mlp + size_t(m.tp_rank) * ls.Fl, ls.Ff, kEpiSwiGLU,
                n_rows, s.d_error, m.sm_count, st);
    tp_gather(m, s, s.mlp, n_rows, ls.Ff, ls.Fl);
    launch_gemv(w.down, ls.Hs, ls.Ff, s.mlp, ls.Ff, nullptr, d.eps, s.x + ls.h0, H, kEpiResidual, n_rows, s.d_error,
                m.sm_count, st);
    tp_gather(m, s, s.x, n_rows, H, ls.Hs);
    dump_hidden(s, l + 1, n_rows);
  }
  project(m, s, s.x, H, false, n_rows, phase, s.logits);
}

void rows_step(Session &s, const int *rows, const int32_t *tokens, int n, int phase) {
  if (n < 1) throw Error("ValueError", "rows_step needs at least one row");
  int hi = 0;
  for (int i = 0; i < n; ++i) {
    check_row(s, rows[i]);
    hi = std::max(hi, rows[i] + 1);
    if (tokens[i] < 0 || tokens[i] >= s.m->d.vocab) throw Error("ValueError", "Token is outside the model vocabulary");
    if (s.pos[rows[i]] + 1 > s.capacity[rows[i]])
      throw Error("ValueError", "KV cache capacity exceeded; generation was not shortened");
  }
  phase_rows(s.m->d, phase);
  std::vector<int> active(hi, 0), tok(hi, 0);
  for (int i = 0; i < n; ++i) {
    active[rows[i]] = 1;
    tok[rows[i]] = tokens[i];
  }
  cudaStream_t st = s.stream;
  YAR_CUDA(cudaMemcpyAsync(s.d_active, active.data(), hi * sizeof(int), cudaMemcpyHostToDevice, st));
  YAR_CUDA(cudaMemcpyAsync(s.d_token, tok.data(), hi * sizeof(int), cudaMemcpyHostToDevice, st));
  YAR_CUDA(cudaMemsetAsync(s.d_error, 0, sizeof(int), st));
  reset_step_sync(s);
  decode_forward(s, hi, phase);
  s.tp_epoch_steps += 1;
  YAR_CUDA(cudaStreamSynchronize(st));
  int err = 0;
  YAR_CUDA(cudaMemcpy(&err, s.d_error, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) {
    // The step is void: the rows keep their positions (the device latch may have advanced)
    // and the session stays usable for the next call.
    YAR_CUDA(cudaMemcpyAsync(s.d_pos, s.pos.data(), s.max_rows * sizeof(int), cudaMemcpyHostToDevice, st));
    YAR_CUDA(cudaStreamSynchronize(st));
    throw Error("RuntimeError", "device error flags " + std::to_string(err));
  }
  for (int i = 0; i < n; ++i) s.pos[rows[i]] += 1;
}

// The per-token step (sampler, then the forward of the sampled token), captured once
// per (rows, requests, phase) and replayed.
static cudaGraphExec_t step_graph(Session &s, int n_rows, int n_requests, int phase) {
  const int pers = use_persistent(s, n_rows) ? 1 : 0;
  for (auto &g : s.graphs)
    if (g.rows == n_rows && g.requests == n_requests && g.phase == phase && g.persistent == pers) return g.exec;
  cudaStream_t st = s.stream;
  YAR_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  cudaGraph_t graph;
  try {
    launch_sampler(*s.m, s, n_requests, st);
    decode_forward(s, n_rows, phase);
  } catch (...) {
    cudaStreamEndCapture(st, &graph);
    throw;
  }
  YAR_CUDA(cudaStreamEndCapture(st, &graph));
  cudaGraphExec_t exec;
  YAR_CUDA(cudaGraphInstantiate(&exec, graph, 0));
  YAR_CUDA(cudaGraphDestroy(graph));
  s.graphs.push_back({n_rows, n_requests, phase, pers, exec});
  return exec;
}

void fill_penalty_alpha(RequestState &r, double penalty, bool legacy) {
  const double base = legacy ? double(round_bf16(float(penalty))) : double(float(penalty));
  for (int i = 0; i <= kMaxPenaltyWindow; ++i) {
    const float a = float(std::pow(base, double(i)));
    r.alpha[i] = legacy ? round_bf16(a) : a;
  }
}

static RequestState make_request(const Model &m, const Session &s, int row_c, int row_u, int phase,
                                 const ::yar_sampling &smp, double cfg_scale, uint64_t seed, uint32_t stream,
                                 bool legacy) {
  RequestState r;
  std::memset(&r, 0, sizeof(r));
  r.row_c = row_c;
  r.row_u = row_u;
  r.phase = phase;
  r.width = phase_rows(m.d, phase).width();
  r.end_local = phase == kPhaseAbc ? kEOD : phase == kPhaseSemantic ? 0 : -1;
  r.temperature = float(smp.temperature);
  r.top_p = float(smp.top_p);
  r.cfg_scale = float(cfg_scale);
  r.top_k = smp.top_k;
  r.window = smp.penalty_window;
  r.min_tokens = smp.min_tokens;
  r.max_tokens = smp.max_tokens;
  r.penalty_on = smp.repetition_penalty != 1.0;
  r.legacy = legacy ? 1 : 0;
  fill_penalty_alpha(r, smp.repetition_penalty, legacy);
  r.seed_lo = uint32_t(seed);
  r.seed_hi = uint32_t(seed >> 32);
  r.stream = stream;
  (void)s;
  return r;
}

void validate_sampling(const ::yar_sampling &s) {
  auto finite = [](double v) { return std::isfinite(v); };
  if (!finite(s.temperature) || !finite(s.top_p) || !finite(s.repetition_penalty))
    throw Error("ValueError", "Sampling numbers must be finite");
  if (!(s.temperature >= 0 && s.temperature <= 5) || !(s.top_p > 0 && s.top_p <= 1) || s.top_k < 1)
    throw Error("ValueError", "Invalid sampling temperature/top_p/top_k");
  if (s.repetition_penalty <= 0 || s.penalty_window < 1 || s.penalty_window > 100)
    throw Error("ValueError", "Invalid repetition penalty/window");
  if (!(0 <= s.min_tokens && s.min_tokens <= s.max_tokens) || s.max_tokens < 1)
    throw Error("ValueError", "Require 0 <= min_tokens <= max_tokens");
  if (s.temperature > 0 && s.top_k > kCandCap)
    throw Error("ValueError", "top_k above 2048 is not supported by the device sampler");
}

std::string generate(Session &s, const int32_t *prefix, int n_prefix, const ::yar_sampling &smp, uint64_t seed,
                     int phase, const int32_t *negative, int n_negative, double cfg_scale, int legacy_off,
                     int (*cancel)(void *), void *cancel_ctx, void (*on_token)(void *, int, int32_t),
                     void *token_ctx, int32_t *out_tokens, int *n_out, int *truncated) {
  const Model &m = *s.m;
  phase_rows(m.d, phase);
  validate_sampling(smp);
  if (seed >= (uint64_t(1) << 63)) throw Error("ValueError", "seed must be an integer in [0, 2**63)");
  if (n_prefix < 1) throw Error("ValueError", "AR prefix must contain at least one token");
  if (size_t(n_prefix) + size_t(smp.max_tokens) > size_t(m.d.context))
    throw Error("ValueError", "Prefix + requested generation budget exceeds 24576; no implicit truncation");
  const bool cfg = cfg_scale != 1.0;
  if (cfg && n_negative < 1) throw Error("ValueError", "CFG requires a negative prefix");
  if (n_negative > 0 && size_t(n_negative) + size_t(smp.max_tokens) > size_t(m.d.context))
    throw Error("ValueError", "Negative prefix + generation budget exceeds context");
  const int rows = cfg ? 2 : 1;
  if (rows > s.max_rows) throw Error("ValueError", "CFG needs a session with at least two rows");
  if (n_prefix + smp.max_tokens > s.max_ctx || (cfg && n_negative + smp.max_tokens > s.max_ctx))
    throw Error("ValueError", "KV cache capacity exceeded; generation was not shortened");
  if (smp.max_tokens > s.out_cap) throw Error("ValueError", "max_tokens exceeds the session output capacity");
  if (cancel && cancel(cancel_ctx)) throw Error("InterruptedError", "Cancelled before prefill");

  YAR_CUDA(cudaSetDevice(m.device));
  YAR_CUDA(cudaStreamSynchronize(s.stream));
  const double t0 = now_s();
  row_reset(s, 0, n_prefix + smp.max_tokens);
  row_prefill(s, 0, prefix, n_prefix, phase, 0, cancel, cancel_ctx);
  if (cfg) {
    row_reset(s, 1, n_negative + smp.max_tokens);
    row_prefill(s, 1, negative, n_negative, phase, 0, cancel, cancel_ctx);
  }
  const double prefill_seconds = now_s() - t0;

  const RequestState req = make_request(m, s, 0, cfg ? 1 : -1, phase, smp, cfg_scale, seed, 0, legacy_off != 0);
  cudaStream_t st = s.stream;
  YAR_CUDA(cudaMemcpyAsync(s.d_req, &req, sizeof(req), cudaMemcpyHostToDevice, st));
  std::vector<int> act(rows, 1);
  YAR_CUDA(cudaMemcpyAsync(s.d_active, act.data(), rows * sizeof(int), cudaMemcpyHostToDevice, st));
  YAR_CUDA(cudaMemsetAsync(s.d_error, 0, sizeof(int), st));
  reset_step_sync(s);
  YAR_CUDA(cudaStreamSynchronize(st));
  cudaGraphExec_t exec = step_graph(s, rows, 1, phase);

  // Replay in chunks; after each chunk read the request's progress (done, tokens).
  const int kChunk = 16;
  int steps = 0, reported = 0;
  bool done = false, eos = false;
  double ttft = -1;
  std::vector<int32_t> toks;
  struct Progress {
    int done, n_out, error, step;
  };
  auto *hp = reinterpret_cast<int *>(s.h_pinned);
  // Device time of the decode loop (graph replays only), on the engine's stream.
  cudaEvent_t ev0, ev1;
  YAR_CUDA(cudaEventCreate(&ev0));
  YAR_CUDA(cudaEventCreate(&ev1));
  YAR_CUDA(cudaEventRecord(ev0, st));
  float decode_ms = 0.f;
  double host_launch_s = 0;  // host time spent enqueuing the graph replays
  while (steps < smp.max_tokens && !done) {
    if (cancel && cancel(cancel_ctx)) throw Error("InterruptedError", std::string("Cancelled during ") +
                                                                          (phase == kPhaseAbc ? "abc" : "semantic"));
    const int k = std::min(kChunk, smp.max_tokens - steps);
    YAR_CUDA(cudaEventRecord(ev0, st));
    const double h0 = now_s();
    for (int i = 0; i < k; ++i) YAR_CUDA(cudaGraphLaunch(exec, st));
    host_launch_s += now_s() - h0;
    s.tp_epoch_steps += k;
    YAR_CUDA(cudaEventRecord(ev1, st));
    steps += k;
    YAR_CUDA(cudaMemcpyAsync(hp, &s.d_req[0].step, 4 * sizeof(int), cudaMemcpyDeviceToHost, st));
    YAR_CUDA(cudaMemcpyAsync(hp + 4, s.d_error, sizeof(int), cudaMemcpyDeviceToHost, st));
    YAR_CUDA(cudaStreamSynchronize(st));
    {
      float ms = 0.f;
      YAR_CUDA(cudaEventElapsedTime(&ms, ev0, ev1));
      decode_ms += ms;
    }
    if (ttft < 0) ttft = now_s() - t0;
    const int dstep = hp[0], ddone = hp[1], dn = hp[2], derr = hp[3];
    if (derr || hp[4]) throw Error("RuntimeError", "device sampler/forward error " + std::to_string(derr) + "/" +
                                                       std::to_string(hp[4]));
    if (dn > reported) {
      toks.resize(dn);
      YAR_CUDA(cudaMemcpy(toks.data() + reported, s.d_out_tokens + reported, (dn - reported) * sizeof(int32_t),
                          cudaMemcpyDeviceToHost));
      if (on_token)
        for (int i = reported; i < dn; ++i) on_token(token_ctx, phase, toks[i]);
      reported = dn;
    }
    if (ddone) {
      done = true;
      eos = dstep > dn;  // the end token was sampled (it is not stored)
    }
    if (dstep >= smp.max_tokens) done = true;
  }
  if (eos && on_token) {
    const int end_native = phase == kPhaseAbc ? kAbcEnd : phase == kPhaseSemantic ? kMusicEnd : -1;
    on_token(token_ctx, phase, end_native);
  }
  YAR_CUDA(cudaStreamSynchronize(st));
  YAR_CUDA(cudaEventDestroy(ev0));
  YAR_CUDA(cudaEventDestroy(ev1));
  const double seconds = now_s() - t0;
  std::copy(toks.begin(), toks.end(), out_tokens);
  *n_out = int(toks.size());
  *truncated = eos ? 0 : 1;
  // Release the request's pages (caches are request-local, sampling.cpp:208-210).
  for (int r = 0; r < rows; ++r) {
    for (int p : s.row_pages[r]) s.free_pages.push_back(p);
    s.row_pages[r].clear();
    s.capacity[r] = 0;
  }
  nlohmann::json timing = {{"seconds", seconds},
                           {"prefill_seconds", prefill_seconds},
                           {"ttft_seconds", ttft},
                           {"output_tokens", int(toks.size()) + int(eos)},
                           {"content_tokens", int(toks.size())},
                           {"output_tps", (toks.size() + int(eos)) / seconds},
                           {"prefix_tokens", n_prefix},
                           {"cfg_branches", cfg ? 2 : 1},
                           {"execution", "cuda_graph"},
                           {"attention", "split_kv"},
                           {"tensor_parallel", s.m->tp_world},
                           {"tp_exchange", s.m->tp_world == 1 ? "none" : s.tp_mapped ? "peer_stores" : "nccl"},
                           {"backend", "cuda-sm100a"},
                           {"decode_steps", steps},
                           {"decode_device_ms", decode_ms},
                           {"host_launch_ms", 1000 * host_launch_s}};
  return timing.dump();
}

// Sampler on host logits (parity tests of the filter chain and the draw).
void sample_host(Model &m, const uint16_t *cond, const uint16_t *uncond, int n, double cfg_scale,
                 const ::yar_sampling &smp, const int32_t *history, int n_history, int step, int phase,
                 uint64_t seed, int legacy_off, int32_t *token, float *scores) {
  validate_sampling(smp);
  const int expected = phase == kPhaseAbc ? kEOD + 1 : phase == kPhaseSemantic ? kCodecSize + 1 : n;
  if (phase != kPhaseAbc && phase != kPhaseSemantic && phase != kPhaseFull)
    throw Error("ValueError", "phase must be 'abc' or 'semantic'");
  if (n < 1 || n != expected) throw Error("ValueError", "Incorrect projected phase vocabulary size");
  YAR_CUDA(cudaSetDevice(m.device));
  const int stride = (n + 7) & ~7;
  bf16 *logits = dmalloc<bf16>(size_t(2) * stride);
  float *sc = dmalloc<float>(stride);
  RequestState *req = dmalloc<RequestState>(1);
  int *tok = dmalloc<int>(2), *act = dmalloc<int>(2);
  int32_t *picked = dmalloc<int32_t>(1);
  try {
    YAR_CUDA(cudaMemcpy(logits, cond, size_t(n) * 2, cudaMemcpyHostToDevice));
    const bool cfg = uncond && cfg_scale != 1.0;
    if (cfg) YAR_CUDA(cudaMemcpy(logits + stride, uncond, size_t(n) * 2, cudaMemcpyHostToDevice));
    RequestState r;
    std::memset(&r, 0, sizeof(r));
    r.row_c = 0;
    r.row_u = cfg ? 1 : -1;
    r.phase = phase;
    r.width = n;
    r.end_local = phase == kPhaseAbc ? kEOD : phase == kPhaseSemantic ? 0 : -1;
    r.temperature = float(smp.temperature);
    r.top_p = float(smp.top_p);
    r.cfg_scale = float(cfg_scale);
    r.top_k = smp.top_k;
    r.window = smp.penalty_window;
    r.min_tokens = smp.min_tokens;
    r.max_tokens = step + 1;
    r.penalty_on = smp.repetition_penalty != 1.0;
    r.legacy = legacy_off ? 1 : 0;
    fill_penalty_alpha(r, smp.repetition_penalty, legacy_off != 0);
    r.seed_lo = uint32_t(seed);
    r.seed_hi = uint32_t(seed >> 32);
    r.step = step;
    const int keep = std::min(n_history, kHistCap);
    r.n_out = n_history;
    for (int i = n_history - keep; i < n_history; ++i) r.hist[i % kHistCap] = history[i];
    YAR_CUDA(cudaMemcpy(req, &r, sizeof(r), cudaMemcpyHostToDevice));
    launch_sampler_ex(req, logits, stride, sc, tok, act, nullptr, 0, 1, picked, 1, nullptr);
    YAR_CUDA(cudaDeviceSynchronize());
    int err = 0;
    YAR_CUDA(cudaMemcpy(&err, &req->error, sizeof(int), cudaMemcpyDeviceToHost));
    if (err) throw Error("RuntimeError", err == 1 ? "sampler candidate set exceeds 2048 rows" : "no finite logits");
    YAR_CUDA(cudaMemcpy(token, picked, sizeof(int32_t), cudaMemcpyDeviceToHost));
    if (scores) YAR_CUDA(cudaMemcpy(scores, sc, size_t(n) * 4, cudaMemcpyDeviceToHost));
  } catch (...) {
    cudaFree(logits), cudaFree(sc), cudaFree(req), cudaFree(tok), cudaFree(act), cudaFree(picked);
    throw;
  }
  cudaFree(logits), cudaFree(sc), cudaFree(req), cudaFree(tok), cudaFree(act), cudaFree(picked);
}


// Many independent requests (no CFG) served from a queue on `slots` rows of the session —
// continuous batching. Request i is prefilled on a free row when one is available; every
// step samples all rows' unfinished requests (one sampler CTA each, own seed and sampling)
// and forwards all rows at once (16+ rows use the batched tcgen05 forward). The step graph
// reads each row's request record and activity from device memory, so a row whose request
// ended (end token or its max_tokens) is refilled between decode chunks with the next
// waiting request (its prefill, a fresh record, the row active again) without a new graph.
// Request i's native tokens (end token excluded) land at out_tokens[sum of the earlier
// requests' max_tokens ..].
std::string generate_requests(Session &s, int n_req, int slots, const int32_t *prefixes, const int32_t *prefix_lens,
                              const ::yar_sampling *smps, const uint64_t *seeds, int phase, int legacy_off,
                              int32_t *out_tokens, int *n_out, int *truncated) {
  const Model &m = *s.m;
  phase_rows(m.d, phase);
  if (n_req < 1) throw Error("ValueError", "request count must be at least 1");
  if (slots <= 0) slots = std::min(n_req, s.max_rows);
  if (slots > s.max_rows || slots > n_req) throw Error("ValueError", "slots must be in [1, min(requests, session rows)]");
  std::vector<size_t> starts(n_req), outs(n_req);
  size_t off = 0, out_off = 0;
  for (int r = 0; r < n_req; ++r) {
    validate_sampling(smps[r]);
    const int n = prefix_lens[r], mt = smps[r].max_tokens;
    if (n < 1) throw Error("ValueError", "AR prefix must contain at least one token");
    if (size_t(n) + size_t(mt) > size_t(m.d.context))
      throw Error("ValueError", "Prefix + requested generation budget exceeds 24576; no implicit truncation");
    if (n + mt > s.max_ctx) throw Error("ValueError", "KV cache capacity exceeded; generation was not shortened");
    if (mt > s.out_cap) throw Error("ValueError", "max_tokens exceeds the session output capacity");
    if (seeds[r] >= (uint64_t(1) << 63)) throw Error("ValueError", "seed must be an integer in [0, 2**63)");
    starts[r] = off;
    off += size_t(n);
    outs[r] = out_off;
    out_off += size_t(mt);
  }
  YAR_CUDA(cudaSetDevice(m.device));
  cudaStream_t st = s.stream;
  YAR_CUDA(cudaStreamSynchronize(st));
  const double t0 = now_s();
  double prefill_seconds = 0;
  std::vector<int> slot_req(slots, -1);  // request on each row (-1: none)
  int next = 0, admitted_late = 0;
  // Prefill request r on `row` and arm its sampler record.
  auto admit = [&](int row, int r) {
    const double p0 = now_s();
    row_reset(s, row, prefix_lens[r] + smps[r].max_tokens);
    row_prefill(s, row, prefixes + starts[r], prefix_lens[r], phase, 0, nullptr, nullptr);
    prefill_seconds += now_s() - p0;
    const RequestState req = make_request(m, s, row, -1, phase, smps[r], 1.0, seeds[r], 0, legacy_off != 0);
    YAR_CUDA(cudaMemcpyAsync(s.d_req + row, &req, sizeof(req), cudaMemcpyHostToDevice, st));
    const int one = 1;
    YAR_CUDA(cudaMemcpyAsync(s.d_active + row, &one, sizeof(int), cudaMemcpyHostToDevice, st));
    YAR_CUDA(cudaStreamSynchronize(st));  // the host values above are on the stack
    slot_req[row] = r;
  };
  for (int row = 0; row < slots; ++row) admit(row, next++);
  YAR_CUDA(cudaMemsetAsync(s.d_error, 0, sizeof(int), st));
  reset_step_sync(s);
  YAR_CUDA(cudaStreamSynchronize(st));
  cudaGraphExec_t exec = step_graph(s, slots, slots, phase);

  const int kChunk = 16;
  int steps = 0, finished = 0;
  float decode_ms = 0.f;
  cudaEvent_t ev0, ev1;
  YAR_CUDA(cudaEventCreate(&ev0));
  YAR_CUDA(cudaEventCreate(&ev1));
  std::vector<int> prog(size_t(slots) * 4);  // (step, done, n_out, error) per row's record
  long long total = 0;
  try {
    while (finished < n_req) {
      YAR_CUDA(cudaEventRecord(ev0, st));
      for (int i = 0; i < kChunk; ++i) YAR_CUDA(cudaGraphLaunch(exec, st));
      s.tp_epoch_steps += kChunk;
      YAR_CUDA(cudaEventRecord(ev1, st));
      steps += kChunk;
      YAR_CUDA(cudaMemcpy2DAsync(prog.data(), 4 * sizeof(int), &s.d_req[0].step, sizeof(RequestState),
                                 4 * sizeof(int), slots, cudaMemcpyDeviceToHost, st));
      int derr = 0;
      YAR_CUDA(cudaMemcpyAsync(&derr, s.d_error, sizeof(int), cudaMemcpyDeviceToHost, st));
      YAR_CUDA(cudaStreamSynchronize(st));
      float ms = 0.f;
      YAR_CUDA(cudaEventElapsedTime(&ms, ev0, ev1));
      decode_ms += ms;
      for (int row = 0; row < slots; ++row) {
        const int r = slot_req[row];
        if (r < 0) continue;
        const int *pg = &prog[4 * row];
        if (pg[3] || derr)
          throw Error("RuntimeError", "device sampler/forward error " + std::to_string(pg[3]) + "/" +
                                          std::to_string(derr));
        if (!pg[1] && pg[0] < smps[r].max_tokens) continue;
        // Request r is finished: collect its tokens, release its pages, refill the row.
        const int dn = pg[2];
        YAR_CUDA(cudaMemcpy(out_tokens + outs[r], s.d_out_tokens + size_t(row) * s.out_cap,
                            size_t(dn) * sizeof(int32_t), cudaMemcpyDeviceToHost));
        n_out[r] = dn;
        truncated[r] = pg[0] > dn ? 0 : 1;  // a sampled end token is counted in step, not stored
        total += dn;
        ++finished;
        for (int p : s.row_pages[row]) s.free_pages.push_back(p);
        s.row_pages[row].clear();
        s.capacity[row] = 0;
        slot_req[row] = -1;
        if (next < n_req) {
          admit(row, next++);
          ++admitted_late;
        }
      }
    }
  } catch (...) {
    cudaEventDestroy(ev0);
    cudaEventDestroy(ev1);
    throw;
  }
  YAR_CUDA(cudaEventDestroy(ev0));
  YAR_CUDA(cudaEventDestroy(ev1));
  const double seconds = now_s() - t0;
  nlohmann::json timing = {{"seconds", seconds},
                           {"prefill_seconds", prefill_seconds},
                           {"requests", n_req},
                           {"slots", slots},
                           {"refills", admitted_late},
                           {"content_tokens", total},
                           {"decode_steps", steps},
                           {"decode_device_ms", decode_ms},
                           {"execution", "cuda_graph"},
                           {"forward", slots >= kBatchedRows ? "batched_tcgen05" : "per_row"},
                           {"tensor_parallel", s.m->tp_world},
                           {"tp_exchange", s.m->tp_world == 1 ? "none" : s.tp_mapped ? "peer_stores" : "nccl"},
                           {"backend", "cuda-sm100a"}};
  return timing.dump();
}

// Many independent requests decoded together on rows 0..n-1 (no CFG, one sampling for all):
// generate_requests with one row per request.
std::string generate_batch(Session &s, int n_req, const int32_t *prefixes, const int32_t *prefix_lens,
                           const ::yar_sampling &smp, const uint64_t *seeds, int phase, int legacy_off,
                           int32_t *out_tokens, int *n_out, int *truncated) {
  if (n_req < 1 || n_req > s.max_rows) throw Error("ValueError", "request count must be in [1, session rows]");
  const std::vector<::yar_sampling> smps(n_req, smp);
  return generate_requests(s, n_req, n_req, prefixes, prefix_lens, smps.data(), seeds, phase, legacy_off, out_tokens,
                           n_out, truncated);
}

}  // namespace yar
