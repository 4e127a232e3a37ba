// api.cpp — the C ABI (include/yue2ar.h). Exceptions never cross it: every entry point
// maps lyra-style typed errors to the lyra_status codes (native/include/CLyraCore/lyra.h:18-23)
// and keeps the message for yar_last_error() on the calling thread.
#include <algorithm>
#include <cstring>
#include <string>

#include "engine.h"
#include "yue2ar.h"

namespace yar {
Model *load_model(const std::string &dir, int device, uint32_t flags, int tp_rank = 0, int tp_world = 1,
                  const uint8_t *nccl_id = nullptr);
void free_model(Model *m);
Session *create_session(Model *m, int max_rows, int max_ctx, int page_tokens);
void free_session(Session *s);
void row_reset(Session &s, int row, int capacity);
void row_prefill(Session &s, int row, const int32_t *ids, int n, int phase, int chunk, int (*cancel)(void *),
                 void *cancel_ctx);
void rows_step(Session &s, const int *rows, const int32_t *tokens, int n, int phase);
std::string generate(Session &s, const int32_t *prefix, int n_prefix, const ::yar_sampling &smp, uint64_t seed,
                     int phase, const int32_t *negative, int n_negative, double cfg_scale, int legacy_off,
                     int (*cancel)(void *), void *cancel_ctx, void (*on_token)(void *, int, int32_t),
                     void *token_ctx, int32_t *out_tokens, int *n_out, int *truncated);
void sample_host(Model &m, const uint16_t *cond, const uint16_t *uncond, int n, double cfg_scale,
                 const ::yar_sampling &smp, const int32_t *history, int n_history, int step, int phase,
                 uint64_t seed, int legacy_off, int32_t *token, float *scores);
std::string generate_requests(Session &s, int n_req, int slots, const int32_t *prefixes, const int32_t *prefix_lens,
                              const ::yar_sampling *smps, const uint64_t *seeds, int phase, int legacy_off,
                              int32_t *out_tokens, int *n_out, int *truncated);
std::string generate_batch(Session &s, int n_req, const int32_t *prefixes, const int32_t *prefix_lens,
                           const ::yar_sampling &smp, const uint64_t *seeds, int phase, int legacy_off,
                           int32_t *out_tokens, int *n_out, int *truncated);
void sample_device_noalloc(Model &m, const uint16_t *logits, long long row_stride, int rows, int n,
                           double cfg_scale, const ::yar_sampling &smp, const int32_t *history, int n_history,
                           int step, int phase, uint64_t seed, int32_t *token, float *scores,
                           cudaStream_t st);
}  // namespace yar

struct yar_model {
  yar::Model *m;
};
struct yar_session {
  yar::Session *s;
};

namespace {
thread_local std::string g_error, g_type;

int status_for(const std::string &type) {
  if (type == "ValueError" || type == "FileNotFoundError") return YAR_INVALID_INPUT;
  if (type == "InterruptedError") return YAR_CANCELLED;
  return YAR_FAILURE;
}

template <typename F>
int guarded(F &&f) {
  try {
    f();
    g_error.clear();
    g_type.clear();
    return YAR_OK;
  } catch (const yar::Error &e) {
    g_error = e.what();
    g_type = e.type;
    return status_for(e.type);
  } catch (const std::bad_alloc &) {
    g_error = "host out of memory";
    g_type = "RuntimeError";
    return YAR_FAILURE;
  } catch (const std::exception &e) {
    g_error = e.what();
    g_type = "RuntimeError";
    return YAR_FAILURE;
  } catch (...) {
    g_error = "unknown error";
    g_type = "RuntimeError";
    return YAR_FAILURE;
  }
}

void need(bool ok, const char *msg) {
  if (!ok) throw yar::Error("ValueError", msg);
}
}  // namespace

#pragma GCC visibility push(default)
extern "C" {

const char *yar_last_error(void) { return g_error.c_str(); }
const char *yar_last_error_type(void) { return g_type.c_str(); }
const char *yar_version(void) { return "yue2ar-cuda 0.1 sm_100a"; }

int yar_model_load_ex(const char *dir, int device, uint32_t flags, yar_model **out) {
  return guarded([&] {
    need(dir && out, "dir and out are required");
    *out = nullptr;
    auto *h = new yar_model{yar::load_model(dir, device, flags)};
    *out = h;
  });
}

int yar_model_load(const char *dir, int device, yar_model **out) { return yar_model_load_ex(dir, device, 0, out); }

int yar_model_load_precision(const char *dir, const char *precision, int device, uint32_t flags, yar_model **out) {
  return guarded([&] {
    need(dir && precision && out, "dir, precision and out are required");
    *out = nullptr;
    const std::string p = precision;
    if (p != "bf16" && p != "8bit" && p != "4bit")
      throw yar::Error("ValueError", "precision must be 'bf16', '8bit', or '4bit'");
    flags &= ~uint32_t(YAR_LOAD_8BIT | YAR_LOAD_4BIT);
    if (p == "8bit") flags |= YAR_LOAD_8BIT;
    if (p == "4bit") flags |= YAR_LOAD_4BIT;
    auto *h = new yar_model{yar::load_model(dir, device, flags)};
    *out = h;
  });
}

int yar_model_precision_bits(const yar_model *model, int *bits) {
  return guarded([&] {
    need(model && bits, "model and bits are required");
    *bits = model->m->bits;
  });
}

int yar_tp_unique_id(uint8_t *out) {
  return guarded([&] {
    need(out, "out is required");
    yar::tp_unique_id(out);
  });
}

int yar_tp_plan(int hidden, int heads, int kv_heads, int head_dim, int ffn, int rank, int world, int64_t *plan) {
  return guarded([&] {
    need(plan && hidden > 0 && heads > 0 && kv_heads > 0 && head_dim > 0 && ffn > 0 && heads % kv_heads == 0,
         "positive dims with heads a multiple of kv_heads are required");
    yar::Dims d;
    d.hidden = hidden;
    d.heads = heads;
    d.kv_heads = kv_heads;
    d.head_dim = head_dim;
    d.ffn = ffn;
    const yar::TpPlan p = yar::tp_plan(d, rank, world);
    const int64_t v[8] = {p.q_row0, p.q_rows, p.kv_row0, p.kv_rows, p.ffn_row0, p.ffn_rows, p.h_row0, p.h_rows};
    std::memcpy(plan, v, sizeof(v));
  });
}

int yar_tp_head_slice(int width, int rank, int world, int *begin, int *end) {
  return guarded([&] {
    need(begin && end && width > 0 && world >= 1 && rank >= 0 && rank < world, "width > 0, rank in [0, world)");
    const int slice = yar::tp_head_slice(width, world);
    *begin = std::min(width, rank * slice);
    *end = std::min(width, (rank + 1) * slice);
  });
}

int yar_model_load_tp(const char *dir, int device, int rank, int world, const uint8_t *nccl_id, uint32_t flags,
                      yar_model **out) {
  return guarded([&] {
    need(dir && out && nccl_id, "dir, nccl_id and out are required");
    need(world >= 1 && rank >= 0 && rank < world, "rank must be in [0, world)");
    *out = nullptr;
    auto *h = new yar_model{yar::load_model(dir, device, flags, rank, world, nccl_id)};
    *out = h;
  });
}

int yar_model_free(yar_model *model) {
  return guarded([&] {
    if (!model) return;
    yar::free_model(model->m);
    delete model;
  });
}

int yar_model_dims(const yar_model *model, int64_t *dims) {
  return guarded([&] {
    need(model && dims, "model and dims are required");
    const auto &d = model->m->d;
    const int64_t v[10] = {d.hidden, d.layers, d.heads, d.kv_heads, d.head_dim, d.ffn,
                           d.vocab,  d.context, int64_t(model->m->arena_bytes >> 20), model->m->sm_count};
    std::memcpy(dims, v, sizeof(v));
  });
}

int yar_session_create(yar_model *model, int max_rows, int max_ctx, int page_tokens, yar_session **out) {
  return guarded([&] {
    need(model && out, "model and out are required");
    *out = nullptr;
    *out = new yar_session{yar::create_session(model->m, max_rows, max_ctx, page_tokens)};
  });
}

int yar_session_free(yar_session *session) {
  return guarded([&] {
    if (!session) return;
    yar::free_session(session->s);
    delete session;
  });
}

int yar_session_set_option(yar_session *session, int option, int value) {
  return guarded([&] {
    need(session, "session is required");
    auto &s = *session->s;
    if (option == YAR_OPT_PERSISTENT) {
      s.use_persistent = value != 0;
    } else if (option == YAR_OPT_TRACE) {
      YAR_CUDA(cudaSetDevice(s.m->device));
      YAR_CUDA(cudaStreamSynchronize(s.stream));
      if (s.d_trace) cudaFree(s.d_trace);
      s.d_trace = nullptr;
      s.trace_elems = 0;
      for (auto &g : s.graphs) cudaGraphExecDestroy(g.exec);  // graphs captured the old pointer
      s.graphs.clear();
      if (value) {
        // + sampler phases, + a 64-step log of kernel start/end times
        s.trace_elems = size_t(s.m->sm_count) * (5 * s.m->d.layers + 1) * 8 + 16 + 64 * 4;
        YAR_CUDA(cudaMalloc(&s.d_trace, s.trace_elems * sizeof(unsigned long long)));
        YAR_CUDA(cudaMemset(s.d_trace, 0, s.trace_elems * sizeof(unsigned long long)));
      }
    } else if (option == YAR_OPT_PREFETCH_STAGES) {
      need(value >= 0 && value <= 64, "prefetch stages must be in [0, 64]");
      YAR_CUDA(cudaSetDevice(s.m->device));
      YAR_CUDA(cudaStreamSynchronize(s.stream));
      for (auto &g : s.graphs) cudaGraphExecDestroy(g.exec);  // graphs captured the old value
      s.graphs.clear();
      s.prefetch_stages = value;
    } else if (option == YAR_OPT_MAX_SPLITS) {
      need(value >= 0 && value <= s.max_splits, "attention splits must be in [0, 32]");
      YAR_CUDA(cudaSetDevice(s.m->device));
      YAR_CUDA(cudaStreamSynchronize(s.stream));
      for (auto &g : s.graphs) cudaGraphExecDestroy(g.exec);  // graphs captured the old split plan
      s.graphs.clear();
      s.forced_splits = value;
    } else if (option == YAR_OPT_FAULT_INJECT) {
      need(value >= 0 && value <= 5 * s.m->d.layers, "fault-injection operation outside the step");
      YAR_CUDA(cudaSetDevice(s.m->device));
      YAR_CUDA(cudaStreamSynchronize(s.stream));
      for (auto &g : s.graphs) cudaGraphExecDestroy(g.exec);  // graphs captured the old value
      s.graphs.clear();
      s.inject_op = value;
    } else if (option == YAR_OPT_PREFILL_ATTN_TC) {
      s.prefill_attn_tc = value != 0;
    } else if (option == YAR_OPT_LAYER_DUMP) {
      YAR_CUDA(cudaSetDevice(s.m->device));
      YAR_CUDA(cudaStreamSynchronize(s.stream));
      for (auto &g : s.graphs) cudaGraphExecDestroy(g.exec);  // graphs captured the old pointer
      s.graphs.clear();
      if (s.d_layer_dump) cudaFree(s.d_layer_dump);
      s.d_layer_dump = nullptr;
      if (value) {
        const size_t n = size_t(s.m->d.layers + 1) * s.max_rows * s.m->d.hidden;
        YAR_CUDA(cudaMalloc(&s.d_layer_dump, n * sizeof(yar::bf16)));
        YAR_CUDA(cudaMemset(s.d_layer_dump, 0, n * sizeof(yar::bf16)));
      }
    } else {
      throw yar::Error("ValueError", "unknown session option");
    }
  });
}

int yar_session_trace(yar_session *session, uint64_t *out, size_t n, size_t *n_written) {
  return guarded([&] {
    need(session && out && n_written, "missing argument");
    auto &s = *session->s;
    *n_written = 0;
    if (!s.d_trace) return;
    YAR_CUDA(cudaSetDevice(s.m->device));
    YAR_CUDA(cudaStreamSynchronize(s.stream));
    const size_t k = n < s.trace_elems ? n : s.trace_elems;
    YAR_CUDA(cudaMemcpy(out, s.d_trace, k * sizeof(uint64_t), cudaMemcpyDeviceToHost));
    *n_written = k;
  });
}

int yar_generate(yar_session *session, const int32_t *prefix, int n_prefix, const yar_sampling *sampling,
                 uint64_t seed, int phase, const int32_t *negative, int n_negative, double cfg_scale,
                 int legacy_off, yar_cancel_fn cancel, void *cancel_ctx, yar_token_fn on_token, void *token_ctx,
                 int32_t *out_tokens, int *n_out, int *truncated, char *timing_json, size_t timing_cap) {
  return guarded([&] {
    need(session && prefix && sampling && out_tokens && n_out && truncated, "missing argument");
    need(n_negative == 0 || negative, "negative prefix pointer missing");
    const std::string timing = yar::generate(*session->s, prefix, n_prefix, *sampling, seed, phase, negative,
                                             n_negative, cfg_scale, legacy_off, cancel, cancel_ctx, on_token,
                                             token_ctx, out_tokens, n_out, truncated);
    if (timing_json && timing_cap > 0) {
      const size_t n = timing.size() < timing_cap - 1 ? timing.size() : timing_cap - 1;
      std::memcpy(timing_json, timing.data(), n);
      timing_json[n] = '\0';
    }
  });
}

int yar_generate_batch(yar_session *session, int n_requests, const int32_t *prefixes, const int32_t *prefix_lens,
                       const yar_sampling *sampling, const uint64_t *seeds, int phase, int legacy_off,
                       int32_t *out_tokens, int *n_out, int *truncated, char *timing_json, size_t timing_cap) {
  return guarded([&] {
    need(session && prefixes && prefix_lens && sampling && seeds && out_tokens && n_out && truncated,
         "missing argument");
    const std::string timing = yar::generate_batch(*session->s, n_requests, prefixes, prefix_lens, *sampling, seeds,
                                                   phase, legacy_off, out_tokens, n_out, truncated);
    if (timing_json && timing_cap > 0) {
      const size_t n = timing.size() < timing_cap - 1 ? timing.size() : timing_cap - 1;
      std::memcpy(timing_json, timing.data(), n);
      timing_json[n] = '\0';
    }
  });
}

int yar_generate_requests(yar_session *session, int n_requests, int slots, const int32_t *prefixes,
                          const int32_t *prefix_lens, const yar_sampling *samplings, const uint64_t *seeds, int phase,
                          int legacy_off, int32_t *out_tokens, int *n_out, int *truncated, char *timing_json,
                          size_t timing_cap) {
  return guarded([&] {
    need(session && prefixes && prefix_lens && samplings && seeds && out_tokens && n_out && truncated,
         "missing argument");
    const std::string timing = yar::generate_requests(*session->s, n_requests, slots, prefixes, prefix_lens,
                                                      samplings, seeds, phase, legacy_off, out_tokens, n_out,
                                                      truncated);
    if (timing_json && timing_cap > 0) {
      const size_t n = timing.size() < timing_cap - 1 ? timing.size() : timing_cap - 1;
      std::memcpy(timing_json, timing.data(), n);
      timing_json[n] = '\0';
    }
  });
}

int yar_row_reset(yar_session *session, int row, int capacity) {
  return guarded([&] {
    need(session, "session is required");
    yar::row_reset(*session->s, row, capacity);
  });
}

int yar_row_prefill(yar_session *session, int row, const int32_t *ids, int n, int phase, int chunk) {
  return guarded([&] {
    need(session && ids, "session and ids are required");
    yar::row_prefill(*session->s, row, ids, n, phase, chunk, nullptr, nullptr);
  });
}

int yar_rows_step(yar_session *session, const int *rows, const int32_t *tokens, int n_rows, int phase) {
  return guarded([&] {
    need(session && rows && tokens, "session, rows and tokens are required");
    yar::rows_step(*session->s, rows, tokens, n_rows, phase);
  });
}

int yar_row_logits(yar_session *session, int row, uint16_t *out, int n) {
  return guarded([&] {
    need(session && out, "session and out are required");
    auto &s = *session->s;
    need(row >= 0 && row < s.max_rows && n >= 0 && n <= s.logit_stride, "row or width outside the session");
    YAR_CUDA(cudaSetDevice(s.m->device));
    YAR_CUDA(cudaStreamSynchronize(s.stream));
    YAR_CUDA(cudaMemcpy(out, s.logits + size_t(row) * s.logit_stride, size_t(n) * 2, cudaMemcpyDeviceToHost));
  });
}

int yar_row_kv(yar_session *session, int row, int layer, int start, int count, uint16_t *k, uint16_t *v) {
  return guarded([&] {
    need(session && k && v, "session, k and v are required");
    auto &s = *session->s;
    const auto &d = s.m->d;
    need(row >= 0 && row < s.max_rows && layer >= 0 && layer < d.layers, "row or layer outside the session");
    need(start >= 0 && count >= 0 && start + count <= s.pos[row], "positions outside the row's cache");
    YAR_CUDA(cudaSetDevice(s.m->device));
    YAR_CUDA(cudaStreamSynchronize(s.stream));
    std::vector<int> table(s.pages_per_row);
    YAR_CUDA(cudaMemcpy(table.data(), s.d_page_table + size_t(row) * s.pages_per_row,
                        table.size() * sizeof(int), cudaMemcpyDeviceToHost));
    // One copy per (k|v, head, page): a page holds a contiguous run of positions.
    for (int kv = 0; kv < 2; ++kv)
      for (int h = 0; h < d.kv_heads; ++h)
        for (int i = 0; i < count;) {
          const int pos = start + i, page = table[pos / s.page_tokens], slot = pos % s.page_tokens;
          const int run = std::min(count - i, s.page_tokens - slot);
          const size_t blk = (size_t(layer) * s.num_pages + page) * 2 + kv;
          const yar::bf16 *src = s.kv + blk * s.kv_page_elems + (size_t(h) * s.page_tokens + slot) * d.head_dim;
          uint16_t *dst = (kv ? v : k) + (size_t(h) * count + i) * d.head_dim;
          YAR_CUDA(cudaMemcpy(dst, src, size_t(run) * d.head_dim * 2, cudaMemcpyDeviceToHost));
          i += run;
        }
  });
}

int yar_row_hidden(yar_session *session, int row, int slot, uint16_t *out, int n) {
  return guarded([&] {
    need(session && out, "session and out are required");
    auto &s = *session->s;
    const auto &d = s.m->d;
    need(s.d_layer_dump != nullptr, "the hidden-state record is off (YAR_OPT_LAYER_DUMP)");
    need(row >= 0 && row < s.max_rows && slot >= 0 && slot <= d.layers && n == d.hidden,
         "row, slot or width outside the record");
    YAR_CUDA(cudaSetDevice(s.m->device));
    YAR_CUDA(cudaStreamSynchronize(s.stream));
    YAR_CUDA(cudaMemcpy(out, s.d_layer_dump + (size_t(slot) * s.max_rows + row) * d.hidden, size_t(n) * 2,
                        cudaMemcpyDeviceToHost));
  });
}

int yar_row_position(yar_session *session, int row, int *pos) {
  return guarded([&] {
    need(session && pos, "session and pos are required");
    need(row >= 0 && row < session->s->max_rows, "row outside the session");
    *pos = session->s->pos[row];
  });
}

int yar_sample_host(yar_model *model, const uint16_t *cond, const uint16_t *uncond, int n, double cfg_scale,
                    const yar_sampling *sampling, const int32_t *history, int n_history, int step, int phase,
                    uint64_t seed, int legacy_off, int32_t *token, float *scores) {
  return guarded([&] {
    need(model && cond && sampling && token, "missing argument");
    need(n_history == 0 || history, "history pointer missing");
    yar::sample_host(*model->m, cond, uncond, n, cfg_scale, *sampling, history, n_history, step, phase, seed,
                     legacy_off, token, scores);
  });
}

int yar_sample_device_noalloc(yar_model *model, const uint16_t *logits, int64_t row_stride, int rows, int n,
                              double cfg_scale, const yar_sampling *sampling, const int32_t *history,
                              int n_history, int step, int phase, uint64_t seed, int32_t *token, float *scores,
                              void *stream) {
  return guarded([&] {
    need(model && logits && sampling && token, "missing argument");
    need(n_history == 0 || history, "history pointer missing");
    yar::sample_device_noalloc(*model->m, logits, row_stride, rows, n, cfg_scale, *sampling, history, n_history,
                               step, phase, seed, token, scores, static_cast<cudaStream_t>(stream));
  });
}

}  // extern "C"
#pragma GCC visibility pop
