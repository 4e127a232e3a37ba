/*
 * yue2ar.h — C ABI of the B200 (sm_100a) YuE2 AR engine (libyue2ar_cuda.so).
 *
 * This is the drop-in boundary for the reference's AR engine interface
 * (native/include/lyra/ar.hpp:20-48): model load, prefill, per-step decode with the
 * sampler, the KV cache, and the whole generate_tokens loop. Plain C types only; no
 * exception crosses it. Every function returns a status with the reference's codes
 * (native/include/CLyraCore/lyra.h:18-23): YAR_OK 0, YAR_FAILURE 1, YAR_INVALID_INPUT 2,
 * YAR_CANCELLED 130. The message and the reference's error type name ("ValueError",
 * "FileNotFoundError", "InterruptedError", "RuntimeError"; native/include/lyra/types.hpp:70-74)
 * of the last failure on the calling thread are read with yar_last_error() and
 * yar_last_error_type().
 *
 * Threading: one call at a time per session; callbacks run on the calling thread and
 * must not re-enter the library (native/include/lyra/runtime.hpp:6-9).
 */
#ifndef YUE2AR_H
#define YUE2AR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  YAR_OK = 0,
  YAR_FAILURE = 1,
  YAR_INVALID_INPUT = 2,
  YAR_CANCELLED = 130
};

/* Protocol phases (native/src/sampling.cpp:8-18). YAR_PHASE_FULL projects every
 * vocabulary row; it exists for models whose vocabulary is smaller than the protocol's
 * codec range (the tiny parity model) and is rejected for the pinned checkpoint. */
enum { YAR_PHASE_ABC = 0, YAR_PHASE_SEMANTIC = 1, YAR_PHASE_FULL = 2 };

/* yar_model_load_ex flags. */
enum {
  /* Accept any self-consistent dims instead of the pinned YuE2-3B config
   * (native/src/ar.cpp:164-179 pins them); used by the tiny parity model. */
  YAR_LOAD_ANY_DIMS = 1u << 0,
  /* Load the `8bit` precision (ar-8bit.safetensors: affine 8-bit group-64 linears) instead
   * of bf16, as ARModel(dir, "8bit") (native/src/ar.cpp:150-160, :208-214). One GPU only. */
  YAR_LOAD_8BIT = 1u << 1,
  /* The `4bit` precision (ar-4bit.safetensors: affine 4-bit group-64 linears). One GPU only. */
  YAR_LOAD_4BIT = 1u << 2
};

/* lyra::Sampling (native/include/lyra/types.hpp:78-87), same field meaning and the same
 * validation as upstream protocol.py:31-41. */
typedef struct yar_sampling {
  double temperature;
  double top_p;
  int32_t top_k;
  double repetition_penalty;
  int32_t penalty_window;
  int32_t min_tokens;
  int32_t max_tokens;
} yar_sampling;

typedef struct yar_model yar_model;
typedef struct yar_session yar_session;

/* Cooperative cancellation (lyra::Cancelled): return nonzero to cancel. Checked before
 * prefill, between prefill chunks and between decode chunks; never inside a kernel. */
typedef int (*yar_cancel_fn)(void *ctx);
/* Token callback (lyra::TokenCallback): phase id and native token id, in order. */
typedef void (*yar_token_fn)(void *ctx, int phase, int32_t token);

const char *yar_last_error(void);
const char *yar_last_error_type(void);
const char *yar_version(void);

/* ARModel::ARModel(dir, "bf16", verify=false) — native/src/ar.cpp:133-238: reads
 * conversion.json (schema 1, precisions.bf16 record), config.json (pinned dims),
 * ar-bf16.safetensors (exact key/shape/dtype set), and uploads the weights to `device`
 * in the engine's layout (fused QKV, gate/up interleaved rows). */
int yar_model_load(const char *dir, int device, yar_model **out);
int yar_model_load_ex(const char *dir, int device, uint32_t flags, yar_model **out);
/* ARModel::ARModel(dir, precision) — native/src/ar.cpp:133-238 with its precision argument:
 * "bf16", "8bit" or "4bit" (the manifest's precisions.<precision> record,
 * ar-<precision>.safetensors; quantized, the record must say bits 8 / 4, group_size 64, mode
 * affine, linear_only, and every linear is a U32 [out, in*bits/32] weight with BF16
 * [out, in/64] scales and biases). Quantized weights are streamed as such by the persistent
 * decode kernel (one and two rows); prefill and the batched decode read them dequantized to
 * BF16. */
int yar_model_load_precision(const char *dir, const char *precision, int device, uint32_t flags, yar_model **out);
/* The loaded precision's bits: 0 (bf16), 8 or 4. */
int yar_model_precision_bits(const yar_model *model, int *bits);
int yar_model_free(yar_model *model);
/* Tensor parallelism over `world` GPUs, one process per GPU (no reference counterpart:
 * the reference runs one device; this splits ARModel's layers across GPUs). Every linear
 * is split by output rows with its whole input width: rank r holds KV heads
 * [r*kv/world, (r+1)*kv/world) with their query heads (q/k/v rows), FFN rows
 * [r*ffn/world, (r+1)*ffn/world) of gate/up, hidden rows [r*hidden/world, ...) of O and
 * down, and the embedding, norms and LM head whole (it projects its share of each phase's
 * columns). After each operation the ranks' BF16 outputs are all-gathered over NCCL, so
 * every value is computed by one rank with the one-GPU arithmetic: logits and tokens are
 * those of one GPU, on every rank. Every rank makes the same calls in the same order with
 * the same arguments.
 * `nccl_id` is 128 bytes from yar_tp_unique_id on one rank, passed to all of them.
 * NCCL is opened at run time (libnccl.so.2). With a TP model yar_model_dims reports this
 * rank's heads, kv_heads and ffn. */
int yar_tp_unique_id(uint8_t *nccl_id128);
/* The split itself, without a GPU: plan8 = {q_row0, q_rows, kv_row0, kv_rows, ffn_row0,
 * ffn_rows, h_row0, h_rows} — this rank's rows of q_proj, of k_proj and v_proj, of
 * gate_proj and up_proj, and of o_proj and down_proj, in the whole model's tensors. */
int yar_tp_plan(int hidden, int heads, int kv_heads, int head_dim, int ffn, int rank, int world, int64_t *plan8);
/* This rank's LM-head columns [begin, end) of a `width`-column phase projection. */
int yar_tp_head_slice(int width, int rank, int world, int *begin, int *end);
int yar_model_load_tp(const char *dir, int device, int rank, int world, const uint8_t *nccl_id128,
                      uint32_t flags, yar_model **out);
/* dims[10] = {hidden, layers, heads, kv_heads, head_dim, ffn, vocab, context,
 * device bytes of weights (low 31 bits in MiB), sm count}. */
int yar_model_dims(const yar_model *model, int64_t *dims10);

/* Device memory for up to `max_rows` decode rows (a CFG request takes two rows) with
 * `max_ctx` positions each, in pages of `page_tokens` (256 by default when 0): the
 * paged BF16 KV cache (KVCache, native/src/ar.cpp:98-132, one page table per row),
 * activations, logits, sampler state and the captured decode-step graph. */
int yar_session_create(yar_model *model, int max_rows, int max_ctx, int page_tokens,
                       yar_session **out);
int yar_session_free(yar_session *session);

/* Session options. YAR_OPT_PERSISTENT (default 1): run each decode forward of one or two
 * rows as the single persistent kernel when the model's shapes allow it; 0 selects one
 * kernel per operation (same arithmetic, identical results). YAR_OPT_TRACE (default 0):
 * record the persistent kernel's timeline (per CTA and operation, 8 SM-clock (clock64)
 * stamps: wait done, activations staged, stages consumed, signalled, producer first/last
 * issue; slots 6/7 of operation 0 and of the head hold globaltimer ns and the SM clock
 * at the step's start and end, for converting cycles to time), overwritten by every
 * step that has an active row (so it keeps the last step that did work, not the final
 * launch after a request's last token); read it with yar_session_trace. YAR_OPT_PREFETCH_STAGES (default 2, 0..64): how many
 * 32 KB stages per SM the persistent kernel pulls into L2 ahead of its shared-memory ring
 * (its lookahead while the step waits at operation boundaries). */
enum { YAR_OPT_PERSISTENT = 1, YAR_OPT_TRACE = 2, YAR_OPT_PREFETCH_STAGES = 3, YAR_OPT_MAX_SPLITS = 4,
       YAR_OPT_LAYER_DUMP = 5, YAR_OPT_FAULT_INJECT = 6, YAR_OPT_PREFILL_ATTN_TC = 7 };
/* YAR_OPT_PREFILL_ATTN_TC (default 1): prefill attention for head_dim 128 on tcgen05 tensor
 * cores with TMEM accumulators and TMA-fed K/V; 0 selects the mma.sync kernel (the same
 * quotient; the two differ by rounding: summation order, exp2 of log2-scaled scores and a
 * running maximum raised in steps on the tcgen05 side). */
/* YAR_OPT_MAX_SPLITS (default 0 = automatic, else 1..32): the number of splits each (row,
 * kv head) of the decode attention is cut into at most — 1 puts a row's whole context in
 * one unit (the longest chain of chunks), for parity tests of the split-KV rescaling.
 * YAR_OPT_LAYER_DUMP (default 0): record, on every decode step, each row's residual stream
 * after the embedding and after every layer (read with yar_row_hidden); used by per-layer
 * parity tests (a teacher-forced layer: its input and cache from the engine, its output
 * compared with the CPU oracle's).
 * YAR_OPT_FAULT_INJECT (default 0; testing of the failure path): 1 + 5 * layer + k makes
 * operation k (0 QKV, 1 attention, 2 O, 3 gate/up, 4 down) of that layer wait, in the
 * persistent decode kernel, for a flag that no operation writes, with every wait of the
 * step limited to ~65k polls: the wait expires, the kernel records the error and ends, and
 * the call returns YAR_FAILURE ("RuntimeError"). No fault, trap or hang is involved; the
 * session stays usable (the next call starts from cleared state). */
int yar_session_set_option(yar_session *session, int option, int value);
/* Copy the timeline of the last step with an active row ([sm][5 * layers + 1][8] uint64,
 * then 16 sampler stamps: SM clocks at its phase ends, and globaltimer ns at its start and
 * end in slots 12/13, then a [64][4] step log indexed by the session's decode step count
 * % 64, written on every step: globaltimer ns of the sampler's start and end (request 0)
 * and of the persistent kernel's start and end (CTA 0)) to host. */
int yar_session_trace(yar_session *session, uint64_t *out, size_t n, size_t *n_written);

/* generate_tokens — native/src/sampling.cpp:185-288 (upstream sampling.py:57-154): prefill
 * of `prefix` (and of `negative` when cfg_scale != 1), then up to max_tokens sampled
 * tokens. `out_tokens` receives native ids without the end token (capacity max_tokens);
 * `*n_out` their count, `*truncated` 1 when no end token was sampled. `timing_json`
 * (optional) receives the reference's timing dict. Host buffers in and out. */
int yar_generate(yar_session *session, const int32_t *prefix, int n_prefix,
                 const yar_sampling *sampling, uint64_t seed, int phase,
                 const int32_t *negative, int n_negative, double cfg_scale, int legacy_off,
                 yar_cancel_fn cancel, void *cancel_ctx, yar_token_fn on_token, void *token_ctx,
                 int32_t *out_tokens, int *n_out, int *truncated, char *timing_json,
                 size_t timing_cap);

/* Many independent requests (the reference's per-song generate_tokens, sampling.cpp:185-288,
 * run for n_requests songs at once; no CFG): request r's prefix is prefixes[sum of earlier
 * lengths ..][prefix_lens[r]], it decodes on row r with seed seeds[r], and its native
 * tokens (end token excluded) land in out_tokens[r * max_tokens ..], n_out[r] of them;
 * truncated[r] is 1 when no end token was sampled. All requests step together (from 16
 * rows on, one batched forward reads each weight once per step for every row); a finished
 * request's row is skipped. Needs n_requests <= the session's rows. */
int yar_generate_batch(yar_session *session, int n_requests, const int32_t *prefixes,
                       const int32_t *prefix_lens, const yar_sampling *sampling,
                       const uint64_t *seeds, int phase, int legacy_off, int32_t *out_tokens,
                       int *n_out, int *truncated, char *timing_json, size_t timing_cap);

/* Continuous batching (no reference counterpart: the reference serves one song at a time,
 * native/src/sampling.cpp:185-288): n_requests independent requests (no CFG) served from a
 * queue on `slots` rows of the session (0: min(n_requests, rows)). Request i has its own
 * prefix (prefixes[sum of earlier lengths ..][prefix_lens[i]]), sampling (samplings[i],
 * its own max_tokens) and seed; it is prefilled on the first free row, and a row whose
 * request ended (end token or max_tokens) takes the next waiting request between decode
 * chunks. Request i's native tokens (end token excluded) land at out_tokens[sum of the
 * earlier requests' max_tokens ..], n_out[i] of them; truncated[i] is 1 when no end token
 * was sampled. Every step forwards all `slots` rows at once (from 16 rows on, one batched
 * forward reads each weight once per step for every row). */
int yar_generate_requests(yar_session *session, int n_requests, int slots, const int32_t *prefixes,
                          const int32_t *prefix_lens, const yar_sampling *samplings, const uint64_t *seeds,
                          int phase, int legacy_off, int32_t *out_tokens, int *n_out, int *truncated,
                          char *timing_json, size_t timing_cap);

/* Row-level API (ARModel::hidden/project + KVCache, ar.cpp:246-323), used by batched
 * serving and by parity tests. A row owns a page table and a position. yar_row_prefill and
 * yar_rows_step are the library's prefill and decode-step entries; a sampled step is
 * yar_generate (the whole loop on the device) or, token at a time, yar_rows_step followed
 * by yar_sample_host (or yar_sample_device_noalloc on device-resident logits). */
int yar_row_reset(yar_session *session, int row, int capacity);
/* Prefill `n` ids into `row` at its current position (chunks of `chunk` tokens, 1024 if
 * 0; native/src/sampling.cpp:152-183) and project the last hidden state onto `phase`. */
int yar_row_prefill(yar_session *session, int row, const int32_t *ids, int n, int phase,
                    int chunk);
/* One decode forward of the given token per listed row (the token is written at each
 * row's position), then the phase projection. */
int yar_rows_step(yar_session *session, const int *rows, const int32_t *tokens, int n_rows,
                  int phase);
/* Copy the last projected logits of `row` (BF16 bits, phase-local width) to host. */
int yar_row_logits(yar_session *session, int row, uint16_t *out, int n);
/* Copy `count` positions starting at `start` of layer `layer` K and V (BF16 bits,
 * [kv_heads][count][head_dim]) of `row` to host. */
int yar_row_kv(yar_session *session, int row, int layer, int start, int count, uint16_t *k,
               uint16_t *v);
int yar_row_position(yar_session *session, int row, int *pos);
/* With YAR_OPT_LAYER_DUMP on: the last decode step's residual rows of `row` (n = hidden
 * BF16 values) at `slot` — 0 the embedding, l + 1 the output of layer l. The hidden state
 * between layers of ARModel::hidden (native/src/ar.cpp:262-299), exposed for parity. */
int yar_row_hidden(yar_session *session, int row, int slot, uint16_t *out, int n);

/* The device sampler on host logits (one step), exposed for parity tests of the filter
 * chain and the draw contract. cond/uncond are phase-local BF16 bits of width n
 * (uncond may be NULL). history holds native ids. Returns the local token and, when
 * scores is non-NULL, the FP32 filtered scores (removed rows -inf). */
int yar_sample_host(yar_model *model, const uint16_t *cond, const uint16_t *uncond, int n,
                    double cfg_scale, const yar_sampling *sampling, const int32_t *history,
                    int n_history, int step, int phase, uint64_t seed, int legacy_off,
                    int32_t *token, float *scores);

/* No counterpart in the reference. The sampler step of yar_sample_host for callers that
 * can't allocate device memory: a process whose caching allocator (PyTorch's, for one)
 * already holds the GPU's free memory, and real-time loops that can't afford the
 * device-wide synchronisation cudaFree implies. It calls no cudaMalloc or cudaFree.
 * Inputs and outputs are the caller's DEVICE memory: `logits` holds `rows` BF16 rows of
 * width n (row 0 conditional; row 1, at logits + row_stride elements, unconditional and
 * used when cfg_scale != 1), `token` one int32 (the phase-local token), `scores` (may be
 * NULL) n FP32 filtered scores. `sampling`, `history` and the rest are host values with
 * yar_sample_host's meaning. Runs on `stream` (a cudaStream_t; NULL = default stream) and
 * returns once the step has finished there. Its working memory is one static device array
 * of 769 KiB that every GPU loading the library holds until exit, so n is at most 196608
 * (larger n returns YAR_INVALID_INPUT). The first call for a device looks up that array's
 * address on the device; make it before any stream capture there. Calls share the array:
 * the library serialises its own calls, and calls whose kernels overlapped would race.
 * The calling thread's current device is the same after the call as before it. */
int yar_sample_device_noalloc(yar_model *model, const uint16_t *logits, int64_t row_stride,
                              int rows, int n, double cfg_scale, const yar_sampling *sampling,
                              const int32_t *history, int n_history, int step, int phase,
                              uint64_t seed, int32_t *token, float *scores, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* YUE2AR_H */
