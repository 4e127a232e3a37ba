// engine.h — internal types of the YuE2 AR engine (host C++20 + CUDA sm_100a).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace yar {

using bf16 = __nv_bfloat16;

// Protocol ids (native/include/lyra/types.hpp:63-68).
constexpr int kEOD = 151643, kAbcEnd = 151848, kMusicEnd = 151852;
constexpr int kCodecOffset = 151853, kCodecSize = 32768, kContext = 24576;
constexpr int kPhaseAbc = 0, kPhaseSemantic = 1, kPhaseFull = 2;

// lyra::Error (types.hpp:70-74): a type name the C ABI maps to a status code.
struct Error : std::runtime_error {
  std::string type;
  Error(std::string kind, const std::string &msg) : std::runtime_error(msg), type(std::move(kind)) {}
};
[[noreturn]] void throw_cuda(cudaError_t e, const char *what, const char *file, int line);
#define YAR_CUDA(x)                                                        \
  do {                                                                     \
    cudaError_t _e = (x);                                                  \
    if (_e != cudaSuccess) ::yar::throw_cuda(_e, #x, __FILE__, __LINE__);  \
  } while (0)

struct Dims {
  int hidden = 2048, layers = 28, heads = 16, kv_heads = 8, head_dim = 128, ffn = 6144;
  int vocab = 184704, context = kContext;
  float eps = 1e-6f;
  double theta = 1e6;
  int qdim() const { return heads * head_dim; }
  int kvdim() const { return kv_heads * head_dim; }
  int qkv_rows() const { return qdim() + 2 * kvdim(); }
};

// Device weights of one decoder layer in the engine layout (under tensor parallelism the
// rank's rows of each, with the whole model's input width).
struct LayerWeights {
  const bf16 *qkv;   // [q + k + v rows][hidden]: q_proj, k_proj, v_proj rows stacked
  const bf16 *o;     // [hidden rows][qdim of the whole model]
  const bf16 *gu;    // [2*ffn][hidden]: row 2j = gate_proj row j, row 2j+1 = up_proj row j
  const bf16 *down;  // [hidden rows][ffn of the whole model]
  const bf16 *ln1, *ln2, *qn, *kn;
};

// Stage images of one layer's 8-bit weights (the `8bit` precision), in the fused row
// order of LayerWeights: the layout the 8-bit ring consumer reads (16-row units of
// K / 2048 stages of 34,816 bytes, written by q8_stage_image).
struct QLayer {
  const unsigned char *qkv, *o, *gu, *down;
};

// Splits per (row, kv head) the decode attention's partial buffers hold.
constexpr int kSessionMaxSplits = 32;

struct Model {
  Dims d;
  int device = 0, sm_count = 148;
  void *arena = nullptr;
  size_t arena_bytes = 0;
  const bf16 *embed = nullptr, *lm_head = nullptr, *final_norm = nullptr;
  std::vector<LayerWeights> layers;
  LayerWeights *d_layers = nullptr;  // device copy of `layers` (persistent decode kernel)
  // Device array [layer][4] of the stage maps (128-byte TMA descriptors) of qkv, o, gu and
  // down for the persistent decode kernel; null when the shapes do not fit its ring.
  void *d_wmaps = nullptr;
  const float *rope_cos = nullptr, *rope_sin = nullptr;  // [context][head_dim/2], BF16-rounded values
  // Precision: 0 (BF16 weights), 8 or 4 (affine, group 64). Quantized, the arena holds the
  // weights dequantized to BF16 (prefill, batched and per-operation decode read them) and
  // `qarena` the stage images the persistent decode kernel streams: per layer (d_qlayers)
  // and per phase of the head (this rank's phase rows; null for a phase the vocabulary
  // does not have).
  int bits = 0;
  void *qarena = nullptr;
  size_t qarena_bytes = 0;
  std::vector<QLayer> qlayers;
  QLayer *d_qlayers = nullptr;
  const unsigned char *qhead[3] = {nullptr, nullptr, nullptr};
  // Tensor parallelism: this rank's share of the heads, KV heads and FFN columns is in `d`
  // (the whole model's dims in `full`, the rank's rows in `tp`); `tp_comm` is the NCCL
  // communicator (null: one GPU).
  Dims full;
  int tp_rank = 0, tp_world = 1;
  void *tp_comm = nullptr;
  struct TpRows {
    int q_row0 = 0, q_rows = 0, kv_row0 = 0, kv_rows = 0, ffn_row0 = 0, ffn_rows = 0, h_row0 = 0, h_rows = 0;
  } tp;
};
using TpPlan = Model::TpRows;

// Tensor-parallel share of one rank, in rows of the whole model's tensors. Every linear is
// split by output rows and keeps its whole input width: query rows [q_row0, +q_rows) of
// q_proj, rows [kv_row0, +kv_rows) of k_proj and v_proj (KV heads in equal groups, each
// with its query heads), rows [ffn_row0, +ffn_rows) of gate_proj and up_proj, and rows
// [h_row0, +h_rows) of o_proj and down_proj. Each rank's outputs (attention heads, hidden
// rows, FFN columns) are all-gathered after their operation, so every output value is
// computed by one rank exactly as on one GPU.
TpPlan tp_plan(const Dims &full, int rank, int world);

// Tensor-parallel exchange steps (tp.cpp) and the element-wise kernels around them.
void tp_unique_id(uint8_t *out128);
void tp_init(Model &m, int rank, int world, const uint8_t *id128);
void tp_destroy(Model &m);
void tp_allgather_bf16(const Model &m, const bf16 *send, bf16 *recv, size_t n, cudaStream_t st);
// Map every peer's exchange region (collective: every rank calls it for its session in the
// same order). All ranks take the same outcome: true with the peers mapped and `dst`
// filled, or false with nothing mapped (a peer without P2P loads/stores/atomics, or a
// device of another size) — the engine then exchanges through NCCL only.
bool tp_map_peers(const Model &m, void *region, size_t region_bytes, std::vector<void *> &peers, long long *dst,
                  cudaStream_t st);
void tp_unmap_peers(std::vector<void *> &peers);
// Returns once every rank has reached it with its stream idle.
void tp_barrier(const Model &m, void *scratch, cudaStream_t st);
// send[r][j] = buf[r * stride + col0 + j] for r < n_rows, j < n.
void launch_tp_pack(const bf16 *buf, int stride, int col0, int n, int n_rows, bf16 *send, cudaStream_t st);
// buf[r * stride + k * n + j] = recv[(k * n_rows + r) * n + j] for every rank k, where
// k * n + j < width.
void launch_tp_unpack(const bf16 *recv, int world, int n_rows, int n, int width, bf16 *buf, int stride,
                      cudaStream_t st);
// LM-head columns per rank under tensor parallelism: the phase width split evenly, rounded
// up to 128 columns, so every 128-column block of the head (one tcgen05 tile in the batched
// projection) lies within one rank's range and is computed as on one GPU.
inline int tp_head_slice(int width, int world) { return ((width + world - 1) / world + 127) / 128 * 128; }

// Phase projection of the LM head: rows [row0, row0 + n_main) and, optionally, one extra
// row mapped to local index n_main (native/src/ar.cpp:302-323).
struct PhaseRows {
  int row0 = 0, n_main = 0, extra = -1;
  int width() const { return n_main + (extra >= 0 ? 1 : 0); }
};
PhaseRows phase_rows(const Dims &d, int phase);

// Per-request sampler state in device memory (one CFG request spans two rows).
constexpr int kHistCap = 128;
constexpr int kMaxPenaltyWindow = 100;
struct RequestState {
  int row_c, row_u;  // conditional row, unconditional row (-1: no CFG)
  int phase, width, end_local;
  float temperature, top_p, cfg_scale;
  int top_k, window, min_tokens, max_tokens, penalty_on;
  int legacy;  // legacy_off: the filter chain in BF16, nucleus keeps >= 3 rows
  float alpha[kMaxPenaltyWindow + 1];  // penalty ** count (FP32; BF16 values when legacy)
  uint32_t seed_lo, seed_hi, stream;
  int step, done, n_out, error;
  int hist[kHistCap];  // ring of native ids (the last kHistCap sampled tokens)
};

struct Session;

// Kernel launchers (kernels_*.cu). All run on `stream`.
void launch_embed_rows(const Model &m, Session &s, int n_rows, cudaStream_t st);
// `error` (device int) enables the bulk-copy kernel, which reports expired waits there.
void launch_gemv(const bf16 *W, int N, int K, const bf16 *in, int in_stride, const bf16 *norm_w,
                 float eps, bf16 *out, int out_stride, int epilogue, int n_rows,
                 int *error, int sm_count, cudaStream_t st);
// `max_splits` (0: the session's) caps the splits per (row, kv head); fewer, longer splits
// suit large batches.
void launch_attn_decode(const Model &m, Session &s, int layer, int n_rows, cudaStream_t st, int max_splits = 0);
void launch_sampler(const Model &m, Session &s, int n_requests, cudaStream_t st);
// Prefill (T tokens of one row).
void launch_embed_tokens(const bf16 *embed, const int *ids, int T, int H, bf16 *x, cudaStream_t st);
void launch_rmsnorm_rows(const bf16 *x, const bf16 *w, int T, int H, float eps, bf16 *out,
                         cudaStream_t st);
void launch_gemm(const bf16 *A, int M, int K, const bf16 *W, int N, bf16 *C, int ldc, int epilogue,
                 cudaStream_t st);
// Prefill linears on tcgen05 (kernels_gemm_tc.cu); `error` receives expired-wait flags.
bool gemm_tc_supported(const bf16 *A, int M, int K, const bf16 *W, int N, const bf16 *C, int ldc);
// `ws` (ws_floats FP32 values, may be null) lets small-M shapes split K across CTAs; the
// split count is chosen for `split_n` columns (0: N; negative: never split), so a
// tensor-parallel rank's block of N / world columns splits K, and adds its partial sums,
// as the whole N does on one GPU.
void launch_gemm_tc(const bf16 *A, int M, int K, const bf16 *W, int N, bf16 *C, int ldc, int epilogue, int *error,
                    float *ws, size_t ws_floats, cudaStream_t st, int split_n = 0);
void configure_gemm_tc_kernels();
// A 2-D TMA map of `rows` rows of 128 BF16 at `base` (256-byte pitch), {64, 64} boxes,
// 128-byte swizzle; false when the driver's encoder is unavailable or refuses it.
bool encode_rows128_map(CUtensorMap *map, const bf16 *base, uint64_t rows);
void launch_qkv_post_prefill(const Model &m, Session &s, int layer, int row, int start, int T,
                             cudaStream_t st);
void launch_attn_prefill(const Model &m, Session &s, int layer, int row, int start, int T,
                         cudaStream_t st);

// penalty ** count per window count: FP32 (power in double of the FP32 penalty, rounded
// once), or for legacy_off the BF16 path's BF16(BF16(penalty) ** count).
void fill_penalty_alpha(RequestState &r, double penalty, bool legacy);
void configure_gemv_kernels();
void configure_gemm_kernels();
void configure_attn_kernels();
void configure_attn_tc_kernels();
void configure_gemv_tma_kernels();
void configure_persistent_kernels();
void configure_sampler_kernels();
bool persistent_supported(const Model &m, int n_rows);
// Encodes m.d_wmaps (after the weights are uploaded); leaves it null when a K is not a
// multiple of 2048.
void build_stage_maps(Model &m);
void launch_decode_persistent(const Model &m, Session &s, int n_rows, int phase, cudaStream_t st);
// Quantized weights at load time (kernels_quant.cu): raw packed rows [rows][K * bits / 8]
// (bits 8 or 4) and BF16 scale / bias bits [rows][K / 64] into BF16 weights, or into a
// stage image of q_image_bytes.
size_t q_image_bytes(int rows, int K, int bits);
void launch_q_dequant(const uint8_t *q, const uint16_t *s, const uint16_t *b, long long rows, int K, int bits,
                      bf16 *out, cudaStream_t st);
void launch_q_image(const uint8_t *q, const uint16_t *s, const uint16_t *b, int rows, int K, int bits,
                    unsigned char *img, cudaStream_t st);

enum Epilogue { kEpiStore = 0, kEpiResidual = 1, kEpiSwiGLU = 2 };

struct Session {
  Model *m = nullptr;
  int max_rows = 0, max_ctx = 0, page_tokens = 256, pages_per_row = 0, num_pages = 0;
  int prefill_chunk = 1024;
  cudaStream_t stream = nullptr;
  // Paged KV pool: [layer][page][k|v][kv_head][page_tokens][head_dim] BF16.
  bf16 *kv = nullptr;
  size_t kv_page_elems = 0;  // elements of one (layer, page, k|v) block: kv_heads*P*D
  std::vector<std::vector<int>> row_pages;
  std::vector<int> free_pages;
  int *d_page_table = nullptr;  // [max_rows][pages_per_row]
  int *d_pos = nullptr;         // [max_rows] next position (== tokens in cache)
  int *d_cur_pos = nullptr;     // [max_rows] position of the token being forwarded
  int *d_capacity = nullptr;    // [max_rows]
  int *d_token = nullptr;       // [max_rows]
  int *d_active = nullptr;      // [max_rows]
  int *d_error = nullptr;       // sticky device error flags
  std::vector<int> capacity;    // host mirror
  std::vector<int> pos;         // host mirror
  // Decode activations.
  bf16 *x = nullptr, *qkv = nullptr, *attn = nullptr, *mlp = nullptr;
  bf16 *logits = nullptr;  // [max_rows][logit_stride]
  int logit_stride = 0;
  // Split-KV attention scratch.
  float *attn_part = nullptr;  // [max_rows][heads][max_splits][head_dim + 2]
  int *attn_count = nullptr;   // [max_rows][kv_heads]
  int max_splits = 0;  // kSessionMaxSplits
  // Prefill activations (prefill_chunk rows).
  bf16 *px = nullptr, *ph = nullptr, *pqkv = nullptr, *pq = nullptr, *pattn = nullptr, *pmlp = nullptr;
  int *pids = nullptr;
  // Sampler.
  RequestState *d_req = nullptr;
  int max_requests = 0;
  int32_t *d_out_tokens = nullptr;  // [max_requests][out_cap]
  int out_cap = 0;
  float *d_scores = nullptr;  // [max_requests][logit_stride] sampler scratch
  uint64_t *d_cand = nullptr;  // [max_requests][kCandCap]
  // Captured decode steps keyed by (rows, requests, phase).
  struct Graph {
    int rows, requests, phase, persistent;
    cudaGraphExec_t exec;
  };
  std::vector<Graph> graphs;
  int *h_pinned = nullptr;  // pinned staging for small D2H reads
  // Persistent decode kernel: operation counters and the completed-step epoch.
  bool use_persistent = true;
  bool prefill_attn_tc = true;  // head_dim 128 prefill attention on tcgen05 (else mma.sync)
  int persistent_ok[3] = {-1, -1, -1};  // per row count: unknown / no / yes
  int *d_ctr = nullptr;
  int *d_epoch = nullptr;
  int n_ctr = 0;
  float *gemm_ws = nullptr;  // split-K partials of the tcgen05 GEMM
  size_t gemm_ws_floats = 0;
  int prefetch_stages = 2;  // persistent kernel: L2 prefetch distance beyond the ring
  int forced_splits = 0;    // decode attention splits per (row, kv head); 0 = automatic
  int inject_op = 0;        // persistent kernel: operation whose wait is made to expire (0 = none)
  // Hidden-state record of the last decode step (when enabled): [layers + 1][max_rows][hidden]
  // BF16 — the embedding rows, then the residual rows after each layer.
  bf16 *d_layer_dump = nullptr;
  unsigned long long *d_trace = nullptr;  // persistent-kernel timeline (when enabled)
  // Tensor parallelism: a rank's block of rows before ([rows][n]) and after
  // ([world][rows][n]) the all-gather.
  bf16 *tp_send = nullptr, *tp_recv = nullptr;
  // The exchange region (one allocation: x, attn, mlp, logits, the persistent kernel's
  // counters). Under tensor parallelism every peer's region is mapped here (CUDA IPC) and
  // tp_dst[i] is the byte offset from this region to peer i's (ranks in order, self left
  // out), so the persistent kernel stores its outputs straight into the peers' buffers.
  char *xregion = nullptr;
  size_t xregion_bytes = 0;
  // Flagged-word activations of the persistent kernel (in the exchange region; rows up to
  // 2): residual rows, raw q/k/v, attention heads, FFN activations; ll_bytes in all.
  uint2 *x_ll = nullptr, *qkv_ll = nullptr, *attn_ll = nullptr, *mlp_ll = nullptr;
  // The decode attention's split partials as flagged words ([rows][heads][max_splits]
  // [head_dim + 2]; rank-local, after the exchanged buffers in the same region).
  uint2 *part_ll = nullptr;
  size_t ll_bytes = 0;
  bool tp_mapped = false;
  long long tp_dst[7] = {};
  std::vector<void *> tp_peer_regions;
  long long tp_epoch_steps = 0;  // persistent steps since the counters were last zeroed
  size_t trace_elems = 0;
};

constexpr int kCandCap = 2048;

// Splits per (row, kv head) of the decode attention for one or two rows (the persistent
// kernel and the per-operation path alike): about one unit per SM, so a long context runs
// in one round of longer units instead of two rounds of short ones. Counted with the whole
// model's KV heads, so tensor-parallel ranks split each head's positions as one GPU does.
inline int decode_max_splits(const Model &m, const Session &s, int n_rows) {
  if (s.forced_splits > 0) return s.forced_splits < s.max_splits ? s.forced_splits : s.max_splits;
  const int per = m.sm_count / (m.full.kv_heads * (n_rows > 0 ? n_rows : 1));
  return per < 1 ? 1 : per < s.max_splits ? per : s.max_splits;
}

}  // namespace yar
