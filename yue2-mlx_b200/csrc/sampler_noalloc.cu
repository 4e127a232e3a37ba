// sampler_noalloc.cu — one device sampler step that allocates no device memory.
//
// Some callers can't call cudaMalloc or cudaFree: a process whose caching allocator
// (PyTorch's, for one) already holds the GPU's free memory, so a side allocation fails
// or fragments its pool, and real-time token loops, where cudaFree's implicit device-wide
// synchronisation would stall every other stream on the GPU. yar_sample_host allocates
// and frees six buffers per call. This variant runs the same k_sampler launch on logits,
// a token slot and an optional score row that the caller already owns, and keeps its
// own working memory — the request record and the FP32 score row the filter chain
// works in — in one static device array.
//
// That array (NoAllocScratch below, 769 KiB for at most kNoAllocMaxColumns columns) is
// part of this library's device image: every GPU that loads the library holds it until
// the process exits. In host code its name is only a host-side stand-in, so the host
// side resolves its device address with cudaGetSymbolAddress once per device, with that
// device current, on the first call made for that device; that first call should
// therefore come before any stream capture on the device.
//
// Every call shares the one array and finds the previous call's contents in it. Each
// call rewrites the whole request record first (its step, done and error words start at
// zero), and the kernel writes score columns [0, n) before it reads them, so nothing
// stale is read. Two calls whose kernels overlapped on the GPU would race on the array:
// a process-wide lock, held until the call's step has finished on its stream, keeps this
// entry point's own calls from overlapping.
//
// The call runs with the model's device current and gives the calling thread back the
// current device it had on entry, on success and on error alike.
#include <climits>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "yue2ar.h"

namespace yar {

void validate_sampling(const ::yar_sampling &s);
void launch_sampler_ex(RequestState *req, const bf16 *logits, int logit_stride, float *scores, int *token,
                       int *active, int32_t *out_tokens, int out_cap, int write_scores, int32_t *picked,
                       int n_requests, cudaStream_t st);

// Widest score row the array holds: the pinned model's whole 184,704-row vocabulary
// (every phase) fits.
constexpr int kNoAllocMaxColumns = 196608;

struct NoAllocScratch {
  RequestState req;
  int token[2];   // per-row sampled token (the decode loop's feedback slot; unused here)
  int active[2];  // per-row active flag (likewise)
  alignas(16) float scores[kNoAllocMaxColumns];
};

static __device__ __align__(256) NoAllocScratch g_sampler_scratch[1];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_lock;
NoAllocScratch *g_scratch_addr[kMaxDevices] = {};

// Makes `device` current for the guard's lifetime and gives the calling thread back its
// own current device on every exit path (a PyTorch caller keeps its tensors and launches
// on the device it had selected, whichever device the model lives on).
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int device) {
    YAR_CUDA(cudaGetDevice(&prev));
    if (prev != device) YAR_CUDA(cudaSetDevice(device));
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
  DeviceGuard(const DeviceGuard &) = delete;
  DeviceGuard &operator=(const DeviceGuard &) = delete;
};

// Device address of this device's copy of the array; the caller holds the lock and has
// made `device` current.
NoAllocScratch *scratch_for(int device) {
  if (device < 0 || device >= kMaxDevices) throw Error("RuntimeError", "device ordinal outside 0..63");
  if (!g_scratch_addr[device]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_sampler_scratch);
    if (e != cudaSuccess || !p)
      throw Error("RuntimeError", std::string("cudaGetSymbolAddress of the sampler scratch failed: ") +
                                      cudaGetErrorString(e));
    g_scratch_addr[device] = static_cast<NoAllocScratch *>(p);
  }
  return g_scratch_addr[device];
}
}  // namespace

void sample_device_noalloc(Model &m, const uint16_t *logits, long long row_stride, int rows, int n,
                           double cfg_scale, const ::yar_sampling &smp, const int32_t *history, int n_history,
                           int step, int phase, uint64_t seed, int32_t *token, float *scores,
                           cudaStream_t st) {
  validate_sampling(smp);
  if (phase != kPhaseAbc && phase != kPhaseSemantic && phase != kPhaseFull)
    throw Error("ValueError", "phase must be 'abc' or 'semantic'");
  const int expected = phase == kPhaseAbc ? kEOD + 1 : phase == kPhaseSemantic ? kCodecSize + 1 : n;
  if (n < 1 || n != expected) throw Error("ValueError", "Incorrect projected phase vocabulary size");
  if (n > kNoAllocMaxColumns)
    throw Error("ValueError", "yar_sample_device_noalloc: " + std::to_string(n) +
                                  " columns exceed its fixed scratch of " + std::to_string(kNoAllocMaxColumns));
  if (rows != 1 && rows != 2) throw Error("ValueError", "rows must be 1 (conditional) or 2 (with unconditional)");
  if (rows == 2 && (row_stride < n || row_stride > INT_MAX))
    throw Error("ValueError", "row_stride must be at least n and fit in 31 bits");
  if (step < 0 || n_history < 0) throw Error("ValueError", "step and n_history must be non-negative");

  // The request record: same fields and values as the host entry point builds.
  RequestState r;
  std::memset(&r, 0, sizeof(r));
  const bool cfg = rows == 2 && cfg_scale != 1.0;
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
  fill_penalty_alpha(r, smp.repetition_penalty, false);
  r.seed_lo = uint32_t(seed);
  r.seed_hi = uint32_t(seed >> 32);
  r.step = step;
  const int keep = n_history < kHistCap ? n_history : kHistCap;
  r.n_out = n_history;
  for (int i = n_history - keep; i < n_history; ++i) r.hist[i % kHistCap] = history[i];

  std::lock_guard<std::mutex> lock(g_scratch_lock);
  DeviceGuard on_model_device(m.device);
  NoAllocScratch *scr = scratch_for(m.device);
  YAR_CUDA(cudaMemcpyAsync(&scr->req, &r, sizeof(r), cudaMemcpyHostToDevice, st));
  launch_sampler_ex(&scr->req, reinterpret_cast<const bf16 *>(logits), cfg ? int(row_stride) : n, scr->scores,
                    scr->token, scr->active, nullptr, 0, 1, token, 1, st);
  if (scores) YAR_CUDA(cudaMemcpyAsync(scores, scr->scores, size_t(n) * 4, cudaMemcpyDeviceToDevice, st));
  int err = 0;
  YAR_CUDA(cudaMemcpyAsync(&err, &scr->req.error, sizeof(int), cudaMemcpyDeviceToHost, st));
  YAR_CUDA(cudaStreamSynchronize(st));
  if (err) throw Error("RuntimeError", err == 1 ? "sampler candidate set exceeds 2048 rows" : "no finite logits");
}

}  // namespace yar
