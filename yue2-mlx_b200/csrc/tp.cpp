// tp.cpp — the tensor-parallel exchange steps over NCCL.
//
// Tensor parallelism (one process per GPU, `world` ranks) splits every linear of a layer
// by output rows — q/k/v by KV-head group, O and down by hidden rows, gate/up by FFN
// columns, the LM head by phase columns — and keeps its whole input width, so each output
// value is computed by one rank with exactly the one-GPU arithmetic. After each operation
// the ranks' output blocks are all-gathered (BF16), leaving every rank with the whole
// activation: attention heads before O, the residual rows after O and after down, the FFN
// activations before down, the logits before sampling. Every rank then samples the same
// token from identical logits with the same Philox key.
//
// NCCL is opened at run time (dlopen of libnccl.so.2: the copy already in the process —
// PyTorch's, when it is loaded — else the system one), so the library itself has no
// link-time NCCL dependency and loads on hosts without it. Only the types come from
// nccl.h; the few entry points used are resolved by name.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <string>
#include <vector>

#include "engine.h"

namespace yar {

namespace {
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
  std::string failure;
};

const NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      const char *e = dlerror();
      api.failure = std::string("cannot open libnccl.so.2: ") + (e ? e : "unknown error");
      return;
    }
    auto sym = [&](const char *name) {
      void *p = dlsym(h, name);
      if (!p && api.failure.empty()) api.failure = std::string("libnccl.so.2 lacks ") + name;
      return p;
    };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank_config =
        reinterpret_cast<decltype(api.comm_init_rank_config)>(sym("ncclCommInitRankConfig"));
    api.comm_get_async_error = reinterpret_cast<decltype(api.comm_get_async_error)>(sym("ncclCommGetAsyncError"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
  });
  if (!api.failure.empty()) throw Error("RuntimeError", "tensor parallelism needs NCCL: " + api.failure);
  return api;
}

void check(ncclResult_t r, const char *what) {
  if (r == ncclSuccess) return;
  const char *msg = nccl().error_string ? nccl().error_string(r) : "unknown";
  throw Error("RuntimeError", std::string(what) + " failed: " + msg);
}

// Seconds the ranks get to join a communicator (YAR_TP_JOIN_TIMEOUT_S, default 300), and
// to finish any later call the non-blocking communicator reports as in progress.
double join_timeout_s() {
  const char *v = std::getenv("YAR_TP_JOIN_TIMEOUT_S");
  const double t = v ? std::atof(v) : 0.0;
  return t > 0 ? t : 300.0;
}

// The communicator is non-blocking (so a rank whose peers never arrive can give up): a
// call may return ncclInProgress, after which its state is polled until it settles or the
// deadline passes — then the communicator is aborted and the call fails.
void settle(ncclComm_t comm, ncclResult_t r, const char *what, double timeout_s) {
  const auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress) {
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
      nccl().comm_abort(comm);
      throw Error("RuntimeError", std::string(what) + ": tensor-parallel ranks did not join within " +
                                      std::to_string(int(timeout_s)) + " s (communicator aborted)");
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
    check(nccl().comm_get_async_error(comm, &r) == ncclSuccess ? ncclSuccess : ncclSystemError, what);
  }
  check(r, what);
}
}  // namespace

void tp_unique_id(uint8_t *out) {
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId id;
  check(nccl().get_unique_id(&id), "ncclGetUniqueId");
  std::memcpy(out, &id, sizeof(id));
}

void tp_init(Model &m, int rank, int world, const uint8_t *id_bytes) {
  ncclUniqueId id;
  std::memcpy(&id, id_bytes, sizeof(id));
  YAR_CUDA(cudaSetDevice(m.device));
  ncclComm_t comm = nullptr;
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  const ncclResult_t r = nccl().comm_init_rank_config(&comm, world, id, rank, &config);
  if (r != ncclSuccess && r != ncclInProgress) check(r, "ncclCommInitRankConfig");
  settle(comm, r, "ncclCommInitRankConfig", join_timeout_s());
  m.tp_comm = comm;
}

void tp_destroy(Model &m) {
  if (!m.tp_comm) return;
  nccl().comm_destroy(static_cast<ncclComm_t>(m.tp_comm));
  m.tp_comm = nullptr;
}

void tp_allgather_bf16(const Model &m, const bf16 *send, bf16 *recv, size_t n, cudaStream_t st) {
  auto comm = static_cast<ncclComm_t>(m.tp_comm);
  settle(comm, nccl().all_gather(send, recv, n, ncclBfloat16, comm, st), "ncclAllGather", join_timeout_s());
}

namespace {
// Every rank's `bytes` of host data (rank order) through one all-gather.
std::vector<char> allgather_host(const Model &m, const void *mine, size_t bytes, cudaStream_t st) {
  const int W = m.tp_world;
  char *d = nullptr;
  YAR_CUDA(cudaMalloc(&d, bytes * (W + 1)));
  std::vector<char> out(bytes * W);
  try {
    YAR_CUDA(cudaMemcpyAsync(d + bytes * W, mine, bytes, cudaMemcpyHostToDevice, st));
    auto comm = static_cast<ncclComm_t>(m.tp_comm);
    settle(comm, nccl().all_gather(d + bytes * W, d, bytes, ncclInt8, comm, st), "ncclAllGather", join_timeout_s());
    YAR_CUDA(cudaMemcpyAsync(out.data(), d, bytes * W, cudaMemcpyDeviceToHost, st));
    YAR_CUDA(cudaStreamSynchronize(st));
  } catch (...) {
    cudaFree(d);
    throw;
  }
  cudaFree(d);
  return out;
}
bool all_ranks_agree(const Model &m, bool ok, cudaStream_t st) {
  const int mine = ok ? 1 : 0;
  const std::vector<char> v = allgather_host(m, &mine, sizeof(int), st);
  for (int k = 0; k < m.tp_world; ++k) {
    int x;
    std::memcpy(&x, v.data() + k * sizeof(int), sizeof(int));
    if (!x) return false;
  }
  return true;
}
}  // namespace

bool tp_map_peers(const Model &m, void *region, size_t region_bytes, std::vector<void *> &peers, long long *dst,
                  cudaStream_t st) {
  struct Entry {
    cudaIpcMemHandle_t handle;
    int device, sm_count;
    unsigned long long bytes;
  };
  const int W = m.tp_world, rank = m.tp_rank;
  if (W > 8) return false;  // dst holds at most 7 peers (the same answer on every rank)
  Entry mine{};
  const bool have_handle = cudaIpcGetMemHandle(&mine.handle, region) == cudaSuccess;
  cudaGetLastError();
  mine.device = m.device;
  mine.sm_count = m.sm_count;
  mine.bytes = region_bytes;
  const std::vector<char> raw = allgather_host(m, &mine, sizeof(Entry), st);
  std::vector<Entry> e(W);
  std::memcpy(e.data(), raw.data(), raw.size());
  // Direct loads, stores and atomics to every peer, the same grid everywhere (the
  // persistent kernel's counter targets assume it) and regions of the same size (the same
  // session shape, hence the same layout: outputs are stored at their own offset).
  bool ok = have_handle;
  for (int k = 0; k < W; ++k) ok = ok && e[k].bytes == region_bytes;
  for (int k = 0; k < W && ok; ++k) {
    if (k == rank) continue;
    int access = 0, atomics = 0;
    ok = cudaDeviceCanAccessPeer(&access, m.device, e[k].device) == cudaSuccess && access &&
         cudaDeviceGetP2PAttribute(&atomics, cudaDevP2PAttrNativeAtomicSupported, m.device, e[k].device) ==
             cudaSuccess &&
         atomics && e[k].sm_count == m.sm_count;
  }
  cudaGetLastError();
  if (!all_ranks_agree(m, ok, st)) return false;
  peers.assign(W, nullptr);
  bool opened = true;
  for (int k = 0; k < W && opened; ++k) {
    if (k == rank) continue;
    opened = cudaIpcOpenMemHandle(&peers[k], e[k].handle, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
  }
  cudaGetLastError();
  if (!all_ranks_agree(m, opened, st)) {
    tp_unmap_peers(peers);
    return false;
  }
  for (int k = 0, i = 0; k < W; ++k)
    if (k != rank) dst[i++] = static_cast<char *>(peers[k]) - static_cast<char *>(region);
  return true;
}

void tp_unmap_peers(std::vector<void *> &peers) {
  for (void *p : peers)
    if (p) cudaIpcCloseMemHandle(p);
  peers.clear();
}

void tp_barrier(const Model &m, void *scratch, cudaStream_t st) {
  YAR_CUDA(cudaStreamSynchronize(st));
  bf16 *b = static_cast<bf16 *>(scratch);
  tp_allgather_bf16(m, b, b + 1, 1, st);
  YAR_CUDA(cudaStreamSynchronize(st));
}

}  // namespace yar
