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

#include <cstring>
#include <mutex>
#include <string>

#include "engine.h"

namespace yar {

namespace {
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
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
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
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
  check(nccl().comm_init_rank(&comm, world, id, rank), "ncclCommInitRank");
  m.tp_comm = comm;
}

void tp_destroy(Model &m) {
  if (!m.tp_comm) return;
  nccl().comm_destroy(static_cast<ncclComm_t>(m.tp_comm));
  m.tp_comm = nullptr;
}

void tp_allgather_bf16(const Model &m, const bf16 *send, bf16 *recv, size_t n, cudaStream_t st) {
  check(nccl().all_gather(send, recv, n, ncclBfloat16, static_cast<ncclComm_t>(m.tp_comm), st), "ncclAllGather");
}

}  // namespace yar
