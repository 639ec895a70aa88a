// tp.cu — tensor parallelism across the GPUs of one node (one process per
// GPU): an NCCL communicator and the all-reduce (sum) that follows o_proj and
// down_proj when a model's heads and FFN columns are split across ranks
// (Megatron-style; the reference has no multi-GPU path).
//
// NCCL is opened at run time (libnccl.so.2): in a process that already has
// PyTorch's NCCL loaded, that same library is used; otherwise the system's.
// The all-reduce is enqueued on the device's stream, so it is captured into
// the decode graphs with the kernels around it.

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "runtime.h"

struct tb200_tp {
  tb200_device* dev = nullptr;
  int rank = 0, world = 1;
  ncclComm_t comm = nullptr;
};

namespace {

struct Nccl {
  void* lib = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

std::mutex g_nccl_mu;
Nccl g_nccl;

int load_nccl(Nccl** out) {
  std::lock_guard<std::mutex> lock(g_nccl_mu);
  if (!g_nccl.lib) {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return rt::fail(TB200_ERR_CUDA, std::string("tensor parallelism needs libnccl.so.2: ") + dlerror());
    Nccl n;
    n.lib = h;
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(h, "ncclAllReduce"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    n.comm_abort = reinterpret_cast<decltype(n.comm_abort)>(dlsym(h, "ncclCommAbort"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!n.get_unique_id || !n.comm_init_rank || !n.all_reduce || !n.comm_destroy || !n.comm_abort ||
        !n.error_string)
      return rt::fail(TB200_ERR_CUDA, "libnccl.so.2 lacks an expected entry point");
    g_nccl = n;
  }
  *out = &g_nccl;
  return TB200_OK;
}

int nccl_fail(Nccl* n, ncclResult_t r, const char* what) {
  return rt::fail(TB200_ERR_CUDA, std::string(what) + ": " + n->error_string(r));
}

}  // namespace

namespace rt {

int tp_allreduce(tb200_tp* tp, float* buf, size_t n, cudaStream_t s) {
  Nccl* nc = nullptr;
  if (int rc = load_nccl(&nc)) return rc;
  ncclResult_t r = nc->all_reduce(buf, buf, n, ncclFloat32, ncclSum, tp->comm, s);
  if (r != ncclSuccess) return nccl_fail(nc, r, "all-reduce");
  return TB200_OK;
}

}  // namespace rt

extern "C" {

int tb200_tp_unique_id(uint8_t* out, size_t len) {
  ARG_CHECK(out && len == NCCL_UNIQUE_ID_BYTES, "the id is " + std::to_string(NCCL_UNIQUE_ID_BYTES) + " bytes");
  Nccl* nc = nullptr;
  if (int rc = load_nccl(&nc)) return rc;
  ncclUniqueId id;
  ncclResult_t r = nc->get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(nc, r, "ncclGetUniqueId");
  std::memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
  return TB200_OK;
}

int tb200_tp_init(tb200_device* dev, int rank, int world, const uint8_t* id, size_t len, tb200_tp** out) {
  ARG_CHECK(dev && id && out, "null argument");
  ARG_CHECK(len == NCCL_UNIQUE_ID_BYTES, "the id is " + std::to_string(NCCL_UNIQUE_ID_BYTES) + " bytes");
  ARG_CHECK(world >= 1 && rank >= 0 && rank < world, "bad rank or world size");
  if (int rc = rt::use(dev)) return rc;
  Nccl* nc = nullptr;
  if (int rc = load_nccl(&nc)) return rc;
  ncclUniqueId uid;
  std::memcpy(uid.internal, id, NCCL_UNIQUE_ID_BYTES);
  auto* tp = new tb200_tp;
  tp->dev = dev;
  tp->rank = rank;
  tp->world = world;
  ncclResult_t r = nc->comm_init_rank(&tp->comm, world, uid, rank);
  if (r != ncclSuccess) {
    delete tp;
    return nccl_fail(nc, r, "ncclCommInitRank");
  }
  *out = tp;
  return TB200_OK;
}

int tb200_tp_free(tb200_tp* tp) {
  if (!tp) return TB200_OK;
  Nccl* nc = nullptr;
  if (load_nccl(&nc) == TB200_OK && tp->comm) {
    cudaSetDevice(tp->dev->ordinal);
    cudaStreamSynchronize(tp->dev->stream);
    nc->comm_destroy(tp->comm);
  }
  delete tp;
  return TB200_OK;
}

int tb200_tp_rank(const tb200_tp* tp) { return tp ? tp->rank : -1; }
int tb200_tp_world(const tb200_tp* tp) { return tp ? tp->world : 0; }

int tb200_tp_allreduce(tb200_tp* tp, tb200_buffer* buf) {
  ARG_CHECK(tp && buf, "null argument");
  if (int rc = rt::use(tp->dev)) return rc;
  if (int rc = rt::tp_allreduce(tp, buf->ptr, buf->len, tp->dev->stream)) return rc;
  CUDA_TRY(cudaStreamSynchronize(tp->dev->stream));
  return TB200_OK;
}

}  // extern "C"
