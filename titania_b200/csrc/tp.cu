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

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

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
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
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
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    n.comm_abort = reinterpret_cast<decltype(n.comm_abort)>(dlsym(h, "ncclCommAbort"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!n.get_unique_id || !n.comm_init_rank || !n.all_reduce || !n.all_gather || !n.comm_destroy ||
        !n.comm_abort || !n.error_string)
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

int tp_world(const tb200_tp* tp) { return tp ? tp->world : 1; }

int tp_allreduce(tb200_tp* tp, float* buf, size_t n, cudaStream_t s) {
  Nccl* nc = nullptr;
  if (int rc = load_nccl(&nc)) return rc;
  ncclResult_t r = nc->all_reduce(buf, buf, n, ncclFloat32, ncclSum, tp->comm, s);
  if (r != ncclSuccess) return nccl_fail(nc, r, "all-reduce");
  return TB200_OK;
}

namespace {

// What a rank tells the others at set-up: its receive region, its GPU, and
// whether it can take part.
struct P2pCard {
  cudaIpcMemHandle_t handle;
  unsigned char uuid[16];
  int ready;
  int pad[3];
};

// Releases what set-up built; `barrier`: wait for every rank first, so that
// no rank frees its region while another still maps it.
void p2p_release(tb200_model* m, bool barrier) {
  TpP2p& p = m->p2p;
  for (int r = 0; r < 8; r++)
    if (p.peer[r] && p.peer[r] != p.region) cudaIpcCloseMemHandle(p.peer[r]);
  if (barrier && m->tp) {
    Nccl* nc = nullptr;
    if (load_nccl(&nc) == TB200_OK) {
      int* one = nullptr;
      if (cudaMalloc(&one, sizeof(int)) == cudaSuccess) {
        nc->all_reduce(one, one, 1, ncclInt32, ncclSum, m->tp->comm, m->dev->stream);
        cudaStreamSynchronize(m->dev->stream);
        cudaFree(one);
      }
    }
  }
  cudaFree(p.region);
  cudaFree(p.tickets);
  cudaFree(p.epoch);
  p = TpP2p{};
}

}  // namespace

// The partial sums of o_proj and down_proj go to every rank by peer stores
// when every rank's GPU is distinct and can map the others' memory; the
// ranks agree (an all-reduce of their readiness) before any uses it.
// TB200_TP_ALLREDUCE=nccl keeps NCCL for them.
int tp_p2p_setup(tb200_model* m) {
  tb200_tp* tp = m->tp;
  if (!tp || tp->world < 2 || tp->world > 8) return TB200_OK;
  Nccl* nc = nullptr;
  if (int rc = load_nccl(&nc)) return rc;
  const char* env = getenv("TB200_TP_ALLREDUCE");
  const bool wanted = !(env && std::string(env) == "nccl");
  TpP2p& p = m->p2p;
  p = TpP2p{};
  const int W = tp->world;
  const size_t H = m->c.hidden_size, L = m->c.num_hidden_layers;
  p.world = W;
  p.rank = tp->rank;
  p.off_d = size_t(W) * H * 4;
  p.off_flags = 2 * size_t(W) * H * 4;
  p.off_po = (p.off_flags + 2 * L * W * 4 + 255) / 256 * 256;
  p.off_pd = p.off_po + size_t(W) * m->c.num_key_value_heads * H * 8;
  p.off_pk = p.off_pd + size_t(W) * H * 8;
  const size_t bytes = p.off_pk + size_t(W) * 2 * 8;
  cudaStream_t s = m->dev->stream;
  P2pCard card{};
  bool ok = wanted;
  if (ok) ok = cudaMalloc(&p.region, bytes) == cudaSuccess && cudaMemset(p.region, 0, bytes) == cudaSuccess;
  if (ok) ok = cudaIpcGetMemHandle(&card.handle, p.region) == cudaSuccess;
  cudaDeviceProp prop{};
  if (ok) ok = cudaGetDeviceProperties(&prop, m->dev->ordinal) == cudaSuccess;
  if (ok) std::memcpy(card.uuid, prop.uuid.bytes, 16);
  card.ready = ok ? 1 : 0;
  // Every rank's card, through the group (every rank takes these collective steps).
  P2pCard* dcards = nullptr;
  CUDA_TRY(cudaMalloc(&dcards, sizeof(P2pCard) * (W + 1)));
  CUDA_TRY(cudaMemcpy(dcards + W, &card, sizeof(card), cudaMemcpyHostToDevice));
  ncclResult_t r = nc->all_gather(dcards + W, dcards, sizeof(P2pCard), ncclUint8, tp->comm, s);
  std::vector<P2pCard> cards(W);
  if (r == ncclSuccess) r = cudaStreamSynchronize(s) == cudaSuccess ? ncclSuccess : ncclUnhandledCudaError;
  if (r == ncclSuccess) cudaMemcpy(cards.data(), dcards, sizeof(P2pCard) * W, cudaMemcpyDeviceToHost);
  cudaFree(dcards);
  if (r != ncclSuccess) {
    p2p_release(m, false);
    return nccl_fail(nc, r, "tensor-parallel set-up: all-gather");
  }
  // Distinct GPUs only: kernels that wait on one another must not share one.
  for (int i = 0; i < W && ok; i++) {
    ok = cards[i].ready == 1;
    for (int j = 0; j < i && ok; j++) ok = std::memcmp(cards[i].uuid, cards[j].uuid, 16) != 0;
  }
  for (int i = 0; i < W && ok; i++) {
    if (i == tp->rank) {
      p.peer[i] = p.region;
    } else {
      void* ptr = nullptr;
      ok = cudaIpcOpenMemHandle(&ptr, cards[i].handle, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
      p.peer[i] = ptr;
    }
  }
  if (ok) ok = cudaMalloc(&p.tickets, 2 * L * 4) == cudaSuccess && cudaMemset(p.tickets, 0, 2 * L * 4) == cudaSuccess;
  if (ok) {
    static const unsigned one = 1u;  // flags start at 0, so the first step's tag is 1
    ok = cudaMalloc(&p.epoch, 4) == cudaSuccess && cudaMemcpy(p.epoch, &one, 4, cudaMemcpyHostToDevice) == cudaSuccess;
  }
  cudaGetLastError();  // a refused mapping is an answer, not an error to keep
  // All ranks or none.
  int* dflag = nullptr;
  CUDA_TRY(cudaMalloc(&dflag, sizeof(int)));
  const int mine = ok ? 1 : 0;
  CUDA_TRY(cudaMemcpy(dflag, &mine, sizeof(int), cudaMemcpyHostToDevice));
  r = nc->all_reduce(dflag, dflag, 1, ncclInt32, ncclMin, tp->comm, s);
  int all = 0;
  if (r == ncclSuccess && cudaStreamSynchronize(s) == cudaSuccess) cudaMemcpy(&all, dflag, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(dflag);
  if (r != ncclSuccess) {
    p2p_release(m, false);
    return nccl_fail(nc, r, "tensor-parallel set-up: all-reduce");
  }
  if (all != 1) {
    p2p_release(m, true);
    return TB200_OK;  // NCCL it is
  }
  p.on = true;
  return TB200_OK;
}

void tp_p2p_free(tb200_model* m) {
  if (m->p2p.region || m->p2p.tickets || m->p2p.epoch) p2p_release(m, m->p2p.on);
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

int tb200_model_tp_peer_exchange(const tb200_model* m) { return m && m->p2p.on ? 1 : 0; }

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
