// runtime.h — the handles behind include/titania_b200.h and the helpers the
// C ABI files share (runtime.cu: device, trait ops, single-token path;
// forward.cu: the many-token and many-sequence paths).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"

struct tb200_tp;  // tp.cu

struct tb200_device {
  int ordinal = 0;
  int sms = 0;
  cudaStream_t stream = nullptr;
  uint32_t* tokens = nullptr;  // device scratch for embed's token ids
  size_t tokens_cap = 0;
  unsigned long long* best = nullptr;  // argmax scratch
  // matmul over several tokens: the input split into three bf16 planes
  uint16_t* split = nullptr;  // [3][split_cap]
  size_t split_cap = 0;
  int max_cluster = 1;        // largest split-K cluster (gemm_max_cluster, at most 8)
  int* err = nullptr;         // device error word of the trait ops
  // Pinned staging buffers of the safetensors loader (loader.cu), two per
  // worker thread, allocated on first use and kept until the device closes:
  // page-locking costs about as much as the copies it serves.
  std::vector<void*> stage;
  // Workspace of the standalone decode attention (attn_op.cu), grown on
  // demand and kept until the device closes.
  float* ao_part = nullptr;        // split-context partials
  size_t ao_part_cap = 0;          // floats
  unsigned* ao_ticket = nullptr;   // one per (sequence, kv head), zero between launches
  size_t ao_ticket_cap = 0;
  int* ao_meta = nullptr;          // [2][cap]: position, sequence of each query row
  size_t ao_meta_cap = 0;
  std::vector<int> ao_meta_host;   // what ao_meta holds
  uint16_t* ao_planes = nullptr;   // [3][rows][q_dim] attention output planes
  size_t ao_planes_cap = 0;        // elements
  const void* ao_map_base = nullptr;  // the cache the tensor map describes
  size_t ao_map_rows = 0;
  CUtensorMap ao_map{};
};

struct tb200_buffer {
  float* ptr = nullptr;
  size_t len = 0, cap = 0;
};

struct tb200_weight {
  uint16_t* ptr = nullptr;
  std::vector<size_t> shape;
  size_t numel = 0;
  bool has_map = false;
  CUtensorMap map{};  // operand map of a matrix for the tensor-core contraction
};

struct FusedLayer {
  const uint16_t *attn_norm, *mlp_norm, *q_norm, *k_norm;
  uint16_t* wqkv = nullptr;  // [q_dim + 2 kv_dim][H], owned
  uint16_t* wgu = nullptr;   // [2F][H] gate/up rows interleaved, owned
  const uint16_t *wo, *wd;
  uint16_t* wo_packed = nullptr;  // o_proj packed per (kv group, output slice), owned
  // operand maps of the tensor-core contraction
  CUtensorMap m_qkv{}, m_o{}, m_gu{}, m_down{};
};

// Tensor parallelism without NCCL on the single-token path: each rank's
// receive buffers for the o_proj and down_proj partial sums of every rank,
// the flag words that say a rank's slot is written, and the other ranks'
// buffers mapped into this process (CUDA IPC over NVLink).
struct TpP2p {
  bool on = false;
  int world = 1, rank = 0;
  // this rank's: recv_o [world][H], recv_d [world][H] f32, flags [2L][world]; then the persistent
  // kernel's tagged words: o_proj partials [world * Hkv][H], down_proj partials [world][H], argmax keys
  void* region = nullptr;
  void* peer[8] = {};                   // every rank's region as mapped here (this rank's: region)
  size_t off_d = 0, off_flags = 0;      // byte offsets of recv_d and the flags in a region
  size_t off_po = 0, off_pd = 0;        // byte offsets of the persistent kernel's partials
  size_t off_pk = 0;                    // ... and of its vocabulary-split argmax keys [world][2]
  unsigned* tickets = nullptr;          // [2L] arrival counters of the publishing launches
  unsigned* epoch = nullptr;            // this step's flag value; advanced by the lm_head
  uint32_t ps_epoch = 1;                // tag base of the persistent kernel's next launch (every rank alike)
};

struct tb200_model {
  tb200_device* dev = nullptr;
  int live_states = 0;          // states built on this model
  bool free_requested = false;  // tb200_model_free came while states lived
  tb200_config c{};
  std::map<std::string, const tb200_weight*> bound;
  bool finalized = false;
  std::vector<FusedLayer> layers;
  const uint16_t *embed = nullptr, *norm = nullptr, *lm_head = nullptr;
  CUtensorMap m_lm{};
  tb200_tp* tp = nullptr;  // tensor-parallel group: this model holds one rank's heads and FFN columns
  TpP2p p2p;               // single-token partial sums by peer stores (tp.cu), when every rank can
  size_t q_dim = 0, kv_dim = 0;
  int attn_o_slices = 0;  // output slices per kv group of the fused attention + o_proj
};

// Operands of the many-token path's contractions, each three bf16 planes:
// normalised residual [cap][H], attention output [cap][q_dim], silu(g)*u [cap][F].
enum { kOpXn = 0, kOpAtt, kOpH, kOps };

struct tb200_state {
  tb200_model* m = nullptr;
  tb200_device* dev = nullptr;
  size_t max_len = 0;
  size_t n_seqs = 1;       // sequences, each with its own cache
  size_t seq_stride = 0;   // cache elements per sequence
  int kv_f32 = 0;          // cache element: 0 bf16, 1 f32
  size_t host_pos = 0;     // the position the next step runs at, as the host knows it
  unsigned char* kv = nullptr;  // [seq][L][2][Hkv][max_len][head_dim], bf16 or f32
  float* rope = nullptr;   // [max_len][head_dim]
  float *x = nullptr, *qkv = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr;
  float *x2 = nullptr, *part_o = nullptr;  // mid-layer residual; per-group o_proj partials
  float *part_tp = nullptr, *part_tp2 = nullptr;  // tensor parallel: o_proj / down_proj partial sums [H]
  float* part = nullptr;
  unsigned* attn_ticket = nullptr;
  unsigned long long* mv_partial = nullptr;
  unsigned* mv_ticket = nullptr;
  int* io = nullptr;          // device: [0] token, [1] pos, [2] step, [3] error
  int* tokens_out = nullptr;  // device: [max_len]
  int* io_host = nullptr;     // pinned: [max_len][2] staged (token, pos) + [4] readback
  int max_split = 1;
  tb::MvPlan p_qkv{}, p_o{}, p_gu{}, p_down{}, p_lm{};
  tb::Trace trace{};       // device trace buffer while tracing
  uint32_t trace_next = 0;  // next free record slot while capturing
  cudaGraphExec_t graph = nullptr;        // positions >= kAttnOMaxCtx
  cudaGraphExec_t graph_short = nullptr;  // positions < kAttnOMaxCtx (fused attention + o_proj)
  // ---- single-token path as one persistent kernel (persist.cu)
  int decode_mode = TB200_DECODE_FUSED;  // TB200_DECODE_*: what single-token steps run
  void* ps_words = nullptr;   // tagged words the phases exchange, zeroed once
  size_t ps_nwords = 0;
  void* ps_ctl = nullptr;     // argmax key, ticket
  uint32_t ps_epoch = 0;      // tag base of the next launch
  int ps_grid = 0;            // CTAs of the last launch
  bool ps_traced = false;     // a persistent launch ran while tracing
  bool ps_dirty = false;      // a launch may have stopped mid-step: reset the argmax key and ticket first

  // ---- many-token / many-sequence path (forward.cu), allocated on first use
  int cap = 0;                 // tokens per pass
  float *bx = nullptr, *bqkv = nullptr, *blogits = nullptr;  // [cap][H], [cap][q+2kv], [n_seqs][V]
  float* bpart = nullptr;      // tensor parallel: o_proj / down_proj partial sums [cap][H]
  float* ssq_a = nullptr;      // [cap][H/128] partial sums of squares of x before attention (RMSNorm input)
  float* ssq_b = nullptr;      // ... and before the MLP
  uint16_t* bact = nullptr;    // the kOps operands' planes, one allocation
  int* bmeta = nullptr;        // device [3][cap]: token, position, sequence of each row
  int* bmeta_host = nullptr;   // pinned [3][cap] + readback words
  float* rows_part = nullptr;  // decode attention split partials
  unsigned* rows_ticket = nullptr;
  int rows_parts = 0;
  unsigned long long* bbest = nullptr;  // device [n_seqs] argmax keys of the lm_head contraction
  int* bstep = nullptr;        // device [0] step, [1] ticket
  int* bout = nullptr;         // device [max_len][n_seqs] generated tokens
  CUtensorMap act[kOps][3]{};  // per operand and plane
  CUtensorMap cache_map{};     // bf16 cache as rows of head_dim, for the tensor-core decode attention
  bool has_cache_map = false;
  cudaGraphExec_t bgraph = nullptr;  // one decode step of every sequence
};

namespace rt {

// Records `msg` for tb200_last_error and returns `code`.
int fail(int code, const std::string& msg);
// The last launch's error, recorded with `what`.
int launched(const char* what);
// Makes `d` the current device.
int use(tb200_device* d);
// model.rs:239-250, on the host.
std::vector<float> rope_table(size_t max_len, size_t head_dim, float theta);
const char* last_error();

// forward.cu: Model::forward (model.rs:83-91) for `n` tokens of sequence
// `seq` at positions pos.. through the tensor-core path; the last token's
// logits go to `logits` (host, or null) and its greedy choice to *next.
int forward_tokens(tb200_state* st, size_t seq, const uint32_t* tokens, size_t n, size_t pos, float* logits,
                   uint32_t* next);
// Sums `n` floats at `buf` over the tensor-parallel group, on stream `s`.
int tp_allreduce(tb200_tp* tp, float* buf, size_t n, cudaStream_t s);
// Ranks in the group (1 for a null group).
int tp_world(const tb200_tp* tp);
// Sets up m->p2p (every rank calls it at finalize; all ranks agree whether
// to use it, else they keep NCCL) and releases it.
int tp_p2p_setup(tb200_model* m);
void tp_p2p_free(tb200_model* m);

// persist.cu: why the persistent single-token step cannot run model m with
// state st ("" when it can); enqueues `steps` greedy steps from st->io as
// one launch (the last step's logits to st->logits when `logits`); the trace
// slots one step uses.
std::string persist_unsupported(const tb200_model* m, const tb200_state* st);
int persist_enqueue(tb200_state* st, size_t steps, bool logits, float* logits_to = nullptr);
size_t persist_trace_slots(const tb200_state* st);
// persist_wide.cu: the same for models wider than 3072 (up to 10240).
std::string persist_wide_unsupported(const tb200_model* m, const tb200_state* st);
int persist_wide_enqueue(tb200_state* st, size_t steps, bool logits, float* logits_to = nullptr);

// Frees what the many-token path allocated on a state.
void free_batch(tb200_state* st);
// Destroys the batched decode graph (it is captured again on next use).
void drop_batch_graph(tb200_state* st);

}  // namespace rt

#define CUDA_TRY(expr)                                                                                    \
  do {                                                                                                    \
    cudaError_t e_ = (expr);                                                                              \
    if (e_ != cudaSuccess) return rt::fail(TB200_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)

#define ARG_CHECK(cond, msg)                            \
  do {                                                  \
    if (!(cond)) return rt::fail(TB200_ERR_ARG, (msg)); \
  } while (0)
