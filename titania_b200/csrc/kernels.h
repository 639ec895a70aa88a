// kernels.h — host-side launchers for the CUDA kernels (ops.cu: one kernel
// per Device-trait op; fused.cu: the fused decode path).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "common.cuh"

namespace tb {

// Records `msg` for tb200_last_error on this thread and returns `code`.
int record_error(int code, const std::string& msg);

// ---- Device-trait ops (model/cpu.rs:34-155 semantics) ----------------------
void launch_copy(cudaStream_t s, float* dst, const float* src, size_t n);
void launch_embed(cudaStream_t s, float* out, const uint16_t* table, size_t dim, const uint32_t* tokens, size_t n);
void launch_matmul(cudaStream_t s, float* out, const uint16_t* w, size_t rows, size_t cols, const float* x, size_t n);
void launch_add(cudaStream_t s, float* x, const float* y, size_t n);
void launch_rmsnorm(cudaStream_t s, float* x, size_t rows, const uint16_t* w, size_t dim, float eps);
void launch_rope(cudaStream_t s, float* x, size_t n_tokens, const float* table, size_t pos, size_t n_heads,
                 size_t head_dim);
void launch_attention(cudaStream_t s, float* out, const float* q, size_t n_tokens, const float* k_cache,
                      const float* v_cache, size_t pos, size_t n_heads, size_t head_dim, size_t n_kv_heads);
void launch_silu_mul(cudaStream_t s, float* g, const float* u, size_t n);
// Writes the argmax key (see argmax_key) of x[0..n) into *best, which the
// caller zeroes first.
void launch_argmax(cudaStream_t s, const float* x, size_t n, unsigned long long* best, int sms);

// ---- fused decode path ------------------------------------------------------

// Epilogues of the fused matrix-vector kernel.
enum MvEpilogue {
  kMvStore = 0,   // out[r] = w_r · x
  kMvResidual,    // out[r] += w_r · x            (residual stream update)
  kMvSiluPair,    // rows interleaved (gate, up): out[r/2] = silu(g) * u
  kMvArgmax,      // out[r] = w_r · x, plus the greedy choice over all rows
};

struct MvArgs {
  const uint16_t* w;       // [rows][cols] bf16
  int rows, cols;
  int row_align;           // CTA row ranges start at multiples of this
  const float* x;          // [cols] input
  const float* partials;   // npartials vectors of [cols] added to x first (fixed order), or null
  int npartials;
  float* x_out;            // receives x + partials (written by CTA 0), or null
  const uint16_t* norm_w;  // RMSNorm weight applied to x first, or null
  float eps;
  float* out;
  const float* resid_src;  // kMvResidual: the residual read (null: out itself)
  // kMvArgmax only:
  unsigned long long* partial;  // [grid] per-CTA best key
  unsigned* ticket;             // zero between launches
  int* token;                   // next input token (written)
  int* pos;                     // position (incremented)
  int* step;                    // generated-token counter (incremented)
  int* tokens_out;              // [tokens_cap] generated tokens
  int tokens_cap;
  int* err;
  Trace trace;
  uint32_t trace_base;  // first record slot of this launch
  uint32_t tag;
  // Tensor parallelism without NCCL (the o_proj / down_proj partial sums,
  // see P2P below): a kMvStore launch with npeers > 0 stores row r of its
  // output at peer_out[p][r] for every rank p instead of out[r] (peer_out[p]
  // is this rank's slot of rank p's receive buffer), and its last CTA then
  // writes *epoch into peer_flag[p] (this rank's flag word at rank p). A
  // launch with nwait > 0 first waits, bounded, until wait_flags[0 .. nwait)
  // all hold *epoch (every rank's slots of its input are written). A kMvArgmax
  // launch with epoch set advances *epoch once its step is done.
  float* peer_out[8];
  unsigned* peer_flag[8];
  int npeers;
  unsigned* p2p_ticket;  // with npeers: zero between launches
  const unsigned* wait_flags;
  int nwait;
  unsigned* epoch;
};

// Rows a CTA of a residual-epilogue launch may own (staged in shared memory).
constexpr int kMaxResidualRows = 64;
// Most partial vectors a matrix-vector kernel sums into its input.
constexpr int kMaxPartials = 8;

struct MvPlan {
  int grid, chunk_rows, stage_rows, slots;
  size_t smem;
  int max_rows;  // most rows any CTA owns
};
MvPlan plan_mv(int rows, int cols, int row_align, bool norm, int sms, size_t smem_budget);
// Raises the shared-memory limit of every matrix-vector kernel to what a
// block can opt into; call once per device before capturing or launching them.
cudaError_t init_fused_kernels(int max_smem_optin);
void launch_mv(cudaStream_t s, const MvPlan& plan, int epilogue, const MvArgs& a, bool pdl);

struct AttnArgs {
  const float* qkv;         // [q_dim | kv_dim | kv_dim] raw projections
  const uint16_t* q_norm;   // [head_dim] bf16 or null
  const uint16_t* k_norm;   // [head_dim] bf16 or null
  float eps;
  const float* rope;        // [max_len][head_dim] (cos, sin) pairs
  void* k_cache;            // [Hkv][max_len][head_dim], bf16 or f32
  void* v_cache;
  int kv_f32;               // cache element: 0 bf16, 1 f32
  int max_len, n_heads, n_kv_heads;
  const int* pos;           // position of the token (device)
  float* out;               // [n_heads][head_dim]
  float* part;              // [Hkv][max_split][group][head_dim + 2]
  unsigned* ticket;         // [Hkv], zero between launches
  int max_split;
  int* err;
  Trace trace;
  uint32_t trace_base;
  uint32_t tag;
};
// Fused attention + o_proj for short contexts (positions < kAttnOMaxCtx):
// CTA (kv group g, output slice s) computes the group's attention and its
// share of o_proj, writing part[g][rows of s]; the next kernel sums the
// per-group partials in order.
constexpr int kAttnOMaxCtx = 64;
struct AttnOArgs {
  const float* qkv;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  float eps;
  const float* rope;
  void* k_cache;
  void* v_cache;
  int kv_f32;
  int max_len, n_heads, n_kv_heads;
  const int* pos;
  const uint16_t* wo_packed;  // [Hkv][nslices][rows_per_slice][group * head_dim]
  int hidden, rows_per_slice, nslices;
  float* part;                // [Hkv][hidden]
  int* err;
  Trace trace;
  uint32_t trace_base;
  uint32_t tag;
};
size_t attn_o_smem_bytes(int rows_per_slice, int group, bool kv_f32);
void launch_attn_o(cudaStream_t s, const AttnOArgs& a, bool pdl);
// Output slices per kv group for the fused attention + o_proj: the largest
// slice of at most 48 KB of packed o_proj weights that divides `hidden`.
int attn_o_slices(int hidden, int group);
// Packs o_proj [hidden][n_heads * head_dim] into [Hkv][nslices][rows][group * head_dim].
void launch_pack_wo(cudaStream_t s, uint16_t* dst, const uint16_t* wo, int hidden, int n_kv_heads, int group,
                    int nslices);

// Context positions per attention CTA; a state's max_len / kAttnChunk
// (rounded up) splits cover every position.
constexpr int kAttnChunk = 64;
size_t attn_smem_bytes(bool kv_f32);
void launch_attn_decode(cudaStream_t s, const AttnArgs& a, bool pdl);

// io[0] = token, io[1] = pos, io[2] = 0 (the step's input and counters).
void launch_set_io(cudaStream_t s, int* io, int token, int pos);

// out = table[*token] as f32; a token outside [0, vocab) records TB200_ERR_ARG.
void launch_embed_token(cudaStream_t s, float* out, const uint16_t* table, int dim, const int* token, int vocab,
                        int* err, bool pdl);

// Packs gate [F][H] and up [F][H] into rows interleaved g0,u0,g1,u1,...
void launch_interleave_rows(cudaStream_t s, uint16_t* dst, const uint16_t* a, const uint16_t* b, size_t rows,
                            size_t cols);
// bf16 [rows][cols] -> f32, for reading the cache in tests.
void launch_bf16_to_f32(cudaStream_t s, float* dst, const uint16_t* src, size_t n);

// ---- tensor-core contraction for many tokens (gemm.cu) ---------------------

enum GemmEpilogue {
  kGemmStore = 0,  // out[t][r] = acc
  kGemmResid,      // out[t][r] += acc                    (residual stream)
  kGemmSilu,       // rows interleaved (gate, up): planes [t][r/2] = split3(silu(g) * u)
  kGemmResidNorm,  // out[t][r] += acc, then the next RMSNorm's input: planes of
                   // out[t][r] * next_w[r] and per-tile sums of squares out_ssq[t][tile]
  kGemmQkv,        // q|k|v rows, 128-row tile = one head: QK-norm, RoPE at the
                   // token's position; q to out[t][r], k and v into the cache
};
struct GemmArgs {
  int M, K, T;              // weight rows, columns (reduction), tokens
  int kb_per_split, splits, stages, mtiles, ntiles;  // set by launch_gemm from the plan
  float* out;               // kGemmStore / kGemmResid: [T][ldo]
  int ldo;
  uint16_t* out_split;      // kGemmSilu: three bf16 planes [T][ldh], `plane` elements apart
  size_t plane;
  int ldh;
  unsigned long long* best;  // kGemmStore: per token, the argmax key (argmax_key) of its
                             // outputs is folded in with atomicMax; null: none
  // The input's RMSNorm scale, folded into every epilogue: acc *= 1 /
  // sqrt(sum_p in_ssq[act_row0 + t][p] / in_dim + eps); null: none.
  const float* in_ssq;
  int in_parts, in_dim;
  float eps;
  int act_row0;             // first activation row (token) the contraction reads
  // kGemmResidNorm: the next RMSNorm's weight, its input planes (`next_plane`
  // apart, rows of ldo) and the sums of squares [T][mtiles].
  const uint16_t* next_w;
  uint16_t* next_split;
  size_t next_plane;
  float* out_ssq;
  // kGemmQkv: QK-norm weights, RoPE table, cache, token rows.
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  const float* rope;
  void* kv;                 // this layer's cache block of sequence 0
  size_t seq_stride;
  int kv_f32, max_len, n_heads, n_kv_heads, n_seqs;
  const int* tok_pos;
  const int* tok_seq;
  int* err;
  TraceAt trace;  // CTA index blockIdx.x + gridDim.x (blockIdx.y + gridDim.y blockIdx.z)
};
struct GemmPlan {
  int mtiles, ntiles;  // 128-row weight tiles, 64-token tiles
  int splits;          // K ranges per tile = cluster size (1: persistent CTAs over all tiles)
  int kb_per_split;    // 64-column K blocks per range
  int stages;          // shared-memory ring depth
  dim3 grid;           // split-K: (row tiles, token tiles, splits); persistent: (CTAs)
};
// Tensor map of a row-major bf16 matrix [rows][cols] in boxes of 64 columns
// by box_rows rows, 128-byte swizzle: the operand layout of the kernel.
int encode_tmap_bf16(CUtensorMap* map, const void* base, size_t rows, size_t cols, int box_rows,
                     std::string* why);
// Box rows (tokens per tile) of the activation maps.
int gemm_box_rows();
// max_cluster: the largest cluster the GPU schedules for this kernel
// (gemm_max_cluster).
GemmPlan plan_gemm(int M, int K, int T, int sms, int max_cluster);
cudaError_t init_gemm_kernels();
// Largest split-K cluster (<= 16) with every CTA at full shared memory that
// the device can run.
int gemm_max_cluster();
// tw: weight map (box rows 128); tx[0..2]: the activation's three planes
// (box rows gemm_box_rows()).
void launch_gemm(cudaStream_t s, const GemmPlan& p, int epilogue, const CUtensorMap& tw, const CUtensorMap* tx,
                 const GemmArgs& a, bool pdl);

// ---- many-token forward around the contractions (batch.cu) ------------------

cudaError_t init_batch_kernels();
// Query heads per kv head that the batched attention kernels handle.
bool batch_group_supported(int group);
// Cache positions per chunk of the decode attention (launch_attn_rows).
int attn_rows_chunk(bool kv_f32);

// x[0..n) -> three bf16 planes (store_split3), `plane` elements apart.
void launch_split_rows(cudaStream_t s, const float* x, uint16_t* out, size_t plane, size_t n, bool pdl);
// planes row r = split3(rmsnorm(x row row0 + r, w)), r < rows; plane =
// elements between planes. With `add` (may be null), x row += add row first.
void launch_norm_split(cudaStream_t s, float* x, const float* add, int row0, int rows, int dim, const uint16_t* w,
                       float eps, uint16_t* out, size_t plane, bool pdl, const TraceAt& tr = TraceAt{});

// x rows = embedding rows of tok[0..tokens), planes of x * w, ssq[t] = sum of
// squares of row t (the first RMSNorm's input in the fused layer sequence).
void launch_embed_split(cudaStream_t s, float* x, const uint16_t* table, int dim, const int* tok, int vocab,
                        const uint16_t* w, uint16_t* out, size_t plane, float* ssq, int* err, int tokens, bool pdl,
                        const TraceAt& tr = TraceAt{});


struct AttnRowsArgs {
  const float* q;           // [T][ldq], query heads (normed, rotated) from column 0
  int ldq;
  const void* kv;           // this layer's cache block of sequence 0
  size_t seq_stride;
  int kv_f32, max_len, n_kv_heads, n_seqs;
  const int* pos;
  const int* seq;
  uint16_t* out;            // [3 planes][T][ldo] attention output, split3
  size_t plane;
  int ldo;
  float* part;              // [T][Hkv][parts][group][head_dim + 2]
  unsigned* ticket;         // [T][Hkv], zero between launches
  int parts;                // CTAs per (token, kv group): attn_rows_parts
  int* err;
  // bf16 cache on the tensor cores (attn_rows_tensor_cores): a map of the
  // whole cache as rows of head_dim (box 64 x 64, 128-byte swizzle), and the
  // row of this layer's block of sequence 0.
  const CUtensorMap* cache_map;
  int layer_rows;
  TraceAt trace;  // CTA index blockIdx.x + gridDim.x (blockIdx.y + gridDim.y blockIdx.z)
};
// Whether launch_attn_rows runs the tensor-core kernel (bf16 cache, 1 or 2
// query heads per kv head; it needs AttnRowsArgs::cache_map).
bool attn_rows_tensor_cores(bool kv_f32, int group);
// Context parts per (token, kv group) for launch_attn_rows: one when the
// batch alone gives two CTAs per SM.
int attn_rows_parts(int tokens, int n_kv_heads, int max_len, bool kv_f32, int sms);
// Rows (positions) of the boxes the tensor-core decode attention loads from
// a bf16 cache: the cache_map of AttnRowsArgs uses this box height.
int attn_cache_box_rows();
void launch_attn_rows(cudaStream_t s, const AttnRowsArgs& a, int tokens, int group, bool pdl);

struct AttnPrefillArgs {
  const float* q;           // [T][ldq]
  int ldq;
  const void* kv;           // this layer's cache block of the sequence
  int kv_f32, max_len, n_kv_heads;
  int T, pos0;              // tokens at positions pos0 .. pos0 + T - 1, already in the cache
  uint16_t* out;            // [3 planes][T][ldo]
  size_t plane;
  int ldo;
};
void launch_attn_prefill(cudaStream_t s, const AttnPrefillArgs& a, int group, bool pdl);

// The greedy choice after a contraction that folded argmax keys into
// best[rows] (GemmArgs::best): writes each row's token id (to next, tok and
// the step's output row), advances positions and the step, zeroes best.
void launch_argmax_finish(cudaStream_t s, const struct ArgmaxRowsArgs& a, unsigned long long* best, int rows,
                          bool pdl);

struct ArgmaxRowsArgs {
  const float* logits;      // [rows][V]
  int V;
  int* next;                // [rows] greedy token, or null
  int* tok;                 // [rows] next step's input token, or null
  int* pos;                 // [rows] incremented, or null
  int* out;                 // [out_cap][rows] tokens by step, or null
  int* step;                // step counter (with out), or null
  unsigned* ticket;         // with step: zero between launches
  int out_cap;
  int* err;                 // launch_argmax_finish: set when a row got no key
  TraceAt trace;
};

}  // namespace tb
