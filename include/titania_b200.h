/*
 * titania_b200.h — C ABI of the B200 (sm_100a) backend for Titania's model.
 *
 * Two layers of entry points:
 *
 *  1. The `Device` trait, one function per method (reference:
 *     model/device.rs:9-89). A Rust `model/b200.rs` implementing `Device`
 *     binds these one to one, exactly as model/titania.rs:99-220 binds a
 *     Titania GPU. Buffers hold f32 activations, weights hold bf16 bits.
 *     Operations are enqueued in order on the device's stream; `tb200_read`
 *     waits for them, so results are observed exactly as the synchronous
 *     reference devices give them.
 *
 *  2. A fused model path with no trait counterpart: the Qwen3 forward pass of
 *     model/model.rs:83-149 run as a handful of fused kernels per layer,
 *     replayed from a CUDA graph, with a bf16 key/value cache and an
 *     on-device greedy sampler. A caller builds it from weights it already
 *     uploaded through (1), naming them as model/model.rs:48-72 does.
 *
 * Errors: the reference panics on a violated assertion (model/cpu.rs:22,40,
 * 52-53; model/titania.rs:125,140,147,156-157,186-188,204-205). Every
 * function here instead returns a nonzero TB200_ERR_* code and keeps a
 * message for tb200_last_error(); a Rust wrapper panics on it.
 *
 * Threading: as in the reference (the trait needs neither Send nor Sync),
 * one thread drives a device at a time.
 */
#ifndef TITANIA_B200_H
#define TITANIA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TB200_API __attribute__((visibility("default")))
#else
#define TB200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  TB200_OK = 0,
  TB200_ERR_ARG = 1,     /* an argument violates the op's contract (a reference panic) */
  TB200_ERR_CUDA = 2,    /* a CUDA runtime error */
  TB200_ERR_TIMEOUT = 3, /* a bounded wait inside a kernel gave up: the state's cache and step
                          * position may be partly advanced (a decode step stops where its
                          * wait gave up); forward the sequence again from a known position
                          * (its prompt) before decoding it further */
  TB200_ERR_IO = 4,      /* a file could not be opened or read (Weights' io::Error) */
  TB200_ERR_FORMAT = 5,  /* a file is not a valid safetensors checkpoint of bf16 tensors */
};

typedef struct tb200_device tb200_device; /* a Device on one GPU */
typedef struct tb200_buffer tb200_buffer; /* Device::Buffer, f32 (model/device.rs:13) */
typedef struct tb200_weight tb200_weight; /* Device::Weight, bf16 (model/device.rs:15) */
typedef struct tb200_model tb200_model;   /* fused-path model (no trait counterpart) */
typedef struct tb200_state tb200_state;   /* fused-path State (model/model.rs:156-172) */
typedef struct tb200_tp tb200_tp;         /* a tensor-parallel group (one rank per process and GPU) */
typedef struct tb200_sampler tb200_sampler; /* top-k / top-p / temperature sampling state on the device */

/* Message for the last nonzero return on this thread. */
TB200_API const char* tb200_last_error(void);

/* Opens the device with CUDA ordinal `ordinal`; replaces `Titania::new`
 * (model/titania.rs:58-68) / the `Cpu` unit value (model/cpu.rs:9). */
TB200_API int tb200_device_open(int ordinal, tb200_device** out);
TB200_API int tb200_device_close(tb200_device* dev);
/* Waits for every enqueued operation; reports a kernel-side timeout. */
TB200_API int tb200_sync(tb200_device* dev);
/* The cudaStream_t all operations run on (for callers that time them). */
TB200_API void* tb200_device_stream(tb200_device* dev);
/* Number of SMs; kernels size their grids to it. */
TB200_API int tb200_device_sms(tb200_device* dev);

/* The RoPE table State::new uploads (model/model.rs:239-250): for each
 * position < max_len and pair i < head_dim/2, (cos, sin) of
 * pos / theta^(2i/head_dim), in f32 with the platform libm as the reference
 * computes it. `out` holds max_len * head_dim floats. */
TB200_API int tb200_rope_table(size_t max_len, size_t head_dim, float theta, float* out);

/* ---- Device trait (model/device.rs) ------------------------------------ */

/* device.rs:18 `upload(&self, tensor: Tensor) -> Weight`; `data` holds the
 * product of `shape` bf16 values, row-major (model/weights.rs:14-17). */
TB200_API int tb200_upload(tb200_device* dev, const uint16_t* data, const size_t* shape, size_t ndim, tb200_weight** out);
/* Weights::open + Weights::read + Device::upload for many tensors at once
 * (model/weights.rs:35-81, model/device.rs:18; the reads Model::load makes,
 * model/model.rs:42,251-254), with no host-side conversion: the safetensors
 * file at `path` is parsed once and the `n` tensors `names` go from the file
 * to device memory through pinned staging buffers on `threads` host threads
 * (0: up to 8), reading overlapped with copying. The staging buffers (two of
 * 8 MB per thread) are page-locked on first use and kept by the device until
 * tb200_device_close, so later loads skip that cost. out[i] is NULL where the file
 * has no tensor names[i] (Weights::contains is false; the caller decides
 * whether it was required). A tensor that is not BF16 fails as Weights::read
 * does ("tensor 'x' is F32, expected BF16", TB200_ERR_FORMAT); so does one
 * whose byte range lies outside the file or does not hold two bytes per
 * element of its shape. An unreadable file is TB200_ERR_IO. On any error no
 * weight stays allocated and every out[i] is NULL. Returns once every byte
 * is on the device. */
TB200_API int tb200_upload_safetensors(tb200_device* dev, const char* path, const char* const* names, size_t n,
                                       int threads, tb200_weight** out);
/* The header entry of tensor `name` in the safetensors file at `path`
 * (model/weights.rs:35-57), parsed as tb200_upload_safetensors parses it:
 * *found = 0 when there is none; otherwise its dtype (NUL-terminated, at
 * most dtype_cap bytes), its shape (*ndim <= max_ndim values in `shape`)
 * and its bytes in the file (*offset from the file's start, *bytes long).
 * Host only. */
/* A window of a 2-D checkpoint tensor: rows [row0, row0 + rows) and columns
 * [col0, col0 + cols); rows = cols = 0 takes the tensor whole (any rank). */
typedef struct tb200_window {
  size_t row0, rows, col0, cols;
} tb200_window;
/* tb200_upload_safetensors for one window of each tensor (no counterpart in
 * the reference: a tensor-parallel rank's share of a checkpoint, e.g. the
 * q/k/v/gate/up rows and o/down columns it holds). out[i] has shape
 * [rows, cols], packed, or the tensor's own shape for a whole window. A
 * window of whole rows is read as one run; a column window reads whole rows
 * and copies their middle out (rows up to 4M elements). A window outside
 * its tensor, or one on a tensor that is not a matrix, is TB200_ERR_ARG. */
TB200_API int tb200_upload_safetensors_windows(tb200_device* dev, const char* path, const char* const* names,
                                               const tb200_window* windows, size_t n, int threads,
                                               tb200_weight** out);
/* The shape of a weight as uploaded: *ndim <= max_ndim values in `shape`.
 * Host only. */
TB200_API int tb200_weight_shape(const tb200_weight* w, size_t* shape, size_t max_ndim, size_t* ndim);
TB200_API int tb200_safetensors_entry(const char* path, const char* name, int* found, char* dtype, size_t dtype_cap,
                                      size_t* shape, size_t max_ndim, size_t* ndim, uint64_t* offset, uint64_t* bytes);
/* device.rs:21 `alloc(&self, len) -> Buffer`: a zeroed buffer. */
TB200_API int tb200_alloc(tb200_device* dev, size_t len, tb200_buffer** out);
/* device.rs:26 `resize(&self, &mut Buffer, len)`: len <= allocated length. */
TB200_API int tb200_resize(tb200_device* dev, tb200_buffer* buf, size_t len);
/* The buffer's current length (Vec::len of `read`'s result). */
TB200_API size_t tb200_buffer_len(const tb200_buffer* buf);
/* device.rs:29 `read(&self, &Buffer) -> Vec<f32>`; `len` must equal the
 * buffer's length. Waits for the device. */
TB200_API int tb200_read(tb200_device* dev, const tb200_buffer* buf, float* out, size_t len);
/* device.rs:32 `write(&self, &mut Buffer, &[f32])`; `len` must equal the
 * buffer's length. */
TB200_API int tb200_write(tb200_device* dev, tb200_buffer* buf, const float* data, size_t len);
/* device.rs:35-42 `copy`: dst[dst_offset..][..len] = src[src_offset..][..len]. */
TB200_API int tb200_copy(tb200_device* dev, tb200_buffer* dst, size_t dst_offset, const tb200_buffer* src, size_t src_offset,
               size_t len);
/* device.rs:46 `embed(&self, out, table, tokens)`. */
TB200_API int tb200_embed(tb200_device* dev, tb200_buffer* out, const tb200_weight* table, const uint32_t* tokens, size_t n);
/* device.rs:51 `matmul(&self, out, w, x)`: out[t] = w · x[t]. */
TB200_API int tb200_matmul(tb200_device* dev, tb200_buffer* out, const tb200_weight* w, const tb200_buffer* x);
/* device.rs:54 `add(&self, x, y)`: x += y. */
TB200_API int tb200_add(tb200_device* dev, tb200_buffer* x, const tb200_buffer* y);
/* device.rs:58 `rmsnorm(&self, x, weight, eps)`: rows of weight's length. */
TB200_API int tb200_rmsnorm(tb200_device* dev, tb200_buffer* x, const tb200_weight* weight, float eps);
/* device.rs:66 `rope(&self, x, table, pos, n_heads, head_dim)`. */
TB200_API int tb200_rope(tb200_device* dev, tb200_buffer* x, const tb200_buffer* table, size_t pos, size_t n_heads,
               size_t head_dim);
/* device.rs:75-85 `attention(&self, out, q, k_cache, v_cache, pos, n_heads,
 * head_dim, n_kv_heads)`; caches laid out [position][kv head][head_dim]. */
TB200_API int tb200_attention(tb200_device* dev, tb200_buffer* out, const tb200_buffer* q, const tb200_buffer* k_cache,
                    const tb200_buffer* v_cache, size_t pos, size_t n_heads, size_t head_dim, size_t n_kv_heads);
/* Device::attention (device.rs:75-85, model/cpu.rs:113-149) for one query
 * token in each of `batch` sequences, over a bf16 key/value cache in the
 * layout the model path keeps (no trait counterpart: the trait's caches are
 * f32, [position][kv head][head_dim]): `cache` has shape
 * [batch, 2 (K, V), n_kv_heads, max_len, 128]; q[b] (n_heads x 128 f32,
 * after QK-norm and RoPE) at positions[b] attends to cached positions
 * 0..positions[b] of sequence b; out[b] receives n_heads x 128 f32. q and out
 * hold batch * n_heads * 128 values; 1, 2, 4 or 8 query heads per kv head.
 * Runs the batched decode step's tensor-core attention kernel. */
TB200_API int tb200_attention_cache(tb200_device* dev, tb200_buffer* out, const tb200_buffer* q,
                                    const tb200_weight* cache, const size_t* positions, size_t batch, size_t n_heads);
/* device.rs:88 `silu_mul(&self, gate, up)`. */
TB200_API int tb200_silu_mul(tb200_device* dev, tb200_buffer* gate, const tb200_buffer* up);

/* The trait has no free (handles live as long as the process, as with
 * Titania, model/titania.rs:43-55); these let a caller give memory back. */
TB200_API int tb200_free_buffer(tb200_device* dev, tb200_buffer* buf);
TB200_API int tb200_free_weight(tb200_device* dev, tb200_weight* w);

/* Greedy sampling (model/sampler.rs:21-33 at temperature 0) on the device:
 * the index of the largest element under IEEE total order, ties to the
 * lowest index. */
TB200_API int tb200_argmax(tb200_device* dev, const tb200_buffer* logits, uint32_t* out);

/* Greedy argmax like tb200_argmax, for callers that cannot allocate device
 * memory: no counterpart in the reference. A caller whose GPU memory belongs
 * to another allocator (say, a framework's caching allocator holding the
 * device's memory), or that keeps cudaMalloc/cudaFree out of its per-token
 * loop because they can synchronize the device, passes logits and an output
 * word it already owns: `logits` is `n` f32 values in device memory, `out` a
 * device uint32 that receives the index of the largest value (IEEE total
 * order, ties to the lowest index). Runs on `stream` (a cudaStream_t; NULL
 * is the default stream) and returns without waiting. It takes no device
 * handle and allocates nothing: its scratch is a static array in the
 * library (about 16 KB per GPU, held until the process exits), which limits
 * `n` to 8,388,608; larger inputs return TB200_ERR_ARG. The first call on a
 * GPU looks the array up on that GPU (set-up, once per device); make that
 * first call before any stream capture. The looked-up address is kept for
 * the life of the process: after a cudaDeviceReset of a GPU (a new primary
 * context), do not call this entry point on that GPU again. Calls share the
 * array, so calls whose work overlaps on the GPU (other streams, other
 * threads) race and must be ordered by the caller. */
TB200_API int tb200_argmax_noalloc(const float* logits, size_t n, uint32_t* out, void* stream);

/* ---- Fused model path --------------------------------------------------- */

/* The config.json fields the model reads (model/config.rs:10-35); head_dim
 * resolved by the caller as Config::head_dim does. */
typedef struct tb200_config {
  size_t hidden_size;
  size_t intermediate_size;
  size_t num_hidden_layers;
  size_t num_attention_heads;
  size_t num_key_value_heads;
  size_t head_dim;
  float rms_norm_eps;
  float rope_theta;
  size_t vocab_size;
  int tie_word_embeddings;
} tb200_config;

/* Starts a fused model for `config` on `dev` (Model::load,
 * model/model.rs:40-77, after its uploads). */
TB200_API int tb200_model_create(tb200_device* dev, const tb200_config* config, tb200_model** out);
/* Names an uploaded weight with its checkpoint tensor name
 * (model/model.rs:48-72, e.g. "model.layers.3.self_attn.q_proj.weight"). */
TB200_API int tb200_model_bind(tb200_model* model, const char* name, const tb200_weight* w);
/* Checks that every tensor is bound with the right shape and packs the fused
 * layouts (q|k|v rows, gate/up rows interleaved). */
TB200_API int tb200_model_finalize(tb200_model* model);
TB200_API int tb200_model_free(tb200_model* model);

/* Element type of the fused path's key/value cache. The reference caches
 * f32 (model/model.rs:206-207); bf16 halves the bytes attention reads. */
enum { TB200_KV_BF16 = 0, TB200_KV_F32 = 1 };

/* State::new (model/model.rs:176-211) for the fused path: a key/value cache
 * of `kv_dtype` (TB200_KV_*) for `max_len` positions and the RoPE table
 * (model/model.rs:239-250). A state keeps its model alive: tb200_model_free
 * on a model with states defers the free to the last tb200_state_free. */
TB200_API int tb200_state_new(tb200_model* model, size_t max_len, int kv_dtype, tb200_state** out);
TB200_API int tb200_state_free(tb200_state* state);

/* Model::forward (model/model.rs:83-91): runs `tokens`, the first at `pos`,
 * adding their keys and values to the cache, and writes the logits for the
 * token after the last one to `logits` (vocab_size floats, host memory; may
 * be NULL) and the greedy choice to `next_token` (may be NULL). */
TB200_API int tb200_forward(tb200_model* model, tb200_state* state, const uint32_t* tokens, size_t n, size_t pos,
                  float* logits, uint32_t* next_token);

/* ---- tensor parallelism (no counterpart in the reference) ------------------- */

/* A model split over `world` GPUs of one node, one process per GPU
 * (Megatron-style): rank r holds q/k/v rows of its num_key_value_heads/world
 * kv heads and their query heads, the matching o_proj columns, gate/up rows
 * r*F/world .. (r+1)*F/world and the matching down_proj columns; norms,
 * embedding and lm_head are replicated. o_proj and down_proj then produce
 * partial sums, which are added over the group (NCCL all-reduce over NVLink)
 * before they join the residual stream; every rank computes the same logits.
 *
 * Rank 0 makes a group id (tb200_tp_unique_id, 128 bytes) and the caller
 * hands it to every rank (for instance with torch.distributed); every rank
 * then calls tb200_tp_init at the same time. A rank's model is created with
 * its local head and FFN counts (the config divided by world), its local
 * tensors are bound, and tb200_model_set_tp attaches the group before
 * tb200_model_finalize. All ranks must then make the same calls in the same
 * order (each forward step runs the group's collectives). NCCL is loaded at
 * run time (libnccl.so.2). */
TB200_API int tb200_tp_unique_id(uint8_t* out, size_t len);
TB200_API int tb200_tp_init(tb200_device* dev, int rank, int world, const uint8_t* id, size_t len, tb200_tp** out);
TB200_API int tb200_tp_free(tb200_tp* tp);
TB200_API int tb200_tp_rank(const tb200_tp* tp);
TB200_API int tb200_tp_world(const tb200_tp* tp);
/* Sums a buffer over the group in place (all ranks call it); waits. */
TB200_API int tb200_tp_allreduce(tb200_tp* tp, tb200_buffer* buf);
/* Attaches the group to a model before tb200_model_finalize. */
TB200_API int tb200_model_set_tp(tb200_model* model, tb200_tp* tp);
/* 1 when a finalized tensor-parallel model adds the single-token step's
 * o_proj and down_proj partial sums by peer stores instead of NCCL: each
 * rank's kernel stores its rows into every rank's receive buffer (CUDA IPC
 * over NVLink, plain stores) and raises a per-step flag there; the next
 * kernel waits (bounded: TB200_ERR_TIMEOUT after a second) for every rank's
 * flag and sums the slots in rank order, so every rank computes the same
 * values. tb200_model_finalize sets it up when every rank has its own GPU
 * and can map the others' memory (all ranks agree, else all keep NCCL;
 * TB200_TP_ALLREDUCE=nccl in the environment keeps NCCL). Prompts and the
 * batched path keep NCCL. 0 otherwise. */
TB200_API int tb200_model_tp_peer_exchange(const tb200_model* model);

/* ---- many sequences ------------------------------------------------------- */

/* A state of `n_seqs` independent sequences, each with its own key/value
 * cache of `max_len` positions: what `n_seqs` separate State::new
 * (model/model.rs:176-211) would hold, in one allocation, so that one decode
 * step runs every sequence at once. A one-sequence state from tb200_state_new
 * is the case n_seqs = 1. The single-token entry points (tb200_generate,
 * tb200_decode_enqueue, tb200_enqueue_op, tracing) take one-sequence states. */
TB200_API int tb200_batch_state_new(tb200_model* model, size_t n_seqs, size_t max_len, int kv_dtype,
                                    tb200_state** out);
TB200_API size_t tb200_state_seqs(const tb200_state* state);

/* Model::forward (model/model.rs:83-91) for sequence `seq` of the state: as
 * tb200_forward. Prompts (n >= 2, here and in tb200_forward) run all their
 * tokens at once through the tensor-core path. */
TB200_API int tb200_forward_seq(tb200_model* model, tb200_state* state, size_t seq, const uint32_t* tokens,
                                size_t n, size_t pos, float* logits, uint32_t* next_token);

/* One decode step of every sequence: token tokens[i] of sequence i at
 * positions[i] (n_seqs each). Writes the logits of every sequence to
 * `logits` ([n_seqs][vocab_size] floats, host; may be NULL) and the greedy
 * choices to `next_tokens` (n_seqs, host; may be NULL). */
TB200_API int tb200_forward_batch(tb200_model* model, tb200_state* state, const uint32_t* tokens,
                                  const size_t* positions, float* logits, uint32_t* next_tokens);

/* Greedy decoding of every sequence on the device: feeds tokens[i] at
 * positions[i], then each chosen token, `steps` times; writes the chosen
 * tokens to `out` ([steps][n_seqs], host). */
TB200_API int tb200_generate_batch(tb200_model* model, tb200_state* state, const uint32_t* tokens,
                                   const size_t* positions, size_t steps, uint32_t* out);

/* What tb200_generate_batch runs, without its copy back or final wait. */
TB200_API int tb200_decode_batch_enqueue(tb200_model* model, tb200_state* state, const uint32_t* tokens,
                                         const size_t* positions, size_t steps);

/* Key (which = 0) or value (1) cache row of sequence `seq` at (layer, pos),
 * kv_heads * head_dim values as f32. */
TB200_API int tb200_batch_read_kv(tb200_state* state, size_t seq, size_t layer, int which, size_t pos, float* out);

/* ---- single sequence, single token --------------------------------------- */

/* Greedy decoding entirely on the device (model/chat.rs:149-196 with
 * temperature 0): feeds `token` at `pos`, then each chosen token, `steps`
 * times; writes the `steps` chosen tokens to `out` (host memory). */
TB200_API int tb200_generate(tb200_model* model, tb200_state* state, uint32_t token, size_t pos, size_t steps,
                   uint32_t* out);
/* What a one-sequence state's single-token steps run (tb200_forward with one
 * token, tb200_generate, tb200_decode_enqueue; no counterpart in the
 * reference, whose Model::forward is one path, model/model.rs:83-149):
 *  - TB200_DECODE_FUSED: 2 + 5 * layers fused kernels per step, replayed from
 *    a CUDA graph (every model this library runs, tensor-parallel included);
 *  - TB200_DECODE_PERSISTENT: one persistent kernel (one CTA per SM) runs all
 *    of a step's phases, the phases exchanging tagged vectors instead of
 *    ending kernels, and tb200_generate / tb200_decode_enqueue run all their
 *    steps in one launch. Needs an unsharded model (or a tensor-parallel
 *    group of one) with head_dim 128, hidden / FFN / query widths up to
 *    10240, at most 4 query heads per kv head, at most 8 kv heads and 64
 *    layers (Qwen3-0.6B and Qwen3-4B fit).
 * tb200_state_new picks PERSISTENT where the model allows it, else FUSED.
 * Both give the same tokens and logits within the tolerance of their
 * different summation orders. */
enum { TB200_DECODE_FUSED = 0, TB200_DECODE_PERSISTENT = 1 };
/* Selects the single-token path of a one-sequence state; TB200_ERR_ARG (with
 * the reason) when the state's model cannot run it. */
TB200_API int tb200_state_set_decode(tb200_state* state, int mode);
/* The state's single-token path (TB200_DECODE_*), -1 for a null state. */
TB200_API int tb200_state_decode(const tb200_state* state);

/* tb200_generate through the persistent kernel whatever the state's decode
 * mode (see TB200_DECODE_PERSISTENT; TB200_ERR_ARG with the reason where the
 * model cannot run it): `steps` greedy tokens from `token` at `pos` into
 * tokens_out (host). With logits_out ([steps][vocab] floats, host; may be
 * NULL) every step is its own launch and its logits are copied back, for
 * checking. */
TB200_API int tb200_decode_persistent(tb200_model* model, tb200_state* state, uint32_t token, size_t pos,
                                      size_t steps, uint32_t* tokens_out, float* logits_out);

/* Enqueues greedy decode steps on the device's stream without waiting or
 * copying anything back: feeds `token` at `pos`, then each chosen token,
 * `steps` times (what tb200_generate runs, minus its copies and wait). For
 * callers that time the device or overlap it with host work. */
TB200_API int tb200_decode_enqueue(tb200_model* model, tb200_state* state, uint32_t token, size_t pos, size_t steps);

/* The fused kernels of one decode step, for tb200_enqueue_op. A step runs
 * EMBED, then per layer QKV, ATTENTION_O, GATE_UP_SUM, DOWN while the
 * position is below 64, or QKV, ATTENTION, O, GATE_UP, DOWN beyond it, then
 * LM_HEAD. GATE_UP(_SUM) also stores its input residual (x, or x plus the
 * partials) to the X2 buffer, which DOWN adds back. */
enum {
  TB200_OP_EMBED = 0,     /* x = embed[token]                               */
  TB200_OP_QKV = 1,       /* q|k|v = W_qkv . rmsnorm(x)                     */
  TB200_OP_ATTENTION = 2, /* QK-norm, RoPE, K/V append, attention           */
  TB200_OP_O = 3,         /* x += W_o . att                                 */
  TB200_OP_GATE_UP = 4,   /* h = silu(W_g . rmsnorm(x)) * (W_u . rmsnorm(x)) */
  TB200_OP_DOWN = 5,      /* x += W_d . h                                   */
  TB200_OP_LM_HEAD = 6,   /* logits = W_lm . rmsnorm(x); greedy token; pos++ */
  TB200_OP_ATTENTION_O = 7, /* short contexts: attention and o_proj per kv group -> partials */
  TB200_OP_GATE_UP_SUM = 8, /* like GATE_UP on x + the summed o_proj partials */
};

/* Enqueues one fused kernel of the decode step (of layer `layer` for ops
 * 1-5) on the device's stream, exactly as the step's graph runs it, without
 * waiting: for timing and testing kernels one at a time. */
TB200_API int tb200_enqueue_op(tb200_model* model, tb200_state* state, int op, size_t layer);

/* ---- sampling (model/sampler.rs) ------------------------------------------- */

/* Sampler::new (model/sampler.rs:12-19) for `rows` rows of `vocab` logits:
 * temperature, top_k (clamped to [1, vocab] as sampler.rs:29; at most 64 here)
 * and top_p as the reference's; row i's xorshift64* state starts at
 * max(seeds[i], 1) and lives in device memory. */
TB200_API int tb200_sampler_new(tb200_device* dev, size_t rows, size_t vocab, float temperature, size_t top_k,
                                float top_p, const uint64_t* seeds, tb200_sampler** out);
TB200_API int tb200_sampler_free(tb200_sampler* sampler);
/* Sampler::sample (model/sampler.rs:21-59) for every row of `logits`
 * ([rows][vocab] f32, the buffer at least that long): one token per row into
 * tokens[rows]; waits. Exact logit ties go to the lowest token id. */
TB200_API int tb200_sample(tb200_sampler* sampler, const tb200_buffer* logits, uint32_t* tokens);
/* The same without the copy back or the wait (tokens stay on the device). */
TB200_API int tb200_sample_enqueue(tb200_sampler* sampler, const tb200_buffer* logits);
/* The generator states, rows x u64 (sampler.rs:63-77's Rng). */
TB200_API int tb200_sampler_state(tb200_sampler* sampler, uint64_t* out);

/* ---- tracing ------------------------------------------------------------ */

/* Events a traced kernel records, one per CTA. */
enum {
  TB200_TRACE_START = 0,   /* the CTA began (it may still wait on the previous kernel) */
  TB200_TRACE_WAITED = 1,  /* the previous kernel's results became visible */
  TB200_TRACE_INPUT = 2,   /* the input vector is staged (and normalized) */
  TB200_TRACE_WEIGHTS = 3, /* the CTA's first weight chunk is in shared memory */
  TB200_TRACE_DONE = 4,         /* the CTA finished its rows */
  TB200_TRACE_ISSUED = 5,       /* the CTA's last weight copy was issued */
  TB200_TRACE_LAST_WEIGHTS = 6, /* the CTA's last weight chunk is in shared memory */
  TB200_TRACE_REDUCE = 7,       /* a split-K CTA's cluster holds every partial tile (reduction starts) */
};

/* Kernels of a state's batched decode step (tb200_forward_batch and friends),
 * as the op half of their trace tags. */
enum {
  TB200_TRACE_OP_EMBED = 16,    /* embedding + the first RMSNorm's input */
  TB200_TRACE_OP_NORM = 17,     /* rmsnorm + split before q|k|v (tensor parallel) */
  TB200_TRACE_OP_QKV = 18,      /* q|k|v contraction */
  TB200_TRACE_OP_QKV_POST = 19, /* (no longer launched: QK-norm, RoPE and the cache append run in the q|k|v epilogue) */
  TB200_TRACE_OP_ATTENTION = 20,
  TB200_TRACE_OP_O = 21,        /* o_proj contraction (+ residual) */
  TB200_TRACE_OP_NORM2 = 22,    /* rmsnorm + split before gate|up (tensor parallel) */
  TB200_TRACE_OP_GATE_UP = 23,  /* gate|up contraction (+ silu) */
  TB200_TRACE_OP_DOWN = 24,     /* down contraction (+ residual) */
  TB200_TRACE_OP_FINAL_NORM = 25, /* (tensor parallel) */
  TB200_TRACE_OP_LM_HEAD = 26,  /* lm_head contraction (+ argmax keys) */
  TB200_TRACE_OP_ARGMAX = 27,
};

/* Phases of the persistent single-token step (TB200_DECODE_PERSISTENT), as
 * the op half of their trace tags. A traced CTA records INPUT when its input
 * vector is complete and DONE when it has written its rows. */
enum {
  TB200_TRACE_OP_P_QKV = 32,   /* q|k|v = W_qkv . rmsnorm(x)                         */
  TB200_TRACE_OP_P_ATTO = 33,  /* QK-norm, RoPE, append, attention, o_proj partial   */
  TB200_TRACE_OP_P_GU = 34,    /* x' = x + partials; h = silu(gate) * up             */
  TB200_TRACE_OP_P_DOWN = 35,  /* x = x' + W_d . h                                   */
  TB200_TRACE_OP_P_LM = 36,    /* lm_head rows and their greedy choice              */
  TB200_TRACE_OP_P_START = 37, /* the CTA began (START)                              */
  TB200_TRACE_OP_P_TOKEN = 38, /* the last CTA published the step's token (DONE)     */
};

/* One trace record: tag = op << 16 | layer (TB200_OP_* for the single-token
 * step, TB200_TRACE_OP_* for the batched one), the CTA index, the event, the
 * SM, and the GPU's global timer in nanoseconds. */
typedef struct tb200_trace_record {
  uint32_t tag, cta, event, sm;
  uint64_t ns;
} tb200_trace_record;

/* Starts recording the state's decode step (the single-token step of a
 * one-sequence state, and the batched step of any state): every kernel of the
 * step's graph owns fixed record slots (8 per CTA), so a replay overwrites
 * the previous one and the buffer holds the last step. `capacity` records
 * are allocated; the graphs are rebuilt to carry the buffer. */
TB200_API int tb200_trace_start(tb200_state* state, size_t capacity);
/* Stops recording, copies up to `cap` record slots to `out` (slots with
 * ns == 0 were not written) and the number of slots one step uses to `*n`. */
TB200_API int tb200_trace_stop(tb200_state* state, tb200_trace_record* out, size_t cap, size_t* n);

/* The fused path's activation buffers, for tb200_state_read/write. */
enum {
  TB200_BUF_X = 0,      /* residual stream, hidden_size */
  TB200_BUF_QKV = 1,    /* raw q|k|v projections, (heads + 2 kv_heads) * head_dim */
  TB200_BUF_ATT = 2,    /* attention output, heads * head_dim */
  TB200_BUF_H = 3,      /* silu(gate) * up, intermediate_size */
  TB200_BUF_LOGITS = 4, /* vocab_size (a persistent step that wrote its logits
                         * straight to page-locked host memory leaves it as it was) */
  TB200_BUF_X2 = 5,     /* residual stream after attention, hidden_size */
  TB200_BUF_PART = 6,   /* o_proj partials, kv_heads * hidden_size */
};

/* Copies a state buffer to the host (`n` must be its length); waits for the
 * device. For testing the fused kernels one at a time. */
TB200_API int tb200_state_read(tb200_state* state, int which, float* out, size_t n);
/* Overwrites a state buffer from the host (`n` must be its length). */
TB200_API int tb200_state_write(tb200_state* state, int which, const float* data, size_t n);
/* Sets the token and position the next step (or tb200_enqueue_op) reads. */
TB200_API int tb200_state_set_position(tb200_state* state, uint32_t token, size_t pos);

/* Reads position `pos` of layer `layer`'s key (which=0) or value (which=1)
 * cache as f32, Hkv*head_dim values, for tests. Waits for the device. */
TB200_API int tb200_state_read_kv(tb200_state* state, size_t layer, int which, size_t pos, float* out);

#ifdef __cplusplus
}
#endif

#endif /* TITANIA_B200_H */
