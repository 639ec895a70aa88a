// runtime.cu — the C ABI of include/titania_b200.h: device handles, buffers
// and weights (the Device trait, model/device.rs), and the fused model path
// (model/model.rs) with its CUDA graph.
//
// Every entry point validates its arguments the way the reference asserts
// them (model/cpu.rs, model/titania.rs) and returns TB200_ERR_ARG with a
// message instead of panicking.

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "runtime.h"

namespace rt {

namespace {
thread_local std::string g_err;
}  // namespace

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TB200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return TB200_OK;
}

int use(tb200_device* d) {
  if (!d) return fail(TB200_ERR_ARG, "null device");
  CUDA_TRY(cudaSetDevice(d->ordinal));
  return TB200_OK;
}

// model.rs:239-250, on the host exactly as the reference computes it.
std::vector<float> rope_table(size_t max_len, size_t head_dim, float theta) {
  size_t half = head_dim / 2;
  std::vector<float> t;
  t.reserve(max_len * head_dim);
  for (size_t pos = 0; pos < max_len; pos++)
    for (size_t i = 0; i < half; i++) {
      float freq = 1.0f / powf(theta, float(2 * i) / float(head_dim));
      float a = float(pos) * freq;
      t.push_back(cosf(a));
      t.push_back(sinf(a));
    }
  return t;
}

const char* last_error() { return g_err.c_str(); }

}  // namespace rt

using rt::fail;
using rt::launched;
using rt::use;
using rt::rope_table;

namespace {

std::string shape_str(const std::vector<size_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); i++) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

}  // namespace

int tb::record_error(int code, const std::string& msg) { return fail(code, msg); }

namespace {

// Several tokens: the tensor-core contraction (gemm.cu). The input is split
// into three bf16 planes in device scratch; the weight's operand map is made
// once.
int matmul_tokens(tb200_device* d, tb200_buffer* out, const tb200_weight* w, const tb200_buffer* x, size_t rows,
                  size_t cols, size_t n) {
  cudaStream_t s = d->stream;
  std::string why;
  auto* wm = const_cast<tb200_weight*>(w);
  if (!wm->has_map) {
    if (int rc = tb::encode_tmap_bf16(&wm->map, w->ptr, rows, cols, 128, &why)) return fail(rc, "matmul: " + why);
    wm->has_map = true;
  }
  const size_t need = n * cols;
  if (need > d->split_cap) {
    CUDA_TRY(cudaStreamSynchronize(s));
    cudaFree(d->split);
    d->split = nullptr;
    d->split_cap = 0;
    CUDA_TRY(cudaMalloc(&d->split, 3 * need * sizeof(uint16_t)));
    d->split_cap = need;
  }
  const tb::GemmPlan p = tb::plan_gemm(int(rows), int(cols), int(n), d->sms, d->max_cluster);
  CUtensorMap tx[3];
  for (int i = 0; i < 3; i++)
    if (int rc = tb::encode_tmap_bf16(&tx[i], d->split + i * d->split_cap, n, cols, tb::gemm_box_rows(), &why))
      return fail(rc, "matmul: " + why);
  tb::launch_split_rows(s, x->ptr, d->split, d->split_cap, need, false);
  if (int rc = launched("matmul split")) return rc;
  tb::GemmArgs a{};
  a.M = int(rows);
  a.K = int(cols);
  a.T = int(n);
  a.out = out->ptr;
  a.ldo = int(rows);
  a.err = d->err;
  tb::launch_gemm(s, p, tb::kGemmStore, wm->map, tx, a, false);
  if (int rc = launched("matmul")) return rc;
  // A kernel-side error (a wait that timed out) is reported here.
  int err = 0;
  CUDA_TRY(cudaMemcpyAsync(&err, d->err, sizeof(int), cudaMemcpyDeviceToHost, s));
  CUDA_TRY(cudaStreamSynchronize(s));
  if (err) {
    cudaMemsetAsync(d->err, 0, sizeof(int), s);
    return fail(TB200_ERR_TIMEOUT, "matmul: a wait inside the contraction timed out");
  }
  return TB200_OK;
}

}  // namespace

extern "C" {

const char* tb200_last_error(void) { return rt::last_error(); }

int tb200_device_open(int ordinal, tb200_device** out) {
  ARG_CHECK(out, "null output handle");
  int n = 0;
  CUDA_TRY(cudaGetDeviceCount(&n));
  ARG_CHECK(ordinal >= 0 && ordinal < n, "no CUDA device " + std::to_string(ordinal));
  CUDA_TRY(cudaSetDevice(ordinal));
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, ordinal));
  if (prop.major != 10 || prop.minor != 0)
    return fail(TB200_ERR_CUDA, std::string("titania_b200 is built for sm_100a (B200); device is ") + prop.name +
                                    " sm_" + std::to_string(prop.major) + std::to_string(prop.minor));
  cudaError_t e = tb::init_fused_kernels(int(prop.sharedMemPerBlockOptin));
  if (e == cudaSuccess) e = tb::init_gemm_kernels();
  if (e == cudaSuccess) e = tb::init_batch_kernels();
  if (e != cudaSuccess) return fail(TB200_ERR_CUDA, std::string("kernel setup: ") + cudaGetErrorString(e));
  auto* d = new tb200_device;
  d->ordinal = ordinal;
  d->sms = prop.multiProcessorCount;
  e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&d->best, sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMalloc(&d->err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(d->err, 0, sizeof(int));
  if (e != cudaSuccess) {
    cudaFree(d->best);
    cudaFree(d->err);
    delete d;
    return fail(TB200_ERR_CUDA, std::string("device setup: ") + cudaGetErrorString(e));
  }
  d->max_cluster = std::min(8, tb::gemm_max_cluster());
  *out = d;
  return TB200_OK;
}

int tb200_device_close(tb200_device* d) {
  if (!d) return TB200_OK;
  cudaSetDevice(d->ordinal);
  cudaStreamSynchronize(d->stream);
  cudaFree(d->tokens);
  cudaFree(d->best);
  cudaFree(d->split);
  cudaFree(d->err);
  cudaFree(d->ao_part);
  cudaFree(d->ao_ticket);
  cudaFree(d->ao_meta);
  cudaFree(d->ao_planes);
  for (void* p : d->stage) cudaFreeHost(p);
  cudaStreamDestroy(d->stream);
  delete d;
  return TB200_OK;
}

int tb200_sync(tb200_device* d) {
  if (int rc = use(d)) return rc;
  CUDA_TRY(cudaStreamSynchronize(d->stream));
  return TB200_OK;
}

void* tb200_device_stream(tb200_device* d) { return d ? static_cast<void*>(d->stream) : nullptr; }
int tb200_device_sms(tb200_device* d) { return d ? d->sms : 0; }

// model.rs:239-250: the RoPE table a State uploads, computed on the host.
int tb200_rope_table(size_t max_len, size_t head_dim, float theta, float* out) {
  ARG_CHECK(out || max_len == 0, "null output");
  ARG_CHECK(head_dim % 2 == 0, "rope table: odd head_dim");
  std::vector<float> t = rope_table(max_len, head_dim, theta);
  std::memcpy(out, t.data(), t.size() * sizeof(float));
  return TB200_OK;
}

// ---- Device trait ------------------------------------------------------------

int tb200_upload(tb200_device* d, const uint16_t* data, const size_t* shape, size_t ndim, tb200_weight** out) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(out && (data || ndim == 0) && (shape || ndim == 0), "null argument");
  auto* w = new tb200_weight;
  w->shape.assign(shape, shape + ndim);
  w->numel = 1;
  for (size_t i = 0; i < ndim; i++) w->numel *= shape[i];
  if (w->numel) {
    cudaError_t e = cudaMalloc(&w->ptr, w->numel * 2);
    if (e == cudaSuccess) e = cudaMemcpyAsync(w->ptr, data, w->numel * 2, cudaMemcpyHostToDevice, d->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) {
      cudaFree(w->ptr);
      delete w;
      return fail(TB200_ERR_CUDA, std::string("upload: ") + cudaGetErrorString(e));
    }
  }
  *out = w;
  return TB200_OK;
}

int tb200_alloc(tb200_device* d, size_t len, tb200_buffer** out) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(out, "null output handle");
  auto* b = new tb200_buffer;
  b->len = b->cap = len;
  if (len) {
    cudaError_t e = cudaMalloc(&b->ptr, len * 4);
    if (e == cudaSuccess) e = cudaMemsetAsync(b->ptr, 0, len * 4, d->stream);
    if (e != cudaSuccess) {
      cudaFree(b->ptr);
      delete b;
      return fail(TB200_ERR_CUDA, std::string("alloc: ") + cudaGetErrorString(e));
    }
  }
  *out = b;
  return TB200_OK;
}

// cpu.rs:17-20 / titania.rs:124-127
int tb200_resize(tb200_device* d, tb200_buffer* b, size_t len) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(b, "null buffer");
  ARG_CHECK(len <= b->cap, "a buffer of " + std::to_string(b->cap) + " activations can't hold " + std::to_string(len));
  b->len = len;
  return TB200_OK;
}

size_t tb200_buffer_len(const tb200_buffer* b) { return b ? b->len : 0; }

int tb200_read(tb200_device* d, const tb200_buffer* b, float* out, size_t len) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(b && (out || len == 0), "null argument");
  ARG_CHECK(len == b->len, "read: buffer holds " + std::to_string(b->len) + " activations, not " + std::to_string(len));
  if (len) CUDA_TRY(cudaMemcpyAsync(out, b->ptr, len * 4, cudaMemcpyDeviceToHost, d->stream));
  CUDA_TRY(cudaStreamSynchronize(d->stream));
  return TB200_OK;
}

// titania.rs:133-137
int tb200_write(tb200_device* d, tb200_buffer* b, const float* data, size_t len) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(b && (data || len == 0), "null argument");
  ARG_CHECK(len == b->len, "write: " + std::to_string(len) + " values into a buffer of " + std::to_string(b->len));
  if (len) CUDA_TRY(cudaMemcpyAsync(b->ptr, data, len * 4, cudaMemcpyHostToDevice, d->stream));
  CUDA_TRY(cudaStreamSynchronize(d->stream));
  return TB200_OK;
}

// cpu.rs:34-36 / titania.rs:139-143
int tb200_copy(tb200_device* d, tb200_buffer* dst, size_t dst_off, const tb200_buffer* src, size_t src_off,
               size_t len) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(dst && src, "null buffer");
  ARG_CHECK(dst_off + len <= dst->len && src_off + len <= src->len, "copy out of range");
  ARG_CHECK(dst != src || dst_off + len <= src_off || src_off + len <= dst_off, "copy: overlapping ranges");
  tb::launch_copy(d->stream, dst->ptr + dst_off, src->ptr + src_off, len);
  return launched("copy");
}

// cpu.rs:38-47 / titania.rs:145-151
int tb200_embed(tb200_device* d, tb200_buffer* out, const tb200_weight* table, const uint32_t* tokens, size_t n) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(out && table && (tokens || n == 0), "null argument");
  ARG_CHECK(table->shape.size() == 2, "embed: table is not a matrix");
  const size_t rows = table->shape[0], dim = table->shape[1];
  ARG_CHECK(out->len == n * dim, "embed: output holds " + std::to_string(out->len) + " activations, expected " +
                                     std::to_string(n * dim));
  for (size_t i = 0; i < n; i++)
    ARG_CHECK(tokens[i] < rows, "embed: token " + std::to_string(tokens[i]) + " is past the table's " +
                                    std::to_string(rows) + " rows");
  if (!n) return TB200_OK;
  if (n > d->tokens_cap) {
    CUDA_TRY(cudaStreamSynchronize(d->stream));
    cudaFree(d->tokens);
    d->tokens = nullptr;
    d->tokens_cap = 0;
    CUDA_TRY(cudaMalloc(&d->tokens, n * 4));
    d->tokens_cap = n;
  }
  CUDA_TRY(cudaMemcpyAsync(d->tokens, tokens, n * 4, cudaMemcpyHostToDevice, d->stream));
  tb::launch_embed(d->stream, out->ptr, table->ptr, dim, d->tokens, n);
  return launched("embed");
}

// cpu.rs:49-77 / titania.rs:153-168
int tb200_matmul(tb200_device* d, tb200_buffer* out, const tb200_weight* w, const tb200_buffer* x) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(out && w && x, "null argument");
  ARG_CHECK(w->shape.size() == 2, "matmul: weight is not a matrix");
  ARG_CHECK(out != x, "matmul: output and input are the same buffer");
  const size_t rows = w->shape[0], cols = w->shape[1];
  ARG_CHECK(cols > 0, "matmul: weight has no columns");
  const size_t n = x->len / cols;
  ARG_CHECK(x->len == n * cols, "matmul: input of " + std::to_string(x->len) + " is not a whole number of " +
                                    std::to_string(cols) + "-wide rows");
  ARG_CHECK(out->len == n * rows, "matmul: output holds " + std::to_string(out->len) + ", expected " +
                                      std::to_string(n * rows));
  if (n >= 2 && cols % 8 == 0 && rows < (size_t(1) << 31) && cols < (size_t(1) << 31) && n < (size_t(1) << 24))
    return matmul_tokens(d, out, w, x, rows, cols, n);
  tb::launch_matmul(d->stream, out->ptr, w->ptr, rows, cols, x->ptr, n);
  return launched("matmul");
}

// cpu.rs:79-83 (zip: the shorter length)
int tb200_add(tb200_device* d, tb200_buffer* x, const tb200_buffer* y) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(x && y, "null buffer");
  tb::launch_add(d->stream, x->ptr, y->ptr, std::min(x->len, y->len));
  return launched("add");
}

// cpu.rs:85-94
int tb200_rmsnorm(tb200_device* d, tb200_buffer* x, const tb200_weight* w, float eps) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(x && w, "null argument");
  ARG_CHECK(w->numel > 0, "rmsnorm: empty weight");
  tb::launch_rmsnorm(d->stream, x->ptr, x->len / w->numel, w->ptr, w->numel, eps);
  return launched("rmsnorm");
}

// cpu.rs:96-111 / titania.rs:184-190
int tb200_rope(tb200_device* d, tb200_buffer* x, const tb200_buffer* table, size_t pos, size_t n_heads,
               size_t head_dim) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(x && table, "null buffer");
  ARG_CHECK(n_heads > 0 && head_dim > 0 && head_dim % 2 == 0, "rope: bad head shape");
  const size_t width = n_heads * head_dim;
  const size_t n = x->len / width;
  if (n == 0) return TB200_OK;
  ARG_CHECK((pos + n) * head_dim <= table->len,
            "rope: position " + std::to_string(pos + n - 1) + " is past the end of the table");
  tb::launch_rope(d->stream, x->ptr, n, table->ptr, pos, n_heads, head_dim);
  return launched("rope");
}

// cpu.rs:113-149 / titania.rs:192-215
int tb200_attention(tb200_device* d, tb200_buffer* out, const tb200_buffer* q, const tb200_buffer* k_cache,
                    const tb200_buffer* v_cache, size_t pos, size_t n_heads, size_t head_dim, size_t n_kv_heads) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(out && q && k_cache && v_cache, "null buffer");
  ARG_CHECK(n_heads > 0 && n_kv_heads > 0 && head_dim > 0 && n_heads % n_kv_heads == 0,
            "attention: bad head counts");
  ARG_CHECK(head_dim <= 256, "attention: head_dim above 256 is not supported");
  const size_t width = n_heads * head_dim;
  const size_t n = q->len / width;
  ARG_CHECK(q->len == n * width, "attention: queries are not a whole number of tokens");
  ARG_CHECK(out->len == q->len, "attention: output length differs from the queries'");
  ARG_CHECK(out != q && out != k_cache && out != v_cache, "attention: output aliases an input");
  const size_t kv_dim = n_kv_heads * head_dim;
  ARG_CHECK((pos + n) * kv_dim <= k_cache->len && (pos + n) * kv_dim <= v_cache->len,
            "attention: position past the end of the cache");
  tb::launch_attention(d->stream, out->ptr, q->ptr, n, k_cache->ptr, v_cache->ptr, pos, n_heads, head_dim,
                       n_kv_heads);
  return launched("attention");
}

// cpu.rs:151-155 (zip: the shorter length)
int tb200_silu_mul(tb200_device* d, tb200_buffer* gate, const tb200_buffer* up) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(gate && up, "null buffer");
  ARG_CHECK(gate != up, "silu_mul: gate and up are the same buffer");
  tb::launch_silu_mul(d->stream, gate->ptr, up->ptr, std::min(gate->len, up->len));
  return launched("silu_mul");
}

int tb200_free_buffer(tb200_device* d, tb200_buffer* b) {
  if (!b) return TB200_OK;
  if (int rc = use(d)) return rc;
  CUDA_TRY(cudaStreamSynchronize(d->stream));
  cudaFree(b->ptr);
  delete b;
  return TB200_OK;
}

int tb200_free_weight(tb200_device* d, tb200_weight* w) {
  if (!w) return TB200_OK;
  if (int rc = use(d)) return rc;
  CUDA_TRY(cudaStreamSynchronize(d->stream));
  cudaFree(w->ptr);
  delete w;
  return TB200_OK;
}

int tb200_argmax(tb200_device* d, const tb200_buffer* logits, uint32_t* out) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(logits && out, "null argument");
  ARG_CHECK(logits->len > 0, "argmax of an empty buffer");
  CUDA_TRY(cudaMemsetAsync(d->best, 0, sizeof(unsigned long long), d->stream));
  tb::launch_argmax(d->stream, logits->ptr, logits->len, d->best, d->sms);
  if (int rc = launched("argmax")) return rc;
  unsigned long long key = 0;
  CUDA_TRY(cudaMemcpyAsync(&key, d->best, sizeof key, cudaMemcpyDeviceToHost, d->stream));
  CUDA_TRY(cudaStreamSynchronize(d->stream));
  *out = 0xFFFFFFFFu - uint32_t(key & 0xFFFFFFFFu);
  return TB200_OK;
}

// ---- fused model ---------------------------------------------------------------

int tb200_model_create(tb200_device* d, const tb200_config* c, tb200_model** out) {
  if (int rc = use(d)) return rc;
  ARG_CHECK(c && out, "null argument");
  ARG_CHECK(c->hidden_size && c->intermediate_size && c->num_hidden_layers && c->num_attention_heads &&
                c->num_key_value_heads && c->head_dim && c->vocab_size,
            "config: zero dimension");
  auto* m = new tb200_model;
  m->dev = d;
  m->c = *c;
  m->q_dim = c->num_attention_heads * c->head_dim;
  m->kv_dim = c->num_key_value_heads * c->head_dim;
  *out = m;
  return TB200_OK;
}

int tb200_model_set_tp(tb200_model* m, tb200_tp* tp) {
  ARG_CHECK(m, "null model");
  ARG_CHECK(!m->finalized, "set the tensor-parallel group before finalizing the model");
  m->tp = tp;
  return TB200_OK;
}

int tb200_model_bind(tb200_model* m, const char* name, const tb200_weight* w) {
  ARG_CHECK(m && name && w, "null argument");
  ARG_CHECK(!m->finalized, "model already finalized");
  m->bound[name] = w;
  return TB200_OK;
}

static int get_bound(tb200_model* m, const std::string& name, std::vector<size_t> shape, bool optional,
                     const tb200_weight** out) {
  auto it = m->bound.find(name);
  if (it == m->bound.end()) {
    if (optional) {
      *out = nullptr;
      return TB200_OK;
    }
    return fail(TB200_ERR_ARG, "missing tensor '" + name + "'");
  }
  if (it->second->shape != shape)
    return fail(TB200_ERR_ARG, "tensor '" + name + "' has shape " + shape_str(it->second->shape) + ", expected " +
                                   shape_str(shape));
  *out = it->second;
  return TB200_OK;
}

int tb200_model_finalize(tb200_model* m) {
  ARG_CHECK(m, "null model");
  if (int rc = use(m->dev)) return rc;
  ARG_CHECK(!m->finalized, "model already finalized");
  const tb200_config& c = m->c;
  const size_t H = c.hidden_size, F = c.intermediate_size, D = c.head_dim, V = c.vocab_size;
  const size_t group = c.num_attention_heads / c.num_key_value_heads;
  ARG_CHECK(D == 128, "the fused path needs head_dim 128 (Qwen3), not " + std::to_string(D));
  ARG_CHECK(c.num_attention_heads % c.num_key_value_heads == 0 && (group == 1 || group == 2 || group == 4 || group == 8),
            "the fused path needs 1, 2, 4 or 8 query heads per kv head");
  ARG_CHECK(H % 8 == 0 && F % 8 == 0, "the fused path needs hidden and FFN sizes divisible by 8");
  ARG_CHECK(H <= 12288 && F <= 12288 && m->q_dim <= 12288, "the fused path supports widths up to 12288");
  cudaStream_t s = m->dev->stream;
  const tb200_weight* w = nullptr;
  if (int rc = get_bound(m, "model.embed_tokens.weight", {V, H}, false, &w)) return rc;
  m->embed = w->ptr;
  if (int rc = get_bound(m, "model.norm.weight", {H}, false, &w)) return rc;
  m->norm = w->ptr;
  if (c.tie_word_embeddings) {
    m->lm_head = m->embed;
  } else {
    if (int rc = get_bound(m, "lm_head.weight", {V, H}, false, &w)) return rc;
    m->lm_head = w->ptr;
  }
  for (size_t i = 0; i < c.num_hidden_layers; i++) {
    const std::string p = "model.layers." + std::to_string(i);
    FusedLayer L{};
    const tb200_weight *q, *k, *v, *o, *g, *u, *dn, *an, *mn, *qn, *kn;
    int rc = get_bound(m, p + ".input_layernorm.weight", {H}, false, &an);
    if (!rc) rc = get_bound(m, p + ".self_attn.q_proj.weight", {m->q_dim, H}, false, &q);
    if (!rc) rc = get_bound(m, p + ".self_attn.k_proj.weight", {m->kv_dim, H}, false, &k);
    if (!rc) rc = get_bound(m, p + ".self_attn.v_proj.weight", {m->kv_dim, H}, false, &v);
    if (!rc) rc = get_bound(m, p + ".self_attn.o_proj.weight", {H, m->q_dim}, false, &o);
    if (!rc) rc = get_bound(m, p + ".self_attn.q_norm.weight", {D}, true, &qn);
    if (!rc) rc = get_bound(m, p + ".self_attn.k_norm.weight", {D}, true, &kn);
    if (!rc) rc = get_bound(m, p + ".post_attention_layernorm.weight", {H}, false, &mn);
    if (!rc) rc = get_bound(m, p + ".mlp.gate_proj.weight", {F, H}, false, &g);
    if (!rc) rc = get_bound(m, p + ".mlp.up_proj.weight", {F, H}, false, &u);
    if (!rc) rc = get_bound(m, p + ".mlp.down_proj.weight", {H, F}, false, &dn);
    if (rc) return rc;
    L.attn_norm = an->ptr;
    L.mlp_norm = mn->ptr;
    L.q_norm = qn ? qn->ptr : nullptr;
    L.k_norm = kn ? kn->ptr : nullptr;
    L.wo = o->ptr;
    L.wd = dn->ptr;
    const size_t rows = m->q_dim + 2 * m->kv_dim;
    CUDA_TRY(cudaMalloc(&L.wqkv, rows * H * 2));
    CUDA_TRY(cudaMemcpyAsync(L.wqkv, q->ptr, m->q_dim * H * 2, cudaMemcpyDeviceToDevice, s));
    CUDA_TRY(cudaMemcpyAsync(L.wqkv + m->q_dim * H, k->ptr, m->kv_dim * H * 2, cudaMemcpyDeviceToDevice, s));
    CUDA_TRY(cudaMemcpyAsync(L.wqkv + (m->q_dim + m->kv_dim) * H, v->ptr, m->kv_dim * H * 2,
                             cudaMemcpyDeviceToDevice, s));
    CUDA_TRY(cudaMalloc(&L.wgu, 2 * F * H * 2));
    tb::launch_interleave_rows(s, L.wgu, g->ptr, u->ptr, F, H);
    if (int rc2 = launched("interleave")) return rc2;
    m->attn_o_slices = tb::attn_o_slices(int(H), int(group));
    CUDA_TRY(cudaMalloc(&L.wo_packed, H * m->q_dim * 2));
    tb::launch_pack_wo(s, L.wo_packed, o->ptr, int(H), int(c.num_key_value_heads), int(group), m->attn_o_slices);
    if (int rc2 = launched("pack o_proj")) return rc2;
    std::string why;
    int rc3 = tb::encode_tmap_bf16(&L.m_qkv, L.wqkv, rows, H, 128, &why);
    if (!rc3) rc3 = tb::encode_tmap_bf16(&L.m_o, L.wo, H, m->q_dim, 128, &why);
    if (!rc3) rc3 = tb::encode_tmap_bf16(&L.m_gu, L.wgu, 2 * F, H, 128, &why);
    if (!rc3) rc3 = tb::encode_tmap_bf16(&L.m_down, L.wd, H, F, 128, &why);
    if (rc3) return fail(rc3, "model: " + why);
    m->layers.push_back(L);
  }
  {
    std::string why;
    if (int rc = tb::encode_tmap_bf16(&m->m_lm, m->lm_head, V, H, 128, &why)) return fail(rc, "model: " + why);
  }
  CUDA_TRY(cudaStreamSynchronize(s));
  if (m->tp)
    if (int rc = rt::tp_p2p_setup(m)) return rc;
  m->finalized = true;
  return TB200_OK;
}

static void delete_model(tb200_model* m) {
  cudaSetDevice(m->dev->ordinal);
  cudaStreamSynchronize(m->dev->stream);
  rt::tp_p2p_free(m);
  for (auto& L : m->layers) {
    cudaFree(L.wqkv);
    cudaFree(L.wgu);
    cudaFree(L.wo_packed);
  }
  delete m;
}

int tb200_model_free(tb200_model* m) {
  if (!m) return TB200_OK;
  // States keep their model alive; the last one to go deletes it.
  if (m->live_states > 0) {
    m->free_requested = true;
    return TB200_OK;
  }
  delete_model(m);
  return TB200_OK;
}

namespace {

// Budget of shared memory per matrix-vector CTA: two consecutive kernels fit
// on one SM (228 KB), so a kernel can stage its weights while the previous
// one runs.
constexpr size_t kMvBudget = 110 * 1024;
constexpr size_t kLmBudget = 160 * 1024;

// Enqueues one fused kernel of the decode step: op 0 embed, 1 q|k|v,
// 2 attention, 3 o_proj, 4 gate|up, 5 down (ops 1-5 of `layer`), 6 lm_head.
void enqueue_op(tb200_state* st, int op, size_t l, bool pdl) {
  tb200_model* m = st->m;
  const tb200_config& c = m->c;
  cudaStream_t s = m->dev->stream;
  const int H = int(c.hidden_size), F = int(c.intermediate_size);
  const size_t kv_layer = 2 * c.num_key_value_heads * st->max_len * c.head_dim;
  int* err = st->io + 3;
  const uint32_t tag = (uint32_t(op) << 16) | uint32_t(l);
  tb::MvArgs a{};
  a.err = err;
  a.trace = st->trace;
  a.tag = tag;
  auto slots_for = [&](uint32_t ctas) {
    const uint32_t base = st->trace_next;
    st->trace_next += ctas * tb::kTraceEvents;
    return base;
  };
  a.eps = c.rms_norm_eps;
  a.row_align = 1;
  // Tensor parallelism by peer stores: slot 0 of a layer is the o_proj
  // partial sums, slot 1 the down_proj ones.
  const TpP2p& pp = m->p2p;
  auto publish = [&](size_t layer, int slot) {
    for (int r = 0; r < pp.world; r++) {
      unsigned char* base = static_cast<unsigned char*>(pp.peer[r]);
      a.peer_out[r] = reinterpret_cast<float*>(base + (slot ? pp.off_d : 0)) + size_t(pp.rank) * H;
      a.peer_flag[r] = reinterpret_cast<unsigned*>(base + pp.off_flags) + (2 * layer + slot) * pp.world + pp.rank;
    }
    a.npeers = pp.world;
    a.p2p_ticket = pp.tickets + 2 * layer + slot;
    a.epoch = pp.epoch;
  };
  auto receive = [&](size_t layer, int slot) {
    unsigned char* base = static_cast<unsigned char*>(pp.region);
    a.partials = reinterpret_cast<const float*>(base + (slot ? pp.off_d : 0));
    a.npartials = pp.world;
    a.wait_flags = reinterpret_cast<const unsigned*>(base + pp.off_flags) + (2 * layer + slot) * pp.world;
    a.nwait = pp.world;
    a.epoch = pp.epoch;
  };
  switch (op) {
    case TB200_OP_EMBED:
      tb::launch_embed_token(s, st->x, m->embed, H, st->io + 0, int(c.vocab_size), err, pdl);
      return;
    case TB200_OP_QKV: {
      const FusedLayer& L = m->layers[l];
      a.w = L.wqkv;
      a.rows = int(m->q_dim + 2 * m->kv_dim);
      a.cols = H;
      a.x = st->x;
      if (m->tp && l > 0) {  // x = x2 + the previous layer's reduced down_proj partial
        a.x = st->x2;
        a.partials = st->part_tp2;
        a.npartials = 1;
        a.x_out = st->x;
        if (pp.on) receive(l - 1, 1);  // ... summed here from every rank's slot
      }
      a.norm_w = L.attn_norm;
      a.out = st->qkv;
      a.trace_base = slots_for(st->p_qkv.grid);
      tb::launch_mv(s, st->p_qkv, tb::kMvStore, a, pdl);
      return;
    }
    case TB200_OP_ATTENTION: {
      const FusedLayer& L = m->layers[l];
      tb::AttnArgs t{};
      t.qkv = st->qkv;
      t.q_norm = L.q_norm;
      t.k_norm = L.k_norm;
      t.eps = c.rms_norm_eps;
      t.rope = st->rope;
      const size_t eb = st->kv_f32 ? 4 : 2;
      t.k_cache = st->kv + l * kv_layer * eb;
      t.v_cache = st->kv + l * kv_layer * eb + kv_layer / 2 * eb;
      t.kv_f32 = st->kv_f32;
      t.max_len = int(st->max_len);
      t.n_heads = int(c.num_attention_heads);
      t.n_kv_heads = int(c.num_key_value_heads);
      t.pos = st->io + 1;
      t.out = st->att;
      t.part = st->part;
      t.ticket = st->attn_ticket;
      t.max_split = st->max_split;
      t.err = err;
      t.trace = st->trace;
      t.tag = tag;
      t.trace_base = slots_for(uint32_t(c.num_key_value_heads * st->max_split));
      tb::launch_attn_decode(s, t, pdl);
      return;
    }
    case TB200_OP_ATTENTION_O: {
      const FusedLayer& L = m->layers[l];
      tb::AttnOArgs t{};
      t.qkv = st->qkv;
      t.q_norm = L.q_norm;
      t.k_norm = L.k_norm;
      t.eps = c.rms_norm_eps;
      t.rope = st->rope;
      const size_t eb = st->kv_f32 ? 4 : 2;
      t.k_cache = st->kv + l * kv_layer * eb;
      t.v_cache = st->kv + l * kv_layer * eb + kv_layer / 2 * eb;
      t.kv_f32 = st->kv_f32;
      t.max_len = int(st->max_len);
      t.n_heads = int(c.num_attention_heads);
      t.n_kv_heads = int(c.num_key_value_heads);
      t.pos = st->io + 1;
      t.wo_packed = L.wo_packed;
      t.hidden = H;
      t.nslices = m->attn_o_slices;
      t.rows_per_slice = H / m->attn_o_slices;
      t.part = st->part_o;
      t.err = err;
      t.trace = st->trace;
      t.tag = tag;
      t.trace_base = slots_for(uint32_t(c.num_key_value_heads * m->attn_o_slices));
      tb::launch_attn_o(s, t, pdl);
      return;
    }
    case TB200_OP_O: {
      a.w = m->layers[l].wo;
      a.rows = H;
      a.cols = int(m->q_dim);
      a.x = st->att;
      a.out = st->x;
      a.trace_base = slots_for(st->p_o.grid);
      if (m->tp) {  // this rank's partial sum; reduced over the group next
        a.out = st->part_tp;
        if (pp.on) publish(l, 0);
        tb::launch_mv(s, st->p_o, tb::kMvStore, a, pdl);
        return;
      }
      tb::launch_mv(s, st->p_o, tb::kMvResidual, a, pdl);
      return;
    }
    case TB200_OP_GATE_UP:
    case TB200_OP_GATE_UP_SUM: {
      a.w = m->layers[l].wgu;
      a.rows = 2 * F;
      a.cols = H;
      a.row_align = 2;
      a.x = st->x;
      a.x_out = st->x2;
      if (op == TB200_OP_GATE_UP_SUM) {
        a.partials = st->part_o;
        a.npartials = int(c.num_key_value_heads);
      } else if (m->tp) {  // x + the reduced o_proj partial
        a.partials = st->part_tp;
        a.npartials = 1;
        if (pp.on) receive(l, 0);
      }
      a.norm_w = m->layers[l].mlp_norm;
      a.out = st->h;
      a.trace_base = slots_for(st->p_gu.grid);
      tb::launch_mv(s, st->p_gu, tb::kMvSiluPair, a, pdl);
      return;
    }
    case TB200_OP_DOWN: {
      a.w = m->layers[l].wd;
      a.rows = H;
      a.cols = F;
      a.x = st->h;
      a.out = st->x;
      a.resid_src = st->x2;
      a.trace_base = slots_for(st->p_down.grid);
      if (m->tp) {  // this rank's partial sum; the next kernel adds it to x2 once reduced
        a.out = st->part_tp2;
        a.resid_src = nullptr;
        if (pp.on) publish(l, 1);
        tb::launch_mv(s, st->p_down, tb::kMvStore, a, pdl);
        return;
      }
      tb::launch_mv(s, st->p_down, tb::kMvResidual, a, pdl);
      return;
    }
    case TB200_OP_LM_HEAD: {
      a.w = m->lm_head;
      a.rows = int(c.vocab_size);
      a.cols = H;
      a.x = st->x;
      if (m->tp) {
        a.x = st->x2;
        a.partials = st->part_tp2;
        a.npartials = 1;
        if (pp.on) receive(c.num_hidden_layers - 1, 1);
      }
      a.norm_w = m->norm;
      a.out = st->logits;
      a.partial = st->mv_partial;
      a.ticket = st->mv_ticket;
      a.token = st->io + 0;
      a.pos = st->io + 1;
      a.step = st->io + 2;
      a.tokens_out = st->tokens_out;
      a.tokens_cap = int(st->max_len);
      a.trace_base = slots_for(st->p_lm.grid);
      tb::launch_mv(s, st->p_lm, tb::kMvArgmax, a, pdl);
      return;
    }
  }
}

// One decode step. `short_ctx`: the position is below kAttnOMaxCtx, so
// attention and o_proj run fused, one kernel per layer less.
int enqueue_step(tb200_state* st, bool short_ctx) {
  st->trace_next = 0;
  // TB200_SERIAL=1 launches the step's kernels without programmatic
  // dependent launch (each waits for the previous to finish): a diagnostic
  // for ordering questions, slower but otherwise identical.
  static const bool pdl = !(getenv("TB200_SERIAL") && getenv("TB200_SERIAL")[0] == '1');
  tb200_model* m = st->m;
  cudaStream_t s = m->dev->stream;
  const size_t H = m->c.hidden_size, Hkv = m->c.num_key_value_heads;
  enqueue_op(st, TB200_OP_EMBED, 0, pdl);
  for (size_t l = 0; l < m->c.num_hidden_layers; l++) {
    enqueue_op(st, TB200_OP_QKV, l, pdl);
    if (short_ctx) {
      enqueue_op(st, TB200_OP_ATTENTION_O, l, pdl);
      if (m->tp)
        if (int rc = rt::tp_allreduce(m->tp, st->part_o, Hkv * H, s)) return rc;
      enqueue_op(st, TB200_OP_GATE_UP_SUM, l, pdl);
    } else {
      enqueue_op(st, TB200_OP_ATTENTION, l, pdl);
      enqueue_op(st, TB200_OP_O, l, pdl);
      if (m->tp && !m->p2p.on)
        if (int rc = rt::tp_allreduce(m->tp, st->part_tp, H, s)) return rc;
      enqueue_op(st, TB200_OP_GATE_UP, l, pdl);
    }
    enqueue_op(st, TB200_OP_DOWN, l, pdl);
    if (m->tp && !m->p2p.on)
      if (int rc = rt::tp_allreduce(m->tp, st->part_tp2, H, s)) return rc;
  }
  enqueue_op(st, TB200_OP_LM_HEAD, 0, pdl);
  return launched("decode step");
}

int capture(tb200_state* st, bool short_ctx, cudaGraphExec_t* out) {
  cudaStream_t s = st->m->dev->stream;
  CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_step(st, short_ctx);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(s, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return fail(TB200_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return fail(TB200_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
  return TB200_OK;
}

int build_graph(tb200_state* st) {
  cudaStream_t s = st->m->dev->stream;
  CUDA_TRY(cudaStreamSynchronize(s));
  for (cudaGraphExec_t* g : {&st->graph, &st->graph_short})
    if (*g) {
      cudaGraphExecDestroy(*g);
      *g = nullptr;
    }
  if (int rc = capture(st, false, &st->graph)) return rc;
  if (st->m->c.num_key_value_heads > size_t(tb::kMaxPartials)) return TB200_OK;
  return capture(st, true, &st->graph_short);
}

// The graph for a step at `pos`: the fused attention + o_proj one for short
// contexts when the model has at most kMaxPartials kv groups.
cudaGraphExec_t step_graph(tb200_state* st, size_t pos) {
  return pos < size_t(tb::kAttnOMaxCtx) && st->graph_short ? st->graph_short : st->graph;
}

// Copies back the io block and reports a kernel-side error.
int finish(tb200_state* st) {
  cudaStream_t s = st->m->dev->stream;
  int* back = st->io_host + 2 * st->max_len;
  CUDA_TRY(cudaMemcpyAsync(back, st->io, 4 * sizeof(int), cudaMemcpyDeviceToHost, s));
  CUDA_TRY(cudaStreamSynchronize(s));
  if (back[3] != 0) st->ps_dirty = true;
  if (back[3] == TB200_ERR_TIMEOUT) return fail(TB200_ERR_TIMEOUT, "a kernel's bounded wait timed out");
  if (back[3] != 0) return fail(TB200_ERR_ARG, "a kernel rejected its input (token or position out of range)");
  return TB200_OK;
}

}  // namespace

namespace {

int state_create(tb200_model* m, size_t n_seqs, size_t max_len, int kv_dtype, tb200_state** out) {
  ARG_CHECK(m && out, "null argument");
  ARG_CHECK(n_seqs > 0 && n_seqs <= 65536, "state: bad number of sequences");
  ARG_CHECK(m->finalized, "model not finalized");
  ARG_CHECK(!m->free_requested, "model already freed");
  ARG_CHECK(kv_dtype == TB200_KV_BF16 || kv_dtype == TB200_KV_F32, "unknown key/value cache type");
  ARG_CHECK(max_len > 0 && max_len < (size_t(1) << 30), "state: bad max_len");
  if (int rc = use(m->dev)) return rc;
  const tb200_config& c = m->c;
  auto* st = new tb200_state;
  st->m = m;
  st->dev = m->dev;
  st->max_len = max_len;
  st->n_seqs = n_seqs;
  st->kv_f32 = kv_dtype == TB200_KV_F32;
  m->live_states++;
  const int sms = m->dev->sms;
  const size_t Hkv = c.num_key_value_heads, D = c.head_dim, L = c.num_hidden_layers;
  const size_t group = c.num_attention_heads / Hkv;
  // Attention splits of kAttnChunk positions cover the whole cache; their
  // merge keeps one weight per (split, head) in the kernel's staging memory.
  st->max_split = int((max_len + tb::kAttnChunk - 1) / tb::kAttnChunk);
  if (size_t(st->max_split) * group * 4 > tb::attn_smem_bytes(kv_dtype == TB200_KV_F32)) {
    m->live_states--;
    delete st;
    return fail(TB200_ERR_ARG, "state: max_len " + std::to_string(max_len) + " is past the longest context (" +
                                   std::to_string(tb::attn_smem_bytes(kv_dtype == TB200_KV_F32) / 4 / group *
                                                  tb::kAttnChunk) + ") of this model's attention kernels");
  }
  std::vector<float> table = rope_table(max_len, D, c.rope_theta);
  cudaError_t e = cudaSuccess;
  auto A = [&](void** p, size_t bytes) {
    if (e == cudaSuccess) e = cudaMalloc(p, bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(*p, 0, bytes, m->dev->stream);
  };
  st->seq_stride = L * 2 * Hkv * max_len * D;
  A((void**)&st->kv, n_seqs * st->seq_stride * (st->kv_f32 ? 4 : 2));
  A((void**)&st->rope, table.size() * 4);
  A((void**)&st->x, c.hidden_size * 4);
  A((void**)&st->qkv, (m->q_dim + 2 * m->kv_dim) * 4);
  A((void**)&st->att, m->q_dim * 4);
  A((void**)&st->h, c.intermediate_size * 4);
  A((void**)&st->x2, c.hidden_size * 4);
  A((void**)&st->part_o, Hkv * c.hidden_size * 4);
  if (m->tp) {
    A((void**)&st->part_tp, c.hidden_size * 4);
    A((void**)&st->part_tp2, c.hidden_size * 4);
  }
  A((void**)&st->logits, c.vocab_size * 4);
  A((void**)&st->part, Hkv * st->max_split * group * tb::kPartStride * 4);
  A((void**)&st->attn_ticket, Hkv * 4);
  A((void**)&st->mv_partial, size_t(sms) * 8);
  A((void**)&st->mv_ticket, 4);
  A((void**)&st->io, 4 * sizeof(int));
  A((void**)&st->tokens_out, max_len * sizeof(int));
  if (e == cudaSuccess) e = cudaHostAlloc((void**)&st->io_host, (2 * max_len + 4) * sizeof(int), cudaHostAllocDefault);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(st->rope, table.data(), table.size() * 4, cudaMemcpyHostToDevice, m->dev->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->dev->stream);
  if (e != cudaSuccess) {
    tb200_state_free(st);
    return fail(TB200_ERR_CUDA, std::string("state: ") + cudaGetErrorString(e));
  }
  const int H = int(c.hidden_size), F = int(c.intermediate_size);
  st->p_qkv = tb::plan_mv(int(m->q_dim + 2 * m->kv_dim), H, 1, true, sms, kMvBudget);
  st->p_o = tb::plan_mv(H, int(m->q_dim), 1, false, sms, kMvBudget);
  st->p_gu = tb::plan_mv(2 * F, H, 2, true, sms, kMvBudget);
  st->p_down = tb::plan_mv(H, F, 1, false, sms, kMvBudget);
  st->p_lm = tb::plan_mv(int(c.vocab_size), H, 1, true, sms, kLmBudget);
  if (st->p_o.max_rows > tb::kMaxResidualRows || st->p_down.max_rows > tb::kMaxResidualRows) {
    tb200_state_free(st);
    return fail(TB200_ERR_ARG, "hidden size too large for the residual kernels on this GPU");
  }
  // The single-token graphs run sequence 0 of a one-sequence state.
  if (n_seqs == 1) {
    if (int rc = build_graph(st)) {
      tb200_state_free(st);
      return rc;
    }
    if (rt::persist_unsupported(m, st).empty()) st->decode_mode = TB200_DECODE_PERSISTENT;
  }
  *out = st;
  return TB200_OK;
}

}  // namespace

int tb200_state_new(tb200_model* m, size_t max_len, int kv_dtype, tb200_state** out) {
  return state_create(m, 1, max_len, kv_dtype, out);
}

int tb200_batch_state_new(tb200_model* m, size_t n_seqs, size_t max_len, int kv_dtype, tb200_state** out) {
  return state_create(m, n_seqs, max_len, kv_dtype, out);
}

size_t tb200_state_seqs(const tb200_state* st) { return st ? st->n_seqs : 0; }

int tb200_state_free(tb200_state* st) {
  if (!st) return TB200_OK;
  cudaSetDevice(st->dev->ordinal);
  cudaStreamSynchronize(st->dev->stream);
  if (st->graph) cudaGraphExecDestroy(st->graph);
  if (st->graph_short) cudaGraphExecDestroy(st->graph_short);
  rt::free_batch(st);
  void* ptrs[] = {st->kv, st->rope, st->x, st->qkv, st->att, st->h, st->logits, st->part, st->attn_ticket,
                  st->mv_partial, st->mv_ticket, st->io, st->tokens_out, st->x2, st->part_o, st->part_tp,
                  st->part_tp2, st->ps_words, st->ps_ctl};
  for (void* p : ptrs) cudaFree(p);
  if (st->io_host) cudaFreeHost(st->io_host);
  tb200_model* m = st->m;
  delete st;
  if (--m->live_states == 0 && m->free_requested) delete_model(m);
  return TB200_OK;
}

// model.rs:83-91
int tb200_forward(tb200_model* m, tb200_state* st, const uint32_t* tokens, size_t n, size_t pos, float* logits,
                  uint32_t* next_token) {
  ARG_CHECK(m && st && st->m == m, "bad model/state");
  ARG_CHECK(st->n_seqs == 1, "tb200_forward runs one-sequence states; use tb200_forward_seq");
  ARG_CHECK(n > 0 && tokens, "no tokens to run");
  ARG_CHECK(pos + n <= st->max_len, "tokens past the end of the cache");
  if (int rc = use(m->dev)) return rc;
  for (size_t i = 0; i < n; i++)
    ARG_CHECK(tokens[i] < m->c.vocab_size, "token " + std::to_string(tokens[i]) + " is past the vocabulary");
  // Several tokens (a prompt): the tensor-core path, all tokens at once.
  if (n >= 2) {
    if (int rc = rt::forward_tokens(st, 0, tokens, n, pos, logits, next_token)) return rc;
    st->host_pos = pos + n;
    return TB200_OK;
  }
  // One token: token, position, step counter and error word in one copy
  // (from the slot finish() reads io back into, which this copy precedes).
  cudaStream_t s = m->dev->stream;
  int* stage = st->io_host + 2 * st->max_len;
  stage[0] = int(tokens[0]);
  stage[1] = int(pos);
  stage[2] = 0;
  stage[3] = 0;
  CUDA_TRY(cudaMemcpyAsync(st->io, stage, 4 * sizeof(int), cudaMemcpyHostToDevice, s));
  // The persistent kernel writes the logits straight into page-locked host
  // memory (as its lm_head rows finish, over PCIe) instead of a copy after it.
  float* direct = nullptr;
  if (logits && st->decode_mode == TB200_DECODE_PERSISTENT) {
    cudaPointerAttributes pa{};
    if (cudaPointerGetAttributes(&pa, logits) == cudaSuccess && pa.type == cudaMemoryTypeHost && pa.devicePointer)
      direct = static_cast<float*>(pa.devicePointer);
    cudaGetLastError();  // a pointer CUDA does not know is an answer, not an error to keep
  }
  if (st->decode_mode == TB200_DECODE_PERSISTENT) {
    if (int rc = rt::persist_enqueue(st, 1, logits != nullptr, direct)) return rc;
  } else {
    CUDA_TRY(cudaGraphLaunch(step_graph(st, pos), s));
  }
  if (logits && !direct)
    CUDA_TRY(cudaMemcpyAsync(logits, st->logits, m->c.vocab_size * 4, cudaMemcpyDeviceToHost, s));
  if (int rc = finish(st)) return rc;
  st->host_pos = pos + n;
  if (next_token) *next_token = uint32_t(st->io_host[2 * st->max_len + 0]);
  return TB200_OK;
}

int tb200_generate(tb200_model* m, tb200_state* st, uint32_t token, size_t pos, size_t steps, uint32_t* out) {
  ARG_CHECK(m && st && st->m == m, "bad model/state");
  ARG_CHECK(st->n_seqs == 1, "the single-token path runs one-sequence states");
  ARG_CHECK(out || steps == 0, "null output");
  ARG_CHECK(pos + steps <= st->max_len, "tokens past the end of the cache");
  ARG_CHECK(token < m->c.vocab_size, "token past the vocabulary");
  if (int rc = use(m->dev)) return rc;
  if (!steps) return TB200_OK;
  cudaStream_t s = m->dev->stream;
  int* stage = st->io_host + 2 * st->max_len;
  stage[0] = int(token);
  stage[1] = int(pos);
  stage[2] = 0;
  stage[3] = 0;
  CUDA_TRY(cudaMemcpyAsync(st->io, stage, 4 * sizeof(int), cudaMemcpyHostToDevice, s));
  if (st->decode_mode == TB200_DECODE_PERSISTENT) {
    if (int rc = rt::persist_enqueue(st, steps, false)) return rc;
  } else {
    for (size_t i = 0; i < steps; i++) CUDA_TRY(cudaGraphLaunch(step_graph(st, pos + i), s));
  }
  static_assert(sizeof(uint32_t) == sizeof(int), "token width");
  CUDA_TRY(cudaMemcpyAsync(out, st->tokens_out, steps * 4, cudaMemcpyDeviceToHost, s));
  if (int rc = finish(st)) return rc;
  st->host_pos = pos + steps;
  return TB200_OK;
}

int tb200_decode_enqueue(tb200_model* m, tb200_state* st, uint32_t token, size_t pos, size_t steps) {
  ARG_CHECK(m && st && st->m == m, "bad model/state");
  ARG_CHECK(st->n_seqs == 1, "the single-token path runs one-sequence states");
  ARG_CHECK(pos + steps <= st->max_len, "decode steps past the end of the cache");
  ARG_CHECK(token < m->c.vocab_size, "token past the vocabulary");
  if (int rc = use(m->dev)) return rc;
  tb::launch_set_io(m->dev->stream, st->io, int(token), int(pos));
  if (int rc = launched("set_io")) return rc;
  if (st->decode_mode == TB200_DECODE_PERSISTENT) {
    if (int rc = rt::persist_enqueue(st, steps, false)) return rc;
  } else {
    for (size_t i = 0; i < steps; i++) CUDA_TRY(cudaGraphLaunch(step_graph(st, pos + i), m->dev->stream));
  }
  st->host_pos = pos + steps;
  return TB200_OK;
}

int tb200_state_set_decode(tb200_state* st, int mode) {
  ARG_CHECK(st, "null state");
  ARG_CHECK(mode == TB200_DECODE_FUSED || mode == TB200_DECODE_PERSISTENT, "unknown decode mode");
  ARG_CHECK(st->n_seqs == 1, "the single-token path runs one-sequence states");
  if (mode == TB200_DECODE_PERSISTENT) {
    const std::string why = rt::persist_unsupported(st->m, st);
    ARG_CHECK(why.empty(), why);
  }
  st->decode_mode = mode;
  return TB200_OK;
}

int tb200_state_decode(const tb200_state* st) { return st ? st->decode_mode : -1; }

int tb200_decode_persistent(tb200_model* m, tb200_state* st, uint32_t token, size_t pos, size_t steps,
                            uint32_t* tokens_out, float* logits_out) {
  ARG_CHECK(m && st && st->m == m, "bad model/state");
  ARG_CHECK(st->n_seqs == 1, "the single-token path runs one-sequence states");
  ARG_CHECK(tokens_out || steps == 0, "null output");
  ARG_CHECK(pos + steps <= st->max_len, "tokens past the end of the cache");
  ARG_CHECK(token < m->c.vocab_size, "token past the vocabulary");
  {
    const std::string why = rt::persist_unsupported(m, st);
    ARG_CHECK(why.empty(), why);
  }
  if (int rc = use(m->dev)) return rc;
  if (!steps) return TB200_OK;
  cudaStream_t s = m->dev->stream;
  int* stage = st->io_host + 2 * st->max_len;
  stage[0] = int(token);
  stage[1] = int(pos);
  stage[2] = 0;
  stage[3] = 0;
  CUDA_TRY(cudaMemcpyAsync(st->io, stage, 4 * sizeof(int), cudaMemcpyHostToDevice, s));
  if (!logits_out) {
    if (int rc = rt::persist_enqueue(st, steps, false)) return rc;
  } else {
    for (size_t i = 0; i < steps; i++) {
      if (int rc = rt::persist_enqueue(st, 1, true)) return rc;
      CUDA_TRY(cudaMemcpyAsync(logits_out + i * m->c.vocab_size, st->logits, m->c.vocab_size * 4,
                               cudaMemcpyDeviceToHost, s));
    }
  }
  CUDA_TRY(cudaMemcpyAsync(tokens_out, st->tokens_out, steps * 4, cudaMemcpyDeviceToHost, s));
  if (int rc = finish(st)) return rc;
  st->host_pos = pos + steps;
  return TB200_OK;
}

int tb200_enqueue_op(tb200_model* m, tb200_state* st, int op, size_t layer) {
  ARG_CHECK(m && st && st->m == m, "bad model/state");
  ARG_CHECK(st->n_seqs == 1, "the single-token path runs one-sequence states");
  ARG_CHECK(op >= TB200_OP_EMBED && op <= TB200_OP_GATE_UP_SUM, "unknown op");
  ARG_CHECK(layer < m->c.num_hidden_layers, "layer out of range");
  if (int rc = use(m->dev)) return rc;
  enqueue_op(st, op, layer, false);
  return launched("enqueue_op");
}

int tb200_trace_start(tb200_state* st, size_t capacity) {
  ARG_CHECK(st && capacity > 0 && capacity < (size_t(1) << 31), "bad trace capacity");
  ARG_CHECK(!st->trace.rec, "already tracing");
  if (int rc = use(st->dev)) return rc;
  CUDA_TRY(cudaStreamSynchronize(st->dev->stream));
  CUDA_TRY(cudaMalloc(&st->trace.rec, capacity * sizeof(tb::TraceRec)));
  CUDA_TRY(cudaMemset(st->trace.rec, 0, capacity * sizeof(tb::TraceRec)));
  st->trace.cap = unsigned(capacity);
  st->ps_traced = false;
  rt::drop_batch_graph(st);  // recaptured with the buffer on next use
  return st->n_seqs == 1 ? build_graph(st) : TB200_OK;
}

int tb200_trace_stop(tb200_state* st, tb200_trace_record* out, size_t cap, size_t* n) {
  ARG_CHECK(st && n && (out || cap == 0), "null argument");
  ARG_CHECK(st->trace.rec, "not tracing");
  static_assert(sizeof(tb200_trace_record) == sizeof(tb::TraceRec), "trace record layout");
  if (int rc = use(st->dev)) return rc;
  CUDA_TRY(cudaStreamSynchronize(st->dev->stream));
  *n = st->ps_traced ? rt::persist_trace_slots(st) : st->trace_next;
  const size_t k = std::min<size_t>(st->trace.cap, cap);
  if (k) CUDA_TRY(cudaMemcpy(out, st->trace.rec, k * sizeof(tb::TraceRec), cudaMemcpyDeviceToHost));
  cudaFree(st->trace.rec);
  st->trace = tb::Trace{};
  rt::drop_batch_graph(st);
  return st->n_seqs == 1 ? build_graph(st) : TB200_OK;
}

static int state_buffer(tb200_state* st, int which, float** p, size_t* len) {
  const tb200_config& c = st->m->c;
  switch (which) {
    case TB200_BUF_X: *p = st->x; *len = c.hidden_size; return TB200_OK;
    case TB200_BUF_QKV: *p = st->qkv; *len = st->m->q_dim + 2 * st->m->kv_dim; return TB200_OK;
    case TB200_BUF_ATT: *p = st->att; *len = st->m->q_dim; return TB200_OK;
    case TB200_BUF_H: *p = st->h; *len = c.intermediate_size; return TB200_OK;
    case TB200_BUF_LOGITS: *p = st->logits; *len = c.vocab_size; return TB200_OK;
    case TB200_BUF_X2: *p = st->x2; *len = c.hidden_size; return TB200_OK;
    case TB200_BUF_PART: *p = st->part_o; *len = c.num_key_value_heads * c.hidden_size; return TB200_OK;
  }
  return fail(TB200_ERR_ARG, "unknown state buffer");
}

int tb200_state_read(tb200_state* st, int which, float* out, size_t n) {
  ARG_CHECK(st && out, "null argument");
  if (int rc = use(st->dev)) return rc;
  float* p;
  size_t len;
  if (int rc = state_buffer(st, which, &p, &len)) return rc;
  ARG_CHECK(n == len, "state buffer holds " + std::to_string(len) + " values, not " + std::to_string(n));
  CUDA_TRY(cudaMemcpyAsync(out, p, n * 4, cudaMemcpyDeviceToHost, st->dev->stream));
  CUDA_TRY(cudaStreamSynchronize(st->dev->stream));
  return TB200_OK;
}

int tb200_state_write(tb200_state* st, int which, const float* data, size_t n) {
  ARG_CHECK(st && data, "null argument");
  if (int rc = use(st->dev)) return rc;
  float* p;
  size_t len;
  if (int rc = state_buffer(st, which, &p, &len)) return rc;
  ARG_CHECK(n == len, "state buffer holds " + std::to_string(len) + " values, not " + std::to_string(n));
  CUDA_TRY(cudaMemcpyAsync(p, data, n * 4, cudaMemcpyHostToDevice, st->dev->stream));
  CUDA_TRY(cudaStreamSynchronize(st->dev->stream));
  return TB200_OK;
}

int tb200_state_set_position(tb200_state* st, uint32_t token, size_t pos) {
  ARG_CHECK(st, "null state");
  ARG_CHECK(st->n_seqs == 1, "the single-token path runs one-sequence states");
  ARG_CHECK(pos < st->max_len && token < st->m->c.vocab_size, "token or position out of range");
  if (int rc = use(st->dev)) return rc;
  tb::launch_set_io(st->dev->stream, st->io, int(token), int(pos));
  st->host_pos = pos;
  return launched("set_position");
}

int tb200_state_read_kv(tb200_state* st, size_t layer, int which, size_t pos, float* out) {
  ARG_CHECK(st && out, "null argument");
  const tb200_config& c = st->m->c;
  ARG_CHECK(layer < c.num_hidden_layers && pos < st->max_len && (which == 0 || which == 1), "out of range");
  if (int rc = use(st->m->dev)) return rc;
  cudaStream_t s = st->m->dev->stream;
  const size_t Hkv = c.num_key_value_heads, D = c.head_dim;
  const size_t kv_layer = 2 * Hkv * st->max_len * D;
  const size_t eb = st->kv_f32 ? 4 : 2;
  std::vector<unsigned char> tmp(Hkv * D * eb);
  for (size_t g = 0; g < Hkv; g++) {
    const unsigned char* src =
        st->kv + (layer * kv_layer + size_t(which) * (kv_layer / 2) + (g * st->max_len + pos) * D) * eb;
    CUDA_TRY(cudaMemcpyAsync(tmp.data() + g * D * eb, src, D * eb, cudaMemcpyDeviceToHost, s));
  }
  CUDA_TRY(cudaStreamSynchronize(s));
  for (size_t i = 0; i < Hkv * D; i++) {
    uint32_t u;
    if (st->kv_f32) {
      std::memcpy(&u, tmp.data() + 4 * i, 4);
    } else {
      uint16_t b;
      std::memcpy(&b, tmp.data() + 2 * i, 2);
      u = uint32_t(b) << 16;
    }
    std::memcpy(out + i, &u, 4);
  }
  return TB200_OK;
}

}  // extern "C"
