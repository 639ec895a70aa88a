// oracle.cpp — TEST INFRASTRUCTURE ONLY. Not part of the product.
//
// A C++ restatement of the Titania reference CPU path, used as the checker
// for the B200 kernels (tests, smoke check) and as the timed CPU baseline
// (bench.py's cpu_baseline leg and `--impl reference` arm). Nothing in the
// titania_b200 package links, imports or calls this file.
//
// Parity status: UNPINNED against the running reference. The reference is
// Rust (edition 2024) and needs cargo plus crates.io dependencies that this
// environment cannot fetch, and it ships no golden vectors. This file is a
// line-by-line restatement of the arithmetic in:
//   model/cpu.rs:9-193      every Device op, incl. the 8-lane dot order
//   model/model.rs:83-250   op sequence, BATCH chunking, last-token head,
//                           State buffers (f32 KV cache), rope_table
//   model/weights.rs:35-81  safetensors reader (BF16 only)
//   model/config.rs:10-35   config.json fields, head_dim default
//   model/sampler.rs:21-77  top-k / top-p / temperature sampling with
//                           the xorshift64* generator (greedy at T = 0)
// It is cross-checked bit-for-bit against an independent numpy restatement
// (tests/golden/gen_golden.py) on the reference's own op-test shapes and
// input generator (model/titania.rs:231-249, 319, 333, 346-359).
//
// Floating-point rules that make the restatement exact:
//  * compile with -ffp-contract=off: Rust never fuses `a += b * c` into an
//    FMA, so neither may we;
//  * Rust's `Iterator::sum` for f32 folds from -0.0 in order;
//  * transcendental calls go to glibc (expf, sqrtf, powf, sinf, cosf), which
//    is what Rust's std uses on x86_64 Linux;
//  * parallelism only where the reference uses rayon (matvec rows,
//    attention heads); the partitions are independent, so results do not
//    depend on the thread count.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ---------------------------------------------------------------------------
// Numerics helpers (model/cpu.rs:159-193)
// ---------------------------------------------------------------------------

// cpu.rs:159-161 — bf16 is the top half of an f32.
inline float bf16(uint16_t bits) {
  uint32_t u = uint32_t(bits) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// cpu.rs:167-177 — eight running sums over chunks of eight, summed in order,
// plus the (sequential) sum of a ragged tail.
float dot(const uint16_t* w, const float* x, size_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t done = n / 8 * 8;
  for (size_t c = 0; c < done; c += 8)
    for (int i = 0; i < 8; i++) acc[i] += bf16(w[c + i]) * x[c + i];
  float rest = -0.0f;
  for (size_t c = done; c < n; c++) rest += bf16(w[c]) * x[c];
  float s = -0.0f;
  for (int i = 0; i < 8; i++) s += acc[i];
  return s + rest;
}

// cpu.rs:179-181
float dot_f32(const float* a, const float* b, size_t n) {
  float s = -0.0f;
  for (size_t i = 0; i < n; i++) s += a[i] * b[i];
  return s;
}

// cpu.rs:183-193 — f32::max ignores NaN like fmaxf.
void softmax(float* x, size_t n) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; i++) mx = fmaxf(mx, x[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; i++) {
    x[i] = expf(x[i] - mx);
    sum += x[i];
  }
  for (size_t i = 0; i < n; i++) x[i] /= sum;
}

[[noreturn]] void panic(const std::string& msg) { throw std::runtime_error(msg); }

// ---------------------------------------------------------------------------
// Device ops (model/cpu.rs:9-156). Buffers are (pointer, len) pairs.
// ---------------------------------------------------------------------------

// cpu.rs:38-47
void op_embed(float* out, size_t out_len, const uint16_t* table, size_t dim, const uint32_t* tokens,
              size_t n) {
  if (out_len != n * dim) panic("embed: output length mismatch");
  for (size_t t = 0; t < n; t++) {
    const uint16_t* row = table + size_t(tokens[t]) * dim;
    for (size_t i = 0; i < dim; i++) out[t * dim + i] = bf16(row[i]);
  }
}

// cpu.rs:49-77. n==1 and n>1 compute the same dot per (row, token), so the
// transposition through `by_row` (cpu.rs:63-76) does not change any value.
void op_matmul(float* out, size_t out_len, const uint16_t* w, size_t rows, size_t cols, const float* x,
               size_t x_len) {
  size_t n = x_len / cols;
  if (x_len != n * cols) panic("matmul: input is not a whole number of rows");
  if (out_len != n * rows) panic("matmul: output length mismatch");
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; r++) {
    const uint16_t* row = w + size_t(r) * cols;
    for (size_t t = 0; t < n; t++) out[t * rows + r] = dot(row, x + t * cols, cols);
  }
}

// cpu.rs:79-83
void op_add(float* x, const float* y, size_t n) {
  for (size_t i = 0; i < n; i++) x[i] += y[i];
}

// cpu.rs:85-94
void op_rmsnorm(float* x, size_t x_len, const uint16_t* weight, size_t dim, float eps) {
  for (size_t r = 0; r + dim <= x_len; r += dim) {
    float* row = x + r;
    float ss = -0.0f;
    for (size_t i = 0; i < dim; i++) ss += row[i] * row[i];
    float mean_square = ss / float(dim);
    float scale = 1.0f / sqrtf(mean_square + eps);
    for (size_t i = 0; i < dim; i++) row[i] *= scale * bf16(weight[i]);
  }
}

// cpu.rs:96-111
void op_rope(float* x, size_t x_len, const float* table, size_t pos, size_t n_heads, size_t head_dim) {
  size_t half = head_dim / 2;
  size_t width = n_heads * head_dim;
  for (size_t t = 0; t * width + width <= x_len; t++) {
    const float* angles = table + (pos + t) * head_dim;
    for (size_t h = 0; h < n_heads; h++) {
      float* head = x + t * width + h * head_dim;
      for (size_t i = 0; i < half; i++) {
        float c = angles[2 * i], s = angles[2 * i + 1];
        float a = head[i], b = head[i + half];
        head[i] = a * c - b * s;
        head[i + half] = b * c + a * s;
      }
    }
  }
}

// cpu.rs:113-149
void op_attention(float* out, const float* q, size_t q_len, const float* k_cache, const float* v_cache,
                  size_t pos, size_t n_heads, size_t head_dim, size_t n_kv_heads) {
  size_t group = n_heads / n_kv_heads;
  size_t kv_dim = n_kv_heads * head_dim;
  float scale = 1.0f / sqrtf(float(head_dim));
  long long items = (long long)(q_len / head_dim);
#pragma omp parallel for schedule(dynamic, 1)
  for (long long i = 0; i < items; i++) {
    size_t token = size_t(i) / n_heads, head = size_t(i) % n_heads;
    size_t len = pos + token + 1;
    size_t kv = head / group * head_dim;
    const float* qh = q + size_t(i) * head_dim;
    std::vector<float> scores(len);
    for (size_t t = 0; t < len; t++) scores[t] = scale * dot_f32(qh, k_cache + t * kv_dim + kv, head_dim);
    softmax(scores.data(), len);
    float* o = out + size_t(i) * head_dim;
    for (size_t d = 0; d < head_dim; d++) o[d] = 0.0f;
    for (size_t t = 0; t < len; t++) {
      const float* v = v_cache + t * kv_dim + kv;
      for (size_t d = 0; d < head_dim; d++) o[d] += scores[t] * v[d];
    }
  }
}

// cpu.rs:151-155
void op_silu_mul(float* g, const float* u, size_t n) {
  for (size_t i = 0; i < n; i++) g[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
}

// model.rs:239-250
std::vector<float> rope_table(size_t max_len, size_t head_dim, float theta) {
  size_t half = head_dim / 2;
  std::vector<float> t;
  t.reserve(max_len * head_dim);
  for (size_t pos = 0; pos < max_len; pos++) {
    for (size_t i = 0; i < half; i++) {
      float freq = 1.0f / powf(theta, float(2 * i) / float(head_dim));
      float a = float(pos) * freq;
      t.push_back(cosf(a));
      t.push_back(sinf(a));
    }
  }
  return t;
}

// ---------------------------------------------------------------------------
// A minimal JSON reader for config.json and the safetensors header
// (model/config.rs:28-30 and model/weights.rs:45-50 use serde_json).
// ---------------------------------------------------------------------------

struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JsonParser {
  const char* p;
  const char* end;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
  }
  [[noreturn]] void fail() { panic("malformed JSON"); }
  std::string string() {
    if (p >= end || *p != '"') fail();
    p++;
    std::string s;
    while (p < end && *p != '"') {
      if (*p == '\\') {
        p++;
        if (p >= end) fail();
        char c = *p++;
        switch (c) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          case 'r': s += '\r'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'u': {
            if (end - p < 4) fail();
            unsigned v = std::strtoul(std::string(p, 4).c_str(), nullptr, 16);
            p += 4;
            if (v < 0x80) s += char(v);
            else if (v < 0x800) { s += char(0xC0 | (v >> 6)); s += char(0x80 | (v & 63)); }
            else { s += char(0xE0 | (v >> 12)); s += char(0x80 | ((v >> 6) & 63)); s += char(0x80 | (v & 63)); }
            break;
          }
          default: s += c;
        }
      } else {
        s += *p++;
      }
    }
    if (p >= end) fail();
    p++;
    return s;
  }
  Json value() {
    ws();
    if (p >= end) fail();
    Json j;
    if (*p == '{') {
      j.kind = Json::Obj;
      p++;
      ws();
      if (p < end && *p == '}') { p++; return j; }
      for (;;) {
        ws();
        std::string k = string();
        ws();
        if (p >= end || *p != ':') fail();
        p++;
        j.obj.emplace_back(k, value());
        ws();
        if (p < end && *p == ',') { p++; continue; }
        if (p < end && *p == '}') { p++; return j; }
        fail();
      }
    }
    if (*p == '[') {
      j.kind = Json::Arr;
      p++;
      ws();
      if (p < end && *p == ']') { p++; return j; }
      for (;;) {
        j.arr.push_back(value());
        ws();
        if (p < end && *p == ',') { p++; continue; }
        if (p < end && *p == ']') { p++; return j; }
        fail();
      }
    }
    if (*p == '"') { j.kind = Json::Str; j.str = string(); return j; }
    if (end - p >= 4 && !std::strncmp(p, "true", 4)) { j.kind = Json::Bool; j.b = true; p += 4; return j; }
    if (end - p >= 5 && !std::strncmp(p, "false", 5)) { j.kind = Json::Bool; p += 5; return j; }
    if (end - p >= 4 && !std::strncmp(p, "null", 4)) { p += 4; return j; }
    char* e = nullptr;
    std::string tmp(p, std::min<size_t>(64, size_t(end - p)));
    j.num = std::strtod(tmp.c_str(), &e);
    if (e == tmp.c_str()) fail();
    j.kind = Json::Num;
    p += (e - tmp.c_str());
    return j;
  }
};

Json parse_json(const std::string& s) {
  JsonParser jp{s.data(), s.data() + s.size()};
  return jp.value();
}

std::string read_file(const std::string& path) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) panic("can't open " + path);
  std::fseek(f, 0, SEEK_END);
  long size = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  std::string s(size_t(size > 0 ? size : 0), '\0');
  size_t got = size > 0 ? std::fread(&s[0], 1, s.size(), f) : 0;
  std::fclose(f);
  if (got != s.size()) panic("short read of " + path);
  return s;
}

// ---------------------------------------------------------------------------
// Config (model/config.rs:10-35)
// ---------------------------------------------------------------------------

struct Config {
  size_t hidden_size, intermediate_size, num_hidden_layers, num_attention_heads, num_key_value_heads;
  size_t head_dim_opt = 0;  // 0 = absent
  float rms_norm_eps, rope_theta;
  size_t vocab_size;
  bool tie_word_embeddings = false;
  size_t head_dim() const { return head_dim_opt ? head_dim_opt : hidden_size / num_attention_heads; }
};

Config load_config(const std::string& path) {
  Json j = parse_json(read_file(path));
  auto need = [&](const char* k) -> const Json& {
    const Json* v = j.get(k);
    if (!v || v->kind != Json::Num) panic(std::string("config.json: missing field ") + k);
    return *v;
  };
  Config c;
  c.hidden_size = size_t(need("hidden_size").num);
  c.intermediate_size = size_t(need("intermediate_size").num);
  c.num_hidden_layers = size_t(need("num_hidden_layers").num);
  c.num_attention_heads = size_t(need("num_attention_heads").num);
  c.num_key_value_heads = size_t(need("num_key_value_heads").num);
  if (const Json* h = j.get("head_dim"); h && h->kind == Json::Num) c.head_dim_opt = size_t(h->num);
  c.rms_norm_eps = float(need("rms_norm_eps").num);
  c.rope_theta = float(need("rope_theta").num);
  c.vocab_size = size_t(need("vocab_size").num);
  if (const Json* t = j.get("tie_word_embeddings"); t && t->kind == Json::Bool) c.tie_word_embeddings = t->b;
  return c;
}

// ---------------------------------------------------------------------------
// Weights (model/weights.rs:14-81)
// ---------------------------------------------------------------------------

struct Tensor {
  std::vector<size_t> shape;
  std::vector<uint16_t> data;
};

struct Weights {
  std::string blob;  // whole file; the reference seeks per tensor instead
  size_t data_start = 0;
  struct Entry {
    std::string dtype;
    std::vector<size_t> shape;
    uint64_t start, end;
  };
  std::map<std::string, Entry> entries;

  explicit Weights(const std::string& path) {
    blob = read_file(path);
    if (blob.size() < 8) panic("safetensors: file too short");
    uint64_t len = 0;
    for (int i = 7; i >= 0; i--) len = (len << 8) | uint8_t(blob[i]);
    if (8 + len > blob.size()) panic("safetensors: header past end of file");
    Json h = parse_json(blob.substr(8, len));
    for (auto& kv : h.obj) {
      if (kv.first == "__metadata__") continue;
      Entry e;
      const Json* dt = kv.second.get("dtype");
      const Json* sh = kv.second.get("shape");
      const Json* off = kv.second.get("data_offsets");
      if (!dt || !sh || !off || off->arr.size() != 2) panic("safetensors: bad entry " + kv.first);
      e.dtype = dt->str;
      for (auto& d : sh->arr) e.shape.push_back(size_t(d.num));
      e.start = uint64_t(off->arr[0].num);
      e.end = uint64_t(off->arr[1].num);
      entries[kv.first] = e;
    }
    data_start = 8 + len;
  }
  bool contains(const std::string& name) const { return entries.count(name) != 0; }
  Tensor read(const std::string& name) const {
    auto it = entries.find(name);
    if (it == entries.end()) panic("missing tensor '" + name + "'");
    const Entry& e = it->second;
    if (e.dtype != "BF16") panic("tensor '" + name + "' is " + e.dtype + ", expected BF16");
    if (data_start + e.end > blob.size() || e.end < e.start) panic("tensor '" + name + "' past end of file");
    Tensor t;
    t.shape = e.shape;
    t.data.resize((e.end - e.start) / 2);
    const unsigned char* b = reinterpret_cast<const unsigned char*>(blob.data() + data_start + e.start);
    for (size_t i = 0; i < t.data.size(); i++) t.data[i] = uint16_t(b[2 * i] | (b[2 * i + 1] << 8));
    return t;
  }
};

// ---------------------------------------------------------------------------
// Model and State (model/model.rs:8-250)
// ---------------------------------------------------------------------------

constexpr size_t BATCH = 64;  // model.rs:8

struct Layer {
  Tensor attn_norm, q, k, v, o, mlp_norm, gate, up, down;
  bool has_q_norm = false, has_k_norm = false;
  Tensor q_norm, k_norm;
};

struct Model {
  Config c;
  Tensor embed, norm, lm_head;
  bool has_lm_head = false;
  std::vector<Layer> layers;
};

// A buffer with the reference's length/capacity behaviour (cpu.rs:17-24).
struct Buf {
  std::vector<float> v;
  size_t len = 0;
  void alloc(size_t n) { v.assign(n, 0.0f); len = n; }
  void resize(size_t n) {
    if (n > v.size()) panic("a buffer can't hold that many activations");
    for (size_t i = len; i < n; i++) v[i] = 0.0f;  // Vec::resize fills with 0.0
    len = n;
  }
  float* p() { return v.data(); }
};

struct State {
  size_t widths[8];
  Buf x, xb, q, k, v, att, gate, up, logits, rope;
  std::vector<Buf> k_cache, v_cache;
  size_t max_len;
};

Model* load_model(const std::string& dir) {
  auto m = std::make_unique<Model>();
  m->c = load_config(dir + "/config.json");
  Weights w(dir + "/model.safetensors");
  for (size_t i = 0; i < m->c.num_hidden_layers; i++) {
    std::string p = "model.layers." + std::to_string(i);
    Layer L;
    L.attn_norm = w.read(p + ".input_layernorm.weight");
    L.q = w.read(p + ".self_attn.q_proj.weight");
    L.k = w.read(p + ".self_attn.k_proj.weight");
    L.v = w.read(p + ".self_attn.v_proj.weight");
    L.o = w.read(p + ".self_attn.o_proj.weight");
    if (w.contains(p + ".self_attn.q_norm.weight")) { L.q_norm = w.read(p + ".self_attn.q_norm.weight"); L.has_q_norm = true; }
    if (w.contains(p + ".self_attn.k_norm.weight")) { L.k_norm = w.read(p + ".self_attn.k_norm.weight"); L.has_k_norm = true; }
    L.mlp_norm = w.read(p + ".post_attention_layernorm.weight");
    L.gate = w.read(p + ".mlp.gate_proj.weight");
    L.up = w.read(p + ".mlp.up_proj.weight");
    L.down = w.read(p + ".mlp.down_proj.weight");
    m->layers.push_back(std::move(L));
  }
  if (!m->c.tie_word_embeddings) { m->lm_head = w.read("lm_head.weight"); m->has_lm_head = true; }
  m->embed = w.read("model.embed_tokens.weight");
  m->norm = w.read("model.norm.weight");
  return m.release();
}

State* new_state(const Model& m, size_t max_len) {
  const Config& c = m.c;
  auto s = std::make_unique<State>();
  size_t q_dim = c.num_attention_heads * c.head_dim();
  size_t kv_dim = c.num_key_value_heads * c.head_dim();
  size_t widths[8] = {c.hidden_size, c.hidden_size, q_dim, kv_dim, kv_dim, q_dim, c.intermediate_size,
                      c.intermediate_size};
  std::memcpy(s->widths, widths, sizeof widths);
  Buf* bufs[8] = {&s->x, &s->xb, &s->q, &s->k, &s->v, &s->att, &s->gate, &s->up};
  for (int i = 0; i < 8; i++) bufs[i]->alloc(BATCH * widths[i]);
  std::vector<float> table = rope_table(max_len, c.head_dim(), c.rope_theta);
  s->rope.alloc(table.size());
  std::memcpy(s->rope.p(), table.data(), table.size() * 4);
  s->logits.alloc(c.vocab_size);
  s->k_cache.resize(c.num_hidden_layers);
  s->v_cache.resize(c.num_hidden_layers);
  for (size_t i = 0; i < c.num_hidden_layers; i++) {
    s->k_cache[i].alloc(max_len * kv_dim);
    s->v_cache[i].alloc(max_len * kv_dim);
  }
  s->max_len = max_len;
  return s.release();
}

void matmul(Buf& out, const Tensor& w, Buf& x) {
  op_matmul(out.p(), out.len, w.data.data(), w.shape[0], w.shape[1], x.p(), x.len);
}
void rmsnorm(Buf& x, const Tensor& w, float eps) { op_rmsnorm(x.p(), x.len, w.data.data(), w.data.size(), eps); }
void copy(Buf& dst, size_t doff, Buf& src, size_t soff, size_t len) {
  if (doff + len > dst.len || soff + len > src.len) panic("copy out of range");
  std::memmove(dst.p() + doff, src.p() + soff, len * 4);
}

// model.rs:93-149
void forward_batch(const Model& m, State& s, const uint32_t* tokens, size_t n, size_t pos, float* logits_out) {
  const Config& c = m.c;
  float eps = c.rms_norm_eps;
  size_t head_dim = c.head_dim();
  size_t kv_dim = c.num_key_value_heads * head_dim;
  if (n > BATCH) panic("a batch of more than BATCH tokens");
  Buf* bufs[8] = {&s.x, &s.xb, &s.q, &s.k, &s.v, &s.att, &s.gate, &s.up};
  for (int i = 0; i < 8; i++) bufs[i]->resize(n * s.widths[i]);

  op_embed(s.x.p(), s.x.len, m.embed.data.data(), m.embed.shape[1], tokens, n);
  for (size_t i = 0; i < c.num_hidden_layers; i++) {
    const Layer& L = m.layers[i];
    copy(s.xb, 0, s.x, 0, n * c.hidden_size);
    rmsnorm(s.xb, L.attn_norm, eps);
    matmul(s.q, L.q, s.xb);
    matmul(s.k, L.k, s.xb);
    matmul(s.v, L.v, s.xb);
    if (L.has_q_norm) rmsnorm(s.q, L.q_norm, eps);
    if (L.has_k_norm) rmsnorm(s.k, L.k_norm, eps);
    op_rope(s.q.p(), s.q.len, s.rope.p(), pos, c.num_attention_heads, head_dim);
    op_rope(s.k.p(), s.k.len, s.rope.p(), pos, c.num_key_value_heads, head_dim);
    copy(s.k_cache[i], pos * kv_dim, s.k, 0, n * kv_dim);
    copy(s.v_cache[i], pos * kv_dim, s.v, 0, n * kv_dim);
    op_attention(s.att.p(), s.q.p(), s.q.len, s.k_cache[i].p(), s.v_cache[i].p(), pos, c.num_attention_heads,
                 head_dim, c.num_key_value_heads);
    matmul(s.xb, L.o, s.att);
    op_add(s.x.p(), s.xb.p(), s.x.len);
    copy(s.xb, 0, s.x, 0, n * c.hidden_size);
    rmsnorm(s.xb, L.mlp_norm, eps);
    matmul(s.gate, L.gate, s.xb);
    matmul(s.up, L.up, s.xb);
    op_silu_mul(s.gate.p(), s.up.p(), s.gate.len);
    matmul(s.xb, L.down, s.gate);
    op_add(s.x.p(), s.xb.p(), s.x.len);
  }
  s.xb.resize(c.hidden_size);
  copy(s.xb, 0, s.x, (n - 1) * c.hidden_size, c.hidden_size);
  rmsnorm(s.xb, m.norm, eps);
  matmul(s.logits, m.has_lm_head ? m.lm_head : m.embed, s.xb);
  std::memcpy(logits_out, s.logits.p(), s.logits.len * 4);
}

// model.rs:83-91
void forward(const Model& m, State& s, const uint32_t* tokens, size_t n, size_t pos, float* logits_out) {
  if (n == 0) panic("no tokens to run");
  if (pos + n > s.max_len) panic("tokens past the end of the cache");
  for (size_t i = 0; i * BATCH < n; i++) {
    size_t len = std::min(BATCH, n - i * BATCH);
    forward_batch(m, s, tokens + i * BATCH, len, pos + i * BATCH, logits_out);
  }
}

// Rust's f32::total_cmp key: flips the magnitude bits of negatives so that
// signed integer order is the IEEE total order.
inline int32_t total_key(float f) {
  int32_t b;
  std::memcpy(&b, &f, 4);
  return b ^ int32_t(uint32_t(b >> 31) >> 1);
}

thread_local std::string g_err;

}  // namespace

// ---------------------------------------------------------------------------
// C ABI used by the tests and by bench.py's CPU baseline.
// Every function returns 0 on success, nonzero after a reference panic (the
// message is kept for orc_last_error).
// ---------------------------------------------------------------------------

#define ORC_TRY(body)                      \
  try {                                    \
    body;                                  \
    return 0;                              \
  } catch (const std::exception& e) {      \
    g_err = e.what();                      \
    return 1;                              \
  }

extern "C" {

const char* orc_last_error() { return g_err.c_str(); }

void orc_set_threads(int n) {
#ifdef _OPENMP
  omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int orc_max_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

int orc_embed(float* out, size_t out_len, const uint16_t* table, size_t dim, const uint32_t* tokens, size_t n) {
  ORC_TRY(op_embed(out, out_len, table, dim, tokens, n))
}
int orc_matmul(float* out, size_t out_len, const uint16_t* w, size_t rows, size_t cols, const float* x,
               size_t x_len) {
  ORC_TRY(op_matmul(out, out_len, w, rows, cols, x, x_len))
}
int orc_add(float* x, const float* y, size_t n) { ORC_TRY(op_add(x, y, n)) }
int orc_rmsnorm(float* x, size_t x_len, const uint16_t* w, size_t dim, float eps) {
  ORC_TRY(op_rmsnorm(x, x_len, w, dim, eps))
}
int orc_rope(float* x, size_t x_len, const float* table, size_t pos, size_t n_heads, size_t head_dim) {
  ORC_TRY(op_rope(x, x_len, table, pos, n_heads, head_dim))
}
int orc_attention(float* out, const float* q, size_t q_len, const float* k, const float* v, size_t pos,
                  size_t n_heads, size_t head_dim, size_t n_kv_heads) {
  ORC_TRY(op_attention(out, q, q_len, k, v, pos, n_heads, head_dim, n_kv_heads))
}
int orc_silu_mul(float* g, const float* u, size_t n) { ORC_TRY(op_silu_mul(g, u, n)) }
int orc_rope_table(float* out, size_t max_len, size_t head_dim, float theta) {
  ORC_TRY({
    std::vector<float> t = rope_table(max_len, head_dim, theta);
    std::memcpy(out, t.data(), t.size() * 4);
  })
}

// sampler.rs:21-33 at temperature 0: the candidate with the largest logit
// under total_cmp. The reference leaves exact ties to an unstable selection;
// this restatement breaks them toward the lowest token id.
uint32_t orc_sample_greedy(const float* logits, size_t n) {
  size_t best = 0;
  for (size_t i = 1; i < n; i++)
    if (total_key(logits[i]) > total_key(logits[best])) best = i;
  return uint32_t(best);
}

// sampler.rs:21-59 (Sampler::sample) with its xorshift64* generator
// (sampler.rs:63-77), one call per token; *rng is the generator state (the
// reference starts it at max(seed, 1)). The top-k candidates are the k
// largest logits under total_cmp in descending order; exact ties (which the
// reference leaves to an unstable selection) go to the lowest token id.
// Every float step is the reference's, in its order: (logit - max) / T, expf,
// a sequential f32 sum, p / sum, the running total while it is below top_p,
// then r = next_f32() * total and r -= p until r <= 0.
uint32_t orc_sample(const float* logits, size_t n, float temperature, size_t top_k, float top_p, uint64_t* rng) {
  const size_t k = top_k < 1 ? 1 : (top_k > n ? n : top_k);
  std::vector<uint32_t> idx(n);
  for (size_t i = 0; i < n; i++) idx[i] = uint32_t(i);
  auto better = [&](uint32_t a, uint32_t b) {
    const int64_t ka = total_key(logits[a]), kb = total_key(logits[b]);
    return ka != kb ? ka > kb : a < b;
  };
  std::partial_sort(idx.begin(), idx.begin() + k, idx.end(), better);
  if (temperature == 0.0f) return idx[0];
  const float max = logits[idx[0]];
  std::vector<float> probs(k);
  for (size_t i = 0; i < k; i++) probs[i] = expf((logits[idx[i]] - max) / temperature);
  float sum = -0.0f;
  for (size_t i = 0; i < k; i++) sum += probs[i];
  float cumulative = 0.0f;
  size_t m = 0;
  for (size_t i = 0; i < k; i++) {
    probs[i] /= sum;
    if (cumulative < top_p) {
      cumulative += probs[i];
      m++;
    }
  }
  uint64_t x = *rng;
  x ^= x >> 12;
  x ^= x << 25;
  x ^= x >> 27;
  *rng = x;
  const float u = float((x * 0x2545F4914F6CDD1DULL) >> 40) / float(1u << 24);
  float r = u * cumulative;
  for (size_t i = 0; i < m; i++) {
    r -= probs[i];
    if (r <= 0.0f) return idx[i];
  }
  return idx[m > 0 ? m - 1 : 0];  // m == 0 (top_p <= 0) panics in the reference
}

void* orc_model_load(const char* dir) {
  try {
    return load_model(dir);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}
void orc_model_free(void* m) { delete static_cast<Model*>(m); }
int orc_model_dims(void* mp, size_t* out /* [hidden, inter, layers, heads, kv_heads, head_dim, vocab] */) {
  const Config& c = static_cast<Model*>(mp)->c;
  size_t v[7] = {c.hidden_size, c.intermediate_size, c.num_hidden_layers, c.num_attention_heads,
                 c.num_key_value_heads, c.head_dim(), c.vocab_size};
  std::memcpy(out, v, sizeof v);
  return 0;
}

void* orc_state_new(void* m, size_t max_len) {
  try {
    return new_state(*static_cast<Model*>(m), max_len);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}
void orc_state_free(void* s) { delete static_cast<State*>(s); }

int orc_forward(void* m, void* s, const uint32_t* tokens, size_t n, size_t pos, float* logits) {
  ORC_TRY(forward(*static_cast<Model*>(m), *static_cast<State*>(s), tokens, n, pos, logits))
}

// Reads layer `layer`'s key or value cache rows [0, len) (f32) for tests.
int orc_state_kv(void* sp, size_t layer, int which, float* out, size_t len) {
  ORC_TRY({
    State& s = *static_cast<State*>(sp);
    if (layer >= s.k_cache.size()) panic("layer out of range");
    Buf& b = which ? s.v_cache[layer] : s.k_cache[layer];
    if (len > b.len) panic("length out of range");
    std::memcpy(out, b.p(), len * 4);
  })
}

}  // extern "C"
