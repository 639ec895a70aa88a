// forward.cu — the many-token and many-sequence paths of the C ABI:
//
//   prompts     Model::forward (model/model.rs:83-91) over n >= 2 tokens of
//               one sequence: every token of a pass at once through the
//               tensor-core contractions (gemm.cu) and the tiled causal
//               attention (batch.cu). The reference cuts prompts into chunks
//               of BATCH = 64 tokens (model.rs:86-89); a pass here takes up
//               to `cap` tokens, which changes nothing but speed: every
//               token's result depends only on the tokens before it.
//   batches     one decode step of every sequence of a state at once (each
//               sequence with its own cache and position, as many
//               independent Model::forward calls would run), captured as a
//               CUDA graph, and a greedy token loop on the device.
//
// A pass over T tokens (model.rs:100-147), five kernels per layer:
//   embed: x, and the first RMSNorm's input (planes of x * w, sums of squares)
//   gemm(qkv, xn) * norm scale, QK-norm, RoPE  -> q, cache
//   attention(q, cache)                        -> att (three planes)
//   gemm(o, att): x += o, the MLP norm's input  -> xn, sums of squares
//   gemm(gate|up, xn) * norm scale, silu * up   -> h
//   gemm(down, h): x += d, the next norm's input -> xn, sums of squares
// then lm_head (* the final norm's scale, argmax keys folded in) and the
// greedy choice for the rows that need logits. Each RMSNorm (cpu.rs:85-94)
// is split between the kernel that produces its input (x * w and per-tile
// sums of squares) and the contraction that consumes it (the per-token
// scale applied to the accumulator). Tensor parallel runs the norms as
// kernels of their own, after the all-reduce of the partial sums.

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>

#include "runtime.h"

using rt::fail;
using rt::launched;
using rt::use;

namespace {

bool use_pdl() {
  // TB200_SERIAL=1: launch without programmatic dependent launch (a
  // diagnostic for ordering questions; slower, otherwise identical).
  static const bool pdl = !(getenv("TB200_SERIAL") && getenv("TB200_SERIAL")[0] == '1');
  return pdl;
}

size_t round_up(size_t x, size_t m) { return (x + m - 1) / m * m; }

int* meta_tok(tb200_state* st) { return st->bmeta; }
int* meta_pos(tb200_state* st) { return st->bmeta + st->cap; }
int* meta_seq(tb200_state* st) { return st->bmeta + 2 * st->cap; }

// Width of an operand of the contractions (kOp*).
size_t width(const tb200_state* st, int op) {
  const tb200_model* m = st->m;
  return op == kOpXn ? m->c.hidden_size : op == kOpAtt ? m->q_dim : m->c.intermediate_size;
}
// Elements between an operand's three planes.
size_t plane(const tb200_state* st, int op) { return size_t(st->cap) * width(st, op); }
// An operand's first plane.
uint16_t* operand(tb200_state* st, int op) {
  uint16_t* p = st->bact;
  for (int i = 0; i < op; i++) p += 3 * plane(st, i);
  return p;
}

// Allocates the many-token workspace on first use.
int ensure_batch(tb200_state* st) {
  if (st->cap) return TB200_OK;
  tb200_model* m = st->m;
  const tb200_config& c = m->c;
  const size_t H = c.hidden_size, F = c.intermediate_size, V = c.vocab_size, D = c.head_dim;
  const size_t Hkv = c.num_key_value_heads, group = c.num_attention_heads / Hkv;
  ARG_CHECK(tb::batch_group_supported(int(group)), "the many-token path needs 1, 2, 4 or 8 query heads per kv head");
  const size_t cap = round_up(std::max(st->n_seqs, std::min<size_t>(st->max_len, 1024)), 128);
  const size_t qkv_w = m->q_dim + 2 * m->kv_dim;
  const size_t parts = size_t(tb::attn_rows_parts(int(st->n_seqs), int(Hkv), int(st->max_len), st->kv_f32 != 0,
                                                      m->dev->sms));
  cudaStream_t s = m->dev->stream;
  cudaError_t e = cudaSuccess;
  auto A = [&](void** p, size_t bytes) {
    if (e == cudaSuccess) e = cudaMalloc(p, bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(*p, 0, bytes, s);
  };
  st->cap = int(cap);
  A((void**)&st->bx, cap * H * 4);
  A((void**)&st->bqkv, cap * qkv_w * 4);
  if (m->tp) A((void**)&st->bpart, cap * H * 4);
  const size_t hparts = std::max<size_t>(1, (H + 127) / 128);
  A((void**)&st->ssq_a, cap * hparts * 4);
  A((void**)&st->ssq_b, cap * hparts * 4);
  A((void**)&st->blogits, st->n_seqs * V * 4);
  A((void**)&st->bact, 3 * cap * (H + m->q_dim + F) * 2);
  A((void**)&st->bmeta, 3 * cap * 4);
  A((void**)&st->rows_part, st->n_seqs * Hkv * parts * group * tb::kPartStride * 4);
  A((void**)&st->rows_ticket, st->n_seqs * Hkv * 4);
  A((void**)&st->bstep, 4 * 4);
  A((void**)&st->bbest, st->n_seqs * 8);
  A((void**)&st->bout, st->max_len * st->n_seqs * 4);
  // Staging: a region per prompt position (passes of one call never share
  // one), then a decode step's rows.
  if (e == cudaSuccess)
    e = cudaHostAlloc((void**)&st->bmeta_host, (3 * (st->max_len + cap) + 3 * cap + 16) * sizeof(int),
                      cudaHostAllocDefault);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    rt::free_batch(st);
    return fail(TB200_ERR_CUDA, std::string("batch workspace: ") + cudaGetErrorString(e));
  }
  st->rows_parts = int(parts);
  if (!st->kv_f32) {
    std::string why;
    const size_t rows = st->n_seqs * st->seq_stride / D;
    if (int rc = tb::encode_tmap_bf16(&st->cache_map, st->kv, rows, D, tb::attn_cache_box_rows(), &why)) {
      rt::free_batch(st);
      return fail(rc, "batch workspace: " + why);
    }
    st->has_cache_map = true;
  }
  for (int op = 0; op < kOps; op++)
    for (int pl = 0; pl < 3; pl++) {
      std::string why;
      uint16_t* base = operand(st, op) + pl * plane(st, op);
      if (int rc = tb::encode_tmap_bf16(&st->act[op][pl], base, cap, width(st, op), tb::gemm_box_rows(), &why)) {
        rt::free_batch(st);
        return fail(rc, "batch workspace: " + why);
      }
    }
  return TB200_OK;
}

// Host words the kernels' results are read back into.
int* readback(tb200_state* st) { return st->bmeta_host + 3 * (st->max_len + size_t(st->cap)) + 3 * size_t(st->cap); }

// One contraction over T rows: weights `w`, activation operand `op`; the
// kGemmSilu epilogue writes operand kOpH.
// Trace slots for a launch of `ctas` CTAs (kTraceEvents each) while a
// traced graph is captured; no slots otherwise.
tb::TraceAt trace_slots(tb200_state* st, bool on, int op, size_t layer, uint32_t ctas) {
  if (!on || !st->trace.rec) return tb::TraceAt{};
  tb::TraceAt t{st->trace, st->trace_next, (uint32_t(op) << 16) | uint32_t(layer)};
  st->trace_next += ctas * tb::kTraceEvents;
  return t;
}

void gemm(tb200_state* st, int T, int M, int K, const CUtensorMap& w, int op, int epi, float* out, int ldo,
          bool pdl, unsigned long long* best = nullptr, bool traced = false, int top = 0, size_t layer = 0,
          const tb::GemmArgs* extra = nullptr) {
  tb200_device* d = st->dev;
  const tb::GemmPlan p = tb::plan_gemm(M, K, T, d->sms, d->max_cluster);
  tb::GemmArgs a = extra ? *extra : tb::GemmArgs{};
  a.M = M;
  a.K = K;
  a.T = T;
  a.out = out;
  a.ldo = ldo;
  if (epi == tb::kGemmSilu) {
    a.out_split = operand(st, kOpH);
    a.plane = plane(st, kOpH);
    a.ldh = int(width(st, kOpH));
  }
  a.err = st->io + 3;
  a.best = best;
  a.trace = trace_slots(st, traced, top, layer, p.grid.x * p.grid.y * p.grid.z);
  tb::launch_gemm(d->stream, p, epi, w, st->act[op], a, pdl);
}

// The transformer layers over T rows whose token, position and sequence are
// in bmeta. prefill: the rows are tokens pos0 .. pos0 + T - 1 of sequence
// `seq`; otherwise each row is one token of its own sequence.
int enqueue_layers(tb200_state* st, int T, bool prefill, size_t seq, size_t pos0, bool pdl) {
  tb200_model* m = st->m;
  const tb200_config& c = m->c;
  cudaStream_t s = m->dev->stream;
  const int H = int(c.hidden_size), F = int(c.intermediate_size);
  const int qkv_w = int(m->q_dim + 2 * m->kv_dim), qd = int(m->q_dim);
  const int group = int(c.num_attention_heads / c.num_key_value_heads);
  const int hparts = std::max(1, (H + 127) / 128);
  const size_t eb = st->kv_f32 ? 4 : 2;
  const size_t kv_layer = 2 * c.num_key_value_heads * st->max_len * c.head_dim;
  int* err = st->io + 3;
  const bool tr = !prefill;  // the batched step is traced (its graph is captured once)
  const bool fused = !m->tp;  // RMSNorms folded into the contractions (tensor parallel adds partials first)
  uint16_t* xn = operand(st, kOpXn);
  uint16_t* att = operand(st, kOpAtt);
  const size_t xn_plane = plane(st, kOpXn), att_plane = plane(st, kOpAtt);
  if (fused)
    tb::launch_embed_split(s, st->bx, m->embed, H, meta_tok(st), int(c.vocab_size), m->layers[0].attn_norm, xn,
                           xn_plane, st->ssq_a, err, T, pdl, trace_slots(st, tr, TB200_TRACE_OP_EMBED, 0, uint32_t(T)));
  else
    tb::launch_embed(s, st->bx, m->embed, c.hidden_size, reinterpret_cast<const uint32_t*>(meta_tok(st)), size_t(T));
  for (size_t l = 0; l < c.num_hidden_layers; l++) {
    const FusedLayer& L = m->layers[l];
    // q|k|v with QK-norm, RoPE and the cache append in its epilogue.
    tb::GemmArgs q{};
    q.eps = c.rms_norm_eps;
    q.q_norm = L.q_norm;
    q.k_norm = L.k_norm;
    q.rope = st->rope;
    q.kv = st->kv + l * kv_layer * eb;
    q.seq_stride = st->seq_stride;
    q.kv_f32 = st->kv_f32;
    q.max_len = int(st->max_len);
    q.n_heads = int(c.num_attention_heads);
    q.n_kv_heads = int(c.num_key_value_heads);
    q.n_seqs = int(st->n_seqs);
    q.tok_pos = meta_pos(st);
    q.tok_seq = meta_seq(st);
    if (fused) {
      q.in_ssq = st->ssq_a;
      q.in_parts = l == 0 ? 1 : hparts;
      q.in_dim = H;
    } else {
      // Tensor parallel: the previous layer's reduced down_proj partial joins x here.
      tb::launch_norm_split(s, st->bx, l > 0 ? st->bpart : nullptr, 0, T, H, L.attn_norm, c.rms_norm_eps, xn,
                            xn_plane, pdl, trace_slots(st, tr, TB200_TRACE_OP_NORM, l, uint32_t(T)));
    }
    gemm(st, T, qkv_w, H, L.m_qkv, kOpXn, tb::kGemmQkv, st->bqkv, qkv_w, pdl, nullptr, tr, TB200_TRACE_OP_QKV, l, &q);
    if (prefill) {
      tb::AttnPrefillArgs a{};
      a.q = st->bqkv;
      a.ldq = qkv_w;
      a.kv = st->kv + (seq * st->seq_stride + l * kv_layer) * eb;
      a.kv_f32 = st->kv_f32;
      a.max_len = int(st->max_len);
      a.n_kv_heads = int(c.num_key_value_heads);
      a.T = T;
      a.pos0 = int(pos0);
      a.out = att;
      a.plane = att_plane;
      a.ldo = qd;
      tb::launch_attn_prefill(s, a, group, pdl);
    } else {
      tb::AttnRowsArgs a{};
      a.q = st->bqkv;
      a.ldq = qkv_w;
      a.kv = st->kv + l * kv_layer * eb;
      a.seq_stride = st->seq_stride;
      a.kv_f32 = st->kv_f32;
      a.max_len = int(st->max_len);
      a.n_kv_heads = int(c.num_key_value_heads);
      a.n_seqs = int(st->n_seqs);
      a.pos = meta_pos(st);
      a.seq = meta_seq(st);
      a.out = att;
      a.plane = att_plane;
      a.ldo = qd;
      a.part = st->rows_part;
      a.ticket = st->rows_ticket;
      a.parts = st->rows_parts;
      a.err = err;
      a.cache_map = st->has_cache_map ? &st->cache_map : nullptr;
      a.layer_rows = int(l * kv_layer / c.head_dim);
      a.trace = trace_slots(st, tr, TB200_TRACE_OP_ATTENTION, l,
                            uint32_t(a.parts) * uint32_t(c.num_key_value_heads) * uint32_t(T));
      tb::launch_attn_rows(s, a, T, group, pdl);
    }
    if (fused) {
      // x += o_proj; then the MLP RMSNorm's input (planes of x * w, sums of squares).
      tb::GemmArgs o{};
      o.next_w = L.mlp_norm;
      o.next_split = xn;
      o.next_plane = xn_plane;
      o.out_ssq = st->ssq_b;
      gemm(st, T, H, qd, L.m_o, kOpAtt, tb::kGemmResidNorm, st->bx, H, pdl, nullptr, tr, TB200_TRACE_OP_O, l, &o);
      tb::GemmArgs gu{};
      gu.in_ssq = st->ssq_b;
      gu.in_parts = hparts;
      gu.in_dim = H;
      gu.eps = c.rms_norm_eps;
      gemm(st, T, 2 * F, H, L.m_gu, kOpXn, tb::kGemmSilu, nullptr, 0, pdl, nullptr, tr, TB200_TRACE_OP_GATE_UP, l,
           &gu);
      // x += down_proj; then the next layer's (or the final) RMSNorm's input.
      tb::GemmArgs dn{};
      dn.next_w = l + 1 < c.num_hidden_layers ? m->layers[l + 1].attn_norm : m->norm;
      dn.next_split = xn;
      dn.next_plane = xn_plane;
      dn.out_ssq = st->ssq_a;
      gemm(st, T, H, F, L.m_down, kOpH, tb::kGemmResidNorm, st->bx, H, pdl, nullptr, tr, TB200_TRACE_OP_DOWN, l,
           &dn);
    } else {  // partial sums, reduced over the group, added to x by the norm
      gemm(st, T, H, qd, L.m_o, kOpAtt, tb::kGemmStore, st->bpart, H, pdl, nullptr, tr, TB200_TRACE_OP_O, l);
      if (int rc = rt::tp_allreduce(m->tp, st->bpart, size_t(T) * H, s)) return rc;
      tb::launch_norm_split(s, st->bx, st->bpart, 0, T, H, L.mlp_norm, c.rms_norm_eps, xn, xn_plane, pdl,
                            trace_slots(st, tr, TB200_TRACE_OP_NORM2, l, uint32_t(T)));
      gemm(st, T, 2 * F, H, L.m_gu, kOpXn, tb::kGemmSilu, nullptr, 0, pdl, nullptr, tr, TB200_TRACE_OP_GATE_UP, l);
      gemm(st, T, H, F, L.m_down, kOpH, tb::kGemmStore, st->bpart, H, pdl, nullptr, tr, TB200_TRACE_OP_DOWN, l);
      if (int rc = rt::tp_allreduce(m->tp, st->bpart, size_t(T) * H, s)) return rc;
    }
  }
  return TB200_OK;
}

// Final norm, lm_head and greedy choice for rows row0 .. row0 + rows - 1 of
// the pass (model.rs:144-147); logits land in blogits rows 0 .. rows - 1.
// The contraction folds each row's argmax key into bbest as it stores the
// logits; a one-CTA kernel turns the keys into token ids.
void enqueue_head(tb200_state* st, int row0, int rows, tb::ArgmaxRowsArgs am, bool pdl, bool tr) {
  tb200_model* m = st->m;
  const tb200_config& c = m->c;
  const int H = int(c.hidden_size), V = int(c.vocab_size);
  cudaStream_t s = m->dev->stream;
  tb::GemmArgs h{};
  if (m->tp) {
    tb::launch_norm_split(s, st->bx, st->bpart, row0, rows, H, m->norm, c.rms_norm_eps, operand(st, kOpXn),
                          plane(st, kOpXn), pdl, trace_slots(st, tr, TB200_TRACE_OP_FINAL_NORM, 0, uint32_t(rows)));
  } else {
    // The last down_proj left x * w_final as planes at rows row0 ..; the scale comes from the sums of squares.
    h.in_ssq = st->ssq_a;
    h.in_parts = std::max(1, (H + 127) / 128);
    h.in_dim = H;
    h.eps = c.rms_norm_eps;
    h.act_row0 = row0;
  }
  gemm(st, rows, V, H, m->m_lm, kOpXn, tb::kGemmStore, st->blogits, V, pdl, st->bbest, tr, TB200_TRACE_OP_LM_HEAD, 0,
       &h);
  am.err = st->io + 3;
  am.trace = trace_slots(st, tr, TB200_TRACE_OP_ARGMAX, 0, 1);
  tb::launch_argmax_finish(s, am, st->bbest, rows, pdl);
}

// One decode step of every sequence; rows' tokens and positions in bmeta.
int enqueue_decode_step(tb200_state* st) {
  const bool pdl = use_pdl();
  tb200_model* m = st->m;
  const int T = int(st->n_seqs);
  st->trace_next = 0;
  if (int rc = enqueue_layers(st, T, false, 0, 0, pdl)) return rc;
  tb::ArgmaxRowsArgs am{};
  am.logits = st->blogits;
  am.V = int(m->c.vocab_size);
  am.tok = meta_tok(st);
  am.pos = meta_pos(st);
  am.out = st->bout;
  am.step = st->bstep;
  am.ticket = reinterpret_cast<unsigned*>(st->bstep + 1);
  am.out_cap = int(st->max_len);
  enqueue_head(st, 0, T, am, pdl, true);
  return launched("batched decode step");
}

int decode_graph(tb200_state* st) {
  if (st->bgraph) return TB200_OK;
  cudaStream_t s = st->m->dev->stream;
  CUDA_TRY(cudaStreamSynchronize(s));
  CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_decode_step(st);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(s, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return fail(TB200_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
  e = cudaGraphInstantiate(&st->bgraph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    st->bgraph = nullptr;
    return fail(TB200_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
  }
  return TB200_OK;
}

// Reads the error word after the stream drains.
int finish(tb200_state* st) {
  cudaStream_t s = st->m->dev->stream;
  int* back = readback(st);
  CUDA_TRY(cudaMemcpyAsync(back, st->io + 3, sizeof(int), cudaMemcpyDeviceToHost, s));
  CUDA_TRY(cudaStreamSynchronize(s));
  const int err = back[0];
  if (err == TB200_ERR_TIMEOUT) return fail(TB200_ERR_TIMEOUT, "a kernel's bounded wait timed out");
  if (err != 0) return fail(TB200_ERR_ARG, "a kernel rejected its input (token, position or sequence out of range)");
  return TB200_OK;
}

// Stages one decode step's rows (token i of sequence i at positions[i]).
int stage_rows(tb200_state* st, const uint32_t* tokens, const size_t* positions) {
  const size_t n = st->n_seqs, cap = size_t(st->cap);
  int* h = st->bmeta_host + 3 * (st->max_len + cap);
  for (size_t i = 0; i < n; i++) {
    h[i] = int(tokens[i]);
    h[cap + i] = int(positions[i]);
    h[2 * cap + i] = int(i);
  }
  cudaStream_t s = st->m->dev->stream;
  CUDA_TRY(cudaMemcpyAsync(st->bmeta, h, 3 * cap * sizeof(int), cudaMemcpyHostToDevice, s));
  CUDA_TRY(cudaMemsetAsync(st->io + 3, 0, sizeof(int), s));
  CUDA_TRY(cudaMemsetAsync(st->bstep, 0, sizeof(int), s));
  return TB200_OK;
}

int check_rows(tb200_state* st, const uint32_t* tokens, const size_t* positions, size_t steps) {
  const tb200_config& c = st->m->c;
  for (size_t i = 0; i < st->n_seqs; i++) {
    ARG_CHECK(tokens[i] < c.vocab_size, "token " + std::to_string(tokens[i]) + " is past the vocabulary");
    ARG_CHECK(positions[i] + steps <= st->max_len && positions[i] < st->max_len,
              "sequence " + std::to_string(i) + ": positions past the end of the cache");
  }
  return TB200_OK;
}

}  // namespace

namespace rt {

void drop_batch_graph(tb200_state* st) {
  if (st->bgraph) cudaGraphExecDestroy(st->bgraph);
  st->bgraph = nullptr;
}

void free_batch(tb200_state* st) {
  drop_batch_graph(st);
  void* ptrs[] = {st->bx, st->bqkv, st->blogits, st->bact, st->bmeta, st->rows_part, st->rows_ticket, st->bstep,
                  st->bout, st->bbest, st->bpart, st->ssq_a, st->ssq_b};
  for (void* p : ptrs) cudaFree(p);
  if (st->bmeta_host) cudaFreeHost(st->bmeta_host);
  st->bx = st->bqkv = st->blogits = st->rows_part = nullptr;
  st->bact = nullptr;
  st->bmeta = st->bmeta_host = st->bstep = st->bout = nullptr;
  st->bbest = nullptr;
  st->bpart = st->ssq_a = st->ssq_b = nullptr;
  st->rows_ticket = nullptr;
  st->cap = 0;
}

int forward_tokens(tb200_state* st, size_t seq, const uint32_t* tokens, size_t n, size_t pos, float* logits,
                   uint32_t* next) {
  if (int rc = ensure_batch(st)) return rc;
  tb200_model* m = st->m;
  cudaStream_t s = m->dev->stream;
  const bool pdl = use_pdl();
  const size_t cap = size_t(st->cap);
  CUDA_TRY(cudaMemsetAsync(st->io + 3, 0, sizeof(int), s));
  size_t last = 0;
  for (size_t c0 = 0; c0 < n; c0 += cap) {
    const size_t T = std::min(cap, n - c0);
    int* h = st->bmeta_host + 3 * (pos + c0);  // this pass's own staging region
    for (size_t i = 0; i < T; i++) {
      h[i] = int(tokens[c0 + i]);
      h[T + i] = int(pos + c0 + i);
      h[2 * T + i] = int(seq);
    }
    CUDA_TRY(cudaMemcpyAsync(st->bmeta, h, T * sizeof(int), cudaMemcpyHostToDevice, s));
    CUDA_TRY(cudaMemcpyAsync(st->bmeta + cap, h + T, T * sizeof(int), cudaMemcpyHostToDevice, s));
    CUDA_TRY(cudaMemcpyAsync(st->bmeta + 2 * cap, h + 2 * T, T * sizeof(int), cudaMemcpyHostToDevice, s));
    if (int rc = enqueue_layers(st, int(T), true, seq, pos + c0, pdl)) return rc;
    last = T;
  }
  tb::ArgmaxRowsArgs am{};
  am.logits = st->blogits;
  am.V = int(m->c.vocab_size);
  am.next = st->bstep + 2;
  enqueue_head(st, int(last) - 1, 1, am, pdl, false);
  if (int rc = launched("prompt pass")) return rc;
  if (logits) CUDA_TRY(cudaMemcpyAsync(logits, st->blogits, m->c.vocab_size * 4, cudaMemcpyDeviceToHost, s));
  int* back = readback(st) + 1;
  CUDA_TRY(cudaMemcpyAsync(back, st->bstep + 2, sizeof(int), cudaMemcpyDeviceToHost, s));
  if (int rc = finish(st)) return rc;
  if (next) *next = uint32_t(back[0]);
  return TB200_OK;
}

}  // namespace rt

extern "C" {

int tb200_forward_seq(tb200_model* m, tb200_state* st, size_t seq, const uint32_t* tokens, size_t n, size_t pos,
                      float* logits, uint32_t* next_token) {
  ARG_CHECK(m && st && st->m == m, "bad model/state");
  ARG_CHECK(seq < st->n_seqs, "sequence " + std::to_string(seq) + " is not in this state");
  ARG_CHECK(n > 0 && tokens, "no tokens to run");
  ARG_CHECK(pos + n <= st->max_len, "tokens past the end of the cache");
  if (int rc = use(m->dev)) return rc;
  for (size_t i = 0; i < n; i++)
    ARG_CHECK(tokens[i] < m->c.vocab_size, "token " + std::to_string(tokens[i]) + " is past the vocabulary");
  return rt::forward_tokens(st, seq, tokens, n, pos, logits, next_token);
}

int tb200_forward_batch(tb200_model* m, tb200_state* st, const uint32_t* tokens, const size_t* positions,
                        float* logits, uint32_t* next_tokens) {
  ARG_CHECK(m && st && st->m == m, "bad model/state");
  ARG_CHECK(tokens && positions, "null argument");
  if (int rc = use(m->dev)) return rc;
  if (int rc = check_rows(st, tokens, positions, 1)) return rc;
  if (int rc = ensure_batch(st)) return rc;
  if (int rc = decode_graph(st)) return rc;
  cudaStream_t s = m->dev->stream;
  if (int rc = stage_rows(st, tokens, positions)) return rc;
  CUDA_TRY(cudaGraphLaunch(st->bgraph, s));
  if (logits) CUDA_TRY(cudaMemcpyAsync(logits, st->blogits, st->n_seqs * m->c.vocab_size * 4, cudaMemcpyDeviceToHost, s));
  if (next_tokens) CUDA_TRY(cudaMemcpyAsync(next_tokens, st->bout, st->n_seqs * 4, cudaMemcpyDeviceToHost, s));
  return finish(st);
}

int tb200_generate_batch(tb200_model* m, tb200_state* st, const uint32_t* tokens, const size_t* positions,
                         size_t steps, uint32_t* out) {
  ARG_CHECK(m && st && st->m == m, "bad model/state");
  ARG_CHECK(tokens && positions && (out || steps == 0), "null argument");
  if (int rc = use(m->dev)) return rc;
  if (int rc = check_rows(st, tokens, positions, steps)) return rc;
  if (!steps) return TB200_OK;
  if (int rc = ensure_batch(st)) return rc;
  if (int rc = decode_graph(st)) return rc;
  cudaStream_t s = m->dev->stream;
  if (int rc = stage_rows(st, tokens, positions)) return rc;
  for (size_t i = 0; i < steps; i++) CUDA_TRY(cudaGraphLaunch(st->bgraph, s));
  CUDA_TRY(cudaMemcpyAsync(out, st->bout, steps * st->n_seqs * 4, cudaMemcpyDeviceToHost, s));
  return finish(st);
}

int tb200_decode_batch_enqueue(tb200_model* m, tb200_state* st, const uint32_t* tokens, const size_t* positions,
                               size_t steps) {
  ARG_CHECK(m && st && st->m == m, "bad model/state");
  ARG_CHECK(tokens && positions, "null argument");
  if (int rc = use(m->dev)) return rc;
  if (int rc = check_rows(st, tokens, positions, steps)) return rc;
  if (int rc = ensure_batch(st)) return rc;
  if (int rc = decode_graph(st)) return rc;
  cudaStream_t s = m->dev->stream;
  // The staging buffer is reused: the previous call's copy must have run.
  CUDA_TRY(cudaStreamSynchronize(s));
  if (int rc = stage_rows(st, tokens, positions)) return rc;
  for (size_t i = 0; i < steps; i++) CUDA_TRY(cudaGraphLaunch(st->bgraph, s));
  return TB200_OK;
}

int tb200_batch_read_kv(tb200_state* st, size_t seq, size_t layer, int which, size_t pos, float* out) {
  ARG_CHECK(st && out, "null argument");
  const tb200_config& c = st->m->c;
  ARG_CHECK(seq < st->n_seqs && layer < c.num_hidden_layers && pos < st->max_len && (which == 0 || which == 1),
            "out of range");
  if (int rc = use(st->m->dev)) return rc;
  cudaStream_t s = st->m->dev->stream;
  const size_t Hkv = c.num_key_value_heads, D = c.head_dim;
  const size_t kv_layer = 2 * Hkv * st->max_len * D;
  const size_t eb = st->kv_f32 ? 4 : 2;
  std::vector<unsigned char> tmp(Hkv * D * eb);
  for (size_t g = 0; g < Hkv; g++) {
    const unsigned char* src = st->kv + (seq * st->seq_stride + layer * kv_layer + size_t(which) * (kv_layer / 2) +
                                         (g * st->max_len + pos) * D) * eb;
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
