// attn_op.cu — GQA decode attention as a standalone op over a bf16
// key/value cache in the model path's layout: Device::attention
// (model/cpu.rs:113-149) for one query token per sequence, each sequence at
// its own position, the cache laid out [sequence][K|V][kv head][max_len][128].
//
// It runs the batched decode step's attention kernel (batch.cu: tensor
// cores over TMA-loaded bf16 chunks), whose output is the f32 result as
// three bf16 planes; a second kernel adds them back into f32 rows (exactly:
// the planes of an f32 value sum to it).
#include <algorithm>
#include <string>

#include "runtime.h"

namespace {

__global__ void k_planes_to_f32(const uint16_t* __restrict__ planes, size_t plane, float* __restrict__ out, size_t n) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = (tb::bf16f(planes[i]) + tb::bf16f(planes[plane + i])) + tb::bf16f(planes[2 * plane + i]);
}

// Grows a device allocation to at least `n` elements of T (contents lost;
// zeroed when `zero`).
template <class T>
int grow(T** p, size_t* cap, size_t n, bool zero, cudaStream_t s) {
  if (*cap >= n) return TB200_OK;
  CUDA_TRY(cudaStreamSynchronize(s));
  cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  CUDA_TRY(cudaMalloc(p, n * sizeof(T)));
  if (zero) CUDA_TRY(cudaMemsetAsync(*p, 0, n * sizeof(T), s));
  *cap = n;
  return TB200_OK;
}

}  // namespace

extern "C" {

int tb200_attention_cache(tb200_device* d, tb200_buffer* out, const tb200_buffer* q, const tb200_weight* cache,
                          const size_t* positions, size_t batch, size_t n_heads) {
  constexpr size_t D = 128;
  ARG_CHECK(d && out && q && cache && positions, "null argument");
  ARG_CHECK(cache->shape.size() == 5 && cache->shape[1] == 2 && cache->shape[4] == D,
            "the cache must have shape [batch, 2, n_kv_heads, max_len, 128]");
  ARG_CHECK(batch > 0 && cache->shape[0] == batch, "the cache holds a different number of sequences");
  const size_t n_kv_heads = cache->shape[2], max_len = cache->shape[3];
  ARG_CHECK(n_kv_heads > 0 && n_heads % n_kv_heads == 0, "n_heads must be a multiple of the cache's kv heads");
  const size_t group = n_heads / n_kv_heads;
  ARG_CHECK(group == 1 || group == 2 || group == 4 || group == 8, "1, 2, 4 or 8 query heads per kv head");
  ARG_CHECK(max_len > 0 && batch * 2 * n_kv_heads * max_len < (size_t(1) << 31), "cache too large");
  const size_t qd = n_heads * D;
  ARG_CHECK(q->len == batch * qd && out->len == batch * qd, "q and out must hold batch * n_heads * 128 values");
  for (size_t b = 0; b < batch; b++) ARG_CHECK(positions[b] < max_len, "position past the end of the cache");
  const void* kv = cache->ptr;
  const bool f32 = false;
  if (int rc = rt::use(d)) return rc;
  cudaStream_t s = d->stream;
  const int parts = tb::attn_rows_parts(int(batch), int(n_kv_heads), int(max_len), f32, d->sms);
  if (int rc = grow(&d->ao_part, &d->ao_part_cap, batch * n_kv_heads * parts * group * tb::kPartStride, false, s))
    return rc;
  if (int rc = grow(&d->ao_ticket, &d->ao_ticket_cap, batch * n_kv_heads, true, s)) return rc;
  if (int rc = grow(&d->ao_planes, &d->ao_planes_cap, 3 * batch * qd, false, s)) return rc;
  if (d->ao_meta_cap < 2 * batch) {
    if (int rc = grow(&d->ao_meta, &d->ao_meta_cap, 2 * batch, false, s)) return rc;
    d->ao_meta_host.clear();
  }
  // Positions and sequence rows: copied only when they change, so that
  // repeated calls enqueue nothing but the two kernels.
  std::vector<int> meta(2 * batch);
  for (size_t b = 0; b < batch; b++) {
    meta[b] = int(positions[b]);
    meta[batch + b] = int(b);
  }
  if (meta != d->ao_meta_host) {
    CUDA_TRY(cudaMemcpyAsync(d->ao_meta, meta.data(), meta.size() * sizeof(int), cudaMemcpyHostToDevice, s));
    d->ao_meta_host = meta;
  }
  const size_t rows = batch * 2 * n_kv_heads * max_len;  // cache rows of 128 elements
  if (d->ao_map_base != kv || d->ao_map_rows != rows) {
    std::string why;
    if (int rc = tb::encode_tmap_bf16(&d->ao_map, kv, rows, D, tb::attn_cache_box_rows(), &why))
      return rt::fail(rc, "attention: " + why);
    d->ao_map_base = kv;
    d->ao_map_rows = rows;
  }
  tb::AttnRowsArgs a{};
  a.q = q->ptr;
  a.ldq = int(qd);
  a.kv = kv;
  a.seq_stride = 2 * n_kv_heads * max_len * D;
  a.kv_f32 = f32;
  a.max_len = int(max_len);
  a.n_kv_heads = int(n_kv_heads);
  a.n_seqs = int(batch);
  a.pos = d->ao_meta;
  a.seq = d->ao_meta + batch;
  a.out = d->ao_planes;
  a.plane = batch * qd;
  a.ldo = int(qd);
  a.part = d->ao_part;
  a.ticket = d->ao_ticket;
  a.parts = parts;
  a.err = d->err;
  a.cache_map = &d->ao_map;
  a.layer_rows = 0;
  tb::launch_attn_rows(s, a, int(batch), int(group), false);
  if (int rc = rt::launched("attention")) return rc;
  const size_t n = batch * qd;
  k_planes_to_f32<<<unsigned((n + 255) / 256), 256, 0, s>>>(d->ao_planes, batch * qd, out->ptr, n);
  return rt::launched("attention output");
}

}  // extern "C"
