// ops.cu — one kernel per Device-trait operation (model/device.rs:17-88),
// matching the reference CPU device (model/cpu.rs) in meaning. These serve
// the op-by-op drop-in path and its parity tests; the fused decode path in
// fused.cu is the fast one.
//
// Numerics: f32 accumulation throughout. Where the reference's operation
// order is the natural parallel one (embed, add, copy, rope), the result is
// bit-identical; reductions (matmul, rmsnorm, attention) sum in a different
// order and land within a few ulps.

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tb {

namespace {

__global__ void k_copy(float* __restrict__ dst, const float* __restrict__ src, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}

// cpu.rs:38-47
__global__ void k_embed(float* __restrict__ out, const uint16_t* __restrict__ table, size_t dim,
                        const uint32_t* __restrict__ tokens) {
  size_t t = blockIdx.x;
  const uint16_t* row = table + size_t(tokens[t]) * dim;
  for (size_t i = threadIdx.x; i < dim; i += blockDim.x) out[t * dim + i] = bf16f(row[i]);
}

// cpu.rs:49-77: out[t][r] = w[r] · x[t]. One warp per row, up to 8 tokens per
// warp so each weight row is read once per 8 tokens.
constexpr int kMmTok = 8;
constexpr int kMmWarps = 8;

template <bool kVec>
__global__ void __launch_bounds__(kMmWarps * 32) k_matmul(float* __restrict__ out, const uint16_t* __restrict__ w,
                                                          int rows, int cols, const float* __restrict__ x, int n) {
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int r = blockIdx.x * kMmWarps + warp;
  int t0 = blockIdx.y * kMmTok;
  if (r >= rows) return;
  int nt = min(kMmTok, n - t0);
  const uint16_t* wr = w + size_t(r) * cols;
  float acc[kMmTok];
#pragma unroll
  for (int t = 0; t < kMmTok; t++) acc[t] = 0.f;
  if (kVec) {
    for (int c = lane * 8; c < cols; c += 256) {
      uint4 wv = __ldg(reinterpret_cast<const uint4*>(wr + c));
#pragma unroll
      for (int t = 0; t < kMmTok; t++) {
        if (t < nt) {
          const float* xt = x + size_t(t0 + t) * cols + c;
          float4 a = __ldg(reinterpret_cast<const float4*>(xt));
          float4 b = __ldg(reinterpret_cast<const float4*>(xt + 4));
          acc[t] = dot8(wv, a, b, acc[t]);
        }
      }
    }
  } else {
    for (int c = lane; c < cols; c += 32) {
      float wf = bf16f(wr[c]);
#pragma unroll
      for (int t = 0; t < kMmTok; t++)
        if (t < nt) acc[t] = fmaf(wf, x[size_t(t0 + t) * cols + c], acc[t]);
    }
  }
#pragma unroll
  for (int t = 0; t < kMmTok; t++) {
    float v = warp_sum(acc[t]);
    if (lane == t && t < nt) out[size_t(t0 + t) * rows + r] = v;
  }
}

__global__ void k_add(float* __restrict__ x, const float* __restrict__ y, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    x[i] = __fadd_rn(x[i], y[i]);
}

// cpu.rs:151-155: g = g / (1 + exp(-g)) * u
__global__ void k_silu_mul(float* __restrict__ g, const float* __restrict__ u, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    float v = g[i];
    g[i] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u[i]);
  }
}

// cpu.rs:85-94, one block per row.
__global__ void k_rmsnorm(float* __restrict__ x, const uint16_t* __restrict__ w, int dim, float eps) {
  __shared__ float red[32];
  float* row = x + size_t(blockIdx.x) * dim;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(row[i], row[i], ss);
  ss = warp_sum(ss);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < nw; i++) tot += red[i];
  float scale = 1.0f / sqrtf(tot / float(dim) + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) row[i] = __fmul_rn(row[i], __fmul_rn(scale, bf16f(w[i])));
}

// cpu.rs:96-111: block per (token, head), thread per pair (i, i + half).
__global__ void k_rope(float* __restrict__ x, int n_heads, int head_dim, const float* __restrict__ table,
                       size_t pos) {
  int t = blockIdx.x / n_heads, h = blockIdx.x % n_heads;
  int half = head_dim / 2;
  float* head = x + (size_t(t) * n_heads + h) * head_dim;
  const float* ang = table + (pos + t) * head_dim;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float c = ang[2 * i], s = ang[2 * i + 1];
    float a = head[i], b = head[i + half];
    head[i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    head[i + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
  }
}

// cpu.rs:113-149: one block of 4 warps per (token, head). Each warp runs an
// online softmax over every 4th position; the warps' partial results are
// merged at the end. head_dim <= 256, elements lane + 32*j per lane.
constexpr int kAttWarps = 4;

__global__ void __launch_bounds__(kAttWarps * 32)
    k_attention(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ kc,
                const float* __restrict__ vc, size_t pos, int n_heads, int head_dim, int n_kv_heads) {
  __shared__ float sm_m[kAttWarps], sm_l[kAttWarps];
  __shared__ float sm_acc[kAttWarps][256];
  int i = blockIdx.x;
  int token = i / n_heads, head = i % n_heads;
  int group = n_heads / n_kv_heads;
  size_t kv_dim = size_t(n_kv_heads) * head_dim;
  size_t kv = size_t(head / group) * head_dim;
  size_t len = pos + token + 1;
  float scale = 1.0f / sqrtf(float(head_dim));
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int per = (head_dim + 31) / 32;
  float qv[8], acc[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    int d = lane + 32 * j;
    qv[j] = (j < per && d < head_dim) ? q[size_t(i) * head_dim + d] : 0.f;
    acc[j] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (size_t t = warp; t < len; t += kAttWarps) {
    const float* kr = kc + t * kv_dim + kv;
    float d0 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      int d = lane + 32 * j;
      if (j < per && d < head_dim) d0 = fmaf(qv[j], kr[d], d0);
    }
    float s = scale * warp_sum(d0);
    float mn = fmaxf(m, s);
    float corr = expf(m - mn);
    float p = expf(s - mn);
    l = l * corr + p;
    const float* vr = vc + t * kv_dim + kv;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      int d = lane + 32 * j;
      if (j < per && d < head_dim) acc[j] = acc[j] * corr + p * vr[d];
    }
    m = mn;
  }
  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = l;
  }
#pragma unroll
  for (int j = 0; j < 8; j++) {
    int d = lane + 32 * j;
    if (j < per && d < head_dim) sm_acc[warp][d] = acc[j];
  }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < kAttWarps; w++) M = fmaxf(M, sm_m[w]);
  float L = 0.f;
  float wgt[kAttWarps];
  for (int w = 0; w < kAttWarps; w++) {
    wgt[w] = sm_m[w] == -INFINITY ? 0.f : expf(sm_m[w] - M);
    L += sm_l[w] * wgt[w];
  }
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float o = 0.f;
    for (int w = 0; w < kAttWarps; w++) o += sm_acc[w][d] * wgt[w];
    out[size_t(i) * head_dim + d] = o / L;
  }
}

__global__ void k_argmax(const float* __restrict__ x, size_t n, unsigned long long* best) {
  __shared__ unsigned long long red[32];
  unsigned long long b = 0;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    unsigned long long k = argmax_key(x[i], uint32_t(i));
    b = k > b ? k : b;
  }
  b = warp_umax64(b);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = b;
  __syncthreads();
  if (warp == 0) {
    b = lane < int(blockDim.x >> 5) ? red[lane] : 0ull;
    b = warp_umax64(b);
    if (lane == 0) atomicMax(best, b);
  }
}

__global__ void k_interleave(uint16_t* __restrict__ dst, const uint16_t* __restrict__ a,
                             const uint16_t* __restrict__ b, size_t rows, size_t cols) {
  size_t total = rows * cols * 2;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
    size_t r2 = i / cols, c = i % cols;
    size_t r = r2 >> 1;
    dst[i] = (r2 & 1) ? b[r * cols + c] : a[r * cols + c];
  }
}

__global__ void k_bf16_to_f32(float* __restrict__ dst, const uint16_t* __restrict__ src, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    dst[i] = bf16f(src[i]);
}

int grid_for(size_t n, int block) {
  size_t g = (n + block - 1) / block;
  return int(std::min<size_t>(std::max<size_t>(g, 1), 148 * 16));
}

}  // namespace

void launch_copy(cudaStream_t s, float* dst, const float* src, size_t n) {
  if (n) k_copy<<<grid_for(n, 256), 256, 0, s>>>(dst, src, n);
}

void launch_embed(cudaStream_t s, float* out, const uint16_t* table, size_t dim, const uint32_t* tokens, size_t n) {
  if (n) k_embed<<<unsigned(n), 256, 0, s>>>(out, table, dim, tokens);
}

void launch_matmul(cudaStream_t s, float* out, const uint16_t* w, size_t rows, size_t cols, const float* x,
                   size_t n) {
  if (!n || !rows) return;
  dim3 grid(unsigned((rows + kMmWarps - 1) / kMmWarps), unsigned((n + kMmTok - 1) / kMmTok));
  bool vec = (cols % 8 == 0) && (reinterpret_cast<uintptr_t>(w) % 16 == 0) &&
             (reinterpret_cast<uintptr_t>(x) % 16 == 0);
  if (vec)
    k_matmul<true><<<grid, kMmWarps * 32, 0, s>>>(out, w, int(rows), int(cols), x, int(n));
  else
    k_matmul<false><<<grid, kMmWarps * 32, 0, s>>>(out, w, int(rows), int(cols), x, int(n));
}

void launch_add(cudaStream_t s, float* x, const float* y, size_t n) {
  if (n) k_add<<<grid_for(n, 256), 256, 0, s>>>(x, y, n);
}

void launch_silu_mul(cudaStream_t s, float* g, const float* u, size_t n) {
  if (n) k_silu_mul<<<grid_for(n, 256), 256, 0, s>>>(g, u, n);
}

void launch_rmsnorm(cudaStream_t s, float* x, size_t rows, const uint16_t* w, size_t dim, float eps) {
  if (rows) k_rmsnorm<<<unsigned(rows), dim >= 1024 ? 512 : 128, 0, s>>>(x, w, int(dim), eps);
}

void launch_rope(cudaStream_t s, float* x, size_t n_tokens, const float* table, size_t pos, size_t n_heads,
                 size_t head_dim) {
  if (n_tokens && n_heads) {
    int threads = int(std::min<size_t>(std::max<size_t>(head_dim / 2, 32), 512));
    k_rope<<<unsigned(n_tokens * n_heads), threads, 0, s>>>(x, int(n_heads), int(head_dim), table, pos);
  }
}

void launch_attention(cudaStream_t s, float* out, const float* q, size_t n_tokens, const float* k_cache,
                      const float* v_cache, size_t pos, size_t n_heads, size_t head_dim, size_t n_kv_heads) {
  if (n_tokens && n_heads)
    k_attention<<<unsigned(n_tokens * n_heads), kAttWarps * 32, 0, s>>>(out, q, k_cache, v_cache, pos, int(n_heads),
                                                                        int(head_dim), int(n_kv_heads));
}

void launch_argmax(cudaStream_t s, const float* x, size_t n, unsigned long long* best, int sms) {
  if (n) k_argmax<<<std::min(grid_for(n, 256), sms * 2), 256, 0, s>>>(x, n, best);
}

void launch_interleave_rows(cudaStream_t s, uint16_t* dst, const uint16_t* a, const uint16_t* b, size_t rows,
                            size_t cols) {
  k_interleave<<<grid_for(rows * cols * 2, 256), 256, 0, s>>>(dst, a, b, rows, cols);
}

void launch_bf16_to_f32(cudaStream_t s, float* dst, const uint16_t* src, size_t n) {
  if (n) k_bf16_to_f32<<<grid_for(n, 256), 256, 0, s>>>(dst, src, n);
}

}  // namespace tb
