// sample.cu — model/sampler.rs:21-77 on the device: the next token from a
// row of logits, from the top_k most likely tokens, then the smallest set of
// those whose probability reaches top_p, at a temperature (greedy at 0), with
// the reference's xorshift64* generator. One state per logit row lives in
// device memory, so a decode loop can sample without a host round trip.
//
// Two kernels per call, deterministic (no atomics):
//   k_sample_chunks  CTA (chunk, row): 2048 logits as 64-bit keys (logit in
//                    total order, then the lowest token id) bitonic-sorted in
//                    shared memory; its top k keys go to a candidate list;
//   k_sample_pick    CTA per row: the chunks' candidates sorted the same way;
//                    thread 0 then runs the reference's arithmetic in its
//                    order — (logit - max) / T, expf, a sequential sum, p / sum,
//                    the running total while below top_p, r = next_f32() * total,
//                    r -= p until r <= 0 — and advances the row's state.
// Exact ties in the logits go to the lowest token id (the reference leaves
// them to an unstable selection).

#include "runtime.h"

struct tb200_sampler {
  tb200_device* dev = nullptr;
  size_t rows = 0, vocab = 0;
  float temperature = 0.f, top_p = 1.f;
  int top_k = 1;
  int chunks = 0;                          // ceil(vocab / kSampleChunk)
  unsigned long long* cand = nullptr;      // [rows][chunks][top_k]
  unsigned long long* state = nullptr;     // [rows] xorshift64* states
  uint32_t* tokens = nullptr;              // [rows]
};

namespace tb {
namespace {

constexpr int kSampleChunk = 2048;     // logits per CTA of the first kernel
constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 64;
constexpr int kSampleMaxCand = 8192;   // chunks x top_k sorted by one CTA

// Descending bitonic sort of n keys (n a power of two) in shared memory.
__device__ void sort_desc(unsigned long long* k, int n) {
  for (int size = 2; size <= n; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const unsigned long long a = k[lo], b = k[hi];
        if ((a < b) == desc) {
          k[lo] = b;
          k[hi] = a;
        }
      }
    }
  __syncthreads();
}

// The logit a key was made from (argmax_key's transform is an involution).
__device__ __forceinline__ float key_logit(unsigned long long key) {
  int32_t b = int32_t(uint32_t(key >> 32) ^ 0x80000000u);
  b ^= int32_t(uint32_t(b >> 31) >> 1);
  return __int_as_float(b);
}

__global__ void __launch_bounds__(kSampleThreads) k_sample_chunks(const float* __restrict__ logits, int vocab,
                                                                  int chunks, int k,
                                                                  unsigned long long* __restrict__ cand) {
  __shared__ unsigned long long keys[kSampleChunk];
  const int chunk = blockIdx.x, row = blockIdx.y;
  const float* lg = logits + size_t(row) * vocab;
  for (int i = threadIdx.x; i < kSampleChunk; i += blockDim.x) {
    const int t = chunk * kSampleChunk + i;
    keys[i] = t < vocab ? argmax_key(__ldg(lg + t), uint32_t(t)) : 0ull;  // 0 sorts last
  }
  sort_desc(keys, kSampleChunk);
  if (threadIdx.x < k) cand[(size_t(row) * chunks + chunk) * k + threadIdx.x] = keys[threadIdx.x];
}

__global__ void __launch_bounds__(kSampleThreads) k_sample_pick(const unsigned long long* __restrict__ cand,
                                                                int n, int n_pow2, int k, float temperature,
                                                                float top_p, unsigned long long* state,
                                                                uint32_t* tokens) {
  extern __shared__ unsigned long long keys[];  // [n_pow2]
  const int row = blockIdx.x;
  for (int i = threadIdx.x; i < n_pow2; i += blockDim.x) keys[i] = i < n ? cand[size_t(row) * n + i] : 0ull;
  sort_desc(keys, n_pow2);
  if (threadIdx.x != 0) return;
  uint32_t token = argmax_index(keys[0]);
  if (temperature != 0.0f) {
    float probs[kSampleMaxK];
    const float mx = key_logit(keys[0]);
    for (int i = 0; i < k; i++) probs[i] = expf(__fdiv_rn(__fsub_rn(key_logit(keys[i]), mx), temperature));
    float sum = -0.0f;
    for (int i = 0; i < k; i++) sum = __fadd_rn(sum, probs[i]);
    float cumulative = 0.0f;
    int m = 0;
    for (int i = 0; i < k; i++) {
      probs[i] = __fdiv_rn(probs[i], sum);
      if (cumulative < top_p) {
        cumulative = __fadd_rn(cumulative, probs[i]);
        m++;
      }
    }
    unsigned long long x = state[row];
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    state[row] = x;
    const float u = float((x * 0x2545F4914F6CDD1Dull) >> 40) / 16777216.0f;  // exact: a 24-bit integer / 2^24
    float r = __fmul_rn(u, cumulative);
    token = argmax_index(keys[m > 0 ? m - 1 : 0]);
    for (int i = 0; i < m; i++) {
      r = __fsub_rn(r, probs[i]);
      if (r <= 0.0f) {
        token = argmax_index(keys[i]);
        break;
      }
    }
  }
  tokens[row] = token;
}

int pow2_at_least(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

}  // namespace
}  // namespace tb

extern "C" {

int tb200_sampler_new(tb200_device* dev, size_t rows, size_t vocab, float temperature, size_t top_k, float top_p,
                      const uint64_t* seeds, tb200_sampler** out) {
  ARG_CHECK(dev && seeds && out, "null argument");
  ARG_CHECK(rows >= 1 && rows <= 65535 && vocab >= 1 && vocab <= (size_t(1) << 31), "bad rows or vocabulary");
  ARG_CHECK(temperature >= 0.0f, "temperature must not be negative");
  // sampler.rs:44-59 keeps no candidate when top_p <= 0 and then panics indexing candidates[n - 1].
  ARG_CHECK(temperature == 0.0f || top_p > 0.0f, "top_p must be positive when sampling at a temperature");
  const size_t k = std::min(std::max<size_t>(top_k, 1), vocab);  // sampler.rs:29 clamps top_k to [1, n]
  ARG_CHECK(k <= size_t(tb::kSampleMaxK), "top_k above 64 is not supported on the device");
  const size_t chunks = (vocab + tb::kSampleChunk - 1) / tb::kSampleChunk;
  ARG_CHECK(chunks * k <= size_t(tb::kSampleMaxCand), "vocabulary too large for top_k on the device");
  if (int rc = rt::use(dev)) return rc;
  // The candidate sort may take more than the default 48 KB of shared memory.
  CUDA_TRY(cudaFuncSetAttribute(tb::k_sample_pick, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(tb::kSampleMaxCand * sizeof(unsigned long long))));
  auto* s = new tb200_sampler;
  s->dev = dev;
  s->rows = rows;
  s->vocab = vocab;
  s->temperature = temperature;
  s->top_k = int(k);
  s->top_p = top_p;
  s->chunks = int(chunks);
  std::vector<unsigned long long> st(rows);
  for (size_t i = 0; i < rows; i++) st[i] = seeds[i] ? seeds[i] : 1ull;  // Rng(seed.max(1))
  cudaError_t e = cudaMalloc(&s->cand, rows * chunks * k * 8);
  if (e == cudaSuccess) e = cudaMalloc(&s->state, rows * 8);
  if (e == cudaSuccess) e = cudaMalloc(&s->tokens, rows * 4);
  if (e == cudaSuccess) e = cudaMemcpy(s->state, st.data(), rows * 8, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    tb200_sampler_free(s);
    return rt::fail(TB200_ERR_CUDA, std::string("sampler: ") + cudaGetErrorString(e));
  }
  *out = s;
  return TB200_OK;
}

int tb200_sampler_free(tb200_sampler* s) {
  if (!s) return TB200_OK;
  cudaSetDevice(s->dev->ordinal);
  cudaStreamSynchronize(s->dev->stream);
  cudaFree(s->cand);
  cudaFree(s->state);
  cudaFree(s->tokens);
  delete s;
  return TB200_OK;
}

int tb200_sample_enqueue(tb200_sampler* s, const tb200_buffer* logits) {
  ARG_CHECK(s && logits, "null argument");
  ARG_CHECK(logits->len >= s->rows * s->vocab, "the logits buffer holds fewer than rows x vocabulary values");
  if (int rc = rt::use(s->dev)) return rc;
  cudaStream_t st = s->dev->stream;
  tb::k_sample_chunks<<<dim3(unsigned(s->chunks), unsigned(s->rows)), tb::kSampleThreads, 0, st>>>(
      logits->ptr, int(s->vocab), s->chunks, s->top_k, s->cand);
  const int n = s->chunks * s->top_k, n2 = tb::pow2_at_least(n);
  tb::k_sample_pick<<<unsigned(s->rows), tb::kSampleThreads, size_t(n2) * 8, st>>>(
      s->cand, n, n2, s->top_k, s->temperature, s->top_p, s->state, s->tokens);
  return rt::launched("sample");
}

int tb200_sample(tb200_sampler* s, const tb200_buffer* logits, uint32_t* tokens) {
  ARG_CHECK(tokens, "null argument");
  if (int rc = tb200_sample_enqueue(s, logits)) return rc;
  CUDA_TRY(cudaMemcpyAsync(tokens, s->tokens, s->rows * 4, cudaMemcpyDeviceToHost, s->dev->stream));
  CUDA_TRY(cudaStreamSynchronize(s->dev->stream));
  return TB200_OK;
}

int tb200_sampler_state(tb200_sampler* s, uint64_t* out) {
  ARG_CHECK(s && out, "null argument");
  if (int rc = rt::use(s->dev)) return rc;
  CUDA_TRY(cudaStreamSynchronize(s->dev->stream));
  CUDA_TRY(cudaMemcpy(out, s->state, s->rows * 8, cudaMemcpyDeviceToHost));
  return TB200_OK;
}

}  // extern "C"
