// noalloc.cu — greedy argmax over logits the caller keeps in device memory,
// for callers that cannot allocate device memory.
//
// Who cannot allocate: a caller whose GPU memory is owned by another
// allocator (a framework's caching allocator that has reserved the device's
// memory, where a stray cudaMalloc fails or fragments it), and a caller that
// keeps cudaMalloc/cudaFree out of its per-token loop because those calls can
// synchronize the whole device and stall its other streams. Such a caller
// holds its logits and an output word in memory it already owns and only
// wants the greedy choice computed where the logits are.
//
// tb200_argmax (runtime.cu) needs a tb200_device, whose scratch word is
// cudaMalloc'ed when the device is opened. This variant takes no handle and
// allocates nothing: its scratch is the file-scope array below, which every
// GPU that loads this library holds until the process exits.

#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace tb {

namespace {

constexpr int kArgmaxTile = 4096;       // logits per CTA
constexpr int kArgmaxMaxTiles = 2048;   // scratch slots
constexpr size_t kArgmaxMaxLogits = size_t(kArgmaxTile) * kArgmaxMaxTiles;  // 8 Mi logits
constexpr int kMaxDevices = 64;

// Scratch: one best-key slot per tile, then the arrival counter.
// 2049 x 8 bytes = 16 KB + 8 B per GPU.
static __device__ __align__(256) unsigned long long g_argmax_scratch[kArgmaxMaxTiles + 1];

// One CTA per tile of kArgmaxTile logits writes its best key (IEEE total
// order, ties to the lowest index — the choice tb200_argmax makes) to its
// scratch slot; the last CTA to arrive reduces the slots in index order and
// writes the winning index to *out.
__global__ void __launch_bounds__(256) k_argmax_tiles(const float* __restrict__ x, size_t n,
                                                      unsigned long long* scratch, uint32_t* out) {
  __shared__ unsigned long long red[8];
  __shared__ int is_last;
  const size_t begin = size_t(blockIdx.x) * kArgmaxTile;
  const size_t end = begin + kArgmaxTile < n ? begin + kArgmaxTile : n;
  unsigned long long best = 0ull;
  for (size_t i = begin + threadIdx.x; i < end; i += blockDim.x) {
    const unsigned long long k = argmax_key(x[i], uint32_t(i));
    best = k > best ? k : best;
  }
  best = warp_umax64(best);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < int(blockDim.x >> 5); w++) b = red[w] > b ? red[w] : b;
    scratch[blockIdx.x] = b;
    __threadfence();
    is_last = atomicAdd(&scratch[kArgmaxMaxTiles], 1ull) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last || warp != 0) return;
  __threadfence();
  unsigned long long b = 0ull;
  for (unsigned t = lane; t < gridDim.x; t += 32) {
    const unsigned long long v = __ldcg(scratch + t);
    b = v > b ? v : b;
  }
  b = warp_umax64(b);
  if (lane == 0) *out = argmax_index(b);
}

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

}  // namespace

}  // namespace tb

extern "C" int tb200_argmax_noalloc(const float* logits, size_t n, uint32_t* out, void* stream) {
  using namespace tb;
  if (!logits || !out) return record_error(TB200_ERR_ARG, "argmax_noalloc: null logits or output");
  if (n == 0) return record_error(TB200_ERR_ARG, "argmax_noalloc: no logits");
  if (n > kArgmaxMaxLogits)
    return record_error(TB200_ERR_ARG, "argmax_noalloc: " + std::to_string(n) + " logits exceed the maximum of " +
                                           std::to_string(kArgmaxMaxLogits) + " (its static scratch holds " +
                                           std::to_string(kArgmaxMaxTiles) + " tiles of " +
                                           std::to_string(kArgmaxTile) + ")");
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return record_error(TB200_ERR_CUDA, std::string("argmax_noalloc: ") + cudaGetErrorString(e));
  if (device < 0 || device >= kMaxDevices) return record_error(TB200_ERR_ARG, "argmax_noalloc: device ordinal too large");
  void* scratch = nullptr;
  {
    // Set-up, once per device, with that device current: in host code the
    // array's name only stands in for it, so look up its device address.
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[device]) {
      e = cudaGetSymbolAddress(&g_scratch_addr[device], g_argmax_scratch);
      if (e != cudaSuccess) {
        g_scratch_addr[device] = nullptr;
        return record_error(TB200_ERR_CUDA, std::string("argmax_noalloc: scratch lookup: ") + cudaGetErrorString(e));
      }
    }
    scratch = g_scratch_addr[device];
  }
  auto* slots = static_cast<unsigned long long*>(scratch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The arrival counter must start at zero; the tile slots are all written.
  e = cudaMemsetAsync(slots + kArgmaxMaxTiles, 0, sizeof(unsigned long long), s);
  if (e != cudaSuccess) return record_error(TB200_ERR_CUDA, std::string("argmax_noalloc: ") + cudaGetErrorString(e));
  const unsigned tiles = unsigned((n + kArgmaxTile - 1) / kArgmaxTile);
  k_argmax_tiles<<<tiles, 256, 0, s>>>(logits, n, slots, out);
  e = cudaGetLastError();
  if (e != cudaSuccess) return record_error(TB200_ERR_CUDA, std::string("argmax_noalloc: ") + cudaGetErrorString(e));
  return TB200_OK;
}
