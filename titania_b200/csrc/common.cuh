// common.cuh — device helpers shared by the kernels: bf16 unpacking, warp
// reductions, and thin wrappers over sm_90+/sm_100a PTX (mbarrier,
// cp.async.bulk, programmatic dependent launch). Every wait on an mbarrier
// is bounded (kWaitCycles, about a second); on expiry it records TB200_ERR_TIMEOUT in the
// device's error word and the kernel returns.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/titania_b200.h"

namespace tb {

// The longest any in-kernel wait may take before it gives up: 2e9 SM cycles,
// one second at 2 GHz (longer at lower clocks). Waits count cycles because
// %clock64 reads in a few cycles while a %globaltimer read takes ~100 ns,
// which a spin loop would add to every poll.
constexpr long long kWaitCycles = 2000000000ll;

__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }
// The two bf16 values packed in a 32-bit word, low half first.
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// f32 -> bf16 bits, round to nearest even.
__device__ __forceinline__ uint16_t f2bf(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }

// The operand form of the tensor-core contraction: v = x0 + x1 + x2 with
// x0 = bf16(v), x1 = bf16(v - x0), x2 = bf16(v - x0 - x1) (exact for
// |v| in 2^-100 .. 2^127; the subtractions are exact), stored to planes
// p[at], p[plane + at], p[2 plane + at].
__device__ __forceinline__ void store_split3(uint16_t* p, size_t plane, size_t at, float v) {
  const uint16_t a = f2bf(v);
  const float r = v - bf16f(a);
  const uint16_t b = f2bf(r);
  const uint16_t c = f2bf(r - bf16f(b));
  p[at] = a;
  p[plane + at] = b;
  p[2 * plane + at] = c;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ unsigned long long warp_umax64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  return v;
}

// IEEE total order (Rust's f32::total_cmp) as an unsigned key, with ties
// broken toward the lower index: larger key = preferred.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  int32_t b = __float_as_int(v);
  b ^= int32_t(uint32_t(b >> 31) >> 1);
  uint32_t k = uint32_t(b) ^ 0x80000000u;
  return (static_cast<unsigned long long>(k) << 32) | (0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t argmax_index(unsigned long long key) {
  return 0xFFFFFFFFu - uint32_t(key & 0xFFFFFFFFu);
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- device-side trace -------------------------------------------------------
// When a state is traced, its kernels append one record per (launch, CTA,
// event) with the global timer, so a host tool can lay out the timeline.
struct TraceRec {
  uint32_t tag;    // op << 16 | layer
  uint32_t cta;    // blockIdx.x + blockIdx.y * gridDim.x
  uint32_t event;  // TB200_TRACE_* (include/titania_b200.h)
  uint32_t sm;
  uint64_t ns;
};
struct Trace {
  TraceRec* rec;  // null: tracing off
  unsigned cap;   // records
};
// Record slots per CTA of a traced launch (one per TB200_TRACE_* event).
constexpr uint32_t kTraceEvents = 8;
__device__ __forceinline__ uint32_t sm_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
  return r;
}

// Writes event `ev` of CTA `cta` into the launch's fixed slots (base + cta
// * kTraceEvents + ev), when tracing.
__device__ __forceinline__ void trace_at(const Trace& t, uint32_t base, uint32_t tag, uint32_t cta, uint32_t ev) {
  if (t.rec) {
    const uint32_t i = base + cta * kTraceEvents + ev;
    if (i < t.cap) t.rec[i] = TraceRec{tag, cta, ev, sm_id(), global_ns()};
  }
}
// A launch's trace slots: the buffer, its first slot and its tag (op << 16 | layer).
struct TraceAt {
  Trace t;
  uint32_t base, tag;
  __device__ __forceinline__ void at(uint32_t cta, uint32_t ev) const { trace_at(t, base, tag, cta, ev); }
};

__device__ __forceinline__ void set_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ---- programmatic dependent launch ----------------------------------------
// Kernels launched with cudaLaunchAttributeProgrammaticStreamSerialization may
// start while the previous kernel in the stream still runs. Each kernel calls
// pdl_launch_dependents() first (so the next kernel can start staging its own
// weights) and pdl_wait() before touching anything the previous kernel
// writes. Every CTA must reach pdl_wait() before it exits: completion of a
// kernel then implies completion of every kernel before it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- mbarrier / bulk copy ---------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase with `parity` to complete, at most kWaitCycles.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      set_error(err, TB200_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// An L2 policy that lets streamed-once data (weights) be evicted first, so
// that activations and the key/value cache stay resident.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16.
// Asks L2 to fetch [src, src + bytes) from memory; nothing waits for it.
// src and bytes multiples of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2-D tiled TMA load of box (x = column, y = row) into this CTA's shared
// memory, completing on `bar`. x * element size must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Named barrier over `nthreads` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// A partial attention result of one head over a run of positions: the 128
// output dimensions (unnormalised), then the run's max and sum; 132 floats
// so that every record starts on a 16-byte boundary.
constexpr int kPartStride = 132;

// The merge of `n` partial attention results of GRP heads (split s, head h
// at part + (s GRP + h) kPartStride), run by the last CTA of a
// split-context attention (128 threads): all threads read the splits'
// maxima at once, a warp per head turns them into weights exp(m_s - M)
// (kept in `w`, n GRP floats of shared memory) and the sum L, then a warp
// per head sums the splits' outputs, lane l taking dimensions 4l .. 4l+3
// with one 16-byte load per split, every load independent. The merged head
// h is left in out[h][0..128) (shared memory).
template <int GRP>
__device__ __forceinline__ void merge_splits(const float* part, int n, float* w, float* hsum, float (*out)[128]) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarps = int(blockDim.x) >> 5;
  for (int i = tid; i < n * GRP; i += blockDim.x) w[i] = __ldcg(part + size_t(i) * kPartStride + 128);
  __syncthreads();
  for (int h = warp; h < GRP; h += nwarps) {
    float M = -INFINITY;
    for (int sp = lane; sp < n; sp += 32) M = fmaxf(M, w[sp * GRP + h]);
    M = warp_max(M);
    float L = 0.f;
    for (int sp = lane; sp < n; sp += 32) {
      const float mm = w[sp * GRP + h];
      const float wt = mm == -INFINITY ? 0.f : expf(mm - M);
      L += __ldcg(part + size_t(sp * GRP + h) * kPartStride + 129) * wt;
      w[sp * GRP + h] = wt;
    }
    L = warp_sum(L);
    if (lane == 0) hsum[h] = L;
  }
  __syncthreads();
  for (int h = warp; h < GRP; h += nwarps) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int sp = 0; sp < n; sp++) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(part + size_t(sp * GRP + h) * kPartStride) + lane);
      const float wt = w[sp * GRP + h];
      acc.x += v.x * wt;
      acc.y += v.y * wt;
      acc.z += v.z * wt;
      acc.w += v.w * wt;
    }
    const float inv = 1.0f / hsum[h];
    *reinterpret_cast<float4*>(&out[h][4 * lane]) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  }
  __syncthreads();
}

// 8 bf16 weights (one 16-byte word) dotted with 8 f32 activations, in the
// order w0*x0 + ... accumulated into acc.
// acc + the four products of bf16 pairs w0, w1 with a.
__device__ __forceinline__ float dot4(uint32_t w0, uint32_t w1, float4 a, float acc) {
  acc = fmaf(bf_lo(w0), a.x, acc);
  acc = fmaf(bf_hi(w0), a.y, acc);
  acc = fmaf(bf_lo(w1), a.z, acc);
  acc = fmaf(bf_hi(w1), a.w, acc);
  return acc;
}
__device__ __forceinline__ float dot8(uint4 w, float4 a, float4 b, float acc) {
  acc = fmaf(bf_lo(w.x), a.x, acc);
  acc = fmaf(bf_hi(w.x), a.y, acc);
  acc = fmaf(bf_lo(w.y), a.z, acc);
  acc = fmaf(bf_hi(w.y), a.w, acc);
  acc = fmaf(bf_lo(w.z), b.x, acc);
  acc = fmaf(bf_hi(w.z), b.y, acc);
  acc = fmaf(bf_lo(w.w), b.z, acc);
  acc = fmaf(bf_hi(w.w), b.w, acc);
  return acc;
}

}  // namespace tb
