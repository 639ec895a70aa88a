// fused.cu — the fused batch-1 decode path (model/model.rs:93-149 for n = 1).
//
// One decode step is 2 + 5 * layers kernels, replayed from a CUDA graph:
//   embed_token                      x = table[token]
//   per layer:
//     mv<norm, store>      (q|k|v)   qkv = Wqkv · rmsnorm(x)
//     attn_decode                    QK-norm, RoPE, K/V append, GQA attention
//                                    (split over the context, 64 positions
//                                    per CTA, merged by the last CTA)
//     mv<residual>         (o)       x += Wo · att
//     mv<norm, silu pair>  (gate|up) h = silu(Wg · rmsnorm(x)) * (Wu · ...)
//     mv<residual>         (down)    x += Wd · h
//   mv<norm, argmax>       (lm_head) logits, greedy token, position += 1
//
// At batch 1 every kernel is short and the step is a chain of 142 dependent
// launches, so the design goal is the critical path of each link. Kernels
// are launched with programmatic dependent launch: a kernel starts while its
// predecessor runs, and everything that does not depend on the predecessor
// — its weights (streamed by a producer warp into a shared-memory ring with
// cp.async.bulk, L2 evict-first), norm weights, the RoPE row, the cached
// keys and values of earlier positions — is staged before
// griddepcontrol.wait. After the wait a kernel makes one round trip to L2
// for its input vector, computes from shared memory, and writes.

#include <algorithm>
#include <type_traits>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace tb {

namespace {

constexpr int kMvWarps = 8;                      // consumer warps
constexpr int kMvThreads = (kMvWarps + 1) * 32;  // + one producer warp
constexpr size_t kMvStageBytes = 64 * 1024;      // most bytes in one weight copy
constexpr int kMvKsplitRows = 8;                 // rows per stage of a K-split kernel

// Shared-memory position of input element i (i a multiple of 4).
__device__ __forceinline__ int xperm(int i) { return (i & ~255) + ((i >> 2) & 1) * 128 + ((i >> 3) & 31) * 4; }

__host__ __device__ constexpr size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Trace slots are fixed per (launch, CTA, event): no atomics on the path.
// Each CTA owns rows [r0, r1). The producer warp copies them in stages of
// `stage_rows` rows (large bulk copies: a TMA copy's cost is mostly per copy,
// so a few tens of KB per copy reach far higher per-SM bandwidth than rows
// one at a time). Every consumer warp walks every stage in order and takes
// its own chunk of CH rows in it (stage_rows <= kMvWarps * CH), so a warp
// never waits on a slot's barrier more than one phase ahead of it.
// With NORM, the input is stored pre-multiplied by the norm weight and the
// RMS scale is applied to each dot product: scale * (w · (x ∘ g)), the
// reference's w · (x ∘ (scale * g)) with the scale factored out.
template <int CH, int EPI, bool NORM, bool KS>
__global__ void __launch_bounds__(kMvThreads) mv_kernel(MvArgs a, int stage_rows, int slots) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float red[kMvWarps];
  __shared__ unsigned long long best_sm[kMvWarps];
  __shared__ float resid[kMaxResidualRows];
  __shared__ float ksum[kMvWarps][kMvKsplitRows];
  __shared__ int is_last;

  pdl_launch_dependents();
  const int c = blockIdx.x, G = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, c, TB200_TRACE_START);

  const int cols = a.cols;
  float* xs = reinterpret_cast<float*>(smem);
  float* nw = reinterpret_cast<float*>(smem + (align_up(size_t(cols), 256) * 4));
  unsigned char* ring = smem + (align_up(size_t(cols), 256) * 4) * (NORM ? 2 : 1);
  const uint32_t row_bytes = uint32_t(cols) * 2;
  const uint32_t stage_bytes = uint32_t(stage_rows) * row_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + size_t(slots) * stage_bytes);
  uint64_t* empty = full + slots;

  const int units = a.rows / a.row_align;
  const int r0 = int((long long)c * units / G) * a.row_align;
  const int r1 = int((long long)(c + 1) * units / G) * a.row_align;
  const int nrows = r1 - r0;
  const int nstages = (nrows + stage_rows - 1) / stage_rows;

  if (tid == 0) {
    for (int s = 0; s < slots; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMvWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kMvWarps) {
    // Producer: weights are never written by a kernel, so they are staged
    // before (and while) the previous kernel finishes.
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      for (int i = 0; i < nstages; i++) {
        const int s = i % slots;
        if (i >= slots && !mbar_wait(&empty[s], ((i / slots) - 1) & 1, a.err)) break;
        const int nr = min(stage_rows, nrows - i * stage_rows);
        const uint32_t bytes = uint32_t(nr) * row_bytes;
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(ring + size_t(s) * stage_bytes, a.w + size_t(r0 + i * stage_rows) * cols, bytes, &full[s], pol);
      }
      trace_at(a.trace, a.trace_base, a.tag, c, TB200_TRACE_ISSUED);
    }
    return;
  }

  // Consumers. Norm weights do not depend on the previous kernel either;
  // each thread stages exactly the elements it multiplies below, so no
  // barrier is needed between the two.
  // A 1024-column input that needs no summing or copying out skips shared
  // memory: every warp loads the whole vector into registers, lane l holding
  // the columns it multiplies (256k + 8l .. + 7, k = 0..3), and sums its own
  // squares, so no barrier separates the input from the dot products.
  constexpr int kXregCols = 1024;
  const bool xreg = !KS && EPI != kMvResidual && cols == kXregCols && a.npartials == 0 && !a.x_out;
  uint4 gw[kXregCols / 256];
  if (NORM && xreg) {
#pragma unroll
    for (int k = 0; k < kXregCols / 256; k++) gw[k] = *reinterpret_cast<const uint4*>(a.norm_w + 256 * k + lane * 8);
  } else if (NORM)
    for (int i = tid * 4; i < cols; i += kMvWarps * 32 * 4) {
      const uint2 g = *reinterpret_cast<const uint2*>(a.norm_w + i);
      *reinterpret_cast<float4*>(nw + i) = make_float4(bf_lo(g.x), bf_hi(g.x), bf_lo(g.y), bf_hi(g.y));
    }

  pdl_wait();  // everything below may read what the previous kernel wrote
  unsigned epoch = 0;
  if (a.epoch) epoch = *reinterpret_cast<volatile unsigned*>(a.epoch);
  if (a.nwait > 0) {
    // Every rank's partial sum of this input has landed in our receive
    // buffer once each rank's flag holds this step's epoch. Bounded; after a
    // timeout (or an earlier one, recorded in the error word) the kernel
    // goes on without waiting, and the host reports TB200_ERR_TIMEOUT.
    if (tid == 0) {
      const volatile unsigned* f = a.wait_flags;
      const volatile int* err = a.err;
      const long long t0 = clock64();
      bool ok = *err != 0;
      while (!ok) {
        ok = true;
        for (int p = 0; p < a.nwait; p++) ok = ok && f[p] == epoch;
        if (!ok && clock64() - t0 > kWaitCycles) {
          set_error(a.err, TB200_ERR_TIMEOUT);
          break;
        }
      }
      __threadfence_system();  // acquire: the peers' stores before their flags
    }
    named_sync(1, kMvWarps * 32);
  }
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, c, TB200_TRACE_WAITED);
  // The residual rows, the input and the partials are all requested before
  // any is used, so staging costs one round trip to L2.
  float rres = 0.f;
  if (EPI == kMvResidual && tid < nrows) rres = __ldcg((a.resid_src ? a.resid_src : a.out) + r0 + tid);
  float ss = 0.f;
  float4 xr[kXregCols / 256][2];
  if (xreg) {
#pragma unroll
    for (int k = 0; k < kXregCols / 256; k++) {
      xr[k][0] = __ldcg(reinterpret_cast<const float4*>(a.x + 256 * k + lane * 8));
      xr[k][1] = __ldcg(reinterpret_cast<const float4*>(a.x + 256 * k + lane * 8 + 4));
    }
  }
  for (int i = tid * 4; !xreg && i < cols; i += kMvWarps * 32 * 4) {
    float4 v = __ldcg(reinterpret_cast<const float4*>(a.x + i));
    if (a.npartials > 0) {
      // x + (p0 + p1 + ...): the o_proj output summed in group order, then
      // added to the residual as the reference adds the whole product.
      float4 pv[kMaxPartials];
#pragma unroll
      for (int p = 0; p < kMaxPartials; p++)
        if (p < a.npartials) pv[p] = __ldcg(reinterpret_cast<const float4*>(a.partials + size_t(p) * cols + i));
      float4 t = pv[0];
#pragma unroll
      for (int p = 1; p < kMaxPartials; p++)
        if (p < a.npartials) {
          t.x += pv[p].x;
          t.y += pv[p].y;
          t.z += pv[p].z;
          t.w += pv[p].w;
        }
      v.x += t.x;
      v.y += t.y;
      v.z += t.z;
      v.w += t.w;
    }
    if (a.x_out && c == 0) *reinterpret_cast<float4*>(a.x_out + i) = v;
    if (NORM) {
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      const float4 g = *reinterpret_cast<const float4*>(nw + i);
      v.x *= g.x;
      v.y *= g.y;
      v.z *= g.z;
      v.w *= g.w;
    }
    // Permuted layout: the four values at column i = 256k + 8l + 4h go to
    // 256k + 128h + 4l, so a warp reading a 256-column block (lane l: 8l ..
    // 8l+7) reads two runs of 512 contiguous bytes, free of bank conflicts.
    *reinterpret_cast<float4*>(xs + xperm(i)) = v;
  }
  float scale = 1.0f;
  if (xreg) {
    if (NORM) {
#pragma unroll
      for (int k = 0; k < kXregCols / 256; k++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const float4 v = xr[k][h];
          ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
      ss = warp_sum(ss);
      scale = 1.0f / sqrtf(ss / float(cols) + a.eps);
#pragma unroll
      for (int k = 0; k < kXregCols / 256; k++) {
        const uint4 g = gw[k];
        xr[k][0].x *= bf_lo(g.x);
        xr[k][0].y *= bf_hi(g.x);
        xr[k][0].z *= bf_lo(g.y);
        xr[k][0].w *= bf_hi(g.y);
        xr[k][1].x *= bf_lo(g.z);
        xr[k][1].y *= bf_hi(g.z);
        xr[k][1].z *= bf_lo(g.w);
        xr[k][1].w *= bf_hi(g.w);
      }
    }
  } else {
    if (EPI == kMvResidual && tid < nrows) resid[tid] = rres;
    if (NORM) {
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
    }
    named_sync(1, kMvWarps * 32);
    if (NORM) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kMvWarps; w++) tot += red[w];
      scale = 1.0f / sqrtf(tot / float(cols) + a.eps);
    }
  }
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, c, TB200_TRACE_INPUT);

  unsigned long long best = 0ull;
  for (int st = 0; st < nstages; st++) {
    const int s = st % slots;
    if (!mbar_wait(&full[s], (st / slots) & 1, a.err)) {
      // Give an in-flight copy one more bounded wait to land, then skip the
      // rest; every consumer still reaches the barriers below.
      mbar_wait(&full[s], (st / slots) & 1, nullptr);
      break;
    }
    if (tid == 0 && st == 0) trace_at(a.trace, a.trace_base, a.tag, c, TB200_TRACE_WEIGHTS);
    if (tid == 0 && st == nstages - 1) trace_at(a.trace, a.trace_base, a.tag, c, TB200_TRACE_LAST_WEIGHTS);
    if (KS) {
      // K-split: every warp takes every row of the stage over its share of
      // the columns (8-column units tid, tid + 256, ...); warp sums meet in
      // shared memory and warp 0 finishes the rows.
      const int row0 = st * stage_rows;
      const int nrs = min(stage_rows, nrows - row0);
      const unsigned char* base = ring + size_t(s) * stage_bytes;
      float acc[kMvKsplitRows];
#pragma unroll
      for (int r = 0; r < kMvKsplitRows; r++) acc[r] = 0.f;
      for (int u = tid; u < cols / 8; u += kMvWarps * 32) {
        const float* xb0 = xs + (u >> 5) * 256 + (u & 31) * 4;
        const float4 xa = *reinterpret_cast<const float4*>(xb0);
        const float4 xb = *reinterpret_cast<const float4*>(xb0 + 128);
#pragma unroll
        for (int r = 0; r < kMvKsplitRows; r++)
          if (r < nrs) acc[r] = dot8(*reinterpret_cast<const uint4*>(base + size_t(r) * row_bytes + size_t(u) * 16), xa, xb, acc[r]);
      }
#pragma unroll
      for (int r = 0; r < kMvKsplitRows; r++)
        if (r < nrs) {
          const float v = warp_sum(acc[r]);
          if (lane == 0) ksum[warp][r] = v;
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      named_sync(1, kMvWarps * 32);
      if (warp == 0) {
        float v = 0.f;
        if (lane < nrs) {
#pragma unroll
          for (int w = 0; w < kMvWarps; w++) v += ksum[w][lane];
          v *= scale;
        }
        if (EPI == kMvSiluPair) {
          const float u = __shfl_down_sync(0xffffffffu, v, 1);
          if ((lane & 1) == 0 && lane < nrs) {
            const int row = r0 + row0 + lane;
            a.out[row / 2] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u);
          }
        } else if (lane < nrs) {
          const int row = r0 + row0 + lane;
          if (EPI == kMvResidual) {
            a.out[row] = __fadd_rn(resid[row - r0], v);
          } else if (EPI == kMvStore && a.npeers > 0) {
            for (int p = 0; p < a.npeers; p++) a.peer_out[p][row] = v;
          } else {
            a.out[row] = v;
            if (EPI == kMvArgmax) {
              const unsigned long long k = argmax_key(v, uint32_t(row));
              best = k > best ? k : best;
            }
          }
        }
      }
      named_sync(1, kMvWarps * 32);  // ksum is reused by the next stage
      continue;
    }
    const int first = st * stage_rows + warp * CH;  // this warp's first row, relative to r0
    const int nr = max(0, min(CH, min(nrows, (st + 1) * stage_rows) - first));
    if (nr > 0) {
      const unsigned char* base = ring + size_t(s) * stage_bytes + size_t(warp * CH) * row_bytes;
      // Two accumulators per row (the first and last four products of each
      // eight) and every weight fragment of an iteration loaded before use:
      // short dependency chains, many loads in flight.
      float acc[CH], acc2[CH];
#pragma unroll
      for (int r = 0; r < CH; r++) acc[r] = acc2[r] = 0.f;
      // Columns col .. col + 7 of this warp's rows against x[col .. col + 7] = (xa, xb).
      auto chunk = [&](int col, const float4& xa, const float4& xb) {
        uint4 wv[CH];
#pragma unroll
        for (int r = 0; r < CH; r++)
          wv[r] = r < nr ? *reinterpret_cast<const uint4*>(base + size_t(r) * row_bytes + size_t(col) * 2)
                         : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int r = 0; r < CH; r++) {
          acc[r] = dot4(wv[r].x, wv[r].y, xa, acc[r]);
          acc2[r] = dot4(wv[r].z, wv[r].w, xb, acc2[r]);
        }
      };
      if (xreg) {
#pragma unroll
        for (int k = 0; k < kXregCols / 256; k++) chunk(256 * k + lane * 8, xr[k][0], xr[k][1]);
      } else {
#pragma unroll 4
        for (int col = lane * 8; col < cols; col += 256) {
          const float* xb0 = xs + (col - lane * 8) + lane * 4;
          chunk(col, *reinterpret_cast<const float4*>(xb0), *reinterpret_cast<const float4*>(xb0 + 128));
        }
      }
#pragma unroll
      for (int r = 0; r < CH; r++) acc[r] = warp_sum(acc[r] + acc2[r]) * scale;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);

      const int rb = r0 + first;
      if (EPI == kMvSiluPair) {
        // rows rb + 2p (gate) and rb + 2p + 1 (up) -> out[rb/2 + p]
#pragma unroll
        for (int p = 0; p < CH / 2; p++) {
          if (lane == p && 2 * p < nr) {
            const float g = acc[2 * p], u = acc[2 * p + 1];
            a.out[rb / 2 + p] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
          }
        }
      } else {
        float v = acc[0];
#pragma unroll
        for (int r = 1; r < CH; r++)
          if (lane == r) v = acc[r];
        if (lane < nr) {
          const int row = rb + lane;
          if (EPI == kMvResidual) {
            a.out[row] = __fadd_rn(resid[row - r0], v);
          } else if (EPI == kMvStore && a.npeers > 0) {
            for (int p = 0; p < a.npeers; p++) a.peer_out[p][row] = v;
          } else {
            a.out[row] = v;
            if (EPI == kMvArgmax) {
              const unsigned long long k = argmax_key(v, uint32_t(row));
              best = k > best ? k : best;
            }
          }
        }
      }
    } else {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }

  if (EPI == kMvStore && a.npeers > 0) {
    // Release: every CTA's peer stores, then the last CTA to arrive writes
    // this step's epoch into each rank's flag word for this rank.
    __shared__ int last_p2p;
    __threadfence_system();
    named_sync(1, kMvWarps * 32);
    if (tid == 0) last_p2p = atomicAdd(a.p2p_ticket, 1u) == unsigned(G - 1);
    named_sync(1, kMvWarps * 32);
    if (last_p2p && tid == 0) {
      __threadfence_system();
      *a.p2p_ticket = 0u;
      for (int p = 0; p < a.npeers; p++) *reinterpret_cast<volatile unsigned*>(a.peer_flag[p]) = epoch;
    }
  }
  if (a.trace.rec) {
    named_sync(1, kMvWarps * 32);
    if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, c, TB200_TRACE_DONE);
  }

  if (EPI == kMvArgmax) {
    best = warp_umax64(best);
    if (lane == 0) best_sm[warp] = best;
    named_sync(1, kMvWarps * 32);
    if (tid == 0) {
      unsigned long long b = 0ull;
#pragma unroll
      for (int w = 0; w < kMvWarps; w++) b = best_sm[w] > b ? best_sm[w] : b;
      a.partial[c] = b;
      __threadfence();
      is_last = (atomicAdd(a.ticket, 1u) == unsigned(G - 1));
    }
    named_sync(1, kMvWarps * 32);
    if (is_last && warp == 0) {
      __threadfence();
      unsigned long long b = 0ull;
      for (int k = lane; k < G; k += 32) {
        const unsigned long long v = __ldcg(a.partial + k);
        b = v > b ? v : b;
      }
      b = warp_umax64(b);
      if (lane == 0) {
        const int tok = int(argmax_index(b));
        *a.token = tok;
        const int stp = *a.step;
        if (stp >= 0 && stp < a.tokens_cap) a.tokens_out[stp] = tok;
        *a.step = stp + 1;
        *a.pos = *a.pos + 1;
        *a.ticket = 0u;
        if (a.epoch) *a.epoch = epoch + 1u;  // the next step's tag for the ranks' flags
      }
    }
  }
}

using MvFn = void (*)(MvArgs, int, int);

template <int CH, bool KS>
MvFn pick_epi(int epi, bool norm) {
  switch (epi) {
    case kMvStore: return norm ? mv_kernel<CH, kMvStore, true, KS> : mv_kernel<CH, kMvStore, false, KS>;
    case kMvResidual: return norm ? mv_kernel<CH, kMvResidual, true, KS> : mv_kernel<CH, kMvResidual, false, KS>;
    case kMvSiluPair:
      if (CH < 2 && !KS) return nullptr;
      return norm ? mv_kernel<CH, kMvSiluPair, true, KS> : mv_kernel<CH, kMvSiluPair, false, KS>;
    case kMvArgmax: return norm ? mv_kernel<CH, kMvArgmax, true, KS> : mv_kernel<CH, kMvArgmax, false, KS>;
  }
  return nullptr;
}

// ch == 0: the K-split kernel (stages of up to kMvKsplitRows rows).
MvFn pick_mv(int ch, int epi, bool norm) {
  switch (ch) {
    case 0: return pick_epi<1, true>(epi, norm);
    case 1: return pick_epi<1, false>(epi, norm);
    case 2: return pick_epi<2, false>(epi, norm);
    case 4: return pick_epi<4, false>(epi, norm);
    case 6: return pick_epi<6, false>(epi, norm);
    case 8: return pick_epi<8, false>(epi, norm);
  }
  return nullptr;
}

// ---- attention -------------------------------------------------------------

constexpr int kHd = 128;  // head_dim of the fused path (Qwen3)

// One CTA per (kv head, split of kAttnChunk positions). The key/value cache
// holds bf16 (F32KV false) or f32 (F32KV true) values, laid out
// [kv head][position][head_dim] per layer, so a split's earlier positions
// are one contiguous run, staged by bulk copy before the dependency wait.
template <int GRP, bool F32KV>
__global__ void __launch_bounds__(128) attn_decode(AttnArgs a) {
  using KV = typename std::conditional<F32KV, float, uint16_t>::type;
  extern __shared__ __align__(128) unsigned char smem[];
  KV* ks = reinterpret_cast<KV*>(smem);   // [kAttnChunk][kHd]
  KV* vs = ks + size_t(kAttnChunk) * kHd;  // [kAttnChunk][kHd]
  __shared__ __align__(16) float qs[GRP][kHd];
  __shared__ __align__(16) float kn[kHd];
  __shared__ __align__(16) float vn[kHd];
  __shared__ __align__(16) float qnw[kHd], knw[kHd], rope_row[kHd];
  __shared__ float wm[4][GRP], wl[4][GRP];
  __shared__ __align__(16) float wacc[4][GRP][kHd];
  __shared__ __align__(8) uint64_t kv_bar;
  __shared__ int is_last;

  pdl_launch_dependents();
  const int g = blockIdx.x, split = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t cta = blockIdx.x + blockIdx.y * gridDim.x;
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, cta, TB200_TRACE_START);

  // The position is written only at the end of the previous step, so it
  // and everything derived from it can be read before the wait.
  const int pos = *a.pos;
  const bool pos_ok = pos >= 0 && pos < a.max_len;
  const int ctx = pos + 1;
  const int nsplit = (ctx + kAttnChunk - 1) / kAttnChunk;
  const int p0 = split * kAttnChunk, p1 = min(ctx, p0 + kAttnChunk);
  const bool active = pos_ok && split < nsplit && nsplit <= a.max_split;
  const int cached = active ? max(0, min(p1, pos) - p0) : 0;  // positions already in the cache

  if (active) {
    if (tid == 0) {
      mbar_init(&kv_bar, 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0 && cached > 0) {
      const uint32_t bytes = uint32_t(cached) * kHd * sizeof(KV);
      const size_t at = (size_t(g) * a.max_len + p0) * kHd;
      const uint64_t pol = l2_evict_first();
      mbar_arrive_expect_tx(&kv_bar, 2 * bytes);
      bulk_g2s(ks, static_cast<const KV*>(a.k_cache) + at, bytes, &kv_bar, pol);
      bulk_g2s(vs, static_cast<const KV*>(a.v_cache) + at, bytes, &kv_bar, pol);
    }
    qnw[tid] = a.q_norm ? bf16f(a.q_norm[tid]) : 1.0f;
    knw[tid] = a.k_norm ? bf16f(a.k_norm[tid]) : 1.0f;
    rope_row[tid] = a.rope[size_t(pos) * kHd + tid];
  }

  pdl_wait();
  __syncthreads();  // the staged norm weights are read by other threads below
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, cta, TB200_TRACE_WAITED);
  if (!pos_ok || nsplit > a.max_split) {
    if (g == 0 && split == 0 && tid == 0) set_error(a.err, TB200_ERR_ARG);
    return;
  }
  if (!active) return;

  // QK-norm (rmsnorm over each head, model.rs:111-116) on this group's query
  // heads and on the key head; lane l holds elements 4l .. 4l+3.
  const float* qraw = a.qkv + size_t(g) * GRP * kHd;
  const float* kraw = a.qkv + size_t(a.n_heads) * kHd + size_t(g) * kHd;
  const float* vraw = kraw + size_t(a.n_kv_heads) * kHd;
  // All loads in flight before any is used (GRP + 1 heads over 4 warps).
  const float vval = __ldcg(vraw + tid);
  float4 qkv4[(GRP + 4) / 4];
#pragma unroll
  for (int j = 0; j < (GRP + 4) / 4; j++) {
    const int h = warp + 4 * j;
    if (h < GRP + 1) qkv4[j] = __ldcg(reinterpret_cast<const float4*>(h < GRP ? qraw + h * kHd : kraw) + lane);
  }
  vn[tid] = vval;
#pragma unroll
  for (int j = 0; j < (GRP + 4) / 4; j++) {
    const int h = warp + 4 * j;
    if (h >= GRP + 1) break;
    float4 v = qkv4[j];
    const bool has_norm = h < GRP ? a.q_norm != nullptr : a.k_norm != nullptr;
    if (has_norm) {
      const float* w = h < GRP ? qnw : knw;
      const float s = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
      const float scale = 1.0f / sqrtf(s / float(kHd) + a.eps);
      v.x = __fmul_rn(v.x, __fmul_rn(scale, w[4 * lane + 0]));
      v.y = __fmul_rn(v.y, __fmul_rn(scale, w[4 * lane + 1]));
      v.z = __fmul_rn(v.z, __fmul_rn(scale, w[4 * lane + 2]));
      v.w = __fmul_rn(v.w, __fmul_rn(scale, w[4 * lane + 3]));
    }
    float* dst = h < GRP ? qs[h] : kn;
    *reinterpret_cast<float4*>(dst + 4 * lane) = v;
  }
  __syncthreads();
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, cta, TB200_TRACE_INPUT);
  // RoPE (cpu.rs:96-111) at `pos`: element i pairs with i + 64.
  if (tid < kHd / 2) {
    const float c = rope_row[2 * tid], s = rope_row[2 * tid + 1];
#pragma unroll
    for (int h = 0; h < GRP + 1; h++) {
      float* x = h < GRP ? qs[h] : kn;
      const float u = x[tid], w = x[tid + kHd / 2];
      x[tid] = __fsub_rn(__fmul_rn(u, c), __fmul_rn(w, s));
      x[tid + kHd / 2] = __fadd_rn(__fmul_rn(w, c), __fmul_rn(u, s));
    }
  }
  __syncthreads();
  // A bf16 cache holds the rounded key and value; this step uses the rounded
  // values too, as every later step will.
  {
    const size_t at = (size_t(g) * a.max_len + pos) * kHd + tid;
    if (F32KV) {
      if (p1 == ctx) {
        static_cast<float*>(a.k_cache)[at] = kn[tid];
        static_cast<float*>(a.v_cache)[at] = vn[tid];
      }
    } else {
      const uint16_t kb = f2bf(kn[tid]), vb = f2bf(vn[tid]);
      kn[tid] = bf16f(kb);
      vn[tid] = bf16f(vb);
      if (p1 == ctx) {
        static_cast<uint16_t*>(a.k_cache)[at] = kb;
        static_cast<uint16_t*>(a.v_cache)[at] = vb;
      }
    }
  }
  __syncthreads();
  if (cached > 0 && !mbar_wait(&kv_bar, 0, a.err)) {
    mbar_wait(&kv_bar, 0, nullptr);  // one more bounded wait for the copy in flight
    return;
  }
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, cta, TB200_TRACE_WEIGHTS);

  const float scale = 1.0f / sqrtf(float(kHd));
  float q[GRP][4], acc[GRP][4], m[GRP], l[GRP];
#pragma unroll
  for (int h = 0; h < GRP; h++) {
    const float4 v = *reinterpret_cast<const float4*>(&qs[h][4 * lane]);
    q[h][0] = v.x; q[h][1] = v.y; q[h][2] = v.z; q[h][3] = v.w;
    acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = 0.f;
    m[h] = -INFINITY;
    l[h] = 0.f;
  }
  for (int t = p0 + warp; t < p1; t += 4) {
    float k4[4], v4[4];
    if (t == pos) {
      const float4 kk = *reinterpret_cast<const float4*>(&kn[4 * lane]);
      const float4 vv = *reinterpret_cast<const float4*>(&vn[4 * lane]);
      k4[0] = kk.x; k4[1] = kk.y; k4[2] = kk.z; k4[3] = kk.w;
      v4[0] = vv.x; v4[1] = vv.y; v4[2] = vv.z; v4[3] = vv.w;
    } else if (F32KV) {
      const float* kr = reinterpret_cast<const float*>(ks) + (t - p0) * kHd + 4 * lane;
      const float* vr = reinterpret_cast<const float*>(vs) + (t - p0) * kHd + 4 * lane;
      const float4 kk = *reinterpret_cast<const float4*>(kr);
      const float4 vv = *reinterpret_cast<const float4*>(vr);
      k4[0] = kk.x; k4[1] = kk.y; k4[2] = kk.z; k4[3] = kk.w;
      v4[0] = vv.x; v4[1] = vv.y; v4[2] = vv.z; v4[3] = vv.w;
    } else {
      const uint16_t* kr = reinterpret_cast<const uint16_t*>(ks) + (t - p0) * kHd + 4 * lane;
      const uint16_t* vr = reinterpret_cast<const uint16_t*>(vs) + (t - p0) * kHd + 4 * lane;
      const uint2 kw = *reinterpret_cast<const uint2*>(kr);
      const uint2 vw = *reinterpret_cast<const uint2*>(vr);
      k4[0] = bf_lo(kw.x); k4[1] = bf_hi(kw.x); k4[2] = bf_lo(kw.y); k4[3] = bf_hi(kw.y);
      v4[0] = bf_lo(vw.x); v4[1] = bf_hi(vw.x); v4[2] = bf_lo(vw.y); v4[3] = bf_hi(vw.y);
    }
#pragma unroll
    for (int h = 0; h < GRP; h++) {
      float d = q[h][0] * k4[0];
      d = fmaf(q[h][1], k4[1], d);
      d = fmaf(q[h][2], k4[2], d);
      d = fmaf(q[h][3], k4[3], d);
      const float s = scale * warp_sum(d);
      const float mn = fmaxf(m[h], s);
      const float corr = expf(m[h] - mn);
      const float p = expf(s - mn);
      l[h] = l[h] * corr + p;
#pragma unroll
      for (int e = 0; e < 4; e++) acc[h][e] = acc[h][e] * corr + p * v4[e];
      m[h] = mn;
    }
  }
#pragma unroll
  for (int h = 0; h < GRP; h++) {
    if (lane == 0) {
      wm[warp][h] = m[h];
      wl[warp][h] = l[h];
    }
    *reinterpret_cast<float4*>(&wacc[warp][h][4 * lane]) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
  }
  __syncthreads();

  // Merge the four warps: thread d of each head.
  const int stride = kPartStride;
  for (int h = 0; h < GRP; h++) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; w++) M = fmaxf(M, wm[w][h]);
    float L = 0.f, o = 0.f;
#pragma unroll
    for (int w = 0; w < 4; w++) {
      const float wt = wm[w][h] == -INFINITY ? 0.f : expf(wm[w][h] - M);
      L += wl[w][h] * wt;
      o += wacc[w][h][tid] * wt;
    }
    if (nsplit == 1) {
      a.out[size_t(g * GRP + h) * kHd + tid] = o / L;
    } else {
      float* pp = a.part + ((size_t(g) * a.max_split + split) * GRP + h) * stride;
      pp[tid] = o;
      if (tid == 0) {
        pp[kHd] = M;
        pp[kHd + 1] = L;
      }
    }
  }
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, cta, TB200_TRACE_DONE);
  if (nsplit == 1) return;

  // Split-context combine: the last CTA of this kv head merges the splits.
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = (atomicAdd(a.ticket + g, 1u) == unsigned(nsplit - 1));
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  {
    // The key/value staging area is free now: it holds the merge weights.
    __shared__ float hsum[GRP];
    float(*merged)[128] = reinterpret_cast<float(*)[128]>(wacc);  // the warp sums are consumed
    merge_splits<GRP>(a.part + size_t(g) * a.max_split * GRP * stride, nsplit, reinterpret_cast<float*>(smem), hsum,
                      merged);
#pragma unroll
    for (int h = 0; h < GRP; h++) a.out[size_t(g * GRP + h) * kHd + tid] = merged[h][tid];
  }
  if (tid == 0) a.ticket[g] = 0u;
}

// Fused attention + o_proj for short contexts. CTA (g, sl) stages, before
// the dependency wait, its packed o_proj slice (rows of output slice sl,
// columns of kv group g's query heads) and the group's cached keys and
// values; after the wait it QK-norms and rotates the group's query heads and
// key, appends the key and value (CTA sl == 0 writes the cache), and runs
// the group's attention in three passes (scores, softmax as the reference:
// exp(s - max) / sum, weighted values), then multiplies its o_proj slice by
// the group's attention output into part[g][rows of sl].
template <int GRP, bool F32KV>
__global__ void __launch_bounds__(256) attn_o(AttnOArgs a) {
  using KV = typename std::conditional<F32KV, float, uint16_t>::type;
  constexpr int kCols = GRP * kHd;
  extern __shared__ __align__(128) unsigned char smem[];
  uint16_t* wo = reinterpret_cast<uint16_t*>(smem);  // [rows_per_slice][kCols]
  KV* ks = reinterpret_cast<KV*>(smem + align_up(size_t(a.rows_per_slice) * kCols * 2, 128));
  KV* vs = ks + size_t(kAttnOMaxCtx) * kHd;
  __shared__ __align__(16) float qs[GRP][kHd];
  __shared__ __align__(16) float kn[kHd];
  __shared__ __align__(16) float vn[kHd];
  __shared__ __align__(16) float qnw[kHd], knw[kHd], rope_row[kHd];
  __shared__ float sc[GRP][kAttnOMaxCtx];
  __shared__ __align__(16) float att[kCols];
  __shared__ __align__(8) uint64_t bar;

  pdl_launch_dependents();
  const int g = blockIdx.x, sl = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t cta = blockIdx.x + blockIdx.y * gridDim.x;
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, cta, TB200_TRACE_START);

  const int pos = *a.pos;  // written only at the end of the previous step
  const bool ok = pos >= 0 && pos < a.max_len && pos < kAttnOMaxCtx;
  const uint32_t wo_bytes = uint32_t(a.rows_per_slice) * kCols * 2;
  const uint32_t kv_bytes = ok ? uint32_t(pos) * kHd * sizeof(KV) : 0u;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (ok) {
    if (tid == 0) {
      const uint64_t pol = l2_evict_first();
      mbar_arrive_expect_tx(&bar, wo_bytes + 2 * kv_bytes);
      bulk_g2s(wo, a.wo_packed + (size_t(g) * a.nslices + sl) * a.rows_per_slice * kCols, wo_bytes, &bar, pol);
      if (kv_bytes) {
        const size_t at = size_t(g) * a.max_len * kHd;
        bulk_g2s(ks, static_cast<const KV*>(a.k_cache) + at, kv_bytes, &bar, pol);
        bulk_g2s(vs, static_cast<const KV*>(a.v_cache) + at, kv_bytes, &bar, pol);
      }
    }
    if (tid < kHd) {
      qnw[tid] = a.q_norm ? bf16f(a.q_norm[tid]) : 1.0f;
      knw[tid] = a.k_norm ? bf16f(a.k_norm[tid]) : 1.0f;
      rope_row[tid] = a.rope[size_t(pos) * kHd + tid];
    }
  }

  pdl_wait();
  __syncthreads();
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, cta, TB200_TRACE_WAITED);
  if (!ok) {
    if (g == 0 && sl == 0 && tid == 0) set_error(a.err, TB200_ERR_ARG);
    return;
  }

  // QK-norm and RoPE, as in attn_decode.
  const float* qraw = a.qkv + size_t(g) * GRP * kHd;
  const float* kraw = a.qkv + size_t(a.n_heads) * kHd + size_t(g) * kHd;
  const float* vraw = kraw + size_t(a.n_kv_heads) * kHd;
  // Both loads in flight before either is used.
  const float vval = tid < kHd ? __ldcg(vraw + tid) : 0.f;
  float4 qkv4 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (warp < GRP + 1) qkv4 = __ldcg(reinterpret_cast<const float4*>(warp < GRP ? qraw + warp * kHd : kraw) + lane);
  if (tid < kHd) vn[tid] = vval;
  for (int h = warp; h < GRP + 1; h += 8) {
    float4 v = qkv4;
    const bool has_norm = h < GRP ? a.q_norm != nullptr : a.k_norm != nullptr;
    if (has_norm) {
      const float* w = h < GRP ? qnw : knw;
      const float s = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
      const float scale = 1.0f / sqrtf(s / float(kHd) + a.eps);
      v.x = __fmul_rn(v.x, __fmul_rn(scale, w[4 * lane + 0]));
      v.y = __fmul_rn(v.y, __fmul_rn(scale, w[4 * lane + 1]));
      v.z = __fmul_rn(v.z, __fmul_rn(scale, w[4 * lane + 2]));
      v.w = __fmul_rn(v.w, __fmul_rn(scale, w[4 * lane + 3]));
    }
    float* dst = h < GRP ? qs[h] : kn;
    *reinterpret_cast<float4*>(dst + 4 * lane) = v;
  }
  __syncthreads();
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, cta, TB200_TRACE_INPUT);
  if (tid < kHd / 2) {
    const float c = rope_row[2 * tid], s = rope_row[2 * tid + 1];
#pragma unroll
    for (int h = 0; h < GRP + 1; h++) {
      float* x = h < GRP ? qs[h] : kn;
      const float u = x[tid], w = x[tid + kHd / 2];
      x[tid] = __fsub_rn(__fmul_rn(u, c), __fmul_rn(w, s));
      x[tid + kHd / 2] = __fadd_rn(__fmul_rn(w, c), __fmul_rn(u, s));
    }
  }
  __syncthreads();
  if (tid < kHd) {
    const size_t at = (size_t(g) * a.max_len + pos) * kHd + tid;
    if (F32KV) {
      if (sl == 0) {
        static_cast<float*>(a.k_cache)[at] = kn[tid];
        static_cast<float*>(a.v_cache)[at] = vn[tid];
      }
    } else {
      const uint16_t kb = f2bf(kn[tid]), vb = f2bf(vn[tid]);
      kn[tid] = bf16f(kb);
      vn[tid] = bf16f(vb);
      if (sl == 0) {
        static_cast<uint16_t*>(a.k_cache)[at] = kb;
        static_cast<uint16_t*>(a.v_cache)[at] = vb;
      }
    }
  }
  __syncthreads();
  if (!mbar_wait(&bar, 0, a.err)) {
    mbar_wait(&bar, 0, nullptr);  // one more bounded wait for the copies in flight
    return;
  }
  if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, cta, TB200_TRACE_WEIGHTS);

  // Scores: s = scale * (q_h . k_t), one thread per (position, head), each
  // walking the head dimension from its own starting quad so that threads
  // on different positions hit different shared-memory banks.
  const float scale = 1.0f / sqrtf(float(kHd));
  for (int idx = tid; idx < (pos + 1) * GRP; idx += 256) {
    const int t = idx / GRP, h = idx % GRP;
    const float4* qv = reinterpret_cast<const float4*>(qs[h]);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int j = 0; j < kHd / 4; j++) {
      const int jj = (j + t) & (kHd / 4 - 1);
      float4 kk;
      if (t == pos) {
        kk = reinterpret_cast<const float4*>(kn)[jj];
      } else if (F32KV) {
        kk = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(ks) + t * kHd)[jj];
      } else {
        const uint2 kw = reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(ks) + t * kHd)[jj];
        kk = make_float4(bf_lo(kw.x), bf_hi(kw.x), bf_lo(kw.y), bf_hi(kw.y));
      }
      const float4 qq = qv[jj];
      float& s = acc[j & 3];
      s = fmaf(qq.x, kk.x, s);
      s = fmaf(qq.y, kk.y, s);
      s = fmaf(qq.z, kk.z, s);
      s = fmaf(qq.w, kk.w, s);
    }
    sc[h][t] = scale * ((acc[0] + acc[1]) + (acc[2] + acc[3]));
  }
  __syncthreads();
  // Softmax per head (cpu.rs:183-193): exp(s - max), then divide by the sum.
  for (int h = warp; h < GRP; h += 8) {
    const float s0 = lane <= pos ? sc[h][lane] : -INFINITY;
    const float s1 = lane + 32 <= pos ? sc[h][lane + 32] : -INFINITY;
    const float mx = warp_max(fmaxf(s0, s1));
    const float e0 = lane <= pos ? expf(s0 - mx) : 0.f;
    const float e1 = lane + 32 <= pos ? expf(s1 - mx) : 0.f;
    const float sum = warp_sum(e0 + e1);
    if (lane <= pos) sc[h][lane] = e0 / sum;
    if (lane + 32 <= pos) sc[h][lane + 32] = e1 / sum;
  }
  __syncthreads();
  // Weighted values: att[h][d] = sum_t p[h][t] * v_t[d], four partial sums.
  for (int o = tid; o < kCols; o += 256) {
    const int h = o / kHd, d = o % kHd;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int t = 0; t < pos; t++) {
      const float v = F32KV ? reinterpret_cast<const float*>(vs)[t * kHd + d]
                            : bf16f(reinterpret_cast<const uint16_t*>(vs)[t * kHd + d]);
      acc[t & 3] = fmaf(sc[h][t], v, acc[t & 3]);
    }
    acc[pos & 3] = fmaf(sc[h][pos], vn[d], acc[pos & 3]);
    att[o] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  }
  __syncthreads();
  // This CTA's share of o_proj: rows sl * R .. + R of part[g].
  // Eight rows per warp at a time: the attention output is read once per
  // eight rows and the eight reductions overlap.
  const int R = a.rows_per_slice;
  float* outp = a.part + size_t(g) * a.hidden + size_t(sl) * R;
  for (int base = warp * 8; base < R; base += 64) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.f;
#pragma unroll
    for (int col = lane * 8; col < kCols; col += 256) {
      const float4 xa = *reinterpret_cast<const float4*>(att + col);
      const float4 xb = *reinterpret_cast<const float4*>(att + col + 4);
#pragma unroll
      for (int i = 0; i < 8; i++)
        if (base + i < R) acc[i] = dot8(*reinterpret_cast<const uint4*>(wo + size_t(base + i) * kCols + col), xa, xb, acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = warp_sum(acc[i]);
    if (lane < 8 && base + lane < R) {
      float v = acc[0];
#pragma unroll
      for (int i = 1; i < 8; i++)
        if (lane == i) v = acc[i];
      outp[base + lane] = v;
    }
  }
  if (a.trace.rec) {
    __syncthreads();
    if (tid == 0) trace_at(a.trace, a.trace_base, a.tag, cta, TB200_TRACE_DONE);
  }
}

// dst[g][s][r][c] = wo[s * R + r][g * cols + c], cols = group * head_dim.
__global__ void k_pack_wo(uint16_t* __restrict__ dst, const uint16_t* __restrict__ wo, int hidden, int n_kv_heads,
                          int cols, int nslices) {
  const int R = hidden / nslices;
  const size_t total = size_t(n_kv_heads) * hidden * cols;
  const size_t q_dim = size_t(n_kv_heads) * cols;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
    const size_t c = i % cols;
    const size_t rest = i / cols;  // (g * nslices + s) * R + r
    const size_t r = rest % R;
    const size_t gs = rest / R;
    const size_t s = gs % nslices, g = gs / nslices;
    dst[i] = wo[(s * R + r) * q_dim + g * cols + c];
  }
}

__global__ void k_embed_token(float* __restrict__ out, const uint16_t* __restrict__ table, int dim,
                              const int* __restrict__ token, int vocab, int* err) {
  pdl_launch_dependents();
  pdl_wait();
  int t = *token;
  if (t < 0 || t >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) set_error(err, TB200_ERR_ARG);
    t = 0;
  }
  const uint16_t* row = table + size_t(t) * dim;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) out[i] = bf16f(row[i]);
}

__global__ void k_set_io(int* io, int token, int pos) {
  io[0] = token;
  io[1] = pos;
  io[2] = 0;
}

template <typename... KArgs, typename... Args>
void launch_ex(cudaStream_t s, dim3 grid, dim3 block, size_t smem, bool pdl, void (*kernel)(KArgs...),
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <int G, bool F>
cudaError_t setup_attn() {
  cudaError_t e = cudaFuncSetAttribute(attn_decode<G, F>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(attn_smem_bytes(F)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_decode<G, F>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
  return e;
}

}  // namespace

size_t attn_smem_bytes(bool kv_f32) { return size_t(2) * kAttnChunk * kHd * (kv_f32 ? 4 : 2); }

MvPlan plan_mv(int rows, int cols, int row_align, bool norm, int sms, size_t smem_budget) {
  MvPlan p;
  p.grid = sms;
  const int units = rows / row_align;
  const int rpc = (units + p.grid - 1) / p.grid * row_align;  // most rows any CTA gets
  const size_t row = size_t(cols) * 2;
  const size_t xs = (align_up(size_t(cols), 256) * 4) * (norm ? 2 : 1);
  p.max_rows = rpc;
  // Few rows per CTA (o_proj, down): K-split, one stage, all warps per row.
  if (rpc <= kMvKsplitRows && xs + size_t(kMvKsplitRows) * row + 64 <= smem_budget) {
    p.chunk_rows = 0;
    p.stage_rows = kMvKsplitRows;
    p.slots = 1;
    p.smem = xs + size_t(kMvKsplitRows) * row + 16;
    return p;
  }
  // A CTA whose whole slice fits stages it in one copy: each warp takes up
  // to 8 rows, and the kernel's shared memory stays small enough for the
  // next kernel to stage its own weights on the same SM meanwhile.
  for (int ch : {1, 2, 4, 6, 8}) {
    if (row_align == 2 && ch % 2) continue;
    if (kMvWarps * ch < rpc) continue;
    const size_t stage = size_t(kMvWarps) * ch * row;
    if (xs + stage + 64 <= smem_budget) {
      p.chunk_rows = ch;
      p.stage_rows = kMvWarps * ch;
      p.slots = 1;
      p.smem = xs + stage + 16;
      return p;
    }
    break;
  }
  // Otherwise stream the slice through a ring: a stage is one chunk of CH
  // rows per consumer warp, at most kMvStageBytes (fewer rows, some warps
  // idle, when rows are wide).
  int ch = int(std::min<size_t>(4, std::max<size_t>(1, kMvStageBytes / (kMvWarps * row))));
  if (ch == 3) ch = 4;
  if (row_align == 2 && ch < 2) ch = 2;
  p.chunk_rows = ch;
  int sr = std::min<int>(kMvWarps * ch, int(std::max<size_t>(size_t(ch), kMvStageBytes / row / ch * ch)));
  if (row_align == 2 && sr % 2) sr -= 1;
  p.stage_rows = sr;
  const size_t stage = size_t(sr) * row;
  const int nstages = (rpc + sr - 1) / sr;
  long long fit = (long long)((smem_budget - xs - 64) / (stage + 16));
  int slots = int(std::min<long long>(nstages, fit));
  if (slots < 2) slots = std::min(2, nstages);
  if (slots < 1) slots = 1;
  p.slots = slots;
  p.smem = xs + size_t(slots) * stage + size_t(slots) * 16;
  return p;
}

cudaError_t init_fused_kernels(int max_smem_optin) {
  // Every matrix-vector instantiation may use all the shared memory a block
  // can opt into, less its static shared memory; and every fused kernel asks
  // for the whole unified L1 as shared memory, so that a kernel and the next
  // one (staging its weights) fit on an SM together. Set once per device,
  // outside any stream capture.
  for (int ch : {0, 1, 2, 4, 6, 8})
    for (int epi = kMvStore; epi <= kMvArgmax; epi++)
      for (bool norm : {false, true})
        if (MvFn fn = pick_mv(ch, epi, norm)) {
          cudaFuncAttributes fa;
          cudaError_t e = cudaFuncGetAttributes(&fa, fn);
          if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     max_smem_optin - int(fa.sharedSizeBytes));
          if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     cudaSharedmemCarveoutMaxShared);
          if (e != cudaSuccess) return e;
        }
  cudaError_t e = cudaSuccess;
  for (cudaError_t r : {setup_attn<1, false>(), setup_attn<2, false>(), setup_attn<4, false>(),
                        setup_attn<8, false>(), setup_attn<1, true>(), setup_attn<2, true>(),
                        setup_attn<4, true>(), setup_attn<8, true>()})
    if (r != cudaSuccess) e = r;
  for (void* fn : {(void*)attn_o<1, false>, (void*)attn_o<2, false>, (void*)attn_o<4, false>,
                   (void*)attn_o<8, false>, (void*)attn_o<1, true>, (void*)attn_o<2, true>, (void*)attn_o<4, true>,
                   (void*)attn_o<8, true>}) {
    cudaFuncAttributes fa;
    cudaError_t r = cudaFuncGetAttributes(&fa, fn);
    if (r == cudaSuccess)
      r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               max_smem_optin - int(fa.sharedSizeBytes));
    if (r == cudaSuccess)
      r = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (r != cudaSuccess) e = r;
  }
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_embed_token, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
  return e;
}

void launch_mv(cudaStream_t s, const MvPlan& plan, int epilogue, const MvArgs& a, bool pdl) {
  MvFn fn = pick_mv(plan.chunk_rows, epilogue, a.norm_w != nullptr);
  launch_ex(s, dim3(plan.grid), dim3(kMvThreads), plan.smem, pdl, fn, a, plan.stage_rows, plan.slots);
}

void launch_attn_decode(cudaStream_t s, const AttnArgs& a, bool pdl) {
  const int group = a.n_heads / a.n_kv_heads;
  const dim3 grid(a.n_kv_heads, a.max_split);
  const size_t smem = attn_smem_bytes(a.kv_f32 != 0);
#define TB_ATTN_CASE(G)                                                   \
  case G:                                                                 \
    if (a.kv_f32)                                                         \
      launch_ex(s, grid, dim3(128), smem, pdl, attn_decode<G, true>, a);  \
    else                                                                  \
      launch_ex(s, grid, dim3(128), smem, pdl, attn_decode<G, false>, a); \
    break;
  switch (group) {
    TB_ATTN_CASE(1)
    TB_ATTN_CASE(2)
    TB_ATTN_CASE(4)
    TB_ATTN_CASE(8)
  }
#undef TB_ATTN_CASE
}

size_t attn_o_smem_bytes(int rows_per_slice, int group, bool kv_f32) {
  return align_up(size_t(rows_per_slice) * group * kHd * 2, 128) + size_t(2) * kAttnOMaxCtx * kHd * (kv_f32 ? 4 : 2);
}

int attn_o_slices(int hidden, int group) {
  const size_t row = size_t(group) * kHd * 2;
  for (int ns = 1; ns <= hidden; ns++)
    if (hidden % ns == 0 && size_t(hidden / ns) * row <= 48 * 1024) return ns;
  return hidden;
}

void launch_pack_wo(cudaStream_t s, uint16_t* dst, const uint16_t* wo, int hidden, int n_kv_heads, int group,
                    int nslices) {
  const size_t total = size_t(n_kv_heads) * hidden * group * kHd;
  const int grid = int(std::min<size_t>((total + 255) / 256, 148 * 16));
  k_pack_wo<<<grid, 256, 0, s>>>(dst, wo, hidden, n_kv_heads, group * kHd, nslices);
}

void launch_attn_o(cudaStream_t s, const AttnOArgs& a, bool pdl) {
  const int group = a.n_heads / a.n_kv_heads;
  const dim3 grid(a.n_kv_heads, a.nslices);
  const size_t smem = attn_o_smem_bytes(a.rows_per_slice, group, a.kv_f32 != 0);
#define TB_ATTNO_CASE(G)                                                  \
  case G:                                                                 \
    if (a.kv_f32)                                                         \
      launch_ex(s, grid, dim3(256), smem, pdl, attn_o<G, true>, a);       \
    else                                                                  \
      launch_ex(s, grid, dim3(256), smem, pdl, attn_o<G, false>, a);      \
    break;
  switch (group) {
    TB_ATTNO_CASE(1)
    TB_ATTNO_CASE(2)
    TB_ATTNO_CASE(4)
    TB_ATTNO_CASE(8)
  }
#undef TB_ATTNO_CASE
}

void launch_set_io(cudaStream_t s, int* io, int token, int pos) { k_set_io<<<1, 1, 0, s>>>(io, token, pos); }

void launch_embed_token(cudaStream_t s, float* out, const uint16_t* table, int dim, const int* token, int vocab,
                        int* err, bool pdl) {
  launch_ex(s, dim3((dim + 255) / 256), dim3(256), 0, pdl, k_embed_token, out, table, dim, token, vocab, err);
}

}  // namespace tb
