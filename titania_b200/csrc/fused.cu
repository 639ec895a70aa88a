// fused.cu — the fused batch-1 decode path (model/model.rs:93-149 for n = 1).
//
// One decode step is 2 + 5 * layers kernels, replayed from a CUDA graph:
//   embed_token                      x = table[token]
//   per layer:
//     mv<norm, store>      (q|k|v)   qkv = Wqkv · rmsnorm(x)
//     attn_decode                    QK-norm, RoPE, bf16 K/V append, GQA
//                                    attention (split over the context)
//     mv<residual>         (o)       x += Wo · att
//     mv<norm, silu pair>  (gate|up) h = silu(Wg · rmsnorm(x)) * (Wu · ...)
//     mv<residual>         (down)    x += Wd · h
//   mv<norm, argmax>       (lm_head) logits, greedy token, position += 1
//
// The matrix-vector kernel is the HBM-bound core (1.19 GB of weights per
// token for Qwen3-0.6B). Each CTA owns a contiguous slice of rows; a
// producer warp streams the slice into a shared-memory ring with
// cp.async.bulk (TMA bulk copies, L2 evict-first), and eight consumer warps
// each take whole chunks of rows. Kernels are launched with programmatic
// dependent launch: a kernel starts while its predecessor runs and stages
// its weights (which no kernel writes) before griddepcontrol.wait, so the
// weight stream does not stop at kernel boundaries.

#include <algorithm>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace tb {

namespace {

constexpr int kMvWarps = 8;                     // consumer warps
constexpr int kMvThreads = (kMvWarps + 1) * 32;  // + one producer warp

__host__ __device__ constexpr size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

template <int CH, int EPI, bool NORM>
__global__ void __launch_bounds__(kMvThreads) mv_kernel(MvArgs a, int slots) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float red[kMvWarps];
  __shared__ unsigned long long best_sm[kMvWarps];
  __shared__ int is_last;

  pdl_launch_dependents();

  const int cols = a.cols;
  float* xs = reinterpret_cast<float*>(smem);
  unsigned char* ring = smem + align_up(size_t(cols) * 4, 128);
  const uint32_t slot_bytes = uint32_t(CH) * cols * 2;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + size_t(slots) * slot_bytes);
  uint64_t* empty = full + slots;

  const int G = gridDim.x, c = blockIdx.x;
  const int units = a.rows / a.row_align;
  const int r0 = int((long long)c * units / G) * a.row_align;
  const int r1 = int((long long)(c + 1) * units / G) * a.row_align;
  const int nrows = r1 - r0;
  const int nchunks = (nrows + CH - 1) / CH;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < slots; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kMvWarps) {
    // Producer: weights are never written by a kernel, so they are staged
    // before (and while) the previous kernel finishes.
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      for (int i = 0; i < nchunks; i++) {
        const int s = i % slots;
        if (i >= slots && !mbar_wait(&empty[s], ((i / slots) - 1) & 1, a.err)) break;
        const int nr = min(CH, nrows - i * CH);
        const uint32_t bytes = uint32_t(nr) * cols * 2;
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(ring + size_t(s) * slot_bytes, a.w + size_t(r0 + i * CH) * cols, bytes, &full[s], pol);
      }
    }
    return;
  }

  // Consumers. Everything below may read what the previous kernel wrote.
  pdl_wait();
  const int tid = threadIdx.x;  // 0 .. 255
  float ss = 0.f;
  for (int i = tid * 4; i < cols; i += kMvWarps * 32 * 4) {
    float4 v = __ldcg(reinterpret_cast<const float4*>(a.x + i));
    *reinterpret_cast<float4*>(xs + i) = v;
    if (NORM) ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  if (NORM) {
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    named_sync(1, kMvWarps * 32);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kMvWarps; w++) tot += red[w];
    const float scale = 1.0f / sqrtf(tot / float(cols) + a.eps);
    for (int i = tid; i < cols; i += kMvWarps * 32) xs[i] = __fmul_rn(xs[i], __fmul_rn(scale, bf16f(a.norm_w[i])));
  }
  named_sync(1, kMvWarps * 32);

  unsigned long long best = 0ull;
  for (int i = warp; i < nchunks; i += kMvWarps) {
    const int s = i % slots;
    if (!mbar_wait(&full[s], (i / slots) & 1, a.err)) {
      // Give an in-flight copy one more bounded wait to land, then skip the
      // rest; every consumer still reaches the barriers below.
      mbar_wait(&full[s], (i / slots) & 1, nullptr);
      break;
    }
    const int nr = min(CH, nrows - i * CH);
    const unsigned char* base = ring + size_t(s) * slot_bytes;
    float acc[CH];
#pragma unroll
    for (int r = 0; r < CH; r++) acc[r] = 0.f;
    for (int col = lane * 8; col < cols; col += 256) {
      const float4 xa = *reinterpret_cast<const float4*>(xs + col);
      const float4 xb = *reinterpret_cast<const float4*>(xs + col + 4);
#pragma unroll
      for (int r = 0; r < CH; r++) {
        if (r < nr) {
          const uint4 wv = *reinterpret_cast<const uint4*>(base + (size_t(r) * cols + col) * 2);
          acc[r] = dot8(wv, xa, xb, acc[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < CH; r++) acc[r] = warp_sum(acc[r]);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    const int rb = r0 + i * CH;
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
          a.out[row] = __fadd_rn(__ldcg(a.out + row), v);
        } else {
          a.out[row] = v;
          if (EPI == kMvArgmax) {
            const unsigned long long k = argmax_key(v, uint32_t(row));
            best = k > best ? k : best;
          }
        }
      }
    }
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
        const int st = *a.step;
        if (st >= 0 && st < a.tokens_cap) a.tokens_out[st] = tok;
        *a.step = st + 1;
        *a.pos = *a.pos + 1;
        *a.ticket = 0u;
      }
    }
  }
}

using MvFn = void (*)(MvArgs, int);

template <int CH>
MvFn pick_epi(int epi, bool norm) {
  switch (epi) {
    case kMvStore: return norm ? mv_kernel<CH, kMvStore, true> : mv_kernel<CH, kMvStore, false>;
    case kMvResidual: return norm ? mv_kernel<CH, kMvResidual, true> : mv_kernel<CH, kMvResidual, false>;
    case kMvSiluPair:
      if (CH < 2) return nullptr;
      return norm ? mv_kernel<(CH < 2 ? 2 : CH), kMvSiluPair, true> : mv_kernel<(CH < 2 ? 2 : CH), kMvSiluPair, false>;
    case kMvArgmax: return norm ? mv_kernel<CH, kMvArgmax, true> : mv_kernel<CH, kMvArgmax, false>;
  }
  return nullptr;
}

MvFn pick_mv(int ch, int epi, bool norm) {
  switch (ch) {
    case 1: return pick_epi<1>(epi, norm);
    case 2: return pick_epi<2>(epi, norm);
    case 4: return pick_epi<4>(epi, norm);
  }
  return nullptr;
}

// ---- attention -------------------------------------------------------------

constexpr int kHd = 128;       // head_dim of the fused path (Qwen3)
constexpr int kAttnMinChunk = 64;

template <int GRP>
__global__ void __launch_bounds__(128) attn_decode(AttnArgs a) {
  __shared__ __align__(16) float qs[GRP][kHd];
  __shared__ __align__(16) float kn[kHd];
  __shared__ __align__(16) float vn[kHd];
  __shared__ float wm[4][GRP], wl[4][GRP];
  __shared__ __align__(16) float wacc[4][GRP][kHd];
  __shared__ int is_last;

  pdl_launch_dependents();
  const int g = blockIdx.x, split = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // The position is written only at the end of the previous step.
  const int pos = *a.pos;
  pdl_wait();
  if (pos < 0 || pos >= a.max_len) {
    if (g == 0 && split == 0 && tid == 0) set_error(a.err, TB200_ERR_ARG);
    return;
  }
  const int ctx = pos + 1;
  const int nact = min(a.max_split, (ctx + kAttnMinChunk - 1) / kAttnMinChunk);
  const int chunk = (ctx + nact - 1) / nact;
  const int p0 = split * chunk, p1 = min(ctx, p0 + chunk);
  if (split >= nact || p0 >= p1) return;

  // QK-norm (rmsnorm over each head, model.rs:111-116) on this group's query
  // heads and on the key head; lane l holds elements 4l .. 4l+3.
  const float* qraw = a.qkv + size_t(g) * GRP * kHd;
  const float* kraw = a.qkv + size_t(a.n_heads) * kHd + size_t(g) * kHd;
  const float* vraw = kraw + size_t(a.n_kv_heads) * kHd;
  for (int h = warp; h < GRP + 1; h += 4) {
    const float* src = h < GRP ? qraw + h * kHd : kraw;
    float4 v = __ldcg(reinterpret_cast<const float4*>(src) + lane);
    const uint16_t* nw = h < GRP ? a.q_norm : a.k_norm;
    if (nw) {
      float s = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
      const float scale = 1.0f / sqrtf(s / float(kHd) + a.eps);
      v.x = __fmul_rn(v.x, __fmul_rn(scale, bf16f(nw[4 * lane + 0])));
      v.y = __fmul_rn(v.y, __fmul_rn(scale, bf16f(nw[4 * lane + 1])));
      v.z = __fmul_rn(v.z, __fmul_rn(scale, bf16f(nw[4 * lane + 2])));
      v.w = __fmul_rn(v.w, __fmul_rn(scale, bf16f(nw[4 * lane + 3])));
    }
    float* dst = h < GRP ? qs[h] : kn;
    *reinterpret_cast<float4*>(dst + 4 * lane) = v;
  }
  vn[tid] = __ldcg(vraw + tid);
  __syncthreads();
  // RoPE (cpu.rs:96-111) at `pos`: element i pairs with i + 64.
  if (tid < kHd / 2) {
    const float c = a.rope[size_t(pos) * kHd + 2 * tid], s = a.rope[size_t(pos) * kHd + 2 * tid + 1];
#pragma unroll
    for (int h = 0; h < GRP + 1; h++) {
      float* x = h < GRP ? qs[h] : kn;
      const float u = x[tid], w = x[tid + kHd / 2];
      x[tid] = __fsub_rn(__fmul_rn(u, c), __fmul_rn(w, s));
      x[tid + kHd / 2] = __fadd_rn(__fmul_rn(w, c), __fmul_rn(u, s));
    }
  }
  __syncthreads();
  // The cache holds bf16; this step uses the rounded key and value too, as
  // every later step will.
  {
    const uint16_t kb = f2bf(kn[tid]), vb = f2bf(vn[tid]);
    kn[tid] = bf16f(kb);
    vn[tid] = bf16f(vb);
    if (p1 == ctx) {
      a.k_cache[(size_t(g) * a.max_len + pos) * kHd + tid] = kb;
      a.v_cache[(size_t(g) * a.max_len + pos) * kHd + tid] = vb;
    }
  }
  __syncthreads();

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
  const uint16_t* kbase = a.k_cache + size_t(g) * a.max_len * kHd + 4 * lane;
  const uint16_t* vbase = a.v_cache + size_t(g) * a.max_len * kHd + 4 * lane;
  for (int t = p0 + warp; t < p1; t += 4) {
    float k4[4], v4[4];
    if (t == pos) {
      const float4 kk = *reinterpret_cast<const float4*>(&kn[4 * lane]);
      const float4 vv = *reinterpret_cast<const float4*>(&vn[4 * lane]);
      k4[0] = kk.x; k4[1] = kk.y; k4[2] = kk.z; k4[3] = kk.w;
      v4[0] = vv.x; v4[1] = vv.y; v4[2] = vv.z; v4[3] = vv.w;
    } else {
      const uint2 kw = __ldcg(reinterpret_cast<const uint2*>(kbase + size_t(t) * kHd));
      const uint2 vw = __ldcg(reinterpret_cast<const uint2*>(vbase + size_t(t) * kHd));
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
  const int stride = kHd + 2;
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
    if (nact == 1) {
      a.out[size_t(g * GRP + h) * kHd + tid] = o / L;
    } else {
      float* pp = a.part + ((size_t(g) * a.max_split + split) * GRP + h) * stride;
      pp[2 + tid] = o;
      if (tid == 0) {
        pp[0] = M;
        pp[1] = L;
      }
    }
  }
  if (nact == 1) return;

  // Split-context combine: the last CTA of this kv head merges the splits.
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = (atomicAdd(a.ticket + g, 1u) == unsigned(nact - 1));
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int h = 0; h < GRP; h++) {
    float M = -INFINITY;
    for (int sp = 0; sp < nact; sp++)
      M = fmaxf(M, __ldcg(a.part + ((size_t(g) * a.max_split + sp) * GRP + h) * stride));
    float L = 0.f, o = 0.f;
    for (int sp = 0; sp < nact; sp++) {
      const float* pp = a.part + ((size_t(g) * a.max_split + sp) * GRP + h) * stride;
      const float mm = __ldcg(pp);
      const float wt = mm == -INFINITY ? 0.f : expf(mm - M);
      L += __ldcg(pp + 1) * wt;
      o += __ldcg(pp + 2 + tid) * wt;
    }
    a.out[size_t(g * GRP + h) * kHd + tid] = o / L;
  }
  if (tid == 0) a.ticket[g] = 0u;
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

}  // namespace

MvPlan plan_mv(int rows, int cols, int row_align, int sms, size_t smem_budget) {
  MvPlan p;
  p.grid = sms;
  const int units = rows / row_align;
  const int rpc = (units + p.grid - 1) / p.grid * row_align;  // most rows any CTA gets
  int ch = rpc >= 16 ? 4 : (rpc >= 8 ? 2 : 1);
  if (row_align == 2 && ch < 2) ch = 2;
  p.chunk_rows = ch;
  const size_t slot = size_t(ch) * cols * 2;
  const size_t xs = align_up(size_t(cols) * 4, 128);
  const int nchunks = (rpc + ch - 1) / ch;
  long long fit = (long long)((smem_budget - xs - 64) / (slot + 16));
  int slots = int(std::min<long long>(nchunks, fit));
  if (slots < 2) slots = 2;
  p.slots = slots;
  p.smem = xs + size_t(slots) * slot + size_t(slots) * 16;
  return p;
}

void init_fused_kernels() {
  // Every instantiation may use up to 227 KB of dynamic shared memory; set
  // once, outside any stream capture.
  static std::once_flag once;
  std::call_once(once, [] {
    for (int ch : {1, 2, 4})
      for (int epi = kMvStore; epi <= kMvArgmax; epi++)
        for (bool norm : {false, true})
          if (MvFn fn = pick_mv(ch, epi, norm))
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
}

void launch_mv(cudaStream_t s, const MvPlan& plan, int epilogue, const MvArgs& a, bool pdl) {
  MvFn fn = pick_mv(plan.chunk_rows, epilogue, a.norm_w != nullptr);
  launch_ex(s, dim3(plan.grid), dim3(kMvThreads), plan.smem, pdl, fn, a, plan.slots);
}

void launch_attn_decode(cudaStream_t s, const AttnArgs& a, bool pdl) {
  const int group = a.n_heads / a.n_kv_heads;
  dim3 grid(a.n_kv_heads, a.max_split);
  switch (group) {
    case 1: launch_ex(s, grid, dim3(128), 0, pdl, attn_decode<1>, a); break;
    case 2: launch_ex(s, grid, dim3(128), 0, pdl, attn_decode<2>, a); break;
    case 4: launch_ex(s, grid, dim3(128), 0, pdl, attn_decode<4>, a); break;
    case 8: launch_ex(s, grid, dim3(128), 0, pdl, attn_decode<8>, a); break;
  }
}

void launch_set_io(cudaStream_t s, int* io, int token, int pos) { k_set_io<<<1, 1, 0, s>>>(io, token, pos); }

void launch_embed_token(cudaStream_t s, float* out, const uint16_t* table, int dim, const int* token, int vocab,
                        int* err, bool pdl) {
  launch_ex(s, dim3((dim + 255) / 256), dim3(256), 0, pdl, k_embed_token, out, table, dim, token, vocab, err);
}

}  // namespace tb
