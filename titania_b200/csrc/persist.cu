// persist.cu — batch-1 greedy decode with one persistent kernel per step
// (model/model.rs:83-149 for one token, then the greedy choice of
// model/sampler.rs:31-33), an opt-in alternative to the fused path's chain of
// 2 + 5 * layers kernels.
//
// One CTA per SM for the whole step (a cooperative launch, so CTAs may wait
// on one another); phases exchange vectors as 64-bit (tag << 32 | value bits)
// words, so data and synchronisation cost one L2 round trip together; one
// producer warp streams this CTA's weight rows for every phase of the step
// through a shared-memory ring without draining it at phase boundaries.
// Every wait is bounded, and no control flow depends on a wait's outcome: the
// first wait that gives up sets the CTA's abort flag and the error word,
// every later wait returns at once, and all threads still reach every
// barrier, so the kernel ends promptly and drains its copies in flight.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <string>

#include "runtime.h"

namespace tb::persist {

constexpr int kWarps = 8;
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kSlotBytes = 64 * 1024;
constexpr int kSlots = 3;
constexpr int kMaxLayers = 64;
constexpr int kHd = 128;
constexpr int kMaxCols = 3072;  // widest input vector
constexpr int kKsplitRows = 8;
constexpr int kMaxGrp = 4;      // query heads per kv head
constexpr int kAttnPer = 8;     // cached positions per warp held in registers at a time
// Longest context the entry point accepts: one register chunk of cached
// positions per warp (the chunk loop beyond it is written, not yet checked).
constexpr int kMaxCtx = kWarps * kAttnPer;
constexpr size_t kSmemBytes = size_t(2) * kMaxCols * 4 + size_t(kSlots) * kSlotBytes + 2 * kSlots * 8;

using TW = unsigned long long;  // a tagged word

struct Layer {
  const uint16_t *wqkv, *wo, *wgu, *wd;  // [Q+2KV][H], [H][Q], [2F][H] (gate/up rows interleaved), [H][F]
  const uint16_t *attn_norm, *mlp_norm, *q_norm, *k_norm;
  float *kc, *vc;  // [Hkv][max_len][kHd] f32
};

struct Args {
  Layer layer[kMaxLayers];
  int L, H, Q, KV, F, V, Hq, Hkv;
  float eps;
  const uint16_t *embed, *lm_head, *norm;
  const float* rope;  // [max_len][kHd] (cos, sin) pairs
  int max_len;
  TW *x, *qkv, *att, *h;  // [H], [Q+2KV], [Q], [F]
  int* token;
  int* pos;
  uint32_t* epoch;          // tag base of this step (advanced by the last CTA)
  unsigned long long* best;
  unsigned* ticket;
  int* err;
  float* logits;  // [V] or null: the lm_head rows as well as their argmax
  int* tokens;    // [steps]: token of the step at position p goes to tokens[p - pos0]
  int pos0;
};

enum { P_QKV = 0, P_ATT = 1, P_O = 2, P_GU = 3, P_DOWN = 4, kPerLayer = 5 };
// Tag offset of a phase's output (0 is the embedding).
__host__ __device__ constexpr uint32_t phase_index(int layer, int p) { return 1u + uint32_t(layer) * kPerLayer + p; }

struct Slice {
  const uint16_t* w;
  int r0, n, cols;
};

// Rows [r0, r0 + n) of a matrix phase for CTA `cta` of G (layer == L: lm_head).
__device__ __forceinline__ Slice slice_of(const Args& a, int layer, int p, int cta, int G) {
  const Layer& Ly = a.layer[layer < a.L ? layer : 0];
  int rows, cols, align;
  const uint16_t* w;
  if (layer == a.L) {
    w = a.lm_head, rows = a.V, cols = a.H, align = 1;
  } else if (p == P_QKV) {
    w = Ly.wqkv, rows = a.Q + 2 * a.KV, cols = a.H, align = 1;
  } else if (p == P_O) {
    w = Ly.wo, rows = a.H, cols = a.Q, align = 1;
  } else if (p == P_GU) {
    w = Ly.wgu, rows = 2 * a.F, cols = a.H, align = 2;
  } else {
    w = Ly.wd, rows = a.H, cols = a.F, align = 1;
  }
  const int units = rows / align;
  const int r0 = int((long long)cta * units / G) * align;
  const int r1 = int((long long)(cta + 1) * units / G) * align;
  return Slice{w, r0, r1 - r0, cols};
}

// Rows per stage: a slice of <= kKsplitRows rows is one K-split stage; else
// up to 4 rows per consumer warp, within one slot.
__device__ __forceinline__ int stage_rows(const Slice& s) {
  if (s.n <= kKsplitRows) return s.n;
  const int fit = kSlotBytes / (s.cols * 2);
  return min(fit, kWarps * 4) & ~1;
}

__device__ __forceinline__ void st_tagged(TW* p, float v, uint32_t tag) {
  const TW w = (TW(tag) << 32) | TW(__float_as_uint(v));
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ TW ld_tagged(const TW* p) {
  TW w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Two tagged words; each 64-bit element is read atomically.
__device__ __forceinline__ void ld_tagged2(const TW* p, TW& a, TW& b) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ float tval(TW w) { return __uint_as_float(uint32_t(w)); }
__device__ __forceinline__ uint32_t ttag(TW w) { return uint32_t(w >> 32); }

// Polls *p until it carries `tag`; bounded (see the abort rule above).
__device__ __forceinline__ float wait_word(const TW* p, uint32_t tag, uint64_t t0, int* err, volatile int* abort) {
  for (;;) {
    const TW w = ld_tagged(p);
    if (ttag(w) == tag || *abort) return tval(w);
    if (global_ns() - t0 > kWaitNs) {
      set_error(err, TB200_ERR_TIMEOUT);
      *abort = 1;
      return tval(w);
    }
  }
}

// mbar_wait under the abort rule.
__device__ __forceinline__ void wait_full(uint64_t* bar, uint32_t parity, int* err, volatile int* abort) {
  if (*abort) return;
  if (!mbar_wait(bar, parity, err)) *abort = 1;
}

// Consumer thread `tid` polls its groups of 4 words of vec[0, n) until every
// word carries `tag` and stores the values to xs, permuted as the library's
// matrix-vector kernel stores its input (column 256k + 8l + 4h at
// 256k + 128h + 4l). Bounded.
__device__ void poll_vector(const TW* vec, int n, uint32_t tag, float* xs, int tid, int* err, volatile int* abort) {
  const uint64_t t0 = global_ns();
  for (int i = tid * 4; i < n; i += kWarps * 32 * 4) {
    TW w0, w1, w2, w3;
    for (;;) {
      ld_tagged2(vec + i, w0, w1);
      ld_tagged2(vec + i + 2, w2, w3);
      if ((ttag(w0) == tag && ttag(w1) == tag && ttag(w2) == tag && ttag(w3) == tag) || *abort) break;
      if (global_ns() - t0 > kWaitNs) {
        set_error(err, TB200_ERR_TIMEOUT);
        *abort = 1;
        break;
      }
    }
    const int at = (i & ~255) + ((i >> 2) & 1) * 128 + ((i >> 3) & 31) * 4;
    *reinterpret_cast<float4*>(xs + at) = make_float4(tval(w0), tval(w1), tval(w2), tval(w3));
  }
}

// Attention for kv head g at position pos (model.rs:107-124 for one token):
// QK-norm of the group's query heads and the key, RoPE, K/V append, then the
// softmax-weighted sum of values over positions 0..pos, warps taking
// positions w, w + 8, ... with their own online softmax, merged at the end.
// `sm` holds at least 5000 floats. Run by the 256 consumer threads.
__device__ void attention_phase(const Args& a, const Layer& Ly, int g, int pos, uint32_t in_tag, uint32_t out_tag,
                                float* sm, int tid, volatile int* abort) {
  const int grp = a.Hq / a.Hkv;
  const int warp = tid >> 5, lane = tid & 31;
  float* qs = sm;                           // [grp][kHd]
  float* kn = qs + kMaxGrp * kHd;           // [kHd]
  float* vn = kn + kHd;                     // [kHd]
  float* wm = vn + kHd;                     // [kWarps][kMaxGrp]
  float* wl = wm + kWarps * kMaxGrp;        // [kWarps][kMaxGrp]
  float* wacc = wl + kWarps * kMaxGrp;      // [kWarps][kMaxGrp][kHd]

  // Cached keys and values (positions < pos) do not depend on this step:
  // the first chunk (positions warp + 8 i) is requested before the wait.
  float4 kr[kAttnPer], vr[kAttnPer];
  auto load_chunk = [&](int base) {
#pragma unroll
    for (int i = 0; i < kAttnPer; i++) {
      const int j = base + warp + kWarps * i;
      if (j < pos) {
        const size_t at = (size_t(g) * a.max_len + j) * kHd + 4 * lane;
        kr[i] = __ldcg(reinterpret_cast<const float4*>(Ly.kc + at));
        vr[i] = __ldcg(reinterpret_cast<const float4*>(Ly.vc + at));
      }
    }
  };
  load_chunk(0);

  // q (grp heads), k, v of this group from the tagged q|k|v vector.
  const uint64_t t0 = global_ns();
  for (int i = tid; i < (grp + 2) * kHd; i += kWarps * 32) {
    const int h = i / kHd, d = i % kHd;
    const int at = h < grp ? (g * grp + h) * kHd + d : h == grp ? a.Q + g * kHd + d : a.Q + a.KV + g * kHd + d;
    (h < grp ? qs + h * kHd : h == grp ? kn : vn)[d] = wait_word(a.qkv + at, in_tag, t0, a.err, abort);
  }
  named_sync(1, kWarps * 32);

  // QK-norm (rmsnorm over each head with q_norm / k_norm): warp h takes head h.
  if (warp < grp + 1) {
    float* x = warp < grp ? qs + warp * kHd : kn;
    const uint16_t* nw = warp < grp ? Ly.q_norm : Ly.k_norm;
    if (nw) {
      float4 v = *reinterpret_cast<float4*>(x + 4 * lane);
      const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
      const float scale = 1.0f / sqrtf(ss / float(kHd) + a.eps);
      v.x = __fmul_rn(v.x, __fmul_rn(scale, bf16f(nw[4 * lane + 0])));
      v.y = __fmul_rn(v.y, __fmul_rn(scale, bf16f(nw[4 * lane + 1])));
      v.z = __fmul_rn(v.z, __fmul_rn(scale, bf16f(nw[4 * lane + 2])));
      v.w = __fmul_rn(v.w, __fmul_rn(scale, bf16f(nw[4 * lane + 3])));
      *reinterpret_cast<float4*>(x + 4 * lane) = v;
    }
  }
  named_sync(1, kWarps * 32);
  // RoPE at pos: element i pairs with i + 64.
  if (tid < kHd / 2) {
    const float c = a.rope[size_t(pos) * kHd + 2 * tid], s = a.rope[size_t(pos) * kHd + 2 * tid + 1];
    for (int h = 0; h < grp + 1; h++) {
      float* x = h < grp ? qs + h * kHd : kn;
      const float u = x[tid], w = x[tid + kHd / 2];
      x[tid] = __fsub_rn(__fmul_rn(u, c), __fmul_rn(w, s));
      x[tid + kHd / 2] = __fadd_rn(__fmul_rn(w, c), __fmul_rn(u, s));
    }
  }
  named_sync(1, kWarps * 32);
  if (tid < kHd) {  // append this position's key and value
    const size_t at = (size_t(g) * a.max_len + pos) * kHd + tid;
    Ly.kc[at] = kn[tid];
    Ly.vc[at] = vn[tid];
  }

  // Online softmax per warp over positions warp, warp + 8, ...
  const float sc = 1.0f / sqrtf(float(kHd));
  float m[kMaxGrp], l[kMaxGrp];
  float4 acc[kMaxGrp];
#pragma unroll
  for (int h = 0; h < kMaxGrp; h++) {
    m[h] = -INFINITY;
    l[h] = 0.f;
    acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int base = 0; base <= pos; base += kWarps * kAttnPer) {
    if (base > 0) load_chunk(base);
#pragma unroll
    for (int i = 0; i < kAttnPer; i++) {
    const int j = base + warp + kWarps * i;
    if (j > pos) break;
    const float4 kj = j == pos ? *reinterpret_cast<const float4*>(kn + 4 * lane) : kr[i];
    const float4 vj = j == pos ? *reinterpret_cast<const float4*>(vn + 4 * lane) : vr[i];
#pragma unroll
    for (int h = 0; h < kMaxGrp; h++) {
      if (h >= grp) break;
      const float4 q = *reinterpret_cast<const float4*>(qs + h * kHd + 4 * lane);
      const float s = warp_sum(q.x * kj.x + q.y * kj.y + q.z * kj.z + q.w * kj.w) * sc;
      const float mn = fmaxf(m[h], s);
      const float corr = expf(m[h] - mn), p = expf(s - mn);
      l[h] = l[h] * corr + p;
      acc[h].x = acc[h].x * corr + p * vj.x;
      acc[h].y = acc[h].y * corr + p * vj.y;
      acc[h].z = acc[h].z * corr + p * vj.z;
      acc[h].w = acc[h].w * corr + p * vj.w;
      m[h] = mn;
    }
    }
  }
#pragma unroll
  for (int h = 0; h < kMaxGrp; h++) {
    if (h >= grp) break;
    if (lane == 0) {
      wm[warp * kMaxGrp + h] = m[h];
      wl[warp * kMaxGrp + h] = l[h];
    }
    *reinterpret_cast<float4*>(wacc + (warp * kMaxGrp + h) * kHd + 4 * lane) = acc[h];
  }
  named_sync(1, kWarps * 32);
  for (int i = tid; i < grp * kHd; i += kWarps * 32) {
    const int h = i / kHd, d = i % kHd;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; w++) M = fmaxf(M, wm[w * kMaxGrp + h]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < kWarps; w++) {
      const float e = wl[w * kMaxGrp + h] > 0.f ? expf(wm[w * kMaxGrp + h] - M) : 0.f;
      L += wl[w * kMaxGrp + h] * e;
      O += wacc[(w * kMaxGrp + h) * kHd + d] * e;
    }
    st_tagged(a.att + (g * grp + h) * kHd + d, O / L, out_tag);
  }
  named_sync(1, kWarps * 32);  // the scratch is reused by the next phase
}

__global__ void __launch_bounds__(kThreads, 1) step_kernel(Args a) {
  extern __shared__ __align__(128) unsigned char smem[];
  float* xs = reinterpret_cast<float*>(smem);  // [kMaxCols] permuted input
  float* nw = xs + kMaxCols;                   // [kMaxCols] norm weight (f32)
  unsigned char* ring = reinterpret_cast<unsigned char*>(nw + kMaxCols);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + size_t(kSlots) * kSlotBytes);
  uint64_t* empty = full + kSlots;
  __shared__ float red[kWarps];
  __shared__ float ksum[kWarps][kKsplitRows];
  __shared__ unsigned long long best_sm[kWarps];
  __shared__ volatile int abort_sm;  // a wait gave up (or the arguments are bad): wait no more
  __shared__ volatile int issued_sm;
  __shared__ int is_last;
  __shared__ int pos_ok;

  const int c = blockIdx.x, G = gridDim.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t epoch = *a.epoch;
  const int pos = *a.pos;

  if (tid == 0) {
    for (int s = 0; s < kSlots; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    fence_mbar_init();
    pos_ok = (pos >= 0 && pos < a.max_len && a.Hq / a.Hkv <= kMaxGrp) ? 1 : 0;
    abort_sm = pos_ok ? 0 : 1;
    issued_sm = 0;
    if (!pos_ok && c == 0) set_error(a.err, TB200_ERR_ARG);
  }
  __syncthreads();

  unsigned long long best = 0ull;
  if (warp == kWarps) {
    // ---- producer: every matrix phase's rows of this CTA, in phase order ----
    if (lane == 0 && !abort_sm) {
      const uint64_t pol = l2_evict_first();
      int k = 0;
      for (int layer = 0; layer <= a.L && !abort_sm; layer++)
        for (int p = 0; p < kPerLayer && !abort_sm; p++) {
          if (p == P_ATT) continue;
          if (layer == a.L && p != P_QKV) break;  // the lm_head
          const Slice s = slice_of(a, layer, p, c, G);
          const int sr = stage_rows(s);
          for (int r = 0; r < s.n && !abort_sm; r += sr, k++) {
            const int slot = k % kSlots;
            if (k >= kSlots && !mbar_wait(&empty[slot], ((k / kSlots) - 1) & 1, a.err)) {
              abort_sm = 1;
              break;
            }
            const uint32_t bytes = uint32_t(min(sr, s.n - r)) * uint32_t(s.cols) * 2;
            mbar_arrive_expect_tx(&full[slot], bytes);
            bulk_g2s(ring + size_t(slot) * kSlotBytes, s.w + size_t(s.r0 + r) * s.cols, bytes, &full[slot], pol);
            issued_sm = k + 1;
          }
        }
    }
  } else {
    // ---- consumers: the same control flow whatever the waits return ----
    {  // embedding rows of this CTA (the same rows it owns in o and down)
      const int tok = *a.token;
      const int r0 = int((long long)c * a.H / G), r1 = int((long long)(c + 1) * a.H / G);
      for (int r = r0 + tid; r < r1; r += kWarps * 32) st_tagged(a.x + r, bf16f(a.embed[size_t(tok) * a.H + r]), epoch);
    }
    int k = 0;
    uint32_t x_tag = epoch;  // tag of the residual stream's current version
    for (int layer = 0; layer <= a.L; layer++) {
      const Layer& Ly = a.layer[layer < a.L ? layer : 0];
      const bool head = layer == a.L;
      for (int p = 0; p < kPerLayer; p++) {
        if (head && p != P_QKV) break;
        const uint32_t out_tag = epoch + phase_index(layer, p);
        if (p == P_ATT) {
          // pos_ok is uniform: an invalid position never reaches the cache.
          if (c < a.Hkv && pos_ok)
            attention_phase(a, Ly, c, pos, epoch + phase_index(layer, P_QKV), out_tag, xs, tid, &abort_sm);
          continue;
        }
        const TW* in;
        int n_in;
        uint32_t in_tag;
        const uint16_t* norm = nullptr;
        if (p == P_QKV) {
          in = a.x, n_in = a.H, in_tag = x_tag, norm = head ? a.norm : Ly.attn_norm;
        } else if (p == P_O) {
          in = a.att, n_in = a.Q, in_tag = epoch + phase_index(layer, P_ATT);
        } else if (p == P_GU) {
          in = a.x, n_in = a.H, in_tag = x_tag, norm = Ly.mlp_norm;
        } else {
          in = a.h, n_in = a.F, in_tag = epoch + phase_index(layer, P_GU);
        }
        if (norm)
          for (int i = tid * 4; i < n_in; i += kWarps * 32 * 4) {
            const uint2 g = *reinterpret_cast<const uint2*>(norm + i);
            *reinterpret_cast<float4*>(nw + i) = make_float4(bf_lo(g.x), bf_hi(g.x), bf_lo(g.y), bf_hi(g.y));
          }
        poll_vector(in, n_in, in_tag, xs, tid, a.err, &abort_sm);
        named_sync(1, kWarps * 32);
        float scale = 1.0f;
        if (norm) {
          float ss = 0.f;
          for (int i = tid * 4; i < n_in; i += kWarps * 32 * 4) {
            const int at = (i & ~255) + ((i >> 2) & 1) * 128 + ((i >> 3) & 31) * 4;
            float4 v = *reinterpret_cast<float4*>(xs + at);
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            const float4 g = *reinterpret_cast<const float4*>(nw + i);
            v.x *= g.x, v.y *= g.y, v.z *= g.z, v.w *= g.w;
            *reinterpret_cast<float4*>(xs + at) = v;  // the same thread wrote this float4 above
          }
          ss = warp_sum(ss);
          if (lane == 0) red[warp] = ss;
          named_sync(1, kWarps * 32);
          float tot = 0.f;
          for (int w = 0; w < kWarps; w++) tot += red[w];
          scale = 1.0f / sqrtf(tot / float(n_in) + a.eps);
        }
        // One output row of a matrix phase.
        auto emit = [&](int row, float v) {
          if (head) {
            if (a.logits) a.logits[row] = v;
            const unsigned long long key = argmax_key(v, uint32_t(row));
            best = key > best ? key : best;
          } else if (p == P_QKV) {
            st_tagged(a.qkv + row, v, out_tag);
          } else {  // o_proj and down_proj: the residual add, on rows this CTA owns
            st_tagged(a.x + row, __fadd_rn(tval(ld_tagged(a.x + row)), v), out_tag);
          }
        };
        const Slice s = slice_of(a, layer, p, c, G);
        const int sr = stage_rows(s);
        const size_t rb = size_t(s.cols) * 2;
        for (int r = 0; r < s.n; r += sr, k++) {
          const int slot = k % kSlots;
          wait_full(&full[slot], (k / kSlots) & 1, a.err, &abort_sm);
          const unsigned char* base = ring + size_t(slot) * kSlotBytes;
          const int nrs = min(sr, s.n - r);
          if (s.n <= kKsplitRows) {  // all warps on every row, K split
            float acc[kKsplitRows];
#pragma unroll
            for (int j = 0; j < kKsplitRows; j++) acc[j] = 0.f;
            for (int u = tid; u < s.cols / 8; u += kWarps * 32) {
              const float* xb0 = xs + (u >> 5) * 256 + (u & 31) * 4;
              const float4 xa = *reinterpret_cast<const float4*>(xb0);
              const float4 xb = *reinterpret_cast<const float4*>(xb0 + 128);
#pragma unroll
              for (int j = 0; j < kKsplitRows; j++)
                if (j < nrs) acc[j] = dot8(*reinterpret_cast<const uint4*>(base + j * rb + size_t(u) * 16), xa, xb, acc[j]);
            }
#pragma unroll
            for (int j = 0; j < kKsplitRows; j++) {
              const float v = warp_sum(acc[j]);
              if (lane == 0) ksum[warp][j] = v;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            named_sync(1, kWarps * 32);
            if (warp == 0) {
              float v = 0.f;
              if (lane < nrs) {
                for (int w = 0; w < kWarps; w++) v += ksum[w][lane];
                v *= scale;
              }
              if (p == P_GU && !head) {  // rows 2i (gate), 2i + 1 (up) -> h[i]; stages hold even row counts
                const float up = __shfl_down_sync(0xffffffffu, v, 1);
                if ((lane & 1) == 0 && lane < nrs)
                  st_tagged(a.h + (s.r0 + r + lane) / 2, __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), up), out_tag);
              } else if (lane < nrs) {
                emit(s.r0 + r + lane, v);
              }
            }
            named_sync(1, kWarps * 32);  // ksum is reused
            continue;
          }
          const int first = warp * 4;
          const int nr = max(0, min(4, nrs - first));
          float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
          for (int col = lane * 8; col < s.cols; col += 256) {
            const float* xb0 = xs + (col - lane * 8) + lane * 4;
            const float4 xa = *reinterpret_cast<const float4*>(xb0);
            const float4 xb = *reinterpret_cast<const float4*>(xb0 + 128);
#pragma unroll
            for (int j = 0; j < 4; j++)
              if (j < nr) {
                const uint4 wv = *reinterpret_cast<const uint4*>(base + (first + j) * rb + size_t(col) * 2);
                acc[j] = dot4(wv.x, wv.y, xa, acc[j]);
                acc2[j] = dot4(wv.z, wv.w, xb, acc2[j]);
              }
          }
#pragma unroll
          for (int j = 0; j < 4; j++) acc[j] = warp_sum(acc[j] + acc2[j]) * scale;
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[slot]);
          const int row0 = s.r0 + r + first;
          if (p == P_GU && !head) {  // rows 2i (gate), 2i + 1 (up) -> h[i]
            if (lane < nr / 2) {
              const float gt = lane == 0 ? acc[0] : acc[2], up = lane == 0 ? acc[1] : acc[3];
              st_tagged(a.h + row0 / 2 + lane, __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up), out_tag);
            }
          } else if (lane < nr) {
            float v = acc[0];
#pragma unroll
            for (int j = 1; j < 4; j++)
              if (lane == j) v = acc[j];
            emit(row0 + lane, v);
          }
        }
        if (p == P_O || p == P_DOWN) x_tag = out_tag;
        named_sync(1, kWarps * 32);  // xs / nw are rewritten by the next phase
      }
    }
  }

  __syncthreads();  // producer done issuing (or gave up); consumers done
  if (abort_sm && tid == 0) {
    // Copies may still be landing in the ring: wait (bounded) for the last
    // one issued into each slot before the CTA's shared memory goes away.
    const int n = issued_sm;
    for (int s = 0; s < kSlots; s++) {
      int last = -1;
      for (int kk = n - 1; kk >= 0 && kk >= n - kSlots; kk--)
        if (kk % kSlots == s && last < 0) last = kk;  // the newest issue into slot s
      if (last >= 0) mbar_wait(&full[s], (last / kSlots) & 1, nullptr);
    }
  }

  // lm_head argmax across the grid; the last CTA advances token, position
  // and the tag base.
  if (warp < kWarps) {
    best = warp_umax64(best);
    if (lane == 0) best_sm[warp] = best;
  }
  __syncthreads();
  if (tid == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < kWarps; w++) b = best_sm[w] > b ? best_sm[w] : b;
    atomicMax(a.best, b);
    __threadfence();
    is_last = atomicAdd(a.ticket, 1u) == unsigned(G - 1);
  }
  __syncthreads();
  if (is_last && tid == 0) {
    __threadfence();
    const unsigned long long b = atomicExch(a.best, 0ull);
    if (pos_ok) {  // an invalid position advances nothing (the error word says why)
      *a.token = int(argmax_index(b));
      *a.pos = pos + 1;
      if (pos - a.pos0 >= 0) a.tokens[pos - a.pos0] = int(argmax_index(b));
    }
    *a.ticket = 0u;
    *a.epoch = epoch + phase_index(a.L, 0) + 1u;
  }
}

// One step on `sms` CTAs, all resident (the kernel's shared memory allows
// one per SM), as a cooperative launch.
cudaError_t launch_step(const Args& a, int sms, cudaStream_t s) {
  static bool init[64] = {};  // per device ordinal
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!init[dev]) {
    e = cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
    if (e != cudaSuccess) return e;
    init[dev] = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(sms));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_kernel, a);
}

// The arguments for model m and state st (sequence 0, f32 cache).
// `tagged` holds 2 * H + 2 * Q + 2 * KV + F words (zeroed once); `ctl` 6
// words: [0] tag base, which must start at 1 (a zeroed word carries tag 0,
// so a first step at tag base 0 would take the zeros for its embedding),
// [2..3] argmax key and [4] ticket, zeroed once.
bool make_args(const tb200_model* m, const tb200_state* st, TW* tagged, uint32_t* ctl, float* logits, Args* out) {
  const tb200_config& c = m->c;
  if (!st->kv_f32 || c.num_hidden_layers > size_t(kMaxLayers) || c.head_dim != size_t(kHd) ||
      c.intermediate_size > size_t(kMaxCols) || m->q_dim > size_t(kMaxCols) || c.hidden_size > size_t(kMaxCols) ||
      c.num_attention_heads / c.num_key_value_heads > size_t(kMaxGrp))
    return false;  // unsupported shape or cache type
  Args a{};
  const size_t per = c.num_key_value_heads * st->max_len * kHd;  // one cache tensor of one layer
  for (size_t l = 0; l < c.num_hidden_layers; l++) {
    const FusedLayer& L = m->layers[l];
    float* base = reinterpret_cast<float*>(st->kv) + l * 2 * per;
    a.layer[l] = Layer{L.wqkv, L.wo, L.wgu, L.wd, L.attn_norm, L.mlp_norm, L.q_norm, L.k_norm, base, base + per};
  }
  a.L = int(c.num_hidden_layers), a.H = int(c.hidden_size), a.Q = int(m->q_dim), a.KV = int(m->kv_dim);
  a.F = int(c.intermediate_size), a.V = int(c.vocab_size);
  a.Hq = int(c.num_attention_heads), a.Hkv = int(c.num_key_value_heads);
  a.eps = c.rms_norm_eps;
  a.embed = m->embed, a.lm_head = m->lm_head, a.norm = m->norm;
  a.rope = st->rope, a.max_len = int(st->max_len);
  a.x = tagged, a.qkv = a.x + a.H, a.att = a.qkv + a.Q + 2 * a.KV, a.h = a.att + a.Q;
  a.token = st->io + 0, a.pos = st->io + 1, a.err = st->io + 3;
  a.epoch = ctl, a.best = reinterpret_cast<unsigned long long*>(ctl + 2), a.ticket = ctl + 4;
  a.logits = logits;
  *out = a;
  return true;
}

}  // namespace tb::persist

int tb200_decode_persistent(tb200_model* m, tb200_state* st, uint32_t token, size_t pos, size_t steps,
                            uint32_t* tokens_out, float* logits_out) {
  namespace P = tb::persist;
  ARG_CHECK(m && st && st->m == m, "bad model/state");
  ARG_CHECK(st->n_seqs == 1, "the single-token path runs one-sequence states");
  ARG_CHECK(tokens_out || steps == 0, "null output");
  ARG_CHECK(pos + steps <= st->max_len, "tokens past the end of the cache");
  ARG_CHECK(token < m->c.vocab_size, "token past the vocabulary");
  ARG_CHECK(pos + steps <= size_t(P::kMaxCtx), "persistent decode runs contexts up to " + std::to_string(P::kMaxCtx) +
                                                   " positions");
  if (int rc = rt::use(m->dev)) return rc;
  P::Args probe;
  ARG_CHECK(P::make_args(m, st, nullptr, nullptr, nullptr, &probe),
            "persistent decode needs an f32 cache, head_dim 128, widths up to 3072, at most 4 query heads per "
            "kv head and at most 64 layers");
  if (!steps) return TB200_OK;
  const tb200_config& c = m->c;
  cudaStream_t s = m->dev->stream;
  const size_t words = 2 * c.hidden_size + 2 * m->q_dim + 2 * m->kv_dim + c.intermediate_size;
  P::TW* tagged = nullptr;
  uint32_t* ctl = nullptr;
  int* toks = nullptr;
  float* logits = nullptr;
  auto release = [&](int rc) {
    cudaStreamSynchronize(s);
    cudaFree(tagged);
    cudaFree(ctl);
    cudaFree(toks);
    cudaFree(logits);
    return rc;
  };
  cudaError_t e = cudaMalloc(&tagged, words * sizeof(P::TW));
  if (e == cudaSuccess) e = cudaMalloc(&ctl, 6 * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&toks, steps * sizeof(int));
  if (e == cudaSuccess && logits_out) e = cudaMalloc(&logits, c.vocab_size * sizeof(float));
  if (e == cudaSuccess) e = cudaMemsetAsync(tagged, 0, words * sizeof(P::TW), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(ctl, 0, 6 * sizeof(uint32_t), s);
  int* stage = st->io_host + 2 * st->max_len;  // pinned
  stage[0] = int(token);
  stage[1] = int(pos);
  stage[2] = 0;
  stage[3] = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(st->io, stage, 4 * sizeof(int), cudaMemcpyHostToDevice, s);
  static const uint32_t one = 1u;  // the first tag base (a zeroed word carries tag 0)
  if (e == cudaSuccess) e = cudaMemcpyAsync(ctl, &one, sizeof(one), cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return release(rt::fail(TB200_ERR_CUDA, std::string("persistent decode: ") + cudaGetErrorString(e)));
  P::Args a;
  P::make_args(m, st, tagged, ctl, logits, &a);
  a.tokens = toks;
  a.pos0 = int(pos);
  // Every CTA owns rows of every matrix phase (no CTA can run a phase ahead
  // of a vector it has yet to read; see the kernel's exchange rule).
  const int grid = int(std::min<size_t>({size_t(m->dev->sms), c.hidden_size, c.intermediate_size,
                                         m->q_dim + 2 * m->kv_dim, c.vocab_size}));
  for (size_t i = 0; i < steps && e == cudaSuccess; i++) {
    e = P::launch_step(a, grid, s);
    if (e == cudaSuccess && logits_out)
      e = cudaMemcpyAsync(logits_out + i * c.vocab_size, logits, c.vocab_size * sizeof(float), cudaMemcpyDeviceToHost,
                          s);
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(tokens_out, toks, steps * sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(stage, st->io, 4 * sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return release(rt::fail(TB200_ERR_CUDA, std::string("persistent decode: ") + cudaGetErrorString(e)));
  if (stage[3] == TB200_ERR_TIMEOUT) return release(rt::fail(TB200_ERR_TIMEOUT, "a kernel's bounded wait timed out"));
  if (stage[3] != 0) return release(rt::fail(TB200_ERR_ARG, "persistent decode: the kernel rejected its input"));
  st->host_pos = pos + steps;
  return release(TB200_OK);
}
