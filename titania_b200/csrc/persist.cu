// persist.cu — batch-1 greedy decode as one persistent kernel per launch:
// Model::forward for one token (model/model.rs:93-149) followed by the greedy
// choice (model/sampler.rs:31-33), repeated for `steps` tokens inside the
// launch.
//
// One CTA per SM (a cooperative launch, so CTAs may wait on one another).
// A step has four phases per layer and the lm_head:
//   QKV    qkv   = W_qkv · rmsnorm(x)                      rows split over CTAs
//   ATT_O  CTA (kv group g, member s): QK-norm, RoPE and K/V append of group
//          g, its attention, then rows of part_o[g] = W_o[:, cols of g] · att_g;
//          then each CTA sums x' = x + Σ_g part_o[g] (g in order) on its own
//          residual rows
//   GU     h = silu(W_g · rmsnorm(x')) * (W_u · rmsnorm(x'))
//   DOWN   x  = x' + W_d · h                               rows owned by CTAs
//   LM     logits = W_lm · rmsnorm(x); greedy token over the grid
// Phases exchange vectors as 64-bit (tag << 32 | value bits) words in global
// memory: a reader polls the words it needs until each carries the tag of
// the current (step, layer, phase), so data and synchronisation cost one L2
// round trip together and no grid barrier exists. The vectors every CTA
// reads (x, h) are written in kRep copies, CTA c reading copy c % kRep, which
// spreads the polling over more L2 lines. Attention over a context of up to
// kRedundantCtx positions is computed by every member of the kv group (no
// exchange); past it, member s attends to its share of the positions and
// the members exchange and merge their partial results.
//
// One producer warp streams this CTA's weight rows of every phase of every
// step through a shared-memory ring with cp.async.bulk, never draining at a
// phase boundary: while the consumers wait for a vector, the next phases'
// weights keep arriving. What each CTA computes (its rows of every phase,
// their ring stages) is planned once per launch.
//
// Every wait is bounded, and no control flow depends on a wait's outcome:
// the first wait that gives up sets the CTA's abort flag and the error word,
// every later wait returns at once, and all threads still reach every
// barrier, so the kernel ends promptly and drains its copies in flight.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <string>

#include "runtime.h"

namespace tb::persist {

constexpr int kWarps = 8;                 // consumer warps
constexpr int kConsumers = kWarps * 32;
constexpr int kThreads = kConsumers + 64;  // + the producer warp and the prefetch warp
constexpr int kSlotBytes = 64 * 1024;
constexpr int kSlots = 3;
constexpr int kMaxLayers = 64;
constexpr int kHd = 128;
constexpr int kMaxCols = 3072;       // widest input vector
constexpr int kMaxRowsPerWarp = 8;   // rows a warp takes in one ring stage
constexpr int kMaxGrp = 4;           // query heads per kv head
constexpr int kMaxKv = 8;            // kv heads (o_proj partial vectors summed per residual row)
constexpr int kMaxOwn = 32;          // residual rows a CTA owns
constexpr int kAttnPer = 8;          // cached positions per warp held in registers at a time
constexpr int kRedundantCtx = 256;   // contexts up to this: every group member attends over all of it
constexpr int kPartWords = 132;      // a member's partial per head: acc[128], max, sum, 2 pad
constexpr int kRep = 4;              // copies of the vectors every CTA reads (x, h): CTA c reads copy c % kRep
constexpr int kLmAheadLayers = 8;    // the lm_head's first kLmAheadNum / kLmAheadDen of rows are asked of L2
constexpr int kLmAheadNum = 1, kLmAheadDen = 6;  //   during the last kLmAheadLayers layers (a third measured no better)
constexpr size_t kSmemBytes = size_t(kMaxCols) * 2 * 4 + size_t(kSlots) * kSlotBytes + 2 * kSlots * 8;

using TW = unsigned long long;  // a tagged word

struct Layer {
  const uint16_t *wqkv, *wo_g, *wgu, *wd;  // [Q+2KV][H], [Hkv][H][grp*128], [2F][H] (gate/up interleaved), [H][F]
  const uint16_t *attn_norm, *mlp_norm, *q_norm, *k_norm;
  void *kc, *vc;  // [Hkv][max_len][128], f32 or bf16
};

struct Args {
  Layer layer[kMaxLayers];
  int L, H, Q, KV, F, V, Hq, Hkv, grp;
  float eps;
  const uint16_t *embed, *lm_head, *norm;
  const float* rope;  // [max_len][128] (cos, sin) pairs
  int max_len, kv_f32;
  // x [kRep][H], qkv [Q+2KV], h [kRep][F], part_o [Hkv][H], part_att [Hkv][nsplit][grp][kPartWords], tokw [4]
  TW *x, *qkv, *h, *part_o, *part_att, *tokw;
  int nsplit;         // most members of a kv group (ceil(CTAs / Hkv))
  int* io;            // [0] token, [1] position, [2] generated-token counter, [3] error word
  int* tokens_out;    // [tokens_cap]: generated tokens by counter
  int tokens_cap;
  unsigned long long* best;  // argmax key, zero between steps
  unsigned* ticket;          // zero between steps
  float* logits;             // [V] of the last step, or null
  uint32_t epoch;            // tag base of the first step (tags never repeat: the host advances it)
  int steps;
  Trace trace;
};

// Matrix phases; K_LM is the lm_head, after the last layer.
enum { K_QKV = 0, K_ATTO = 1, K_GU = 2, K_DOWN = 3, K_LM = 4, kKinds = 5, kPhases = 4 };

// Tags of one step, relative to its base: 0 the embedded token's x, then
// 1 + 4 layer + phase, then the chosen token.
__host__ __device__ constexpr uint32_t tags_per_step(int L) { return 2u + 4u * uint32_t(L); }
__device__ __forceinline__ uint32_t phase_tag(uint32_t base, int layer, int p) {
  return base + 1u + 4u * uint32_t(layer) + uint32_t(p);
}
// Trace slot group of a phase: 0 the step's start, 1 + 4 layer + phase, then
// the lm_head and the token.
__device__ __forceinline__ uint32_t trace_base(int layer, int p, int G) {
  return (1u + 4u * uint32_t(layer) + uint32_t(p)) * uint32_t(G) * kTraceEvents;
}

// One CTA's share of a matrix phase: output rows [r0, r0 + n) of `cols`
// columns, the first at row `w0` of the phase's matrix, in `nst` ring stages
// of `sr` rows (the last may hold fewer).
struct Plan {
  int r0, n, cols, sr, nst;
  long long w0;
};

// The kv group and member of CTA c in ATT_O, and the group's member count.
__device__ __forceinline__ void group_of(const Args& a, int c, int G, int& g, int& s, int& ng) {
  g = c % a.Hkv;
  s = c / a.Hkv;
  ng = (G - g + a.Hkv - 1) / a.Hkv;
}

// CTA c's share [r0, r1) of `rows` rows split over G CTAs in units of
// `align` rows, or of `base` rows where that would leave a CTA without any
// (every CTA must own rows of every phase: a CTA that wrote nothing could
// fall a phase behind and find the vector it polls already overwritten).
// Units of four f32 outputs fill 32-byte sectors, so no two CTAs write the
// same sector of a vector: readers then wait for one writer per sector, and
// an all-gather among 148 CTAs measured 1.0 us instead of 1.5 us.
__device__ __forceinline__ void share(int rows, int align, int base, int c, int G, int& r0, int& r1) {
  const int al = rows / align >= G ? align : base;
  const int units = rows / al;
  r0 = int((long long)c * units / G) * al;
  r1 = int((long long)(c + 1) * units / G) * al;
}

// Residual rows CTA c owns (its embedding, x' and down_proj rows).
__device__ __forceinline__ void own_rows(const Args& a, int c, int G, int& r0, int& r1) {
  share(a.H, 4, 1, c, G, r0, r1);
}

__device__ Plan plan_of(const Args& a, int kind, int c, int G) {
  Plan p{};
  int r1;
  if (kind == K_ATTO) {
    int g, s, ng;
    group_of(a, c, G, g, s, ng);
    p.cols = a.grp * kHd;
    share(a.H, 4, 1, s, ng, p.r0, r1);
    p.w0 = (long long)g * a.H + p.r0;
  } else {
    if (kind == K_QKV) share(a.Q + 2 * a.KV, 4, 1, c, G, p.r0, r1), p.cols = a.H;
    else if (kind == K_GU) share(2 * a.F, 8, 2, c, G, p.r0, r1), p.cols = a.H;  // gate/up pairs: 4 h values
    else if (kind == K_DOWN) own_rows(a, c, G, p.r0, r1), p.cols = a.F;
    else share(a.V, 1, 1, c, G, p.r0, r1), p.cols = a.H;
    p.w0 = p.r0;
  }
  p.n = r1 - p.r0;
  // Stages of equal size (even, so that a gate/up pair never straddles two),
  // each at most one slot and kWarps * kMaxRowsPerWarp rows.
  const int maxrows = min((kSlotBytes / (p.cols * 2)) & ~1, kWarps * kMaxRowsPerWarp);
  p.nst = (p.n + maxrows - 1) / maxrows;
  p.sr = p.nst ? (((p.n + p.nst - 1) / p.nst) + 1) & ~1 : 0;
  if (p.sr > maxrows) p.sr = maxrows;
  return p;
}

// The phase's matrix in layer `Ly` (or the lm_head).
__device__ __forceinline__ const uint16_t* matrix_of(const Args& a, const Layer& Ly, int kind) {
  return kind == K_QKV ? Ly.wqkv : kind == K_ATTO ? Ly.wo_g : kind == K_GU ? Ly.wgu : kind == K_DOWN ? Ly.wd
                                                                                                      : a.lm_head;
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
// Four tagged words (32 bytes); each 64-bit element is read atomically.
__device__ __forceinline__ void ld_tagged4(const TW* p, TW (&w)[4]) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(w[0]), "=l"(w[1]) : "l"(p) : "memory");
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(w[2]), "=l"(w[3]) : "l"(p + 2) : "memory");
}
__device__ __forceinline__ void ld_tagged2(const TW* p, TW (&w)[2]) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(w[0]), "=l"(w[1]) : "l"(p) : "memory");
}
__device__ __forceinline__ float tval(TW w) { return __uint_as_float(uint32_t(w)); }
__device__ __forceinline__ uint32_t ttag(TW w) { return uint32_t(w >> 32); }
__device__ __forceinline__ bool tags4(const TW (&w)[4], uint32_t tag) {
  return ttag(w[0]) == tag && ttag(w[1]) == tag && ttag(w[2]) == tag && ttag(w[3]) == tag;
}

// Shared-memory position of input element i (i a multiple of 4): columns
// 256k + 8l .. 8l+3 at 256k + 4l and 8l+4 .. 8l+7 at 256k + 128 + 4l, so
// that lane l reads its eight columns of a 256-column block as two float4.
__device__ __forceinline__ int xperm(int i) { return (i & ~255) + ((i >> 2) & 1) * 128 + ((i >> 3) & 31) * 4; }

// Records a timeout: the error word, and this CTA's abort flag.
__device__ __forceinline__ bool timed_out(long long t0, int* err, volatile int* abort) {
  if (clock64() - t0 <= kWaitCycles) return false;
  set_error(err, TB200_ERR_TIMEOUT);
  *abort = 1;
  return true;
}

// mbar_wait under the abort rule.
__device__ __forceinline__ void wait_full(uint64_t* bar, uint32_t parity, int* err, volatile int* abort) {
  if (*abort) return;
  if (!mbar_wait(bar, parity, err)) *abort = 1;
}

// ---- cross-lane reductions ------------------------------------------------------

// Sums each of the PR values of every lane over the warp, PR - 1 + 5 -
// log2(PR) shuffles in all (a reduce-scatter, then a butterfly over the lanes
// that hold the same value): lane l ends with the sum of value
// row_of_lane<PR>(l). v is clobbered.
template <int PR>
__device__ __forceinline__ float reduce_rows(float (&v)[PR], int lane) {
#pragma unroll
  for (int h = PR / 2, o = 16; h >= 1; h /= 2, o /= 2) {
    const bool upper = lane & o;
#pragma unroll
    for (int i = 0; i < h; i++) {
      const float send = upper ? v[i] : v[i + h];
      const float keep = upper ? v[i + h] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  float r = v[0];
#pragma unroll
  for (int o = 16 / PR; o >= 1; o /= 2) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}
// Which of the PR values lane l holds after reduce_rows (lanes l and
// l ^ m, m < 32 / PR, hold the same one).
template <int PR>
__device__ __forceinline__ int row_of_lane(int lane) {
  int r = 0;
#pragma unroll
  for (int h = PR / 2, o = 16; h >= 1; h /= 2, o /= 2)
    if (lane & o) r += h;
  return r;
}
// The lowest lane that holds value r after reduce_rows.
template <int PR>
__device__ __forceinline__ int lane_of_row(int r) {
  int l = 0;
#pragma unroll
  for (int h = PR / 2, o = 16; h >= 1; h /= 2, o /= 2)
    if (r & h) l += o;
  return l;
}

// ---- the matrix-vector product of one warp's rows -------------------------------

struct WarpRows {
  float v;     // this lane's row's dot product (unscaled)
  int row;     // which of the warp's rows (>= nr: none)
  int stride;  // lanes between consecutive rows' holders
};

// Rows w[0 .. NR) (rb bytes apart, shared memory) dotted with the input in
// xs (xperm layout, cols columns): lane l takes columns 8l .. 8l+7 of every
// 256-column block.
template <int NR>
__device__ __forceinline__ WarpRows dot_rows(const unsigned char* w, int rb, int cols, const float* xs, int lane) {
  constexpr int PR = NR == 1 ? 1 : NR == 2 ? 2 : NR <= 4 ? 4 : 8;
  float acc[PR], acc2[NR];
#pragma unroll
  for (int j = 0; j < PR; j++) acc[j] = 0.f;
#pragma unroll
  for (int j = 0; j < NR; j++) acc2[j] = 0.f;
  const unsigned char* wl = w + lane * 16;
  const float* xl = xs + lane * 4;
  auto block = [&](int col) {
    const float4 xa = *reinterpret_cast<const float4*>(xl + col);
    const float4 xb = *reinterpret_cast<const float4*>(xl + col + 128);
#pragma unroll
    for (int j = 0; j < NR; j++) {
      const uint4 wv = *reinterpret_cast<const uint4*>(wl + j * rb + col * 2);
      acc[j] = dot4(wv.x, wv.y, xa, acc[j]);
      acc2[j] = dot4(wv.z, wv.w, xb, acc2[j]);
    }
  };
  const int whole = cols & ~255;
#pragma unroll 2
  for (int col = 0; col < whole; col += 256) block(col);
  if (whole + lane * 8 < cols) block(whole);  // a last block of fewer than 256 columns
#pragma unroll
  for (int j = 0; j < NR; j++) acc[j] += acc2[j];
  WarpRows r;
  r.v = reduce_rows<PR>(acc, lane);
  r.row = (lane & (32 / PR - 1)) == 0 ? row_of_lane<PR>(lane) : 1 << 20;
  r.stride = 32 / PR;
  return r;
}

// Polls vec[0, n) (n a multiple of 4, at most 4 kConsumers) until every word
// carries `tag`. With a norm weight, the values times the weight go to xs
// (xperm positions) and the thread's sum of squares of the values is
// returned (the RMSNorm's, cpu.rs:85-94); without one, the values
// themselves. All of a thread's loads are issued before any is checked.
// Bounded.
__device__ float poll_vector(const TW* vec, int n, uint32_t tag, const uint16_t* norm, float* xs, int tid, int* err,
                             volatile int* abort) {
  constexpr int kG = 3;  // groups of 4 words per thread (n <= 3072)
  bool done[kG];
#pragma unroll
  for (int k = 0; k < kG; k++) done[k] = tid * 4 + k * kConsumers * 4 >= n;
  float ss = 0.f;
  const long long t0 = clock64();
  for (;;) {
    bool all = true;
#pragma unroll
    for (int k = 0; k < kG; k++) {
      if (done[k]) continue;
      const int i = tid * 4 + k * kConsumers * 4;
      TW w[4];
      ld_tagged4(vec + i, w);
      if (tags4(w, tag) || *abort) {
        float4 v = make_float4(tval(w[0]), tval(w[1]), tval(w[2]), tval(w[3]));
        if (norm) {
          // In arrival order: the same bits whatever the order for up to two
          // groups, and every normed input here (the hidden vector) has at most
          // 2048 (wider models run persist_wide.cu, which adds in group order).
          ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
          const uint2 g = *reinterpret_cast<const uint2*>(norm + i);
          v.x *= bf_lo(g.x), v.y *= bf_hi(g.x), v.z *= bf_lo(g.y), v.w *= bf_hi(g.y);
        }
        *reinterpret_cast<float4*>(xs + xperm(i)) = v;
        done[k] = true;
      } else {
        all = false;
      }
    }
    if (all || timed_out(t0, err, abort)) break;
  }
  return ss;
}

// ---- attention ----------------------------------------------------------------

__device__ __forceinline__ float4 ld_kv(const void* base, size_t at, bool f32) {
  if (f32) return __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(base) + at));
  const uint2 u = __ldcg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + at));
  return make_float4(bf_lo(u.x), bf_hi(u.x), bf_lo(u.y), bf_hi(u.y));
}
__device__ __forceinline__ void st_kv(void* base, size_t at, float4 v, bool f32) {
  if (f32) {
    *reinterpret_cast<float4*>(static_cast<float*>(base) + at) = v;
  } else {
    const uint32_t lo = uint32_t(f2bf(v.x)) | (uint32_t(f2bf(v.y)) << 16);
    const uint32_t hi = uint32_t(f2bf(v.z)) | (uint32_t(f2bf(v.w)) << 16);
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(base) + at) = make_uint2(lo, hi);
  }
}
// What the cache holds for v: v itself (f32) or its bf16 rounding.
__device__ __forceinline__ float4 as_cached(float4 v, bool f32) {
  if (f32) return v;
  return make_float4(bf16f(f2bf(v.x)), bf16f(f2bf(v.y)), bf16f(f2bf(v.z)), bf16f(f2bf(v.w)));
}

// Attention of kv group g at position `pos` (model.rs:107-124 for one
// token; cpu.rs:113-149), run by the consumer warps of member s of the
// group's ng members. Warp w < GRP + 2 polls head w of q (w < GRP), k, v
// from the q|k|v vector, applies QK-norm (model.rs:111-116) and RoPE
// (cpu.rs:96-111) in registers; member 0 appends k and v to the cache. The
// context [lo, hi) this member attends to is all of 0..pos when pos < the
// redundant limit, else its share; warps take positions lo + w, lo + w + 8,
// ... eight at a time: the GRP x 8 dot products of a chunk are reduced
// together (reduce_rows), each lane then owns one (head, position) score for
// the online softmax, and the probabilities are broadcast for the weighted
// sum of values, each lane holding 4 of the 128 dimensions. The warps are
// merged at the end. In split mode the members then exchange partials (tag
// `ptag`) and every member merges all of them in one fixed order. The result,
// GRP heads of 128, goes to xs at xperm positions (the o_proj partial's
// input). `sc` is shared scratch of at least 4960 floats.
template <int GRP>
__device__ void attention_phase(const Args& a, const Layer& Ly, int g, int s, int ng, int pos, uint32_t qtag,
                                uint32_t ptag, float* xs, float* sc, int tid, volatile int* abort, const TraceAt& tr,
                                int cta) {
  constexpr int grp = GRP;
  constexpr int PR = GRP * kAttnPer;  // (head, slot) scores of a chunk
  const int warp = tid >> 5, lane = tid & 31;
  const bool f32 = a.kv_f32 != 0;
  float* qs = sc;                        // [grp][128]
  float* kn = qs + kMaxGrp * kHd;        // [128]
  float* vn = kn + kHd;                  // [128]
  float* wm = vn + kHd;                  // [kWarps][kMaxGrp]
  float* wl = wm + kWarps * kMaxGrp;     // [kWarps][kMaxGrp]
  float* wacc = wl + kWarps * kMaxGrp;   // [kWarps][kMaxGrp][128]
  float* we = wacc + kWarps * kMaxGrp * kHd;  // [kMaxGrp][kWarps] merge weights

  const int ctx = pos + 1;
  const bool split = ctx > kRedundantCtx;
  const int lo = split ? int((long long)s * ctx / ng) : 0;
  const int hi = split ? int((long long)(s + 1) * ctx / ng) : ctx;
  const size_t head0 = size_t(g) * a.max_len * kHd;

  // Cached positions (< pos) do not depend on this step: the first chunk is
  // requested before the wait.
  float4 kr[kAttnPer], vr[kAttnPer];
#pragma unroll
  for (int i = 0; i < kAttnPer; i++) kr[i] = vr[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  auto load_chunk = [&](int base) {
#pragma unroll
    for (int i = 0; i < kAttnPer; i++) {
      const int j = base + warp + kWarps * i;
      if (j < hi && j < pos) {
        const size_t at = head0 + size_t(j) * kHd + 4 * lane;
        kr[i] = ld_kv(Ly.kc, at, f32);
        vr[i] = ld_kv(Ly.vc, at, f32);
      }
    }
  };
  load_chunk(lo);

  // Warp w < grp + 2: head w of q, then k, then v, polled and prepared in registers.
  if (warp < grp + 2) {
    const int at = warp < grp ? (g * grp + warp) * kHd : warp == grp ? a.Q + g * kHd : a.Q + a.KV + g * kHd;
    TW w[4];
    const long long t0 = clock64();
    for (;;) {
      ld_tagged4(a.qkv + at + 4 * lane, w);
      if (tags4(w, qtag) || *abort || timed_out(t0, a.io + 3, abort)) break;
    }
    float4 v = make_float4(tval(w[0]), tval(w[1]), tval(w[2]), tval(w[3]));
    if (warp <= grp) {
      const uint16_t* nw = warp < grp ? Ly.q_norm : Ly.k_norm;
      if (nw) {  // rmsnorm over the head (cpu.rs:85-94 with dim 128)
        const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
        const float scale = 1.0f / sqrtf(ss / float(kHd) + a.eps);
        const uint2 gw = *reinterpret_cast<const uint2*>(nw + 4 * lane);
        v.x = __fmul_rn(v.x, __fmul_rn(scale, bf_lo(gw.x)));
        v.y = __fmul_rn(v.y, __fmul_rn(scale, bf_hi(gw.x)));
        v.z = __fmul_rn(v.z, __fmul_rn(scale, bf_lo(gw.y)));
        v.w = __fmul_rn(v.w, __fmul_rn(scale, bf_hi(gw.y)));
      }
      // RoPE: element i pairs with i + 64, held by lane ^ 16.
      const float4 o = make_float4(__shfl_xor_sync(0xffffffffu, v.x, 16), __shfl_xor_sync(0xffffffffu, v.y, 16),
                                   __shfl_xor_sync(0xffffffffu, v.z, 16), __shfl_xor_sync(0xffffffffu, v.w, 16));
      const int i0 = (4 * lane) & 63;
      const float4 cs0 = *reinterpret_cast<const float4*>(a.rope + size_t(pos) * kHd + 2 * i0);
      const float4 cs1 = *reinterpret_cast<const float4*>(a.rope + size_t(pos) * kHd + 2 * i0 + 4);
      const float c[4] = {cs0.x, cs0.z, cs1.x, cs1.z}, sn[4] = {cs0.y, cs0.w, cs1.y, cs1.w};
      float e[4] = {v.x, v.y, v.z, v.w};
      const float f[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
      for (int q = 0; q < 4; q++)
        e[q] = lane < 16 ? __fsub_rn(__fmul_rn(e[q], c[q]), __fmul_rn(f[q], sn[q]))
                         : __fadd_rn(__fmul_rn(e[q], c[q]), __fmul_rn(f[q], sn[q]));
      v = make_float4(e[0], e[1], e[2], e[3]);
    }
    if (warp >= grp) {
      if (s == 0) {  // member 0 appends this position's key and value
        st_kv(warp == grp ? Ly.kc : Ly.vc, head0 + size_t(pos) * kHd + 4 * lane, v, f32);
        __threadfence();  // a later step of this launch reads it from another CTA
      }
      v = as_cached(v, f32);
    }
    *reinterpret_cast<float4*>((warp < grp ? qs + warp * kHd : warp == grp ? kn : vn) + 4 * lane) = v;
  }
  named_sync(1, kConsumers);
  if (tid == 0) tr.at(cta, TB200_TRACE_WAITED);

  // Online softmax per warp over its positions of [lo, hi), eight at a time.
  const float scale = 1.0f / sqrtf(float(kHd));
  const int myr = row_of_lane<PR>(lane);  // this lane's (head, slot) after the reduction
  const int myh = myr / kAttnPer, myi = myr % kAttnPer;
  float m[GRP], l[GRP];
  float4 acc[GRP], q[GRP];
#pragma unroll
  for (int h = 0; h < GRP; h++) {
    m[h] = -INFINITY;
    l[h] = 0.f;
    acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    q[h] = *reinterpret_cast<const float4*>(qs + h * kHd + 4 * lane);
  }
  const float4 kcur = *reinterpret_cast<const float4*>(kn + 4 * lane);
  const float4 vcur = *reinterpret_cast<const float4*>(vn + 4 * lane);
  for (int base = lo; base < hi; base += kWarps * kAttnPer) {
    if (base > lo) load_chunk(base);
    const int nvalid = min(kAttnPer, (hi - base - warp + kWarps - 1) / kWarps);  // slots of this warp in [lo, hi)
    float sco[PR];
#pragma unroll
    for (int i = 0; i < kAttnPer; i++) {
      if (base + warp + kWarps * i == pos) kr[i] = kcur, vr[i] = vcur;
#pragma unroll
      for (int h = 0; h < GRP; h++)
        sco[h * kAttnPer + i] = q[h].x * kr[i].x + q[h].y * kr[i].y + q[h].z * kr[i].z + q[h].w * kr[i].w;
    }
    float sv = reduce_rows<PR>(sco, lane);
    sv = myi < nvalid ? sv * scale : -INFINITY;
    // The chunk's maximum and probability sum per head: over the lanes
    // holding that head's slots.
    float cm = sv;
#pragma unroll
    for (int b = 0; b < 3; b++) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, (32 / PR) << b));
    float Mn[GRP], corr[GRP];
#pragma unroll
    for (int h = 0; h < GRP; h++) {
      Mn[h] = fmaxf(m[h], __shfl_sync(0xffffffffu, cm, lane_of_row<PR>(h * kAttnPer)));
      corr[h] = Mn[h] == -INFINITY ? 1.f : expf(m[h] - Mn[h]);
    }
    float mine = Mn[0];
#pragma unroll
    for (int h = 1; h < GRP; h++)
      if (myh == h) mine = Mn[h];
    const float p = sv == -INFINITY ? 0.f : expf(sv - mine);
    float ps = p;
#pragma unroll
    for (int b = 0; b < 3; b++) ps += __shfl_xor_sync(0xffffffffu, ps, (32 / PR) << b);
#pragma unroll
    for (int h = 0; h < GRP; h++) {
      l[h] = l[h] * corr[h] + __shfl_sync(0xffffffffu, ps, lane_of_row<PR>(h * kAttnPer));
      m[h] = Mn[h];
      float4 ac = make_float4(acc[h].x * corr[h], acc[h].y * corr[h], acc[h].z * corr[h], acc[h].w * corr[h]);
#pragma unroll
      for (int i = 0; i < kAttnPer; i++) {
        const float pi = __shfl_sync(0xffffffffu, p, lane_of_row<PR>(h * kAttnPer + i));
        ac.x += pi * vr[i].x;
        ac.y += pi * vr[i].y;
        ac.z += pi * vr[i].z;
        ac.w += pi * vr[i].w;
      }
      acc[h] = ac;
    }
  }
#pragma unroll
  for (int h = 0; h < GRP; h++) {
    if (lane == 0) {
      wm[warp * kMaxGrp + h] = m[h];
      wl[warp * kMaxGrp + h] = l[h];
    }
    *reinterpret_cast<float4*>(wacc + (warp * kMaxGrp + h) * kHd + 4 * lane) = acc[h];
  }
  named_sync(1, kConsumers);
  // Merge weights of the warps, one thread per (head, warp).
  if (tid < grp * kWarps) {
    const int h = tid / kWarps, w = tid % kWarps;
    float M = -INFINITY;
#pragma unroll
    for (int u = 0; u < kWarps; u++) M = fmaxf(M, wm[u * kMaxGrp + h]);
    const float lw = wl[w * kMaxGrp + h];
    we[h * kWarps + w] = lw > 0.f ? expf(wm[w * kMaxGrp + h] - M) : 0.f;
  }
  named_sync(1, kConsumers);
  // Merge: thread (h, 4 dims) of the grp * 32 threads.
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  float M = -INFINITY, Ls = 0.f;
  const int mh = tid >> 5, d4 = tid & 31;
  if (tid < grp * 32) {
#pragma unroll
    for (int w = 0; w < kWarps; w++) {
      const float e = we[mh * kWarps + w];
      const float4 aw = *reinterpret_cast<const float4*>(wacc + (w * kMaxGrp + mh) * kHd + 4 * d4);
      Ls += wl[w * kMaxGrp + mh] * e;
      o.x += aw.x * e;
      o.y += aw.y * e;
      o.z += aw.z * e;
      o.w += aw.w * e;
      M = fmaxf(M, wm[w * kMaxGrp + mh]);
    }
  }
  if (split) {
    // Publish this member's partial; then every member merges all of them.
    TW* mine = a.part_att + (size_t(g * a.nsplit + s) * grp) * kPartWords;
    if (tid < grp * 32) {
      TW* p = mine + mh * kPartWords;
      st_tagged(p + 4 * d4 + 0, o.x, ptag);
      st_tagged(p + 4 * d4 + 1, o.y, ptag);
      st_tagged(p + 4 * d4 + 2, o.z, ptag);
      st_tagged(p + 4 * d4 + 3, o.w, ptag);
      if (d4 == 0) {
        st_tagged(p + 128, M, ptag);
        st_tagged(p + 129, Ls, ptag);
        st_tagged(p + 130, 0.f, ptag);
        st_tagged(p + 131, 0.f, ptag);
      }
    }
    // Every member merges all members' partials: the consumer threads form
    // kWarps / grp quarters of (head, 4 dims) threads; quarter q merges
    // members q, q + nq, ... (two requested at once, merged in that order),
    // then the quarters' results are merged in quarter order. The order is
    // fixed, so every member gets the same bits whatever the timing.
    const int nq = kWarps / grp, q = tid / (grp * 32), qh = (tid >> 5) % grp, qd = tid & 31;
    float4 qo = make_float4(0.f, 0.f, 0.f, 0.f);
    float qm = -INFINITY, ql = 0.f;
    auto merge = [](float4& o, float& M, float& L, const TW (&w)[4], const TW (&ml)[2]) {
      const float ms = tval(ml[0]), ls = tval(ml[1]);
      if (ls > 0.f) {
        const float Mn = fmaxf(M, ms);
        const float cold = expf(M - Mn), cnew = expf(ms - Mn);
        o.x = o.x * cold + tval(w[0]) * cnew;
        o.y = o.y * cold + tval(w[1]) * cnew;
        o.z = o.z * cold + tval(w[2]) * cnew;
        o.w = o.w * cold + tval(w[3]) * cnew;
        L = L * cold + ls * cnew;
        M = Mn;
      }
    };
    const long long t0 = clock64();
    for (int sp = q; sp < ng; sp += 2 * nq) {
      const bool two = sp + nq < ng;
      const TW* p0 = a.part_att + (size_t(g * a.nsplit + sp) * grp + qh) * kPartWords;
      const TW* p1 = a.part_att + (size_t(g * a.nsplit + (two ? sp + nq : sp)) * grp + qh) * kPartWords;
      TW w0[4], w1[4], m0[2], m1[2];
      for (;;) {
        ld_tagged4(p0 + 4 * qd, w0);
        ld_tagged2(p0 + 128, m0);
        ld_tagged4(p1 + 4 * qd, w1);
        ld_tagged2(p1 + 128, m1);
        const bool ok = tags4(w0, ptag) && ttag(m0[0]) == ptag && ttag(m0[1]) == ptag && tags4(w1, ptag) &&
                        ttag(m1[0]) == ptag && ttag(m1[1]) == ptag;
        if (ok || *abort || timed_out(t0, a.io + 3, abort)) break;
      }
      merge(qo, qm, ql, w0, m0);
      if (two) merge(qo, qm, ql, w1, m1);
    }
    named_sync(1, kConsumers);  // the warp merge above is done with wacc, wm, wl
    *reinterpret_cast<float4*>(wacc + (q * grp + qh) * kHd + 4 * qd) = qo;
    if (qd == 0) {
      wm[q * kMaxGrp + qh] = qm;
      wl[q * kMaxGrp + qh] = ql;
    }
    named_sync(1, kConsumers);
    o = make_float4(0.f, 0.f, 0.f, 0.f);
    M = -INFINITY;
    Ls = 0.f;
    if (tid < grp * 32) {
      for (int u = 0; u < nq; u++) {
        const float4 v = *reinterpret_cast<const float4*>(wacc + (u * grp + mh) * kHd + 4 * d4);
        const TW w[4] = {TW(__float_as_uint(v.x)), TW(__float_as_uint(v.y)), TW(__float_as_uint(v.z)),
                         TW(__float_as_uint(v.w))};
        const TW ml[2] = {TW(__float_as_uint(wm[u * kMaxGrp + mh])), TW(__float_as_uint(wl[u * kMaxGrp + mh]))};
        merge(o, M, Ls, w, ml);
      }
    }
  }
  if (tid < grp * 32) {
    const float inv = 1.0f / Ls;
    *reinterpret_cast<float4*>(xs + xperm(mh * kHd + 4 * d4)) = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
  }
}

// ---- the kernel -----------------------------------------------------------------

// L2 prefetch of [p, p + bytes) (bytes a multiple of 16) in pieces.
__device__ __forceinline__ void prefetch_range(const void* p, size_t bytes) {
  constexpr size_t kPiece = 32 * 1024;
  const char* b = static_cast<const char*>(p);
  for (size_t o = 0; o < bytes; o += kPiece) bulk_prefetch_l2(b + o, uint32_t(min(kPiece, bytes - o)));
}

// Asks L2 for CTA c's rows of phase `kind` of `layer` in step `step` (the
// lm_head: its first ring's worth) and, for ATT_O, the CTA's cached keys and
// values (positions < pos), so that HBM keeps streaming while the ring is
// full and the consumers wait for a vector.
__device__ void prefetch_phase(const Args& a, const Plan& pl, int c, int G, int pos0, int step, int layer, int kind) {
  if (step >= a.steps) return;
  const Layer& Ly = a.layer[layer < a.L ? layer : 0];
  size_t bytes = size_t(pl.n) * size_t(pl.cols) * 2;
  if (kind == K_LM) bytes = min(bytes, size_t(kSlots) * kSlotBytes);
  prefetch_range(matrix_of(a, Ly, kind) + pl.w0 * pl.cols, bytes);
  if (kind == K_ATTO) {
    int g, s, ng;
    group_of(a, c, G, g, s, ng);
    const int pos = pos0 + step, ctx = pos + 1;
    const bool split = ctx > kRedundantCtx;
    const int lo = split ? int((long long)s * ctx / ng) : 0;
    const int hi = min(pos, split ? int((long long)(s + 1) * ctx / ng) : ctx);
    if (hi > lo) {
      const size_t esz = a.kv_f32 ? 4 : 2;
      const size_t at = (size_t(g) * a.max_len + lo) * kHd * esz, nb = size_t(hi - lo) * kHd * esz;
      prefetch_range(static_cast<const char*>(Ly.kc) + at, nb);
      prefetch_range(static_cast<const char*>(Ly.vc) + at, nb);
    }
  }
}

template <int GRP>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(Args a) {
  extern __shared__ __align__(128) unsigned char smem[];
  float* xs = reinterpret_cast<float*>(smem);  // [kMaxCols] input, xperm layout; attention scratch after 1024
  unsigned char* ring = smem + size_t(kMaxCols) * 2 * 4;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + size_t(kSlots) * kSlotBytes);
  uint64_t* empty = full + kSlots;
  __shared__ float red[kWarps];
  __shared__ float own[kMaxOwn];  // the residual stream x on this CTA's rows, as this CTA last wrote it
  __shared__ unsigned long long best_sm[kWarps];
  __shared__ Plan plan[kKinds];
  __shared__ volatile int abort_sm;  // a wait gave up (or the arguments are bad): wait no more
  __shared__ volatile int issued_sm;
  __shared__ volatile int progress_sm;  // the consumers' last phase with its input complete (prefetch warp)
  __shared__ int tok_sm;

  const int c = blockIdx.x, G = gridDim.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pos0 = a.io[1], tok0 = a.io[0], count0 = a.io[2];
  const uint32_t per_step = tags_per_step(a.L);

  if (tid < kKinds) plan[tid] = plan_of(a, tid, c, G);
  if (tid == 32) {
    for (int s = 0; s < kSlots; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    fence_mbar_init();
    const bool ok = pos0 >= 0 && pos0 + a.steps <= a.max_len && count0 >= 0 && count0 + a.steps <= a.tokens_cap &&
                    tok0 >= 0 && tok0 < a.V;
    abort_sm = ok ? 0 : 1;
    issued_sm = 0;
    progress_sm = -1;
    tok_sm = tok0;
    if (!ok && c == 0) set_error(a.io + 3, TB200_ERR_ARG);
    trace_at(a.trace, 0, uint32_t(TB200_TRACE_OP_P_START) << 16, c, TB200_TRACE_START);
  }
  __syncthreads();
  const bool valid = !abort_sm;  // uniform: nothing is written for invalid arguments

  if (warp == kWarps + 1) {
    // ---- prefetch: each phase one layer ahead, once the consumers have the
    // phase's input (a bulk prefetch waits behind the ring's copies in the
    // copy engine, so it is issued from a thread that has nothing else to
    // do; and after the exchange, which it would slow) ----
    if (lane == 0 && valid) {
      for (int q = 0; q < kPhases; q++) prefetch_phase(a, plan[q], c, G, pos0, 0, 0, q);
      for (int step = 0; step < a.steps && !abort_sm; step++)
        for (int layer = 0; layer <= a.L && !abort_sm; layer++)
          for (int p = 0; p < kPhases && !abort_sm; p++) {
            if (layer == a.L && p != 0) break;
            const int ph = step * (4 * a.L + 1) + 4 * layer + p;  // as the consumers count
            // Bounded; a prefetch that never comes costs time, not results.
            const long long t0 = clock64();
            while (progress_sm < ph && !abort_sm && clock64() - t0 < kWaitCycles) __nanosleep(32);
            if (progress_sm < ph) break;
            if (layer + 1 < a.L) prefetch_phase(a, plan[p], c, G, pos0, step, layer + 1, p);
            // The head of this CTA's lm_head rows, spread over the last
            // layers, whose phases leave HBM idle while they exchange.
            const int j = layer - (a.L - kLmAheadLayers);
            if (j >= 0 && layer < a.L && p == 2) {
              const Plan& lm = plan[K_LM];
              const size_t total = size_t(lm.n) * size_t(lm.cols) * 2 * kLmAheadNum / kLmAheadDen / 16 * 16;
              const size_t c0 = total * size_t(j) / kLmAheadLayers / 16 * 16;
              const size_t c1 = total * size_t(j + 1) / kLmAheadLayers / 16 * 16;
              prefetch_range(reinterpret_cast<const char*>(a.lm_head + lm.w0 * lm.cols) + c0, c1 - c0);
            }
            else if (layer == a.L)
              for (int q = 0; q < kPhases; q++) prefetch_phase(a, plan[q], c, G, pos0, step + 1, 0, q);
          }
    }
  } else if (warp == kWarps) {
    // ---- producer: every matrix phase's rows of this CTA, in phase order ----
    if (lane == 0 && valid) {
      const uint64_t pol = l2_evict_first();
      int k = 0;
      for (int step = 0; step < a.steps && !abort_sm; step++)
        for (int layer = 0; layer <= a.L && !abort_sm; layer++)
          for (int p = 0; p < kPhases && !abort_sm; p++) {
            if (layer == a.L && p != 0) break;
            const int kind = layer == a.L ? K_LM : p;
            const Plan& pl = plan[kind];
            const uint16_t* w = matrix_of(a, a.layer[layer < a.L ? layer : 0], kind) + pl.w0 * pl.cols;
            for (int b = 0; b < pl.nst && !abort_sm; b++, k++) {
              const int slot = k % kSlots;
              if (k >= kSlots && !mbar_wait(&empty[slot], ((k / kSlots) - 1) & 1, a.io + 3)) {
                abort_sm = 1;
                break;
              }
              const int r = b * pl.sr;
              const uint32_t bytes = uint32_t(min(pl.sr, pl.n - r)) * uint32_t(pl.cols) * 2;
              mbar_arrive_expect_tx(&full[slot], bytes);
              bulk_g2s(ring + size_t(slot) * kSlotBytes, w + size_t(r) * pl.cols, bytes, &full[slot], pol);
              issued_sm = k + 1;
            }
            trace_at(a.trace, layer == a.L ? trace_base(a.L, 0, G) : trace_base(layer, p, G),
                     (uint32_t(TB200_TRACE_OP_P_QKV + kind) << 16) | uint32_t(layer), c, TB200_TRACE_ISSUED);
          }
    }
  } else if (valid) {
    // ---- consumers: the same control flow whatever the waits return ----
    int own0, own1;
    own_rows(a, c, G, own0, own1);
    int ag, as, ang;
    group_of(a, c, G, ag, as, ang);
    int k = 0;
    for (int step = 0; step < a.steps; step++) {
      const uint32_t T = a.epoch + uint32_t(step) * per_step;
      const int pos = pos0 + step;
      // The token: the launch's input, or the previous step's choice.
      if (step > 0) {
        if (tid == 0) {
          const long long t0 = clock64();
          TW w = 0;
          for (;;) {
            w = ld_tagged(a.tokw);
            if (ttag(w) == T - 1u || abort_sm || timed_out(t0, a.io + 3, &abort_sm)) break;
          }
          const int t = int(uint32_t(w));
          tok_sm = t >= 0 && t < a.V ? t : 0;
          // Acquire: the cache entries other CTAs appended in earlier steps
          // of this launch are read after this point.
          __threadfence();
        }
        named_sync(1, kConsumers);
      }
      const int tok = tok_sm;
      for (int r = own0 + tid; r < own1; r += kConsumers) {
        const float e = bf16f(a.embed[size_t(tok) * a.H + r]);
        own[r - own0] = e;
#pragma unroll
        for (int q = 0; q < kRep; q++) st_tagged(a.x + q * a.H + r, e, T);
      }
      uint32_t x_tag = T;  // tag of the residual stream's current version

      unsigned long long best = 0ull;
      for (int layer = 0; layer <= a.L; layer++) {
        const Layer& Ly = a.layer[layer < a.L ? layer : 0];
        const bool head = layer == a.L;
        for (int p = 0; p < kPhases; p++) {
          if (head && p != 0) break;
          const int kind = head ? K_LM : p;
          const uint32_t out_tag = phase_tag(T, layer, p);
          const TraceAt tr{a.trace, head ? trace_base(a.L, 0, G) : trace_base(layer, p, G),
                           (uint32_t(TB200_TRACE_OP_P_QKV + kind) << 16) | uint32_t(layer)};
          float scale = 1.0f;
          if (kind == K_ATTO) {
            attention_phase<GRP>(a, Ly, ag, as, ang, pos, phase_tag(T, layer, K_QKV), out_tag, xs, xs + 1024, tid,
                                 &abort_sm, tr, c);
            named_sync(1, kConsumers);
          } else {
            const int n_in = kind == K_DOWN ? a.F : a.H;
            const TW* in = (kind == K_DOWN ? a.h : a.x) + (c % kRep) * n_in;
            const uint32_t in_tag = kind == K_DOWN ? phase_tag(T, layer, K_GU)
                                    : kind == K_GU ? phase_tag(T, layer, K_ATTO)
                                                   : x_tag;
            const uint16_t* norm = kind == K_QKV ? Ly.attn_norm : kind == K_GU ? Ly.mlp_norm : kind == K_LM ? a.norm
                                                                                                             : nullptr;
            float ss = poll_vector(in, n_in, in_tag, norm, xs, tid, a.io + 3, &abort_sm);
            if (norm) {  // rmsnorm (cpu.rs:85-94): x * w stored, the 1/rms scale applied to each dot
              ss = warp_sum(ss);
              if (lane == 0) red[warp] = ss;
            }
            named_sync(1, kConsumers);
            if (norm) {
              float tot = 0.f;
#pragma unroll
              for (int w = 0; w < kWarps; w++) tot += red[w];
              scale = 1.0f / sqrtf(tot / float(n_in) + a.eps);
            }
          }
          if (tid == 0) {
            tr.at(c, TB200_TRACE_INPUT);
            progress_sm = step * (4 * a.L + 1) + 4 * layer + p;
          }
          const Plan pl = plan[kind];
          const int rb = pl.cols * 2;
          for (int b = 0; b < pl.nst; b++, k++) {
            const int slot = k % kSlots;
            const int rs0 = b * pl.sr, nrs = min(pl.sr, pl.n - rs0);
            int rpw = (nrs + kWarps - 1) / kWarps;
            if (kind == K_GU) rpw = (rpw + 1) & ~1;
            const int first = warp * rpw, nr = max(0, min(rpw, nrs - first));
            wait_full(&full[slot], (k / kSlots) & 1, a.io + 3, &abort_sm);
            if (tid == 0 && b == 0) tr.at(c, TB200_TRACE_WEIGHTS);
            if (tid == 0 && b == pl.nst - 1) tr.at(c, TB200_TRACE_LAST_WEIGHTS);
            const unsigned char* wbase = ring + size_t(slot) * kSlotBytes + size_t(first) * rb;
            WarpRows d{0.f, 1 << 20, 32};
            switch (nr) {
              case 1: d = dot_rows<1>(wbase, rb, pl.cols, xs, lane); break;
              case 2: d = dot_rows<2>(wbase, rb, pl.cols, xs, lane); break;
              case 3: d = dot_rows<3>(wbase, rb, pl.cols, xs, lane); break;
              case 4: d = dot_rows<4>(wbase, rb, pl.cols, xs, lane); break;
              case 5: d = dot_rows<5>(wbase, rb, pl.cols, xs, lane); break;
              case 6: d = dot_rows<6>(wbase, rb, pl.cols, xs, lane); break;
              case 7: d = dot_rows<7>(wbase, rb, pl.cols, xs, lane); break;
              case 8: d = dot_rows<8>(wbase, rb, pl.cols, xs, lane); break;
              default: break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            const int row = pl.r0 + rs0 + first + d.row;  // output row of this lane's value
            const float v = d.v * scale;
            if (kind == K_GU) {  // rows 2i (gate), 2i + 1 (up) -> h[i]
              const float up = __shfl_down_sync(0xffffffffu, v, d.stride);
              if (d.row < nr && (d.row & 1) == 0) {
                const float hv = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), up);
#pragma unroll
                for (int q = 0; q < kRep; q++) st_tagged(a.h + q * a.F + row / 2, hv, out_tag);
              }
            } else if (d.row < nr) {
              if (kind == K_QKV) {
                st_tagged(a.qkv + row, v, out_tag);
              } else if (kind == K_ATTO) {
                st_tagged(a.part_o + size_t(ag) * a.H + row, v, out_tag);
              } else if (kind == K_DOWN) {  // the residual add on a row this CTA owns
                const float x1 = __fadd_rn(own[row - own0], v);
                own[row - own0] = x1;
#pragma unroll
                for (int q = 0; q < kRep; q++) st_tagged(a.x + q * a.H + row, x1, out_tag);
              } else {
                if (a.logits) a.logits[row] = v;
                const unsigned long long key = argmax_key(v, uint32_t(row));
                best = key > best ? key : best;
              }
            }
          }
          if (kind == K_ATTO && tid < own1 - own0) {
            // x' = x + the o_proj partials of every kv group, in group order
            // (model.rs:131-132), on this CTA's residual rows: a poll of
            // Hkv words per row, so that the next phase reads x' alone.
            const int r = own0 + tid;
            float xv = own[tid];
            TW w[kMaxKv];
            const long long t0 = clock64();
            for (;;) {
              bool ok = true;
#pragma unroll
              for (int g = 0; g < kMaxKv; g++)
                if (g < a.Hkv) {
                  w[g] = ld_tagged(a.part_o + size_t(g) * a.H + r);
                  ok = ok && ttag(w[g]) == out_tag;
                }
              if (ok || abort_sm || timed_out(t0, a.io + 3, &abort_sm)) break;
            }
#pragma unroll
            for (int g = 0; g < kMaxKv; g++)
              if (g < a.Hkv) xv = __fadd_rn(xv, tval(w[g]));
            own[tid] = xv;
#pragma unroll
            for (int q = 0; q < kRep; q++) st_tagged(a.x + q * a.H + r, xv, out_tag);
          }
          if (kind == K_DOWN) x_tag = out_tag;
          if (tid == 0) tr.at(c, TB200_TRACE_DONE);
          named_sync(1, kConsumers);  // xs and own are rewritten by the next phase
        }
      }

      // The greedy token over the grid; the last CTA to arrive publishes it.
      best = warp_umax64(best);
      if (lane == 0) best_sm[warp] = best;
      named_sync(1, kConsumers);
      if (tid == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < kWarps; w++) b = best_sm[w] > b ? best_sm[w] : b;
        atomicMax(a.best, b);
        __threadfence();
        if (atomicAdd(a.ticket, 1u) == unsigned(G - 1)) {
          __threadfence();
          const unsigned long long bb = atomicExch(a.best, 0ull);
          *a.ticket = 0u;
          const int t = int(argmax_index(bb));
          a.io[0] = t;
          a.io[1] = pos + 1;
          a.io[2] = count0 + step + 1;
          a.tokens_out[count0 + step] = t;
          __threadfence();
          st_tagged(a.tokw, __int_as_float(t), T + per_step - 1u);
          trace_at(a.trace, trace_base(a.L, 1, G), uint32_t(TB200_TRACE_OP_P_TOKEN) << 16, c, TB200_TRACE_DONE);
        }
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
}

// One launch on `sms` CTAs, all resident (the kernel's shared memory allows
// one per SM), as a cooperative launch.
cudaError_t launch(const Args& a, int sms, cudaStream_t s) {
  static bool init[64] = {};  // per device ordinal
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  void (*kern)(Args) = a.grp == 1 ? step_kernel<1> : a.grp == 2 ? step_kernel<2> : step_kernel<4>;
  if (!init[dev]) {
    for (void (*k)(Args) : {step_kernel<1>, step_kernel<2>, step_kernel<4>}) {
      e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
      if (e != cudaSuccess) return e;
    }
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
  return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace tb::persist

namespace rt {

namespace P = tb::persist;

// Why model m and state st cannot run the persistent step ("" when they can).
// Models wider than kMaxCols (hidden, FFN or query width) or with a hidden
// size above 2048 (whose RMSNorm sums would depend on arrival order here),
// and every tensor-parallel rank, go to the wide kernel (persist_wide.cu).
static bool wide_model(const tb200_model* m) {
  return std::max({m->c.hidden_size, m->c.intermediate_size, m->q_dim}) > size_t(P::kMaxCols) ||
         m->c.hidden_size > 2048;
}

std::string persist_unsupported(const tb200_model* m, const tb200_state* st) {
  const tb200_config& c = m->c;
  const int sms = m->dev->sms;
  if (wide_model(m) || tp_world(m->tp) > 1) return persist_wide_unsupported(m, st);
  if (tp_world(m->tp) > 1) return "persistent decode runs unsharded models (no tensor parallelism)";
  if (st->n_seqs != 1) return "persistent decode runs one-sequence states";
  if (c.num_hidden_layers > size_t(P::kMaxLayers)) return "persistent decode runs at most 64 layers";
  if (c.head_dim != size_t(P::kHd)) return "persistent decode needs head_dim 128";
  if (c.intermediate_size > size_t(P::kMaxCols) || m->q_dim > size_t(P::kMaxCols) ||
      c.hidden_size > size_t(P::kMaxCols))
    return "persistent decode needs hidden, FFN and query widths up to 3072";
  const size_t grp = c.num_attention_heads / c.num_key_value_heads;
  if (grp > size_t(P::kMaxGrp) || c.num_key_value_heads > size_t(P::kMaxKv))
    return "persistent decode needs at most 4 query heads per kv head and at most 8 kv heads";
  const size_t G = std::min<size_t>({size_t(sms), c.hidden_size, c.intermediate_size, m->q_dim + 2 * m->kv_dim,
                                     c.vocab_size});
  if (G < c.num_key_value_heads || (c.hidden_size + G - 1) / G > size_t(P::kMaxOwn) ||
      (c.hidden_size / 4 + G - 1) / G * 4 > size_t(P::kMaxOwn))
    return "persistent decode: this GPU's SM count does not fit the model's kv groups and residual rows";
  return "";
}

// The state's persistent-step scratch, allocated on first use: tagged words
// (zeroed once; tags only grow, so stale words never match) and the argmax
// key and ticket.
static size_t persist_grid(const tb200_model* m) {
  const tb200_config& c = m->c;
  return std::min<size_t>({size_t(m->dev->sms), c.hidden_size, c.intermediate_size, m->q_dim + 2 * m->kv_dim,
                           c.vocab_size});
}

static int persist_prepare(tb200_state* st) {
  if (st->ps_words) return TB200_OK;
  const tb200_model* m = st->m;
  const tb200_config& c = m->c;
  const size_t grp = c.num_attention_heads / c.num_key_value_heads;
  const size_t nsplit = (persist_grid(m) + c.num_key_value_heads - 1) / c.num_key_value_heads;
  const size_t words = P::kRep * c.hidden_size + m->q_dim + 2 * m->kv_dim + P::kRep * c.intermediate_size +
                       c.num_key_value_heads * c.hidden_size + c.num_key_value_heads * nsplit * grp * P::kPartWords + 4;
  cudaStream_t s = m->dev->stream;
  CUDA_TRY(cudaMalloc(&st->ps_words, words * 8));
  CUDA_TRY(cudaMemsetAsync(st->ps_words, 0, words * 8, s));
  CUDA_TRY(cudaMalloc(&st->ps_ctl, 16));
  CUDA_TRY(cudaMemsetAsync(st->ps_ctl, 0, 16, s));
  st->ps_nwords = words;
  st->ps_epoch = 1;  // a zeroed word carries tag 0
  return TB200_OK;
}

// Enqueues `steps` greedy steps from the token and position in st->io as
// one launch (io[2] counts generated tokens into st->tokens_out); the last
// step's logits go to st->logits when `logits` (to `logits_to`, a device
// address of page-locked host memory, when given).
int persist_enqueue(tb200_state* st, size_t steps, bool logits, float* logits_to) {
  if (!steps) return TB200_OK;
  if (wide_model(st->m) || tp_world(st->m->tp) > 1) return persist_wide_enqueue(st, steps, logits, logits_to);
  if (int rc = persist_prepare(st)) return rc;
  const tb200_model* m = st->m;
  const tb200_config& c = m->c;
  cudaStream_t s = m->dev->stream;
  const uint32_t per = P::tags_per_step(int(c.num_hidden_layers));
  if (st->ps_dirty) {  // a launch that gave up may have left the grid's argmax half done
    CUDA_TRY(cudaMemsetAsync(st->ps_ctl, 0, 16, s));
    st->ps_dirty = false;
  }
  if (uint64_t(st->ps_epoch) + uint64_t(per) * steps >= 0xFFFF0000ull) {  // tags would wrap: start over
    CUDA_TRY(cudaMemsetAsync(st->ps_words, 0, st->ps_nwords * 8, s));
    st->ps_epoch = 1;
  }
  P::Args a{};
  const size_t eb = st->kv_f32 ? 4 : 2;
  const size_t per_layer = 2 * c.num_key_value_heads * st->max_len * c.head_dim;  // elements
  for (size_t l = 0; l < c.num_hidden_layers; l++) {
    const FusedLayer& L = m->layers[l];
    unsigned char* kb = st->kv + l * per_layer * eb;
    a.layer[l] = P::Layer{L.wqkv, L.wo_packed, L.wgu, L.wd, L.attn_norm, L.mlp_norm, L.q_norm, L.k_norm, kb,
                          kb + per_layer / 2 * eb};
  }
  a.L = int(c.num_hidden_layers), a.H = int(c.hidden_size), a.Q = int(m->q_dim), a.KV = int(m->kv_dim);
  a.F = int(c.intermediate_size), a.V = int(c.vocab_size);
  a.Hq = int(c.num_attention_heads), a.Hkv = int(c.num_key_value_heads), a.grp = a.Hq / a.Hkv;
  a.eps = c.rms_norm_eps;
  a.embed = m->embed, a.lm_head = m->lm_head, a.norm = m->norm;
  a.rope = st->rope, a.max_len = int(st->max_len), a.kv_f32 = st->kv_f32;
  P::TW* w = static_cast<P::TW*>(st->ps_words);
  a.x = w, a.qkv = a.x + P::kRep * a.H, a.h = a.qkv + a.Q + 2 * a.KV, a.part_o = a.h + P::kRep * a.F;
  const int grid = int(persist_grid(m));
  a.nsplit = (grid + a.Hkv - 1) / a.Hkv;
  a.part_att = a.part_o + size_t(a.Hkv) * a.H;
  a.tokw = a.part_att + size_t(a.Hkv) * a.nsplit * a.grp * P::kPartWords;
  a.io = st->io, a.tokens_out = st->tokens_out, a.tokens_cap = int(st->max_len);
  a.best = reinterpret_cast<unsigned long long*>(st->ps_ctl);
  a.ticket = reinterpret_cast<unsigned*>(static_cast<unsigned char*>(st->ps_ctl) + 8);
  a.logits = logits ? (logits_to ? logits_to : st->logits) : nullptr;
  a.epoch = st->ps_epoch;
  a.steps = int(steps);
  a.trace = st->trace;
  st->ps_epoch += per * uint32_t(steps);
  st->ps_grid = grid;
  if (st->trace.rec) st->ps_traced = true;
  cudaError_t e = P::launch(a, grid, s);
  if (e != cudaSuccess) return fail(TB200_ERR_CUDA, std::string("persistent decode: ") + cudaGetErrorString(e));
  return TB200_OK;
}

// Trace slots one persistent step uses.
size_t persist_trace_slots(const tb200_state* st) {
  return (3 + 4 * st->m->c.num_hidden_layers) * size_t(std::max(st->ps_grid, st->m->dev->sms)) * tb::kTraceEvents;
}

}  // namespace rt
