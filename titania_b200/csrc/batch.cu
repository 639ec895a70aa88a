// batch.cu — kernels of the many-token forward (model/model.rs:93-149 run
// over n tokens at once, and over many sequences at once): everything around
// the tensor-core contractions of gemm.cu.
//
//   k_split_rows     x -> three bf16 planes, the operand form of gemm.cu
//   k_norm_split     RMSNorm of each token row (cpu.rs:85-94), then the split
//   k_embed_split    embedding rows -> the first RMSNorm's planes and sums of
//                    squares (QK-norm, RoPE and the cache append run in the
//                    q|k|v contraction's epilogue, gemm.cu)
//   k_attn_rows      decode attention, one query token per sequence: a CTA per
//                    (token, kv group[, part of the context]) streaming the
//                    cache through a ring of bulk copies with an online
//                    softmax (cpu.rs:113-149)
//   k_attn_prefill   causal attention for a run of tokens of one sequence,
//                    tiled: 64 query rows against 64-position key/value tiles
//                    with an online softmax
//   k_argmax_finish  greedy choice per row from the argmax keys the lm_head
//                    contraction folded (sampler.rs:21-33 at temperature 0,
//                    ties to the lowest id), advancing each sequence's
//                    position for the device-side token loop
//
// The key/value cache of a batch is [sequence][layer][k|v][kv head][position]
// [head_dim]; a sequence's block is the single-sequence layout, so the
// single-token fused path reads the same cache.

#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace tb {

namespace {

constexpr int kD = 128;  // head_dim of the batched path (Qwen3)

template <typename... KArgs, typename... Args>
void launch_pdl(cudaStream_t s, dim3 grid, dim3 block, size_t smem, bool pdl, void (*kernel)(KArgs...),
                Args&&... args) {
  cudaLaunchConfig_t cfg{};
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

// ---- operand split and RMSNorm -------------------------------------------------

__global__ void k_split_rows(const float* __restrict__ x, uint16_t* __restrict__ out, size_t plane, size_t n) {
  pdl_launch_dependents();
  pdl_wait();
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    store_split3(out, plane, i, x[i]);
}

// One CTA per output row r: x row (row0 + r) of width dim, normalised as
// cpu.rs:85-94 (mean square, scale = 1/sqrt(ms + eps), v * (scale * w)),
// written split to row r of the three planes. With `add`, the row of `add`
// is first added to x (the residual update x += o, model.rs:121-123) and x
// written back.
__global__ void __launch_bounds__(256) k_norm_split(float* __restrict__ x, const float* __restrict__ add, int row0,
                                                   int dim, const uint16_t* __restrict__ w, float eps,
                                                   uint16_t* __restrict__ out, size_t plane, TraceAt tr) {
  __shared__ float red[8];
  pdl_launch_dependents();
  if (threadIdx.x == 0) tr.at(blockIdx.x, TB200_TRACE_START);
  pdl_wait();
  if (threadIdx.x == 0) tr.at(blockIdx.x, TB200_TRACE_WAITED);
  float* xr = x + size_t(row0 + blockIdx.x) * dim;
  if (add) {
    const float* ar = add + size_t(row0 + blockIdx.x) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) xr[i] = __fadd_rn(xr[i], ar[i]);
    __syncthreads();
  }
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = xr[i];
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; i++) tot += red[i];
  const float scale = 1.0f / sqrtf(tot / float(dim) + eps);
  const size_t row = size_t(blockIdx.x) * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x)
    store_split3(out, plane, row + i, __fmul_rn(xr[i], __fmul_rn(scale, bf16f(w[i]))));
  if (threadIdx.x == 0) tr.at(blockIdx.x, TB200_TRACE_DONE);
}

// One CTA per token: x row = the embedding row of the token (cpu.rs:38-47),
// then the first RMSNorm's input as the contraction consumes it: planes of
// x * w and the row's sum of squares (ssq[t], one part).
__global__ void __launch_bounds__(256) k_embed_split(float* __restrict__ x, const uint16_t* __restrict__ table,
                                                    int dim, const int* __restrict__ tok, int vocab,
                                                    const uint16_t* __restrict__ w, uint16_t* __restrict__ out,
                                                    size_t plane, float* __restrict__ ssq, int* err, TraceAt tr) {
  __shared__ float red[8];
  pdl_launch_dependents();
  if (threadIdx.x == 0) tr.at(blockIdx.x, TB200_TRACE_START);
  pdl_wait();
  int id = tok[blockIdx.x];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) set_error(err, TB200_ERR_ARG);
    id = 0;
  }
  const uint16_t* er = table + size_t(id) * dim;
  float* xr = x + size_t(blockIdx.x) * dim;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = bf16f(er[i]);
    xr[i] = v;
    ss = fmaf(v, v, ss);
    store_split3(out, plane, size_t(blockIdx.x) * dim + i, __fmul_rn(v, bf16f(w[i])));
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < int(blockDim.x >> 5); i++) tot += red[i];
    ssq[blockIdx.x] = tot;
    tr.at(blockIdx.x, TB200_TRACE_DONE);
  }
}

// ---- decode attention: one query token per sequence ------------------------------

template <bool F32KV>
struct RowsCfg {
  using KV = typename std::conditional<F32KV, float, uint16_t>::type;
  static constexpr int kCh = F32KV ? 32 : 64;  // positions per chunk: 16 KB each of K and V
  static constexpr int kStages = 3;            // chunks in flight
  static constexpr size_t kStageBytes = size_t(2) * kCh * kD * sizeof(KV);
  static constexpr size_t kSmem = kStages * kStageBytes;
};

__device__ __forceinline__ void load4(const float* p, float (&o)[4]) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}
__device__ __forceinline__ void load4(const uint16_t* p, float (&o)[4]) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  o[0] = bf_lo(v.x); o[1] = bf_hi(v.x); o[2] = bf_lo(v.y); o[3] = bf_hi(v.y);
}
__device__ __forceinline__ float load1(const float* p) { return *p; }
__device__ __forceinline__ float load1(const uint16_t* p) { return bf16f(*p); }

// CTA (part, kv group g, token t): the token's sequence from position
// part * span up to its own position, in chunks of kCh positions streamed by
// bulk copy through a ring of kStages chunks, with an online softmax
// (running max and sum per head). Per chunk: scores with a thread per
// (position, head) reading key rows in rotated 4-element groups
// (conflict-free), the chunk's statistics per head (a warp per head), then
// the weighted values with a thread per dimension. One part covers the
// whole context when the batch alone fills the GPU; otherwise the parts'
// partial results are combined in part order by the last CTA.
template <int GRP, bool F32KV>
__global__ void __launch_bounds__(128) k_attn_rows(AttnRowsArgs a) {
  using Cf = RowsCfg<F32KV>;
  using KV = typename Cf::KV;
  constexpr int CH = Cf::kCh, NS = Cf::kStages;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(16) float qs[GRP][kD];
  __shared__ float ps[GRP][CH];
  __shared__ float corr_s[GRP], m_s[GRP], l_s[GRP];
  __shared__ __align__(8) uint64_t bar[NS];
  __shared__ int verdict, is_last;
  auto kst = [&](int s) { return reinterpret_cast<KV*>(smem + size_t(s) * Cf::kStageBytes); };
  auto vst = [&](int s) { return kst(s) + size_t(CH) * kD; };

  pdl_launch_dependents();
  const int part = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
  const uint32_t cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  if (threadIdx.x == 0) a.trace.at(cta, TB200_TRACE_START);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Positions and sequence ids change only between steps (the host, or the
  // step's last kernel), so they can be read before the dependency wait.
  const int pos = a.pos[t], seq = a.seq[t];
  const bool ok = pos >= 0 && pos < a.max_len && seq >= 0 && seq < a.n_seqs;
  const int ctx = pos + 1;
  const int span = ((ctx + a.parts - 1) / a.parts + CH - 1) / CH * CH;  // positions per part, whole chunks
  const int nparts = (ctx + span - 1) / span;
  const bool active = ok && part < nparts;
  const int p0 = part * span, p1 = active ? min(ctx, p0 + span) : p0;
  const int nchunks = (p1 - p0 + CH - 1) / CH;
  const size_t head = size_t(seq) * a.seq_stride + size_t(g) * a.max_len * kD;
  const size_t v_off = size_t(a.n_kv_heads) * a.max_len * kD;
  const KV* kc = static_cast<const KV*>(a.kv) + head;
  const KV* vc = kc + v_off;
  const uint64_t pol = l2_evict_first();
  // Chunk i -> stage i % NS, completing on bar[i % NS].
  auto issue = [&](int i) {
    const int c0 = p0 + i * CH, n = min(CH, p1 - c0);
    const uint32_t bytes = uint32_t(n) * kD * sizeof(KV);
    uint64_t* b = &bar[i % NS];
    mbar_arrive_expect_tx(b, 2 * bytes);
    bulk_g2s(kst(i % NS), kc + size_t(c0) * kD, bytes, b, pol);
    bulk_g2s(vst(i % NS), vc + size_t(c0) * kD, bytes, b, pol);
  };

  int issued = 0;
  if (active) {
    if (tid == 0) {
      for (int s = 0; s < NS; s++) mbar_init(&bar[s], 1);
      fence_mbar_init();
      // Chunks before the token's own position were written by earlier
      // steps: they go out before the dependency wait.
      while (issued < NS && issued < nchunks && p0 + (issued + 1) * CH <= pos) issue(issued++);
    }
  }
  pdl_wait();
  if (threadIdx.x == 0) a.trace.at(cta, TB200_TRACE_WAITED);
  if (!ok) {
    if (part == 0 && g == 0 && tid == 0) set_error(a.err, TB200_ERR_ARG);
    return;
  }
  if (!active) return;
  if (tid == 0)
    while (issued < NS && issued < nchunks) issue(issued++);
  for (int i = tid; i < GRP * kD; i += 128) qs[i / kD][i % kD] = a.q[size_t(t) * a.ldq + size_t(g) * GRP * kD + i];
  if (tid < GRP) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
  }

  const float scale = 1.0f / sqrtf(float(kD));
  float acc[GRP], acc2[GRP];  // even and odd positions: two independent chains
#pragma unroll
  for (int h = 0; h < GRP; h++) acc[h] = acc2[h] = 0.f;
  bool failed = false;
  for (int i = 0; i < nchunks; i++) {
    const int s = i % NS;
    const int c0 = p0 + i * CH, n = min(CH, p1 - c0);
    // One thread waits with the time limit and the CTA follows its verdict.
    if (tid == 0) verdict = mbar_wait(&bar[s], (i / NS) & 1, a.err) ? 1 : 0;
    __syncthreads();  // also: qs and the previous chunk's statistics are visible
    if (!verdict) {
      failed = true;
      break;
    }
    mbar_wait(&bar[s], (i / NS) & 1, nullptr);  // the phase is complete: returns at once
    const KV* ks = kst(s);
    const KV* vs = vst(s);
    for (int idx = tid; idx < GRP * CH; idx += 128) {
      const int h = idx / CH, p = idx % CH;
      float sc = -INFINITY;
      if (p < n) {
        const KV* kr = ks + size_t(p) * kD;
        float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;  // four independent chains
#pragma unroll 8
        for (int j = 0; j < 32; j++) {
          const int c = 4 * ((j + p) & 31);
          float k4[4];
          load4(kr + c, k4);
          const float4 q4 = *reinterpret_cast<const float4*>(&qs[h][c]);
          d0 = fmaf(q4.x, k4[0], d0);
          d1 = fmaf(q4.y, k4[1], d1);
          d2 = fmaf(q4.z, k4[2], d2);
          d3 = fmaf(q4.w, k4[3], d3);
        }
        sc = scale * ((d0 + d1) + (d2 + d3));
      }
      ps[h][p] = sc;
    }
    __syncthreads();
    for (int h = warp; h < GRP; h += 4) {
      float mx = -INFINITY;
      for (int p = lane; p < n; p += 32) mx = fmaxf(mx, ps[h][p]);
      mx = warp_max(mx);
      const float mo = m_s[h];
      const float mn = fmaxf(mo, mx);
      float sum = 0.f;
      for (int p = lane; p < n; p += 32) {
        const float e = expf(ps[h][p] - mn);
        ps[h][p] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float c = expf(mo - mn);  // 0 on the first chunk (mo = -inf)
        corr_s[h] = c;
        m_s[h] = mn;
        l_s[h] = l_s[h] * c + sum;
      }
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < GRP; h++) {
      acc[h] *= corr_s[h];
      acc2[h] *= corr_s[h];
    }
    int p = 0;
#pragma unroll 2
    for (; p + 1 < n; p += 2) {
      const float v0 = load1(vs + size_t(p) * kD + tid);
      const float v1 = load1(vs + size_t(p + 1) * kD + tid);
#pragma unroll
      for (int h = 0; h < GRP; h++) {
        acc[h] = fmaf(ps[h][p], v0, acc[h]);
        acc2[h] = fmaf(ps[h][p + 1], v1, acc2[h]);
      }
    }
    if (p < n) {
      const float v0 = load1(vs + size_t(p) * kD + tid);
#pragma unroll
      for (int h = 0; h < GRP; h++) acc[h] = fmaf(ps[h][p], v0, acc[h]);
    }
    __syncthreads();  // every thread is done with stage s and ps
    if (tid == 0 && issued < nchunks) issue(issued++);
  }
  if (failed) {
    // Let the copies in flight land (bounded) before the CTA's memory goes.
    if (tid == 0)
      for (int i = max(0, issued - NS); i < issued; i++) mbar_wait(&bar[i % NS], (i / NS) & 1, nullptr);
    return;
  }

#pragma unroll
  for (int h = 0; h < GRP; h++) acc[h] += acc2[h];
  const size_t out_at = size_t(t) * a.ldo + size_t(g) * GRP * kD + tid;
  if (nparts == 1) {
#pragma unroll
    for (int h = 0; h < GRP; h++) store_split3(a.out, a.plane, out_at + size_t(h) * kD, acc[h] / l_s[h]);
    if (tid == 0) a.trace.at(cta, TB200_TRACE_DONE);
    return;
  }
  const int stride = kPartStride;
  float* pbase = a.part + ((size_t(t) * a.n_kv_heads + g) * a.parts) * GRP * stride;
#pragma unroll
  for (int h = 0; h < GRP; h++) {
    float* pp = pbase + (size_t(part) * GRP + h) * stride;
    pp[tid] = acc[h];
    if (tid == 0) {
      pp[kD] = m_s[h];
      pp[kD + 1] = l_s[h];
    }
  }
  __threadfence();
  __syncthreads();
  unsigned* ticket = a.ticket + size_t(t) * a.n_kv_heads + g;
  if (tid == 0) is_last = atomicAdd(ticket, 1u) == unsigned(nparts - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  {
    // The staging ring is free now: it holds the merge weights, then the merged heads.
    __shared__ float hsum[GRP];
    float* wbuf = reinterpret_cast<float*>(smem);
    float(*merged)[128] = reinterpret_cast<float(*)[128]>(wbuf + ((nparts * GRP + 3) & ~3));  // 16-byte aligned
    merge_splits<GRP>(pbase, nparts, wbuf, hsum, merged);
#pragma unroll
    for (int h = 0; h < GRP; h++) store_split3(a.out, a.plane, out_at + size_t(h) * kD, merged[h][tid]);
  }
  if (tid == 0) *ticket = 0u;
}

// ---- decode attention on the tensor cores (bf16 cache) ---------------------------
//
// The same work as k_attn_rows for a bf16 cache, with the two products on
// mma.sync m16n8k16 (bf16 in, f32 accumulate):
//   scores   S[p][c] = K[p][:] . qc[:]   A = 16 cached keys (ldmatrix), B = the
//            query as columns (column GRP j + h: plane j of head h, q = q0 + q1
//            + q2; padded to blocks of 8 with zeros), kept in registers;
//   values   O[d][c] = V[:][d] . Pc[:]   A = 16 dimensions x 16 positions of V
//            (ldmatrix.trans), B = the probabilities split the same way.
// Scores and outputs are regrouped by head through small per-warp tiles in
// shared memory.
// Every product is exact (bf16 x bf16 in f32) and the planes make q and P
// exact, so only the f32 accumulation order differs from k_attn_rows. Keys
// and values arrive by TMA (128-byte swizzle, so ldmatrix is conflict-free)
// in chunks of 32 positions; warps 2h and 2h + 1 take every other chunk
// (h, h + 2, ...), positions 0..15 and 16..31 of it, each keeping its own
// running max, sum and output; the four warps are combined once at the end.

constexpr int kTcCh = 32;                         // positions per chunk (two warps of 16)
constexpr int kTcStages = 3;
constexpr int kTcBox = kTcCh * 64 * 2;            // one 32-position x 64-dim box: 4 KB
constexpr int kTcStage = 4 * kTcBox;              // K lo/hi dims, V lo/hi dims: 16 KB
// 49 KB of staging: four CTAs fit on an SM, so 148 x 4 = 592 (token, kv group)
// CTAs run at once (64 sequences x 8 kv heads = 512 in one wave).
constexpr size_t kTcSmem = size_t(kTcStages) * kTcStage + 1024;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Byte offset of (row r, 16-byte unit u) in a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t sw128(int r, int u) { return uint32_t(r * 128 + ((u ^ (r & 7)) << 4)); }
__device__ __forceinline__ uint16_t plane_of(float v, int j) {
  const uint16_t a = f2bf(v);
  if (j == 0) return a;
  const float r = v - bf16f(a);
  const uint16_t b = f2bf(r);
  return j == 1 ? b : f2bf(r - bf16f(b));
}

template <int GRP>
__global__ void __launch_bounds__(128, GRP <= 2 ? 4 : 2)
    k_attn_rows_tc(const __grid_constant__ CUtensorMap cache, AttnRowsArgs a) {
  constexpr int NC = 3 * GRP;        // live columns: plane j of head h at column GRP j + h
  constexpr int NB = (NC + 7) / 8;   // MMA column blocks of 8
  constexpr int HP = (GRP + 1) / 2;  // (position, head) pairs per lane: 16 positions x GRP heads / 32 lanes
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // swizzled boxes: 1024-byte aligned
  __shared__ __align__(16) float qs[GRP][kD];
  __shared__ __align__(16) uint16_t pw[4][8 * NB][16];  // per warp: probabilities [column][position]
  __shared__ float sw[4][16][8 * NB + 1];               // per warp: scores [position][column]
  __shared__ float corr_w[4][GRP];
  __shared__ float wm[4][GRP], wl[4][GRP];
  __shared__ __align__(8) uint64_t bar[kTcStages];
  __shared__ int consumed[kTcStages], is_last;
  // The chunk whose load was last issued into each stage. The two warp pairs
  // walk different chunks, so a pair can be two phases of a stage's barrier
  // ahead of its chunk; it waits for its own chunk's issue first.
  __shared__ volatile int stage_chunk[kTcStages];

  pdl_launch_dependents();
  const int part = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
  const uint32_t cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  if (threadIdx.x == 0) a.trace.at(cta, TB200_TRACE_START);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Positions and sequence ids change only between steps (the host, or the
  // step's last kernel), so they can be read before the dependency wait.
  const int pos = a.pos[t], seq = a.seq[t];
  const bool ok = pos >= 0 && pos < a.max_len && seq >= 0 && seq < a.n_seqs;
  const int ctx = pos + 1;
  const int span = ((ctx + a.parts - 1) / a.parts + kTcCh - 1) / kTcCh * kTcCh;
  const int nparts = (ctx + span - 1) / span;
  const bool active = ok && part < nparts;
  const int p0 = part * span, p1 = active ? min(ctx, p0 + span) : p0;
  const int nchunks = (p1 - p0 + kTcCh - 1) / kTcCh;
  // Cache rows (of head_dim elements) of this (sequence, layer, kv head).
  const int krow = int(size_t(seq) * a.seq_stride / kD) + a.layer_rows + g * a.max_len;
  const int vrow = krow + a.n_kv_heads * a.max_len;
  const uint64_t pol = l2_evict_first();
  auto issue = [&](int i) {
    unsigned char* st = sm + size_t(i % kTcStages) * kTcStage;
    uint64_t* b = &bar[i % kTcStages];
    const int c0 = p0 + i * kTcCh;
    stage_chunk[i % kTcStages] = i;
    mbar_arrive_expect_tx(b, kTcStage);
    tma_load_2d(st, &cache, 0, krow + c0, b, pol);
    tma_load_2d(st + kTcBox, &cache, 64, krow + c0, b, pol);
    tma_load_2d(st + 2 * kTcBox, &cache, 0, vrow + c0, b, pol);
    tma_load_2d(st + 3 * kTcBox, &cache, 64, vrow + c0, b, pol);
  };

  int issued = 0;
  if (active && tid == 0) {
    for (int s = 0; s < kTcStages; s++) {
      mbar_init(&bar[s], 1);
      consumed[s] = 0;
      stage_chunk[s] = -1;
    }
    fence_mbar_init();
    // Chunks wholly before the token's own position were written by earlier
    // steps: they go out before the dependency wait.
    while (issued < kTcStages && issued < nchunks && p0 + (issued + 1) * kTcCh <= pos) issue(issued++);
  }
  pdl_wait();
  if (threadIdx.x == 0) a.trace.at(cta, TB200_TRACE_WAITED);
  if (!ok) {
    if (part == 0 && g == 0 && tid == 0) set_error(a.err, TB200_ERR_ARG);
    return;
  }
  if (!active) return;
  if (tid == 0) {
    while (issued < kTcStages && issued < nchunks) issue(issued++);
  }
  for (int i = tid; i < GRP * kD; i += 128) qs[i / kD][i % kD] = a.q[size_t(t) * a.ldq + size_t(g) * GRP * kD + i];
  for (int i = tid; i < 4 * 8 * NB * 16; i += 128) (&pw[0][0][0])[i] = 0;  // pad columns stay zero
  __syncthreads();

  // The query as B fragments: column c = 8 nb + lane / 4, k = dims 16 kb + 2 (lane % 4) (+1, +8, +9).
  const int kq = 2 * (lane & 3);
  uint32_t qb[NB][8][2];
#pragma unroll
  for (int nb = 0; nb < NB; nb++) {
    const int c = 8 * nb + (lane >> 2);
    const int qj = c / GRP, qh = c % GRP;
    const bool live = c < NC;
#pragma unroll
    for (int kb = 0; kb < 8; kb++)
#pragma unroll
      for (int hf = 0; hf < 2; hf++) {
        const int d = 16 * kb + kq + 8 * hf;
        const uint32_t lo = live ? plane_of(qs[qh][d], qj) : 0u;
        const uint32_t hi = live ? plane_of(qs[qh][d + 1], qj) : 0u;
        qb[nb][kb][hf] = lo | (hi << 16);
      }
  }

  // Scores are kept in base-2 units (scaled by log2 e) so the exponentials are exp2.
  const float scale2 = 1.4426950408889634f / sqrtf(float(kD));
  // This lane's (position, head) pairs: position rr of the warp's 16, heads
  // hb + 2 i. The running max per head (shared by the 16 lanes of the head)
  // and this lane's share of the running sum (added up once at the end).
  const int rr = lane & 15, hb = lane >> 4;
  float m[HP], l[HP];
#pragma unroll
  for (int i = 0; i < HP; i++) {
    m[i] = -INFINITY;
    l[i] = 0.f;
  }
  float o[8][NB][4];  // O^T fragments: dims 16 mb + lane / 4 (+8), columns 8 nb + 2 (lane % 4) (+1)
#pragma unroll
  for (int mb = 0; mb < 8; mb++)
#pragma unroll
    for (int nb = 0; nb < NB; nb++) o[mb][nb][0] = o[mb][nb][1] = o[mb][nb][2] = o[mb][nb][3] = 0.f;
  const int r = lane >> 2;
  bool failed = false;
  // The warps go through the chunks independently: each waits for a chunk
  // itself, and the last warp done with a stage issues the chunk kTcStages
  // ahead into it (no block-wide barrier per chunk).
  // Warps 2h and 2h + 1 take chunks h, h + 2, h + 4, ...: positions 0..15 and
  // 16..31 of each.
  for (int i = warp >> 1; i < nchunks; i += 2) {
    const int s = i % kTcStages;
    const int c0 = p0 + i * kTcCh;
    int got = 1;
    if (lane == 0) {
      // This chunk's load was issued (bounded wait), then it landed.
      const long long t0 = clock64();
      while (stage_chunk[s] != i)
        if (clock64() - t0 > kWaitCycles) {
          set_error(a.err, TB200_ERR_TIMEOUT);
          got = 0;
          break;
        }
      if (got) got = mbar_wait(&bar[s], (i / kTcStages) & 1, a.err) ? 1 : 0;
    }
    if (!__shfl_sync(0xffffffffu, got, 0)) {
      failed = true;
      break;
    }
    mbar_wait(&bar[s], (i / kTcStages) & 1, nullptr);  // the phase is complete: returns at once
    const uint32_t kbase = smem_u32(sm + size_t(s) * kTcStage), vbase = kbase + 2 * kTcBox;
    const int pw0 = 16 * (warp & 1);  // the warp's first position in the chunk
    {
      // All eight key fragments first, then two independent accumulation chains.
      const int ar = pw0 + (lane & 7) + 8 * ((lane >> 3) & 1), au = lane >> 4;
      uint32_t af[8][4];
#pragma unroll
      for (int kb = 0; kb < 8; kb++) ldsm_x4(kbase + (kb >> 2) * kTcBox + sw128(ar, 2 * (kb & 3) + au), af[kb]);
      float sc[2][NB][4];
#pragma unroll
      for (int h2 = 0; h2 < 2; h2++)
#pragma unroll
        for (int nb = 0; nb < NB; nb++) sc[h2][nb][0] = sc[h2][nb][1] = sc[h2][nb][2] = sc[h2][nb][3] = 0.f;
#pragma unroll
      for (int kb = 0; kb < 8; kb++)
#pragma unroll
        for (int nb = 0; nb < NB; nb++) mma16816(sc[kb & 1][nb], af[kb], qb[nb][kb][0], qb[nb][kb][1]);
#pragma unroll
      for (int nb = 0; nb < NB; nb++) {
        sw[warp][r][8 * nb + kq] = sc[0][nb][0] + sc[1][nb][0];
        sw[warp][r][8 * nb + kq + 1] = sc[0][nb][1] + sc[1][nb][1];
        sw[warp][r + 8][8 * nb + kq] = sc[0][nb][2] + sc[1][nb][2];
        sw[warp][r + 8][8 * nb + kq + 1] = sc[0][nb][3] + sc[1][nb][3];
      }
    }
    __syncwarp();
    const int n = min(kTcCh, p1 - c0);
    const bool live_pos = pw0 + rr < n;
    float pv[HP];
#pragma unroll
    for (int i2 = 0; i2 < HP; i2++) {
      const int h = hb + 2 * i2;
      float sc = -INFINITY;
      if (h < GRP && live_pos) sc = scale2 * ((sw[warp][rr][h] + sw[warp][rr][GRP + h]) + sw[warp][rr][2 * GRP + h]);
      // Running max of head h over this warp's positions (lanes with the same hb).
      float mx = sc;
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[i2], mx);
      const float corr = (m[i2] == -INFINITY || mn == -INFINITY) ? 0.f : exp2f(m[i2] - mn);
      const float e = sc == -INFINITY ? 0.f : exp2f(sc - mn);
      l[i2] = l[i2] * corr + e;
      m[i2] = mn;
      pv[i2] = e;
      if (rr == 0 && h < GRP) corr_w[warp][h] = corr;
    }
    // Probabilities as B fragments (three planes per head), via the warp's pw.
#pragma unroll
    for (int i2 = 0; i2 < HP; i2++) {
      const int h = hb + 2 * i2;
      if (h < GRP)
#pragma unroll
        for (int j = 0; j < 3; j++) pw[warp][GRP * j + h][rr] = plane_of(pv[i2], j);
    }
    __syncwarp();
    {
      const int vr = pw0 + (lane & 7) + 8 * (lane >> 4), vu = (lane >> 3) & 1;
      uint32_t af[8][4];
#pragma unroll
      for (int mb = 0; mb < 8; mb++) ldsm_x4_t(vbase + (mb >> 2) * kTcBox + sw128(vr, 2 * (mb & 3) + vu), af[mb]);
      uint32_t pb[NB][2];
#pragma unroll
      for (int nb = 0; nb < NB; nb++) {
        pb[nb][0] = *reinterpret_cast<const uint32_t*>(&pw[warp][8 * nb + (lane >> 2)][kq]);
        pb[nb][1] = *reinterpret_cast<const uint32_t*>(&pw[warp][8 * nb + (lane >> 2)][kq + 8]);
      }
#pragma unroll
      for (int mb = 0; mb < 8; mb++)
#pragma unroll
        for (int nb = 0; nb < NB; nb++)
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const int c = 8 * nb + kq + (e & 1);
            o[mb][nb][e] *= c < NC ? corr_w[warp][c % GRP] : 0.f;
          }
#pragma unroll
      for (int mb = 0; mb < 8; mb++)
#pragma unroll
        for (int nb = 0; nb < NB; nb++) mma16816(o[mb][nb], af[mb], pb[nb][0], pb[nb][1]);
    }
    // This warp is done with stage s (its fragments are in registers). The
    // second warp of the chunk to get here refills the stage.
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&consumed[s], 1) == 1) {  // both warps of the chunk are done
        consumed[s] = 0;
        __threadfence_block();  // the reset is seen before the next chunk's issue
        if (i + kTcStages < nchunks) issue(i + kTcStages);
      }
    }
  }
  // Every warp is out of the loop (and done reading the stages) before the
  // stage memory is reused below; a failure anywhere fails the CTA.
  failed = __syncthreads_or(failed);
  if (failed) {
    // Let the copies in flight land (bounded) before the CTA's memory goes.
    if (tid == 0)
      for (int s = 0; s < kTcStages; s++) {
        const int c = stage_chunk[s];  // the last chunk issued into stage s
        if (c >= 0) mbar_wait(&bar[s], (c / kTcStages) & 1, nullptr);
      }
    return;
  }
  // The sums of the 16 lanes of each head.
#pragma unroll
  for (int i2 = 0; i2 < HP; i2++)
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) l[i2] += __shfl_xor_sync(0xffffffffu, l[i2], off);

  // Per warp: publish (m, l) per head and O per (column, dim) into the idle
  // stage memory, then thread d combines the warps and the planes.
  float* ow = reinterpret_cast<float*>(sm);  // [4][8 NB][kD]
#pragma unroll
  for (int mb = 0; mb < 8; mb++)
#pragma unroll
    for (int nb = 0; nb < NB; nb++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int c = 8 * nb + kq + (e & 1), d = 16 * mb + r + 8 * (e >> 1);
        ow[(warp * 8 * NB + c) * kD + d] = o[mb][nb][e];
      }
  if (rr == 0)
#pragma unroll
    for (int i2 = 0; i2 < HP; i2++) {
      const int h = hb + 2 * i2;
      if (h < GRP) {
        wm[warp][h] = m[i2];
        wl[warp][h] = l[i2];
      }
    }
  __syncthreads();
  float res[GRP], rm[GRP], rl[GRP];
#pragma unroll
  for (int h = 0; h < GRP; h++) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; w++) M = fmaxf(M, wm[w][h]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; w++) {
      const float wt = wm[w][h] == -INFINITY ? 0.f : exp2f(wm[w][h] - M);  // base-2 units
      const float* ob = ow + size_t(w * 8 * NB) * kD + tid;
      const float ov = (ob[size_t(h) * kD] + ob[size_t(GRP + h) * kD]) + ob[size_t(2 * GRP + h) * kD];
      L += wl[w][h] * wt;
      O += ov * wt;
    }
    res[h] = O;
    rm[h] = M;
    rl[h] = L;
  }
  const size_t out_at = size_t(t) * a.ldo + size_t(g) * GRP * kD + tid;
  if (nparts == 1) {
#pragma unroll
    for (int h = 0; h < GRP; h++) store_split3(a.out, a.plane, out_at + size_t(h) * kD, res[h] / rl[h]);
    if (tid == 0) a.trace.at(cta, TB200_TRACE_DONE);
    return;
  }
  const int stride = kPartStride;
  float* pbase = a.part + ((size_t(t) * a.n_kv_heads + g) * a.parts) * GRP * stride;
#pragma unroll
  for (int h = 0; h < GRP; h++) {
    float* pp = pbase + (size_t(part) * GRP + h) * stride;
    pp[tid] = res[h];
    if (tid == 0) {
      pp[kD] = rm[h] * 0.6931471805599453f;  // the partial records hold natural-log maxima
      pp[kD + 1] = rl[h];
    }
  }
  __threadfence();
  __syncthreads();
  unsigned* ticket = a.ticket + size_t(t) * a.n_kv_heads + g;
  if (tid == 0) is_last = atomicAdd(ticket, 1u) == unsigned(nparts - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  {
    // The staging ring is free now: it holds the merge weights, then the merged heads.
    __shared__ float hsum[GRP];
    float* wbuf = reinterpret_cast<float*>(sm);
    float(*merged)[128] = reinterpret_cast<float(*)[128]>(wbuf + ((nparts * GRP + 3) & ~3));  // 16-byte aligned
    merge_splits<GRP>(pbase, nparts, wbuf, hsum, merged);
#pragma unroll
    for (int h = 0; h < GRP; h++) store_split3(a.out, a.plane, out_at + size_t(h) * kD, merged[h][tid]);
  }
  if (tid == 0) *ticket = 0u;
}

// ---- causal prefill attention -------------------------------------------------------

constexpr int kPR = 64;     // query rows per CTA (tokens x heads of one kv group)
constexpr int kPK = 64;     // cache positions per tile
constexpr int kPPad = 68;   // padded row of the transposed tiles
struct PrefillSmem {
  float qt[kD][kPPad];   // queries, transposed: [dim][row]
  float kt[kD][kPPad];   // keys, transposed:    [dim][position]
  float vs[kPK][kD];     // values:              [position][dim]
  float ps[kPR][kPPad];  // probabilities:       [row][position]
};

// CTA (query block, kv group g): rows r = token * GRP + head of kPR / GRP
// consecutive tokens; 256 threads, thread (ty, tx) = (tid / 16, tid % 16)
// owns rows 4ty .. 4ty+3, score columns 4tx .. 4tx+3 and output dimensions
// 8tx .. 8tx+7.
template <int GRP, bool F32KV>
__global__ void __launch_bounds__(256) k_attn_prefill(AttnPrefillArgs a) {
  using KV = typename std::conditional<F32KV, float, uint16_t>::type;
  constexpr int QT = kPR / GRP;  // tokens per CTA
  extern __shared__ __align__(128) unsigned char smem[];
  PrefillSmem& S = *reinterpret_cast<PrefillSmem*>(smem);
  pdl_launch_dependents();
  pdl_wait();
  const int nqb = (a.T + QT - 1) / QT;
  const int qb = nqb - 1 - int(blockIdx.x);  // longest rows first
  const int g = blockIdx.y;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int tok0 = qb * QT;
  const int qtok = min(QT, a.T - tok0);
  const int kend = a.pos0 + tok0 + qtok;  // keys [0, kend) cover every row's causal window
  const size_t v_off = size_t(a.n_kv_heads) * a.max_len * kD;
  const KV* kc = static_cast<const KV*>(a.kv) + size_t(g) * a.max_len * kD;
  const KV* vc = kc + v_off;

  for (int i = tid; i < kPR * kD; i += 256) {
    const int r = i / kD, d = i % kD;
    const int tk = r / GRP, h = r % GRP;
    S.qt[d][r] = tk < qtok ? a.q[size_t(tok0 + tk) * a.ldq + size_t(g * GRP + h) * kD + d] : 0.f;
  }
  float o[4][8], m[4], l[4];
  int qpos[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    m[i] = -INFINITY;
    l[i] = 0.f;
    qpos[i] = a.pos0 + tok0 + (4 * ty + i) / GRP;
#pragma unroll
    for (int j = 0; j < 8; j++) o[i][j] = 0.f;
  }
  const float scale = 1.0f / sqrtf(float(kD));
  const int ntiles = (kend + kPK - 1) / kPK;
  for (int kt = 0; kt < ntiles; kt++) {
    const int kp0 = kt * kPK;
    const int kn = min(kPK, kend - kp0);
    __syncthreads();  // previous tile's reads of kt / vs / ps are done
    for (int i = tid; i < kPK * kD; i += 256) {
      const int p = i / kD, d = i % kD;
      float kv = 0.f, vv = 0.f;
      if (p < kn) {
        kv = load1(kc + size_t(kp0 + p) * kD + d);
        vv = load1(vc + size_t(kp0 + p) * kD + d);
      }
      S.kt[d][p] = kv;
      S.vs[p][d] = vv;
    }
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) s[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < kD; d++) {
      const float4 q4 = *reinterpret_cast<const float4*>(&S.qt[d][4 * ty]);
      const float4 k4 = *reinterpret_cast<const float4*>(&S.kt[d][4 * tx]);
      const float qv[4] = {q4.x, q4.y, q4.z, q4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int kp = kp0 + 4 * tx + j;
        s[i][j] = (4 * tx + j < kn && kp <= qpos[i]) ? scale * s[i][j] : -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[i], mx);
      const float corr = expf(m[i] - mn);
      float sum = 0.f;
      float p4[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        p4[j] = expf(s[i][j] - mn);
        sum += p4[j];
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      l[i] = l[i] * corr + sum;
      m[i] = mn;
#pragma unroll
      for (int j = 0; j < 8; j++) o[i][j] *= corr;
      *reinterpret_cast<float4*>(&S.ps[4 * ty + i][4 * tx]) = make_float4(p4[0], p4[1], p4[2], p4[3]);
    }
    __syncthreads();
#pragma unroll 2
    for (int p = 0; p < kn; p++) {
      const float4 va = *reinterpret_cast<const float4*>(&S.vs[p][8 * tx]);
      const float4 vb = *reinterpret_cast<const float4*>(&S.vs[p][8 * tx + 4]);
      const float vv[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float pr = S.ps[4 * ty + i][p];
#pragma unroll
        for (int j = 0; j < 8; j++) o[i][j] = fmaf(pr, vv[j], o[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int r = 4 * ty + i, tk = r / GRP, h = r % GRP;
    if (tk >= qtok) continue;
    const size_t at = size_t(tok0 + tk) * a.ldo + size_t(g * GRP + h) * kD + 8 * tx;
    const float inv = 1.0f / l[i];
#pragma unroll
    for (int j = 0; j < 8; j++) store_split3(a.out, a.plane, at + j, o[i][j] * inv);
  }
}

// ---- greedy choice per row ----------------------------------------------------------

// One CTA: the token ids from the keys a contraction folded into best[],
// which it zeroes for the next step.
__global__ void __launch_bounds__(256) k_argmax_finish(ArgmaxRowsArgs a, unsigned long long* best, int rows) {
  __shared__ int step_s;
  pdl_launch_dependents();
  if (threadIdx.x == 0) a.trace.at(0, TB200_TRACE_START);
  pdl_wait();
  if (threadIdx.x == 0) a.trace.at(0, TB200_TRACE_WAITED);
  if (threadIdx.x == 0) step_s = a.step ? *a.step : 0;
  __syncthreads();
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    const unsigned long long k = best[r];
    best[r] = 0ull;
    int tok = int(argmax_index(k));
    if (k == 0ull || tok < 0 || tok >= a.V) {  // no key arrived: a contraction failed
      set_error(a.err, TB200_ERR_TIMEOUT);
      tok = 0;
    }
    if (a.next) a.next[r] = tok;
    if (a.tok) a.tok[r] = tok;
    if (a.pos) a.pos[r] += 1;
    if (a.out && step_s < a.out_cap) a.out[size_t(step_s) * rows + r] = tok;
  }
  __syncthreads();
  if (threadIdx.x == 0 && a.step) *a.step = step_s + 1;
  if (threadIdx.x == 0) a.trace.at(0, TB200_TRACE_DONE);
}

// ---- causal prompt attention on the tensor cores (bf16 cache) -------------------
//
// CTA (query block, kv group g) of 4 warps; warp w owns query rows 16w ..
// 16w+15 of the block (row r = token r / GRP, head r % GRP of the group).
// For every 64-position tile of keys and values (double-buffered in shared
// memory with cp.async, rows padded to 272 bytes so that ldmatrix reads
// distinct banks): scores S = Q K^T with mma.sync m16n8k16 (Q as two bf16
// planes, q = q0 + q1 to 2^-17, K exact), a base-2 online softmax per row
// (the four lanes of a quad share a row), then O += P V with P as two bf16
// planes taken straight from the score accumulators. The result leaves as
// the three bf16 planes of O / l, the next contraction's operand.
constexpr int kPQR = 64;            // query rows per CTA
constexpr int kPKT = 64;            // cache positions per tile
constexpr int kPRow = kD + 8;       // shared-memory row of a tile, in bf16 elements (272 bytes)
constexpr size_t kPTile = size_t(kPKT) * kPRow * 2;
constexpr size_t kPrefillTcSmem = 4 * kPTile;  // K and V, two stages

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return uint32_t(f2bf(lo)) | (uint32_t(f2bf(hi)) << 16);
}
__device__ __forceinline__ float bf_round(float v) { return bf16f(f2bf(v)); }

template <int GRP>
__global__ void __launch_bounds__(128) k_attn_prefill_tc(AttnPrefillArgs a) {
  extern __shared__ __align__(128) unsigned char smem_pf[];
  uint16_t* tiles = reinterpret_cast<uint16_t*>(smem_pf);  // [stage][K | V][kPKT][kPRow]
  constexpr int QT = kPQR / GRP;  // tokens per CTA
  pdl_launch_dependents();
  pdl_wait();
  const int nqb = (a.T + QT - 1) / QT;
  const int qb = nqb - 1 - int(blockIdx.x);  // longest rows first
  const int g = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gq = lane >> 2, tq = lane & 3;
  const int tok0 = qb * QT;
  const int qtok = min(QT, a.T - tok0);
  const int kend = a.pos0 + tok0 + qtok;  // keys [0, kend) cover every row's causal window
  const uint16_t* kc = static_cast<const uint16_t*>(a.kv) + size_t(g) * a.max_len * kD;
  const uint16_t* vc = kc + size_t(a.n_kv_heads) * a.max_len * kD;

  // This lane's two rows and their positions (the causal limits).
  int rtok[2], rqp[2];
  bool rok[2];
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int r = 16 * warp + gq + 8 * i;
    rtok[i] = r / GRP;
    rok[i] = rtok[i] < qtok;
    rqp[i] = a.pos0 + tok0 + rtok[i];
  }
  auto qval = [&](int i, int d) -> float {
    const int r = 16 * warp + gq + 8 * i;
    return rok[i] ? a.q[size_t(tok0 + rtok[i]) * a.ldq + size_t(g * GRP + r % GRP) * kD + d] : 0.f;
  };
  // Q as A fragments, two planes: a0 = (row gq, dims 2tq, 2tq+1), a1 = row
  // gq + 8, a2 / a3 the same at dims + 8, per 16-dim k-block.
  uint32_t qa[2][8][4];
#pragma unroll
  for (int kb = 0; kb < 8; kb++)
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int i = j & 1, d = 16 * kb + 2 * tq + 8 * (j >> 1);
      const float x0 = qval(i, d), x1 = qval(i, d + 1);
      qa[0][kb][j] = pack2(x0, x1);
      qa[1][kb][j] = pack2(x0 - bf_round(x0), x1 - bf_round(x1));
    }

  auto load_tile = [&](int kt, int stage) {
    uint16_t* ks = tiles + size_t(stage) * 2 * kPKT * kPRow;
    uint16_t* vs = ks + kPKT * kPRow;
    for (int i = tid; i < kPKT * (kD / 8); i += 128) {
      const int r = i / (kD / 8), c = (i % (kD / 8)) * 8;
      const int p = kt * kPKT + r;
      const bool ok = p < a.max_len;
      const size_t at = size_t(ok ? p : 0) * kD + c;
      cp_async16(ks + r * kPRow + c, kc + at, ok);
      cp_async16(vs + r * kPRow + c, vc + at, ok);
    }
    cp_async_commit();
  };

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const float scale2 = 1.4426950408889634f / sqrtf(float(kD));
  const int ntiles = (kend + kPKT - 1) / kPKT;
  load_tile(0, 0);
  for (int kt = 0; kt < ntiles; kt++) {
    if (kt + 1 < ntiles) {
      load_tile(kt + 1, (kt + 1) & 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint16_t* ks = tiles + size_t(kt & 1) * 2 * kPKT * kPRow;
    const uint16_t* vs = ks + kPKT * kPRow;
    // S = Q K^T over the tile's 64 positions: n-block nb = positions 8nb .. 8nb+7.
    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; nb++) {
      s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
#pragma unroll
      for (int kbp = 0; kbp < 4; kbp++) {
        uint32_t b[4];
        ldsm_x4(smem_u32(ks + (nb * 8 + (lane & 7)) * kPRow + 32 * kbp + (lane >> 3) * 8), b);
#pragma unroll
        for (int pl = 0; pl < 2; pl++) {
          mma16816(s[nb], qa[pl][2 * kbp], b[0], b[1]);
          mma16816(s[nb], qa[pl][2 * kbp + 1], b[2], b[3]);
        }
      }
    }
    // Online softmax, base 2: lane holds rows (gq, gq + 8) at positions
    // 8nb + 2tq + {0, 1}; a row's four lanes are a quad.
    float mx[2] = {m[0], m[1]};
#pragma unroll
    for (int nb = 0; nb < 8; nb++)
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int i = j >> 1, p = kt * kPKT + 8 * nb + 2 * tq + (j & 1);
        const float v = (rok[i] && p <= rqp[i]) ? s[nb][j] * scale2 : -INFINITY;
        s[nb][j] = v;
        mx[i] = fmaxf(mx[i], v);
      }
#pragma unroll
    for (int i = 0; i < 2; i++) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 2; i++) corr[i] = mx[i] == -INFINITY ? 1.f : exp2f(m[i] - mx[i]);
#pragma unroll
    for (int nb = 0; nb < 8; nb++)
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int i = j >> 1;
        const float p = s[nb][j] == -INFINITY ? 0.f : exp2f(s[nb][j] - mx[i]);
        s[nb][j] = p;
        rs[i] += p;
      }
#pragma unroll
    for (int i = 0; i < 2; i++) {
      l[i] = l[i] * corr[i] + rs[i];  // this lane's share; the quad sums at the end
      m[i] = mx[i];
    }
#pragma unroll
    for (int n = 0; n < 16; n++) {
      o[n][0] *= corr[0];
      o[n][1] *= corr[0];
      o[n][2] *= corr[1];
      o[n][3] *= corr[1];
    }
    // O += P V: k-block kb = positions 16kb .. 16kb+15 (score n-blocks 2kb, 2kb+1).
#pragma unroll
    for (int kb = 0; kb < 4; kb++) {
      uint32_t pa[2][4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int nb = 2 * kb + (j >> 1), c = (j & 1) * 2;
        const float x0 = s[nb][c], x1 = s[nb][c + 1];
        pa[0][j] = pack2(x0, x1);
        pa[1][j] = pack2(x0 - bf_round(x0), x1 - bf_round(x1));
      }
#pragma unroll
      for (int nbp = 0; nbp < 8; nbp++) {
        uint32_t b[4];
        const int mi = lane >> 3;  // matrix: (positions +0 / +8, dims +0 / +8)
        ldsm_x4_t(smem_u32(vs + (16 * kb + (mi & 1) * 8 + (lane & 7)) * kPRow + 16 * nbp + (mi >> 1) * 8), b);
#pragma unroll
        for (int pl = 0; pl < 2; pl++) {
          mma16816(o[2 * nbp], pa[pl], b[0], b[1]);
          mma16816(o[2 * nbp + 1], pa[pl], b[2], b[3]);
        }
      }
    }
    __syncthreads();  // the stage is reloaded two tiles later
  }
  // Normalise and store the three planes of each output value.
  float inv[2];
#pragma unroll
  for (int i = 0; i < 2; i++) {
    float L = l[i];
    L += __shfl_xor_sync(0xffffffffu, L, 1);
    L += __shfl_xor_sync(0xffffffffu, L, 2);
    inv[i] = L > 0.f ? 1.0f / L : 0.f;
  }
#pragma unroll
  for (int i = 0; i < 2; i++) {
    if (!rok[i]) continue;
    const int r = 16 * warp + gq + 8 * i;
    const size_t row = size_t(tok0 + rtok[i]) * a.ldo + size_t(g * GRP + r % GRP) * kD;
#pragma unroll
    for (int n = 0; n < 16; n++)
#pragma unroll
      for (int j = 0; j < 2; j++) store_split3(a.out, a.plane, row + 8 * n + 2 * tq + j, o[n][2 * i + j] * inv[i]);
  }
}

template <int G>
cudaError_t prefill_tc_attr() {
  return cudaFuncSetAttribute(k_attn_prefill_tc<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(kPrefillTcSmem));
}

template <int G>
cudaError_t tc_attr() {
  return cudaFuncSetAttribute(k_attn_rows_tc<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kTcSmem));
}

template <int G, bool F>
cudaError_t rows_attr() {
  cudaError_t e = cudaFuncSetAttribute(k_attn_rows<G, F>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(RowsCfg<F>::kSmem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_attn_prefill<G, F>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(sizeof(PrefillSmem)));
  return e;
}

}  // namespace

cudaError_t init_batch_kernels() {
  cudaError_t e = cudaSuccess;
#define TB_ATTR(G)                               \
  if (e == cudaSuccess) e = rows_attr<G, true>(); \
  if (e == cudaSuccess) e = rows_attr<G, false>();
  TB_ATTR(1)
  TB_ATTR(2)
  TB_ATTR(4)
  TB_ATTR(8)
#undef TB_ATTR
  if (e == cudaSuccess) e = tc_attr<1>();
  if (e == cudaSuccess) e = tc_attr<2>();
  if (e == cudaSuccess) e = tc_attr<4>();
  if (e == cudaSuccess) e = tc_attr<8>();
  if (e == cudaSuccess) e = prefill_tc_attr<1>();
  if (e == cudaSuccess) e = prefill_tc_attr<2>();
  if (e == cudaSuccess) e = prefill_tc_attr<4>();
  if (e == cudaSuccess) e = prefill_tc_attr<8>();
  return e;
}

bool batch_group_supported(int group) { return group == 1 || group == 2 || group == 4 || group == 8; }

int attn_rows_chunk(bool kv_f32) { return kv_f32 ? RowsCfg<true>::kCh : RowsCfg<false>::kCh; }

int attn_cache_box_rows() { return kTcCh; }

int attn_rows_parts(int tokens, int n_kv_heads, int max_len, bool kv_f32, int sms) {
  // Enough CTAs for two per SM; never a part shorter than one chunk (the
  // tensor-core kernel's chunk is at least as long as the other's). Four per
  // SM measured slower at batch 1 (the last CTA merges twice the partials).
  const int units = std::max(1, tokens * n_kv_heads);
  const int want = (2 * sms + units - 1) / units;
  const int chunk = std::max(attn_rows_chunk(kv_f32), kTcCh);
  const int chunks = (max_len + chunk - 1) / chunk;
  return std::max(1, std::min(want, chunks));
}

void launch_split_rows(cudaStream_t s, const float* x, uint16_t* out, size_t plane, size_t n, bool pdl) {
  const unsigned grid = unsigned(std::min<size_t>((n + 255) / 256, 4096));
  if (n) launch_pdl(s, dim3(grid), dim3(256), 0, pdl, k_split_rows, x, out, plane, n);
}

void launch_norm_split(cudaStream_t s, float* x, const float* add, int row0, int rows, int dim, const uint16_t* w,
                       float eps, uint16_t* out, size_t plane, bool pdl, const TraceAt& tr) {
  if (rows > 0)
    launch_pdl(s, dim3(rows), dim3(256), 0, pdl, k_norm_split, x, add, row0, dim, w, eps, out, plane, tr);
}

void launch_embed_split(cudaStream_t s, float* x, const uint16_t* table, int dim, const int* tok, int vocab,
                        const uint16_t* w, uint16_t* out, size_t plane, float* ssq, int* err, int tokens, bool pdl,
                        const TraceAt& tr) {
  if (tokens > 0)
    launch_pdl(s, dim3(tokens), dim3(256), 0, pdl, k_embed_split, x, table, dim, tok, vocab, w, out, plane, ssq, err,
               tr);
}


bool attn_rows_tensor_cores(bool kv_f32, int group) {
  return !kv_f32 && (group == 1 || group == 2 || group == 4 || group == 8);
}

void launch_attn_rows(cudaStream_t s, const AttnRowsArgs& a, int tokens, int group, bool pdl) {
  if (tokens <= 0) return;
  const dim3 grid(unsigned(a.parts), unsigned(a.n_kv_heads), unsigned(tokens));
  if (attn_rows_tensor_cores(a.kv_f32 != 0, group) && a.cache_map) {
    if (group == 1) launch_pdl(s, grid, dim3(128), kTcSmem, pdl, k_attn_rows_tc<1>, *a.cache_map, a);
    if (group == 2) launch_pdl(s, grid, dim3(128), kTcSmem, pdl, k_attn_rows_tc<2>, *a.cache_map, a);
    if (group == 4) launch_pdl(s, grid, dim3(128), kTcSmem, pdl, k_attn_rows_tc<4>, *a.cache_map, a);
    if (group == 8) launch_pdl(s, grid, dim3(128), kTcSmem, pdl, k_attn_rows_tc<8>, *a.cache_map, a);
    return;
  }
#define TB_ROWS(G)                                                                                   \
  if (group == G) {                                                                                  \
    if (a.kv_f32) launch_pdl(s, grid, dim3(128), RowsCfg<true>::kSmem, pdl, k_attn_rows<G, true>, a); \
    else launch_pdl(s, grid, dim3(128), RowsCfg<false>::kSmem, pdl, k_attn_rows<G, false>, a);       \
    return;                                                                                          \
  }
  TB_ROWS(1)
  TB_ROWS(2)
  TB_ROWS(4)
  TB_ROWS(8)
#undef TB_ROWS
}

void launch_attn_prefill(cudaStream_t s, const AttnPrefillArgs& a, int group, bool pdl) {
  if (a.T <= 0) return;
  if (!a.kv_f32) {  // bf16 cache: the tensor cores
    const int qt = kPQR / group;
    const dim3 grid(unsigned((a.T + qt - 1) / qt), unsigned(a.n_kv_heads));
    if (group == 1) launch_pdl(s, grid, dim3(128), kPrefillTcSmem, pdl, k_attn_prefill_tc<1>, a);
    if (group == 2) launch_pdl(s, grid, dim3(128), kPrefillTcSmem, pdl, k_attn_prefill_tc<2>, a);
    if (group == 4) launch_pdl(s, grid, dim3(128), kPrefillTcSmem, pdl, k_attn_prefill_tc<4>, a);
    if (group == 8) launch_pdl(s, grid, dim3(128), kPrefillTcSmem, pdl, k_attn_prefill_tc<8>, a);
    return;
  }
  const int qt = kPR / group;
  const dim3 grid(unsigned((a.T + qt - 1) / qt), unsigned(a.n_kv_heads));
#define TB_PRE(G)                                                                                          \
  if (group == G) {                                                                                        \
    if (a.kv_f32) launch_pdl(s, grid, dim3(256), sizeof(PrefillSmem), pdl, k_attn_prefill<G, true>, a);   \
    else launch_pdl(s, grid, dim3(256), sizeof(PrefillSmem), pdl, k_attn_prefill<G, false>, a);           \
    return;                                                                                                \
  }
  TB_PRE(1)
  TB_PRE(2)
  TB_PRE(4)
  TB_PRE(8)
#undef TB_PRE
}

void launch_argmax_finish(cudaStream_t s, const ArgmaxRowsArgs& a, unsigned long long* best, int rows, bool pdl) {
  if (rows > 0) launch_pdl(s, dim3(1), dim3(256), 0, pdl, k_argmax_finish, a, best, rows);
}


}  // namespace tb
