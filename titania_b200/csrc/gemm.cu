// gemm.cu — the tensor-core contraction for many tokens at once:
//
//     out[t][r] = Σ_c W[r][c] · x[t][c]          (model/cpu.rs:49-77, n > 1)
//
// W is the bf16 weight [M][K] exactly as uploaded; x is f32. The fifth
// generation tensor cores multiply bf16 by bf16 (kind::f16, f32 accumulate),
// so each activation is carried as three bf16 planes, x = x0 + x1 + x2 with
// x0 = bf16(x), x1 = bf16(x - x0), x2 = bf16(x - x0 - x1): 3 x 8 significant
// bits hold every f32 of magnitude 2^-100 .. 2^127 exactly, and every
// bf16 x bf16 product is exact in f32, so W·x0 + W·x1 + W·x2 differs from the
// reference's dot product only in the order and rounding of the f32
// additions. A tile of 64 tokens stacks its three planes as the 192 columns
// of one MMA (M=128, N=192, K=16), so each weight tile is read from shared
// memory once per K step; the epilogue adds the three column groups.
//
// Roles (192 threads):
//   warp 0      TMA producer: a 128x64 weight box and three 64x64 activation
//               boxes (128-byte swizzle) per stage, into a ring of stages;
//   warp 1      allocates 512 tensor-memory columns (two accumulators of
//               192), and one lane issues tcgen05.mma, committing each stage
//               back to the producer and each finished tile to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld of their 32-lane quadrant, then store
//               (optionally folding each token's argmax key), residual add,
//               or SiLU(gate)·up of interleaved row pairs split again into
//               three bf16 planes for the next contraction.
// Two schedules:
//   persistent  (enough tiles for every SM) one CTA per SM walks tiles
//               blockIdx.x, + gridDim.x, ...; the producer runs ahead across
//               tiles and the two accumulators let the epilogue of one tile
//               overlap the MMAs of the next;
//   split-K     (few tiles: short, wide matrices at decode batch sizes) the
//               K ranges of a tile are the CTAs of one thread-block cluster,
//               which sum their partial tiles over distributed shared memory
//               in split order, so results do not depend on scheduling.
// Every CTA takes more than half an SM's shared memory, so no two share an
// SM and the 512-column allocation never waits.
//
// Every mbarrier wait is bounded (kWaitCycles); on expiry the kernel records
// TB200_ERR_TIMEOUT, lets what it issued drain (bounded), frees its tensor
// memory on every path, and returns.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <initializer_list>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace tb {

namespace {

constexpr int kBM = 128;                 // weight rows per tile (MMA M)
constexpr int kBK = 64;                  // K per stage: one 128-byte swizzle row of bf16
constexpr int kBN = 64;                  // tokens per tile
constexpr int kNP = 3 * kBN;             // MMA N: the tile's three activation planes
constexpr int kGemmThreads = 192;
constexpr int kStageA = kBM * kBK * 2;   // 16 KB
constexpr int kStageB = kNP * kBK * 2;   // 24 KB (three 8 KB plane boxes)
constexpr int kStage = kStageA + kStageB;
constexpr int kMaxStages = 5;
constexpr int kMaxSplitStages = 4;               // split-K: room for the receive buffer
constexpr size_t kRecvBytes = size_t(kBN) * kBM * 4;  // split-K: S slices of 64 / S tokens x 128 rows
// Two splits send 16-byte pieces (4 tokens of a row) into rows padded to
// kRecvLd2 floats ([source][row][token]: conflict-free on both sides); more
// splits send 4-byte values into [source][token][row].
constexpr int kRecvLd2 = kBN / 2 + 4;
__host__ __device__ constexpr size_t recv_bytes_for(int splits) {
  return splits == 2 ? size_t(2) * kBM * kRecvLd2 * 4 : (splits > 1 ? kRecvBytes : 0);
}
constexpr int kAccCols = 256;            // tensor-memory columns per accumulator
constexpr int kTmemCols = 2 * kAccCols;
// Floor of the dynamic shared memory: more than half of an SM's 228 KB.
constexpr size_t kMinSmem = 116 * 1024;

// The epilogue warps' scratch for a group of up to 32 tokens: per-warp
// partial sums, per-token scales, and one head's values per token.
struct EpiScratch {
  float scale[32];
  int pos[32], seq[32];
  float tile[32 * 132];  // [token][row], row stride 128 + 128 / tokens (tile_token_sum)
};

// Shared memory: `stages` tiles, (split-K) the receive buffer, then 8-byte
// slots: full[stages], empty[stages], tfull[2], tempty[2], mdone, the
// tensor-memory address and flags, the receive barrier (6 slots), then the
// epilogue warps' argmax keys [4][kBN] and their EpiScratch; plus alignment
// slack.
size_t smem_for(int stages, int splits) {
  const size_t need = size_t(stages) * kStage + recv_bytes_for(splits) + (2 * size_t(stages) + 11) * 8 +
                      4 * kBN * 8 + sizeof(EpiScratch) + 1024;
  return need > kMinSmem ? need : kMinSmem;
}

// ---- tcgen05 / TMA wrappers -------------------------------------------------

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Whole warp: allocates `cols` tensor-memory columns, address written to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t addr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(addr), "r"(cols) : "memory");
}

// Shared-memory matrix descriptor: K-major operand whose rows are 128 bytes,
// 128-byte swizzle, 8-row groups 1024 bytes apart (the layout a TMA box of
// 64 bf16 columns with CU_TENSOR_MAP_SWIZZLE_128B writes). Bits: start
// address >> 4 [0,14), leading byte offset >> 4 [16,30) (unused for this
// layout, 1), stride byte offset >> 4 [32,46), descriptor version 1 [46,48),
// base offset 0 [49,52) (tiles are 1024-byte aligned), layout 2 = 128-byte
// swizzle [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptor, kind::f16: f32 accumulator [4,6) = 1, A and B bf16
// ([7,10) = 1, [10,13) = 1), both K-major (bits 15, 16 zero), N >> 3 at
// [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
// Arrives on `bar` once every tcgen05.mma this thread issued has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns of tensor memory per warp.
__device__ __forceinline__ void tmem_ld16(uint32_t addr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}


// silu(g) * u = g / (1 + exp(-g)) * u (cpu.rs:151-155), with the fast
// exponential and division (a few ulp from libm's; within every parity bar).
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

// Per-token sums over a tile's 128 rows. Epilogue thread e (row e) left its
// value for token j at tile[j * (128 + G) + e]; then G = 128 / N threads share
// a token, each adding every G-th row, and a G-lane shuffle tree (G-lane groups
// sit inside one warp) finishes the sum, returned on every lane of the group.
// The padded row stride puts the G-thread groups of different tokens on
// distinct banks. One barrier and no per-token warp-wide dependency chain.
template <int N>
__device__ __forceinline__ float tile_token_sum(const float* tile, int e) {
  constexpr int G = 128 / N, ST = 128 + G;
  const int j = e / G, p = e % G;
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < N; k++) s += tile[j * ST + p + k * G];
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// What an epilogue group reads besides its accumulators. The split-K kernel
// loads it while the contraction runs; the persistent one just before use.
template <int N>
struct EpiPre {
  float x[N];    // kGemmResid, kGemmResidNorm: the residual rows of the N tokens
  float w;       // kGemmQkv: the QK-norm weight of this thread's row
  uint2 w4;      // kGemmResidNorm: the next norm's weight, the 4 rows this lane stores
  float2 cs[N];  // kGemmQkv: RoPE cos / sin of each token's position
};

// Loads the EpiPre of N tokens t0 .. of row `row` of tile `mt`, and leaves
// in `es` the input scale per token (in_ssq) and, for kGemmQkv, the tokens'
// positions and sequences. Only results of earlier kernels are read (after
// the dependency wait). es is read only after a later named barrier.
template <int EPI, int N>
__device__ __forceinline__ void epi_prefetch(const GemmArgs& a, int mt, int row, bool row_ok, int q, int lane,
                                             int t0, EpiPre<N>& pre, EpiScratch& es) {
  const int e = int(threadIdx.x) - 64;
  if (a.in_ssq && e < N && t0 + e < a.T) {
    // The input's RMSNorm (cpu.rs:85-94): the scale of each token, from the
    // partial sums of squares the producer of the input left, in order.
    const float* p = a.in_ssq + size_t(a.act_row0 + t0 + e) * a.in_parts;
    float ss = 0.f;
#pragma unroll 4
    for (int i = 0; i < a.in_parts; i++) ss += p[i];
    es.scale[e] = 1.0f / sqrtf(ss / float(a.in_dim) + a.eps);
  }
  if (EPI == kGemmResid || EPI == kGemmResidNorm) {
#pragma unroll
    for (int j = 0; j < N; j++) pre.x[j] = row_ok && t0 + j < a.T ? a.out[size_t(t0 + j) * a.ldo + row] : 0.f;
    if (EPI == kGemmResidNorm) {
      const int r4 = mt * kBM + 4 * lane;  // the rows this lane stores (epi_group's output pass)
      if (r4 + 3 < a.M) {
        pre.w4 = *reinterpret_cast<const uint2*>(a.next_w + r4);
      } else {
        uint16_t h[4];
        for (int i = 0; i < 4; i++) h[i] = r4 + i < a.M ? a.next_w[r4 + i] : uint16_t(0);
        pre.w4 = make_uint2(uint32_t(h[0]) | (uint32_t(h[1]) << 16), uint32_t(h[2]) | (uint32_t(h[3]) << 16));
      }
    }
  }
  if (EPI == kGemmQkv) {
    const int nq = a.n_heads, nk = a.n_kv_heads;
    const int d = 32 * q + lane;
    if (e < N) {
      const bool t_ok = t0 + e < a.T;
      es.pos[e] = t_ok ? a.tok_pos[a.act_row0 + t0 + e] : -1;
      es.seq[e] = t_ok ? a.tok_seq[a.act_row0 + t0 + e] : -1;
    }
    const uint16_t* nw = mt < nq ? a.q_norm : mt < nq + nk ? a.k_norm : nullptr;
    pre.w = nw ? bf16f(nw[d]) : 1.f;
    if (mt < nq + nk) {
      const int i = d & 63;
#pragma unroll
      for (int j = 0; j < N; j++) {
        const int pos = t0 + j < a.T ? a.tok_pos[a.act_row0 + t0 + j] : -1;
        pre.cs[j] = (pos >= 0 && pos < a.max_len) ? *reinterpret_cast<const float2*>(a.rope + size_t(pos) * 128 + 2 * i)
                                                  : make_float2(1.f, 0.f);
      }
    }
  }
}

// The epilogues' output pass: after the values go through shared memory
// (tile[token][row], row stride kEpiLd), each warp writes whole token rows,
// 4 consecutive rows per lane, as 16-byte (f32) or 8-byte (bf16) stores —
// a quarter of the store instructions of one value per lane (the epilogue
// time was measured per store instruction). Rows at or past `rows` are not
// written; `vec` is false when the destination rows are not 16-byte aligned.
constexpr int kEpiLd = 132;
__device__ __forceinline__ void store_f32x4(float* dst, int r0, int rows, float4 v, bool vec) {
  if (vec && r0 + 3 < rows) {
    *reinterpret_cast<float4*>(dst + r0) = v;
  } else {
    const float w[4] = {v.x, v.y, v.z, v.w};
    for (int i = 0; i < 4; i++)
      if (r0 + i < rows) dst[r0 + i] = w[i];
  }
}
// Four values as three bf16 planes (store_split3's split), plane p at dst + p * plane.
__device__ __forceinline__ void store_split3x4(uint16_t* dst, size_t plane, int r0, int rows, float4 v, bool vec) {
  const float in[4] = {v.x, v.y, v.z, v.w};
  uint16_t p0[4], p1[4], p2[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    p0[i] = f2bf(in[i]);
    const float res = in[i] - bf16f(p0[i]);
    p1[i] = f2bf(res);
    p2[i] = f2bf(res - bf16f(p1[i]));
  }
  if (vec && r0 + 3 < rows) {
    *reinterpret_cast<uint2*>(dst + r0) = make_uint2(p0[0] | (uint32_t(p0[1]) << 16), p0[2] | (uint32_t(p0[3]) << 16));
    *reinterpret_cast<uint2*>(dst + plane + r0) =
        make_uint2(p1[0] | (uint32_t(p1[1]) << 16), p1[2] | (uint32_t(p1[3]) << 16));
    *reinterpret_cast<uint2*>(dst + 2 * plane + r0) =
        make_uint2(p2[0] | (uint32_t(p2[1]) << 16), p2[2] | (uint32_t(p2[3]) << 16));
  } else {
    for (int i = 0; i < 4; i++)
      if (r0 + i < rows) {
        dst[r0 + i] = p0[i];
        dst[plane + r0 + i] = p1[i];
        dst[2 * plane + r0 + i] = p2[i];
      }
  }
}
__device__ __forceinline__ bool aligned16(const void* p, size_t ld_elems, size_t elem_bytes) {
  return ((reinterpret_cast<uintptr_t>(p) | (ld_elems * elem_bytes)) & 15) == 0;
}

// The epilogue of N consecutive tokens t0 .. t0 + N - 1 (N <= 32) of row
// `row` = m0 + 32 q + lane of row tile `mt`: v[j] is the accumulator of
// token t0 + j, `pre` what epi_prefetch loaded for the same tokens. All 128
// epilogue threads call it together (named barrier 1). On return v holds the
// values the epilogue produced from (after the input scale; kGemmQkv: after
// QK-norm and RoPE).
template <int EPI, int N>
__device__ __forceinline__ void epi_group(const GemmArgs& a, int mt, int row, bool row_ok, int q, int lane, int t0,
                                          float (&v)[N], const EpiPre<N>& pre, EpiScratch& es) {
  static_assert(N <= 32, "scratch holds 32 tokens");
  const int e = int(threadIdx.x) - 64;  // 0 .. 127 over the epilogue warps
  if (a.in_ssq) {
    named_sync(1, 128);  // es.scale in place
#pragma unroll
    for (int j = 0; j < N; j++) v[j] *= es.scale[j];
    named_sync(1, 128);
  }
  const int r = 32 * q + lane;   // this thread's row of the tile
  const int m0 = mt * kBM;       // the tile's first row
  const int tw = e >> 5;         // output pass: this warp's token of each group of 4
  const int rr = 4 * lane;       // output pass: this lane's 4 rows
  static_assert(N % 4 == 0, "tokens in groups of 4");
  if (EPI == kGemmStore) {
#pragma unroll
    for (int j = 0; j < N; j++) es.tile[j * kEpiLd + r] = v[j];
    named_sync(1, 128);
    const bool vec = aligned16(a.out, size_t(a.ldo), 4);
#pragma unroll
    for (int k = 0; k < N / 4; k++) {
      const int j = 4 * k + tw, t = t0 + j;
      if (t < a.T)
        store_f32x4(a.out + size_t(t) * a.ldo, m0 + rr, a.M,
                    *reinterpret_cast<const float4*>(&es.tile[j * kEpiLd + rr]), vec);
    }
    named_sync(1, 128);  // the tile is read before the next group writes it
  } else if (EPI == kGemmResid || EPI == kGemmResidNorm) {
#pragma unroll
    for (int j = 0; j < N; j++) {
      v[j] = __fadd_rn(pre.x[j], v[j]);  // x += W . input (rows past M are 0 + 0)
      es.tile[j * kEpiLd + r] = v[j];
    }
    named_sync(1, 128);
    const bool vec = aligned16(a.out, size_t(a.ldo), 4);
    const bool vec_h = EPI == kGemmResidNorm && aligned16(a.next_split, size_t(a.ldo), 2) && (a.next_plane & 3) == 0;
#pragma unroll
    for (int k = 0; k < N / 4; k++) {
      const int j = 4 * k + tw, t = t0 + j;
      if (t >= a.T) continue;  // warp-uniform
      const float4 x4 = *reinterpret_cast<const float4*>(&es.tile[j * kEpiLd + rr]);
      store_f32x4(a.out + size_t(t) * a.ldo, m0 + rr, a.M, x4, vec);
      if (EPI == kGemmResidNorm) {
        // The next RMSNorm's input: x * w as planes, and this tile's sum of
        // squares of x per token (its consumer divides by the row length).
        const float ss = warp_sum(((x4.x * x4.x + x4.y * x4.y) + x4.z * x4.z) + x4.w * x4.w);
        if (lane == 0) a.out_ssq[size_t(t) * a.mtiles + mt] = ss;
        const float4 xw = make_float4(__fmul_rn(x4.x, bf_lo(pre.w4.x)), __fmul_rn(x4.y, bf_hi(pre.w4.x)),
                                      __fmul_rn(x4.z, bf_lo(pre.w4.y)), __fmul_rn(x4.w, bf_hi(pre.w4.y)));
        store_split3x4(a.next_split + size_t(t) * a.ldo, a.next_plane, m0 + rr, a.M, xw, vec_h);
      }
    }
    named_sync(1, 128);  // the tile is read before the next group writes it
  } else if (EPI == kGemmSilu) {
    // Lanes 2i (gate) and 2i+1 (up) of hidden row i share tokens: the even
    // lane finishes token j, the odd lane token j + 1.
    static_assert(N % 2 == 0, "token pairs");
    const bool even = (row & 1) == 0;
#pragma unroll
    for (int j = 0; j < N; j += 2) {
      const float other = __shfl_xor_sync(0xffffffffu, even ? v[j + 1] : v[j], 1);
      const float g = even ? v[j] : other, u = even ? other : v[j + 1];
      es.tile[(j + (even ? 0 : 1)) * kEpiLd + (r >> 1)] = silu_mul(g, u);
    }
    named_sync(1, 128);
    // 64 hidden rows per token: 16 lanes x 4 rows, 8 tokens per pass.
    const int hq = 4 * (e & 15), hrows = a.M / 2;
    const bool vec = aligned16(a.out_split, size_t(a.ldh), 2) && (a.plane & 3) == 0;
#pragma unroll
    for (int k = 0; k < (N + 7) / 8; k++) {
      const int j = 8 * k + (e >> 4), t = t0 + j;
      if (j < N && t < a.T)
        store_split3x4(a.out_split + size_t(t) * a.ldh, a.plane, m0 / 2 + hq, hrows,
                       *reinterpret_cast<const float4*>(&es.tile[j * kEpiLd + hq]), vec);
    }
    named_sync(1, 128);  // the tile is read before the next group writes it
  } else {  // kGemmQkv: tile mt is query head mt, key head mt - nq, or value head mt - nq - nk
    const int nq = a.n_heads, nk = a.n_kv_heads;
    const int d = r;  // the head dimension of this row (e is not: warp 2 reads lanes 64..95)
    const bool is_v = mt >= nq + nk;
    if (!is_v) {
      const uint16_t* nw = mt < nq ? a.q_norm : a.k_norm;
      if (nw) {
        // QK-norm over the head (model.rs:111-116 with cpu.rs:85-94).
        constexpr int G = 128 / N, ST = 128 + G;
#pragma unroll
        for (int j = 0; j < N; j++) es.tile[j * ST + d] = v[j] * v[j];
        named_sync(1, 128);
        const float ss = tile_token_sum<N>(es.tile, e);
        if (e % G == 0) es.scale[e / G] = 1.0f / sqrtf(ss / 128.0f + a.eps);
        named_sync(1, 128);
        const float w = pre.w;
#pragma unroll
        for (int j = 0; j < N; j++) v[j] = __fmul_rn(v[j], __fmul_rn(es.scale[j], w));
      }
      // RoPE (cpu.rs:96-111): element d pairs with d ^ 64.
#pragma unroll
      for (int j = 0; j < N; j++) es.tile[j * 128 + d] = v[j];
      named_sync(1, 128);
#pragma unroll
      for (int j = 0; j < N; j++) {
        if (t0 + j >= a.T) continue;
        const float other = es.tile[j * 128 + (d ^ 64)];
        const float2 cs = pre.cs[j];
        v[j] = d < 64 ? __fsub_rn(__fmul_rn(v[j], cs.x), __fmul_rn(other, cs.y))
                      : __fadd_rn(__fmul_rn(v[j], cs.x), __fmul_rn(other, cs.y));
      }
    }
    named_sync(1, 128);  // RoPE's reads are done; es.pos / es.seq in place
#pragma unroll
    for (int j = 0; j < N; j++) es.tile[j * kEpiLd + d] = v[j];
    named_sync(1, 128);
    const bool vec = aligned16(a.out, size_t(a.ldo), 4);
#pragma unroll
    for (int k = 0; k < N / 4; k++) {
      const int j = 4 * k + tw, t = t0 + j;
      if (t >= a.T) continue;  // warp-uniform
      const float4 v4 = *reinterpret_cast<const float4*>(&es.tile[j * kEpiLd + rr]);
      if (mt < nq) {
        store_f32x4(a.out + size_t(t) * a.ldo, m0 + rr, a.M, v4, vec);
        continue;
      }
      const int pos = es.pos[j], sq = es.seq[j];
      if (pos < 0 || pos >= a.max_len || sq < 0 || sq >= a.n_seqs) {
        if (lane == 0) set_error(a.err, TB200_ERR_ARG);
        continue;
      }
      const int kh = is_v ? mt - nq - nk : mt - nq;
      const size_t at = size_t(sq) * a.seq_stride + (is_v ? size_t(nk) * a.max_len * 128 : 0) +
                        (size_t(kh) * a.max_len + pos) * 128 + rr;  // 128 contiguous dims per (token, head)
      if (a.kv_f32) {
        *reinterpret_cast<float4*>(static_cast<float*>(a.kv) + at) = v4;
      } else {
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(a.kv) + at) =
            make_uint2(uint32_t(f2bf(v4.x)) | (uint32_t(f2bf(v4.y)) << 16),
                       uint32_t(f2bf(v4.z)) | (uint32_t(f2bf(v4.w)) << 16));
      }
    }
    named_sync(1, 128);  // es.tile / es.pos / es.seq read before the next group writes them
  }
}

// Folds each token's argmax key over this warp's 32 rows into best[] (one
// atomic per token and warp); all lanes call it.
template <int N>
__device__ __forceinline__ void argmax_tokens(const GemmArgs& a, int row, bool row_ok, int t0, const float (&v)[N],
                                              int lane) {
#pragma unroll
  for (int j = 0; j < N; j++) {
    const unsigned long long key = warp_umax64(row_ok ? argmax_key(v[j], uint32_t(row)) : 0ull);
    if (lane == 0 && t0 + j < a.T) atomicMax(a.best + t0 + j, key);
  }
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The two halves of a cluster barrier, for work placed between them.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// An asynchronous 4-byte store into the shared memory of another CTA of the
// cluster, counted (complete_tx) on that CTA's barrier at `rbar`.
__device__ __forceinline__ void st_async_f32(uint32_t remote, float x, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(remote),
               "r"(__float_as_uint(x)), "r"(rbar)
               : "memory");
}
// The same for 16 bytes (the remote address 16-byte aligned).
__device__ __forceinline__ void st_async_f32x4(uint32_t remote, float4 x, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(remote),
               "r"(__float_as_uint(x.x)), "r"(__float_as_uint(x.y)), "r"(__float_as_uint(x.z)),
               "r"(__float_as_uint(x.w)), "r"(rbar)
               : "memory");
}
// mbar_wait with acquire at cluster scope: what other CTAs' st.async
// delivered before the phase completed is visible afterwards.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      set_error(err, TB200_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}
// The shared::cluster address of offset `saddr` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_cluster(uint32_t saddr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(saddr), "r"(rank));
  return remote;
}

// Sums the three plane column groups of accumulator columns [c, c + 16)
// for this warp's 32 lanes: v[j] = token (c + j) of the tile.
__device__ __forceinline__ void tmem_ld_tokens(uint32_t taddr, int c, float (&v)[16]) {
  float p1[16], p2[16];
  tmem_ld16(taddr + c, v);
  tmem_ld16(taddr + kBN + c, p1);
  tmem_ld16(taddr + 2 * kBN + c, p2);
#pragma unroll
  for (int j = 0; j < 16; j++) v[j] = (v[j] + p1[j]) + p2[j];
}

template <int EPI, int S>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx0,
           const __grid_constant__ CUtensorMap tx1, const __grid_constant__ CUtensorMap tx2, GemmArgs a) {
  extern __shared__ unsigned char smem_raw[];
  // The swizzled tiles need 1024-byte alignment.
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  constexpr bool split = S > 1;  // a.splits == S
  const int stages = a.stages;  // 1 .. kMaxStages (split-K: .. kMaxSplitStages)
  // Split-K: the receive buffer of the other CTAs' partial sums follows the stages.
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + size_t(stages) * kStage + recv_bytes_for(S));
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;  // [2] accumulator ready
  uint64_t* tempty = tfull + 2;      // [2] accumulator drained
  uint64_t* mdone = tempty + 2;      // every MMA of the CTA completed
  uint64_t* rbar = mdone + 5;        // split-K: the other CTAs' partial sums have landed
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mdone + 1);
  int* flags = reinterpret_cast<int*>(tslot + 1);  // [0..3] per epilogue warp
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(mdone + 6);  // [4][kBN]
  EpiScratch& es = *reinterpret_cast<EpiScratch*>(keys + 4 * kBN);
  auto sA = [&](int s) { return sm + size_t(s) * kStage; };
  auto sB = [&](int s) { return sm + size_t(s) * kStage + kStageA; };

  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  if (threadIdx.x == 0) a.trace.at(cta, TB200_TRACE_START);
  constexpr int PER = split ? kBN / S : 16;  // split-K: the tokens of the tile this CTA finishes
  EpiPre<PER> pre;                           // split-K: that slice's epilogue inputs
  const int nkb = (a.K + kBK - 1) / kBK;
  // Tile sequence of this CTA: split-K, one tile (blockIdx) and one K range;
  // persistent, tiles blockIdx.x, blockIdx.x + gridDim.x, ... over all of K.
  const int ntiles = split ? 1 : (a.mtiles * a.ntiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x);
  const int kb0 = split ? int(blockIdx.z) * a.kb_per_split : 0;
  const int nk = split ? max(0, min(nkb, kb0 + a.kb_per_split) - kb0) : nkb;
  auto tile_m = [&](int ti) { return split ? int(blockIdx.x) : (int(blockIdx.x) + ti * int(gridDim.x)) % a.mtiles; };
  auto tile_n = [&](int ti) { return split ? int(blockIdx.y) : (int(blockIdx.x) + ti * int(gridDim.x)) / a.mtiles; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(mdone, 1);
    if (split) {
      mbar_init(rbar, 1);
      mbar_arrive_expect_tx(rbar, uint32_t((S - 1) * PER * kBM * 4));
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tslot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  // Split-K: the receive barriers are initialized before any CTA of the
  // cluster sends to them (every thread waits on this arrival later).
  if constexpr (split) cluster_arrive_relaxed();

  if (warp == 0) {
    if (lane == 0) {
      // Producer. Weights do not depend on earlier kernels: the first
      // tile's first stages of weights go out before the dependency wait.
      const uint64_t pol_w = l2_evict_first(), pol_x = l2_evict_last();
      auto load_b = [&](int s, int kb, int n0) {
        const int y = a.act_row0 + n0;
        tma_load_2d(sB(s), &tx0, kb * kBK, y, &full[s], pol_x);
        tma_load_2d(sB(s) + kBN * 128, &tx1, kb * kBK, y, &full[s], pol_x);
        tma_load_2d(sB(s) + 2 * kBN * 128, &tx2, kb * kBK, y, &full[s], pol_x);
      };
      const int pre = ntiles > 0 ? min(nk, stages) : 0;
      for (int i = 0; i < pre; i++) {
        mbar_arrive_expect_tx(&full[i], kStage);
        tma_load_2d(sA(i), &tw, (kb0 + i) * kBK, tile_m(0) * kBM, &full[i], pol_w);
      }
      pdl_wait();
      for (int i = 0; i < pre; i++) load_b(i, kb0 + i, tile_n(0) * kBN);
      int i = 0, issued = pre;  // i: this CTA's k-block counter over all its tiles
      bool ok = true;
      for (int ti = 0; ti < ntiles && ok; ti++) {
        const int m0 = tile_m(ti) * kBM, n0 = tile_n(ti) * kBN;
        for (int k = 0; k < nk; k++, i++) {
          if (i < pre) continue;
          const int s = i % stages;
          if (!mbar_wait(&empty[s], ((i / stages) & 1) ^ 1, a.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kStage);
          tma_load_2d(sA(s), &tw, (kb0 + k) * kBK, m0, &full[s], pol_w);
          load_b(s, kb0 + k, n0);
          issued = i + 1;
        }
      }
      a.trace.at(cta, TB200_TRACE_ISSUED);
      // Drain: every issued copy has landed before the CTA can exit (on the
      // normal path the MMA warp already waited for each of them).
      for (int j = issued - 1; j >= 0 && j >= issued - stages; j--)
        mbar_wait(&full[j % stages], (j / stages) & 1, nullptr);
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(kBM, kNP);
      int i = 0;
      bool ok = true;
      for (int ti = 0; ti < ntiles && ok; ti++) {
        const int b = ti & 1;
        // The epilogue has drained this accumulator's previous tile.
        if (!mbar_wait(&tempty[b], ((ti >> 1) - 1) & 1, a.err)) break;
        tc_fence_after();
        const uint32_t acc = tmem + uint32_t(b * kAccCols);
        for (int k = 0; k < nk; k++, i++) {
          const int s = i % stages;
          if (!mbar_wait(&full[s], (i / stages) & 1, a.err)) {
            ok = false;
            break;
          }
          if (i == 0) a.trace.at(cta, TB200_TRACE_WEIGHTS);
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA(s)), b0 = smem_u32(sB(s));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; kk++)  // K = 16 bf16 = 32 bytes per MMA in the 128-byte row
            mma_bf16(acc, sw128_desc(a0 + 32 * kk), sw128_desc(b0 + 32 * kk), idesc, (k > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        mma_commit(&tfull[b]);
      }
      a.trace.at(cta, TB200_TRACE_LAST_WEIGHTS);
      // Tensor memory is freed below only after every MMA has completed:
      // a last commit tracks all of them.
      mma_commit(mdone);
      mbar_wait(mdone, 0, nullptr);
    }
    __syncwarp();
  } else {
    // Epilogue: warp w reads tensor-memory lanes 32 (w % 4) .. + 31.
    pdl_wait();
    if (warp == 2 && lane == 0) a.trace.at(cta, TB200_TRACE_WAITED);
    const int q = warp & 3;
    // The four epilogue warps take the same branches: a verdict is shared.
    auto all_ok = [&](bool ok) {
      ok = __all_sync(0xffffffffu, ok);
      if (lane == 0) flags[q] = ok ? 1 : 0;
      named_sync(1, 128);
      ok = flags[0] && flags[1] && flags[2] && flags[3];
      named_sync(1, 128);  // flags[0..3] read before they are written again
      return ok;
    };
    if constexpr (split) {
      // Split-K over the cluster: cluster CTA R finishes tokens R PER .. +
      // PER - 1 of the tile. Every CTA pushes the other CTAs' token slices of
      // its partial sums into their receive buffers (st.async, counted on the
      // receiver's barrier) and keeps its own; then each CTA sums the S slices
      // of its tokens in split order from its own shared memory. No CTA reads
      // another's memory, and each waits for every byte sent to it before it
      // leaves.
      const int R = int(cluster_rank());
      const int rl = 32 * q + lane, row = int(blockIdx.x) * kBM + rl, n0 = int(blockIdx.y) * kBN;
      const bool row_ok = row < a.M;
      float* recv = reinterpret_cast<float*>(sm + size_t(stages) * kStage);  // [source][token][row]
      const uint32_t recv_s = smem_u32(recv), rbar_s = smem_u32(rbar);
      // The epilogue's other inputs, loaded while the contraction runs.
      epi_prefetch<EPI, PER>(a, int(blockIdx.x), row, row_ok, q, lane, n0 + R * PER, pre, es);
      cluster_wait();  // every receive barrier of the cluster is initialized
      auto push = [&](int jt, float x) {
        const int dst = jt / PER;
        const uint32_t off = uint32_t(((R * PER + jt % PER) * kBM + rl) * 4);
        if (dst == R) recv[off / 4] = x;
        else st_async_f32(mapa_cluster(recv_s + off, uint32_t(dst)), x, mapa_cluster(rbar_s, uint32_t(dst)));
      };
      auto push4 = [&](int jt, float4 x) {  // two splits: tokens jt .. jt + 3 of this row
        const int dst = jt / PER;
        const uint32_t off = uint32_t(((R * kBM + rl) * kRecvLd2 + jt % PER) * 4);
        if (dst == R) *reinterpret_cast<float4*>(&recv[off / 4]) = x;
        else st_async_f32x4(mapa_cluster(recv_s + off, uint32_t(dst)), x, mapa_cluster(rbar_s, uint32_t(dst)));
      };
      bool ok = true;
      if (nk > 0) {
        ok = all_ok(mbar_wait(&tfull[0], 0, a.err));
        if (ok) {
          if (warp == 2 && lane == 0) a.trace.at(cta, TB200_TRACE_INPUT);
          tc_fence_after();
          const uint32_t taddr = tmem + (uint32_t(32 * q) << 16);
#pragma unroll 1
          for (int c = 0; c < kBN; c += 16) {
            float v[16];
            tmem_ld_tokens(taddr, c, v);
            if constexpr (S == 2) {
#pragma unroll
              for (int j = 0; j < 16; j += 4) push4(c + j, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
            } else {
#pragma unroll
              for (int j = 0; j < 16; j++) push(c + j, v[j]);
            }
          }
        }
      } else {
        // A split past the end of K adds zeros.
        if constexpr (S == 2) {
#pragma unroll 1
          for (int jt = 0; jt < kBN; jt += 4) push4(jt, make_float4(0.f, 0.f, 0.f, 0.f));
        } else {
#pragma unroll 1
          for (int jt = 0; jt < kBN; jt++) push(jt, 0.f);
        }
      }
      // Every byte sent here lands before the CTA goes, whatever its verdict.
      const bool got = all_ok(mbar_wait_cluster(rbar, 0, a.err));
      if (ok && got) {
        if (threadIdx.x == 64) a.trace.at(cta, TB200_TRACE_REDUCE);
        float v[PER];
        if constexpr (S == 2) {
#pragma unroll
          for (int j = 0; j < PER; j += 4) {
            const float4 p0 = *reinterpret_cast<const float4*>(&recv[rl * kRecvLd2 + j]);
            const float4 p1 = *reinterpret_cast<const float4*>(&recv[(kBM + rl) * kRecvLd2 + j]);
            v[j] = p0.x + p1.x;
            v[j + 1] = p0.y + p1.y;
            v[j + 2] = p0.z + p1.z;
            v[j + 3] = p0.w + p1.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < PER; j++) {
            v[j] = recv[j * kBM + rl];
#pragma unroll
            for (int r = 1; r < S; r++) v[j] += recv[(r * PER + j) * kBM + rl];
          }
        }
        epi_group<EPI, PER>(a, int(blockIdx.x), row, row_ok, q, lane, n0 + R * PER, v, pre, es);
        if (EPI == kGemmStore && a.best) argmax_tokens<PER>(a, row, row_ok, n0 + R * PER, v, lane);
      }
    } else {
      for (int ti = 0; ti < ntiles; ti++) {
        const int b = ti & 1;
        const int m0 = tile_m(ti) * kBM, n0 = tile_n(ti) * kBN;
        const int row = m0 + 32 * q + lane;
        const bool row_ok = row < a.M;
        if (!all_ok(mbar_wait(&tfull[b], (ti >> 1) & 1, a.err))) break;
        if (ti == 0 && warp == 2 && lane == 0) a.trace.at(cta, TB200_TRACE_INPUT);
        tc_fence_after();
        const uint32_t taddr = tmem + uint32_t(b * kAccCols) + (uint32_t(32 * q) << 16);
#pragma unroll 1
        for (int c = 0; c < kBN; c += 16) {
          float v[16];
          EpiPre<16> pre16;
          epi_prefetch<EPI, 16>(a, tile_m(ti), row, row_ok, q, lane, n0 + c, pre16, es);
          tmem_ld_tokens(taddr, c, v);
          epi_group<EPI, 16>(a, tile_m(ti), row, row_ok, q, lane, n0 + c, v, pre16, es);
          if (EPI == kGemmStore && a.best) {
#pragma unroll
            for (int j = 0; j < 16; j++) {
              const unsigned long long key = warp_umax64(row_ok ? argmax_key(v[j], uint32_t(row)) : 0ull);
              if (lane == 0) keys[q * kBN + c + j] = key;
            }
          }
        }
        // The accumulator is drained: the MMA warp may refill it.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
        if (EPI == kGemmStore && a.best) {
          // One atomic per token and tile: the best of the four warps' rows.
          named_sync(1, 128);
          const int j = threadIdx.x - 64;
          if (j < kBN && n0 + j < a.T) {
            unsigned long long key = keys[j];
#pragma unroll
            for (int w = 1; w < 4; w++) key = keys[w * kBN + j] > key ? keys[w * kBN + j] : key;
            atomicMax(a.best + n0 + j, key);
          }
          named_sync(1, 128);  // keys read before the next tile writes them
        }
      }
    }
  }
  if constexpr (split) {
    if (warp < 2) {
      __syncwarp();
      cluster_wait();  // pairs with the arrival at the start
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) a.trace.at(cta, TB200_TRACE_DONE);
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, kTmemCols);
  }
}

// ---- host side -----------------------------------------------------------------

static_assert(kMaxSplitStages <= kMaxStages, "split plans fit the kernels' shared-memory attribute");
static_assert(size_t(kMaxSplitStages) * kStage + recv_bytes_for(2) <= size_t(kMaxStages) * kStage,
              "the two-split receive buffer fits the kernels' shared-memory attribute");

std::mutex g_encode_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

template <int EPI, int S>
cudaError_t set_attrs_one() {
  cudaError_t e = cudaFuncSetAttribute(k_gemm<EPI, S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(smem_for(kMaxStages, 1)));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_gemm<EPI, S>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e;
}
template <int EPI>
cudaError_t set_attrs() {
  cudaError_t e = set_attrs_one<EPI, 1>();
  if (e == cudaSuccess) e = set_attrs_one<EPI, 2>();
  if (e == cudaSuccess) e = set_attrs_one<EPI, 4>();
  if (e == cudaSuccess) e = set_attrs_one<EPI, 8>();
  if (e == cudaSuccess) e = set_attrs_one<EPI, 16>();
  return e;
}

template <int EPI, int S>
void launch_tile(cudaStream_t s, const GemmPlan& p, const CUtensorMap& tw, const CUtensorMap* tx, const GemmArgs& a,
                 bool pdl) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = p.grid;
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem_for(p.stages, p.splits);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (p.splits > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = unsigned(p.splits);
    n++;
  }
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaLaunchKernelEx(&cfg, k_gemm<EPI, S>, tw, tx[0], tx[1], tx[2], a);
}

}  // namespace

int encode_tmap_bf16(CUtensorMap* map, const void* base, size_t rows, size_t cols, int box_rows,
                     std::string* why) {
  {
    std::lock_guard<std::mutex> lock(g_encode_mu);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q{};
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
        *why = "cuTensorMapEncodeTiled is not available from the driver";
        return TB200_ERR_CUDA;
      }
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || (cols * 2) % 16 != 0 || rows == 0 || cols == 0 ||
      box_rows < 1 || box_rows > 256) {
    *why = "tensor map: base must be 16-byte aligned and rows 16-byte multiples";
    return TB200_ERR_ARG;
  }
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols * 2)};
  cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *why = "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")";
    return TB200_ERR_CUDA;
  }
  return TB200_OK;
}

int gemm_box_rows() { return kBN; }

GemmPlan plan_gemm(int M, int K, int T, int sms, int max_cluster) {
  GemmPlan p{};
  p.mtiles = (M + kBM - 1) / kBM;
  p.ntiles = (T + kBN - 1) / kBN;
  const int nkb = (K + kBK - 1) / kBK;
  const int tiles = p.mtiles * p.ntiles;
  int splits = 1;
  // Split K across the CTAs of a cluster (a power of two) when the tiles
  // alone leave SMs idle.
  if (tiles < sms) {
    const int want = std::max(1, std::min({nkb, sms / tiles, max_cluster}));
    while (splits * 2 <= want) splits *= 2;
  }
  p.kb_per_split = (nkb + splits - 1) / splits;
  p.splits = splits;  // a power of two; a split past the end of K contributes zeros
  if (p.splits > 1) {
    p.stages = std::min(kMaxSplitStages, p.kb_per_split);
    p.grid = dim3(unsigned(p.mtiles), unsigned(p.ntiles), unsigned(p.splits));
  } else {
    p.stages = kMaxStages;
    p.grid = dim3(unsigned(std::min(tiles, sms)), 1, 1);
  }
  return p;
}

cudaError_t init_gemm_kernels() {
  cudaError_t e = set_attrs<kGemmStore>();
  if (e == cudaSuccess) e = set_attrs<kGemmResid>();
  if (e == cudaSuccess) e = set_attrs<kGemmSilu>();
  if (e == cudaSuccess) e = set_attrs<kGemmResidNorm>();
  if (e == cudaSuccess) e = set_attrs<kGemmQkv>();
  return e;
}

int gemm_max_cluster() {
  for (unsigned n : {16u, 8u, 4u, 2u}) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(1, 1, n);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = smem_for(kMaxSplitStages, 2);  // the largest split layout
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = n;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, k_gemm<kGemmStore, 2>, &cfg) == cudaSuccess && clusters > 0)
      return int(n);
    cudaGetLastError();  // an unsupported size is not an error of ours
  }
  return 1;
}

void launch_gemm(cudaStream_t s, const GemmPlan& p, int epi, const CUtensorMap& tw, const CUtensorMap* tx,
                 const GemmArgs& a, bool pdl) {
  GemmArgs b = a;
  b.kb_per_split = p.kb_per_split;
  b.splits = p.splits;
  b.stages = p.stages;
  b.mtiles = p.mtiles;
  b.ntiles = p.ntiles;
#define TB_GEMM_S(EPI)                                                      \
  if (epi == EPI) {                                                         \
    if (p.splits == 1) launch_tile<EPI, 1>(s, p, tw, tx, b, pdl);           \
    if (p.splits == 2) launch_tile<EPI, 2>(s, p, tw, tx, b, pdl);           \
    if (p.splits == 4) launch_tile<EPI, 4>(s, p, tw, tx, b, pdl);           \
    if (p.splits == 8) launch_tile<EPI, 8>(s, p, tw, tx, b, pdl);           \
    if (p.splits == 16) launch_tile<EPI, 16>(s, p, tw, tx, b, pdl);         \
  }
  TB_GEMM_S(kGemmStore)
  TB_GEMM_S(kGemmResid)
  TB_GEMM_S(kGemmSilu)
  TB_GEMM_S(kGemmResidNorm)
  TB_GEMM_S(kGemmQkv)
#undef TB_GEMM_S
}

}  // namespace tb
