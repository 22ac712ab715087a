// Prefill / batched projection on the 5th-generation tensor cores:
// D[r][t] = sum_k W[r][k] * X[t][k] for a tile of 128 weight rows and up to
// 256 tokens, accumulated in tensor memory (TMEM) by tcgen05.mma.
//
// Replaces weightTensor.mulBatch (matmul.go:55-95) for Q8_0 and BF16 weights
// with the epilogues of the CUDA-core path (gemm_simt.cuh).
//
// BF16 weights are tensor-core operands as stored: TMA brings the weight tile
// with the activation tiles, and the float32 activations are split exactly
// into three bfloat16 pieces X' = X0 + X1 + X2 (8 + 8 + 8 significant bits),
// so W.X0 + W.X1 + W.X2 (exact products, float32 accumulation) is the
// float32 product. Tiles of up to 128 tokens keep the three pieces within
// one stage buffer.
//
// Q6_K / Q5_K weights: warps 0-15 build three binary16 pieces whose sum is
// the reference's float32 weight (quant_k.go:47-85) times 2^sw, exactly
// whenever its lowest bit lands at or above 2^-24 after scaling: every value
// within 2^14 of the matrix bound 2^13 (tcu_read_values with TCU_DECODE_TC
// checks this bit for bit). Q6_K: the group scale d * sc split into three
// six-bit pieces, each times the integer q - 32 (tc_q6k_pieces; exact
// binary16 products, no float32 decode). Q5_K: the value decoded in float32
// as the reference does, then W' = Wh + Wm + Wl, each piece the rounding of
// what the previous ones leave. Five products W1.Xh + W1.Xl + W2.Xh + W2.Xl +
// W3.Xh are accumulated; the dropped W3.Xl is ~2^-22 of the result.
//
// Q8_0 exactness: a Q8_0 weight
// s*q has at most 19 significant bits and an activation 24, more than one
// binary16 operand holds, so both sides are split into an exact binary16
// pair -- W' = W * 2^sw = Wh + Wl (Wh = fp16(s'q), Wl = fp16(fma(s', q, -Wh)))
// and X' = X * 2^sx(t) = Xh + Xl -- and three products Wh.Xh + Wh.Xl + Wl.Xh
// are accumulated in float32; the dropped terms are ~2^-22 of the result. The
// power-of-two scales keep the low halves out of the subnormal range and are
// removed exactly in the epilogue.
//
// Warps: 0-15 dequantise the weight tile, one row per thread group of 4
// (then run the epilogue from TMEM: the warps with the same w % 4 share TMEM
// lanes 32(w % 4).. and split the columns), warp 16 owns TMEM and issues the
// MMAs (one thread), warp 17 issues the TMA loads of the activation tiles.
// Decoding sets the pace for quantised weights; four decoding warps per SM
// sub-partition hide its load latency (4 -> 8 -> 16 warps: config-4 step
// 2797 -> 2297 -> 2192 ms).
//
// Shared memory holds two rings: decoded weight stages (warps 0-15 fill
// them) and activation stages (TMA fills them; for BF16 each also carries
// the weight tile). The MMA thread frees a stage of each ring with a
// tcgen05.commit once its MMAs have read it. DEEP = false: two stages each,
// freed by one commit. DEEP = true (BF16 and Q8_0 tiles of up to 128
// tokens): as many stages as 227 KB holds, up to four per ring, so the
// activation copies of later stages are in flight while earlier ones are
// multiplied -- one stage's turnaround is the copy's latency plus the MMAs'
// completion, which two stages leave exposed. Every wait is bounded. All
// copies read this GPU's own memory into this CTA's shared memory.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include "common.cuh"
#include "gemv.cuh"
#include "tma.cuh"

namespace tcu {

constexpr int TC_BM = 128;     // weight rows per tile (MMA M)
constexpr int TC_BK = 64;      // K per stage (one 128-byte swizzle atom of binary16)
constexpr int TC_MAXN = 256;   // tokens per tile (MMA N)
constexpr int TC_DQW = 16;     // weight-decoding warps (a multiple of 4)
constexpr int TC_MMA_WARP = TC_DQW, TC_TMA_WARP = TC_DQW + 1;
constexpr int TC_THREADS = TC_DQW * 32 + 64;
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;      // 16 KB per binary16 weight tile
constexpr int TC_MAX_STAGES = 4;                   // per ring
constexpr int TC_SMEM_LIMIT = 227 * 1024;          // a CTA's shared memory
// Weight operand of a GEMM: Q8_0 decoded into a binary16 pair, Q6_K / Q5_K
// into three binary16 pieces, BF16 brought by TMA as stored.
enum TcWeights : int { TCW_Q8 = 0, TCW_KQ = 1, TCW_BF16 = 2 };
// Binary16 weight pieces of a decoded weight stage.
__host__ __device__ constexpr int tc_pieces(int wm) { return wm == TCW_KQ ? 3 : 2; }
// Bytes of one weight stage (none for BF16, whose tile comes by TMA with the
// activations) and of one activation stage (Xh and Xl, or the BF16 weight
// tile and X0, X1, X2) for a tile of n_tile tokens.
__host__ __device__ constexpr int tc_w_stage_bytes(int wm) { return wm == TCW_BF16 ? 0 : tc_pieces(wm) * TC_A_BYTES; }
__host__ __device__ constexpr int tc_x_stage_bytes(int wm, int n_tile) {
  return wm == TCW_BF16 ? TC_A_BYTES + 3 * n_tile * TC_BK * 2 : 2 * n_tile * TC_BK * 2;
}
// Both rings, 1 KB alignment slack, barriers: with two stages each and full
// tiles 193.25 KB (Q8_0, BF16) or 225.25 KB (K-quants).
__host__ __device__ constexpr int tc_smem_bytes(int wm, int n_tile, int ws, int xs) {
  return ws * tc_w_stage_bytes(wm) + xs * tc_x_stage_bytes(wm, n_tile) + 1024 + 256;
}
static_assert(tc_smem_bytes(TCW_KQ, TC_MAXN, 2, 2) <= TC_SMEM_LIMIT, "tensor-core GEMM stages exceed shared memory");
static_assert(tc_smem_bytes(TCW_BF16, 128, 0, 2) <= TC_SMEM_LIMIT, "tensor-core GEMM stages exceed shared memory");
static_assert(TC_DQW * 8 == TC_BM, "one weight row per decoding thread group and stage (the Q6_K prefetch relies on it)");

struct TcArgs {
  DMat W;             // Q8_0 weights [rows][cols]
  int n;              // tokens
  int n_tile;         // tokens per CTA tile (multiple of 16, <= TC_MAXN)
  int n_pad;          // rows of one half of the activation split (hi rows, then lo rows)
  const int* sx;      // [n] per-token power of two of the split
  int sw;             // power of two of the weight split
  // epilogue (as GemmArgs)
  float* out;
  int out_stride;
  int n_plain;
  float* glu_out;
  int glu_stride;
  int glu_act;
  float* resid;
  int resid_stride;
  int k_split;        // EPI_RESID2: K where the second accumulator starts (multiple of TC_BK)
  float* part;        // split K: partial sums [gridDim.z][n][rows] (nullptr: apply the epilogue)
  int k_per_z;        // split K: columns per z slice (multiple of TC_BK)
  int tok_fast;       // grid x = token tiles (else x = weight-row tiles)
  int ws, xs;         // DEEP: stages of the weight ring (0 for BF16) and of the activation ring, <= TC_MAX_STAGES
  int* err;
};

// 2^e exactly, for e in [-126, 127].
__device__ __forceinline__ float tc_pow2(int e) { return __int_as_float((e + 127) << 23); }

__device__ __forceinline__ uint64_t tc_smem_desc(uint32_t saddr) {
  // K-major operand, 128-byte swizzle: 8-row groups 1024 bytes apart (SBO),
  // LBO unused (1), descriptor version 1, layout type 2 (SWIZZLE_128B).
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: float32 accumulator, A and B both binary16 (or
// both bfloat16), both K-major, N = n, M = 128.
__device__ __forceinline__ uint32_t tc_idesc(int n, bool bf16) {
  return (1u << 4) | (bf16 ? (1u << 7) | (1u << 10) : 0u) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// 2-D TMA load of a box at (x = k, y = row) into shared memory, completing on bar.
__device__ __forceinline__ void tc_tma_load(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
                   smem_u32(dst)),
               "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
               : "memory");
}

// Byte offset of element (row, k) (k < 64) in a K-major 128-byte-swizzled
// tile: rows in 8-row groups of 1024 bytes, 16-byte chunk c of row r stored
// at chunk c ^ (r % 8).
__device__ __forceinline__ uint32_t tc_sw128(int row, int k) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((k * 2) >> 4) ^ (row & 7)) << 4) + ((k * 2) & 15));
}

// Binary16 pair of 8 int8 weights times the scale s' (binary16): the eight
// values 1024 + (q ^ 0x80) are built by byte permutation and 1152 subtracted,
// which is exact; Wh = q * s' rounded, Wl = fma(q, s', -Wh) rounded (exact).
__device__ __forceinline__ void tc_dequant8(uint2 q, __half2 s2, uint4& hi, uint4& lo) {
  const uint32_t w[2] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u};
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 2; i++) {
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const uint32_t p = __byte_perm(w[i], 0x64646464u, j == 0 ? 0x7170 : 0x7372);  // bytes (2j, 2j+1) as 0x64xx
      const __half2 qv = __hsub2(*reinterpret_cast<const __half2*>(&p), bias);
      const __half2 wh = __hmul2(qv, s2);
      const __half2 wl = __hfma2(qv, s2, __hneg2(wh));
      h[2 * i + j] = *reinterpret_cast<const uint32_t*>(&wh);
      l[2 * i + j] = *reinterpret_cast<const uint32_t*>(&wl);
    }
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Top six significant bits of a float32 (sign, exponent and five stored
// mantissa bits); x - tc_top6(x) is exact.
__device__ __forceinline__ float tc_top6(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFC0000u); }

// The Q6_K operand of sixteen weights W[r][k0 .. k0 + 16) (k0 % 16 == 0: one
// scale group). The reference's value (quant_k.go:47-85) is
// v = (d * sc) * (q - 32) with d binary16, sc int8 and q six bits: d * sc has
// at most 18 significant bits and |q - 32| <= 32 at most 5, so both float32
// products are exact and v = s * (q - 32) with s = d * sc. The scaled
// s' = s * 2^sw is split into three pieces of at most six significant bits,
// s' = s1 + s2 + s3 (each a masked remainder, exact), and each piece times
// the integer q - 32 has at most 11 bits: an exact binary16 product
// (HMUL2). So p1 + p2 + p3 = v * 2^sw exactly. The raw bytes come with one
// 16-byte load each for the 16 low nibbles and the 16 high-bit pairs
// (tc_q6k_load; the GEMM loads the next stage's while it builds this one).
struct Q6Raw {
  uint4 ql, qh;
  float s;  // d * sc (exact), 0 for rows or columns past the matrix
};

__device__ __forceinline__ Q6Raw tc_q6k_load(const DMat& W, int r, int k0, bool valid) {
  Q6Raw q;
  if (!valid) {
    q.ql = q.qh = make_uint4(0, 0, 0, 0);
    q.s = 0.f;
    return q;
  }
  const uint8_t* blk = W.w + ((size_t)r * (W.cols >> 8) + (k0 >> 8)) * 224;
  const int i0 = k0 & 255;
  q.ql = __ldg(reinterpret_cast<const uint4*>(blk + (i0 >> 7) * 64 + (i0 & 63)));
  q.qh = __ldg(reinterpret_cast<const uint4*>(blk + 128 + (i0 >> 7) * 32 + (i0 & 31)));
  const float d = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(blk + 208))));
  q.s = __fmul_rn(d, (float)(int8_t)__ldg(blk + 192 + (i0 >> 4)));
  return q;
}

__device__ __forceinline__ void tc_q6k_build(const Q6Raw& q, int k0, float wscale, uint4 (&p)[3][2]) {
  const int i0 = k0 & 255;
  const float sc = __fmul_rn(q.s, wscale);
  const float s1 = tc_top6(sc), r1 = __fsub_rn(sc, s1), s2 = tc_top6(r1), s3 = __fsub_rn(r1, s2);
  const __half2 h1 = __float2half2_rn(s1), h2 = __float2half2_rn(s2), h3 = __float2half2_rn(s3);
  const int ls = ((i0 & 127) >> 6) * 4, hs = ((i0 & 127) >> 5) * 2;
  const uint32_t lw[4] = {q.ql.x, q.ql.y, q.ql.z, q.ql.w}, hw[4] = {q.qh.x, q.qh.y, q.qh.z, q.qh.w};
  const __half2 bias = __halves2half2(__ushort_as_half(0x6420), __ushort_as_half(0x6420));  // 1056 = 1024 + 32
  uint32_t o1[8], o2[8], o3[8];
#pragma unroll
  for (int w = 0; w < 4; w++) {
    const uint32_t q4 = ((lw[w] >> ls) & 0x0F0F0F0Fu) | (((hw[w] >> hs) & 0x03030303u) << 4);
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const uint32_t b = __byte_perm(q4, 0x64646464u, j == 0 ? 0x7170 : 0x7372);  // (1024 + q) pairs
      const __half2 qq = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);      // q - 32, exact
      const __half2 a = __hmul2(h1, qq), m = __hmul2(h2, qq), l = __hmul2(h3, qq);
      o1[2 * w + j] = *reinterpret_cast<const uint32_t*>(&a);
      o2[2 * w + j] = *reinterpret_cast<const uint32_t*>(&m);
      o3[2 * w + j] = *reinterpret_cast<const uint32_t*>(&l);
    }
  }
  p[0][0] = make_uint4(o1[0], o1[1], o1[2], o1[3]);
  p[0][1] = make_uint4(o1[4], o1[5], o1[6], o1[7]);
  p[1][0] = make_uint4(o2[0], o2[1], o2[2], o2[3]);
  p[1][1] = make_uint4(o2[4], o2[5], o2[6], o2[7]);
  p[2][0] = make_uint4(o3[0], o3[1], o3[2], o3[3]);
  p[2][1] = make_uint4(o3[4], o3[5], o3[6], o3[7]);
}

__device__ __forceinline__ void tc_q6k_pieces(const DMat& W, int r, int k0, float wscale, uint4 (&p)[3][2]) {
  tc_q6k_build(tc_q6k_load(W, r, k0, true), k0, wscale, p);
}

// The tensor-core operand of sixteen weights W[r][k0 .. k0 + 16), scaled by
// wscale = 2^sw, as binary16 pieces p[piece][half] (eight values per uint4):
//   Q8_0 (WM = TCW_Q8): the exact pair of tc_dequant8; values at or past
//     k_end are zero;
//   Q6_K (WM = TCW_KQ): tc_q6k_pieces;
//   Q5_K (WM = TCW_KQ): each value decoded as kquant_decode8 does (the
//     reference's float32 arithmetic), then split into three pieces,
//     h = fp16(v), m = fp16(v - h), l = fp16(v - h - m).
//   K-quant rows are whole super-blocks (K % 256 == 0, k_end too), so
//   k0 < k_end covers all 16.
// Rows r >= R give zeros. The GEMM's decoding warps and tcu_read_values
// (TCU_DECODE_TC) both call this.
template <int WM>
__device__ __forceinline__ void tc_weight_pieces(const DMat& W, int r, int k0, int k_end, float wscale,
                                                 uint4 (&p)[tc_pieces(WM)][2]) {
#pragma unroll
  for (int j = 0; j < tc_pieces(WM); j++) p[j][0] = p[j][1] = make_uint4(0, 0, 0, 0);
  if (r >= W.rows || k0 >= k_end) return;
  if constexpr (WM == TCW_KQ) {
    if (W.fmt == FMT_Q6_K) {
      tc_q6k_pieces(W, r, k0, wscale, p);
      return;
    }
    float v[16];
    kquant_decode8(W, r, k0, v);
    kquant_decode8(W, r, k0 + 8, v + 8);
    uint32_t hh[8], mm[8], ll[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float x0 = v[2 * i] * wscale, x1 = v[2 * i + 1] * wscale;
      const __half2 h = __floats2half2_rn(x0, x1);
      const float2 hf = __half22float2(h);
      const float r0 = __fsub_rn(x0, hf.x), r1 = __fsub_rn(x1, hf.y);
      const __half2 m = __floats2half2_rn(r0, r1);
      const float2 mf = __half22float2(m);
      const __half2 l = __floats2half2_rn(__fsub_rn(r0, mf.x), __fsub_rn(r1, mf.y));
      hh[i] = *reinterpret_cast<const uint32_t*>(&h);
      mm[i] = *reinterpret_cast<const uint32_t*>(&m);
      ll[i] = *reinterpret_cast<const uint32_t*>(&l);
    }
    p[0][0] = make_uint4(hh[0], hh[1], hh[2], hh[3]);
    p[0][1] = make_uint4(hh[4], hh[5], hh[6], hh[7]);
    p[1][0] = make_uint4(mm[0], mm[1], mm[2], mm[3]);
    p[1][1] = make_uint4(mm[4], mm[5], mm[6], mm[7]);
    p[2][0] = make_uint4(ll[0], ll[1], ll[2], ll[3]);
    p[2][1] = make_uint4(ll[4], ll[5], ll[6], ll[7]);
  } else {
    const uint4 q = *reinterpret_cast<const uint4*>(W.w + (size_t)r * W.cols + k0);
    const float s = __half2float(W.s[(size_t)r * W.sstride + k0 / 32]) * wscale;
    const __half2 s2 = __float2half2_rn(s);
    tc_dequant8(make_uint2(q.x, q.y), s2, p[0][0], p[1][0]);
    tc_dequant8(make_uint2(q.z, q.w), s2, p[0][1], p[1][1]);
    if (k0 + 8 > k_end) p[0][0] = p[1][0] = make_uint4(0, 0, 0, 0);
    if (k0 + 16 > k_end) p[0][1] = p[1][1] = make_uint4(0, 0, 0, 0);
  }
}

// WM: TCW_BF16 takes bfloat16 weight tiles through wmap; TCW_Q8 and TCW_KQ
// weights are decoded by warps 0-15 (wmap unused).
template <int EPI, int WM, bool DEEP>
__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_tc(const __grid_constant__ CUtensorMap xmap,
                                                           const __grid_constant__ CUtensorMap wmap, TcArgs a) {
  constexpr bool WB = WM == TCW_BF16;
  constexpr int NP = tc_pieces(WM);
  extern __shared__ uint8_t tc_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  const int NT = a.n_tile;
  // Ring depths (BF16 has no weight ring: its weight stage is 0 bytes).
  const int WS = DEEP && !WB ? a.ws : 2, XS = DEEP ? a.xs : 2;
  const uint32_t w_stage = (uint32_t)tc_w_stage_bytes(WM), x_stage = (uint32_t)tc_x_stage_bytes(WM, NT);
  const uint32_t x_piece = (uint32_t)NT * TC_BK * 2;  // one activation piece of the tile
  uint8_t* wring = smem;                                        // [WS] decoded weight stages
  uint8_t* xring = smem + (size_t)(WB ? 0 : WS) * w_stage;      // [XS] activation stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(xring + (size_t)XS * x_stage);
  uint64_t* x_full = bars;                       // [XS] activation tiles landed
  uint64_t* x_empty = bars + TC_MAX_STAGES;      // [XS] MMAs reading the activation stage finished
  uint64_t* w_full = bars + 2 * TC_MAX_STAGES;   // [WS] weight tiles written
  // [WS] MMAs reading the weight stage finished; with two stages each, the
  // activation barriers serve both rings.
  uint64_t* w_empty = DEEP ? bars + 3 * TC_MAX_STAGES : x_empty;
  uint64_t* acc_full = bars + 4 * TC_MAX_STAGES;  // accumulators final
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4 * TC_MAX_STAGES + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = a.W.rows, K = a.W.cols;
  // tok_fast: token tiles are the fastest grid index, so the CTAs that share
  // a weight tile run together and read it from L2 rather than HBM.
  const int r0 = (a.tok_fast ? blockIdx.y : blockIdx.x) * TC_BM, t0 = (a.tok_fast ? blockIdx.x : blockIdx.y) * a.n_tile;
  const int k_begin = a.part ? blockIdx.z * a.k_per_z : 0;
  const int k_end = a.part ? min(K, k_begin + a.k_per_z) : K;
  const int iters = (k_end - k_begin + TC_BK - 1) / TC_BK;
  const bool two_acc = (EPI == EPI_RESID2) && !a.part;
  const uint32_t tmem_cols = two_acc ? 2 * TC_MAXN : TC_MAXN;

  if (threadIdx.x == 0) {
    for (int i = 0; i < XS; i++) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < WS; i++) {
      mbar_init(&w_full[i], TC_DQW * 32);
      if (DEEP) mbar_init(&w_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == TC_MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp == TC_TMA_WARP) {
    // ---- activation stages: Xh rows [t0, t0 + NT), Xl rows n_pad + the same.
    // BF16: the weight tile, then pieces X0, X1, X2 (rows p * n_pad + t0).
    if (lane == 0) {
      const uint32_t bytes = WB ? (uint32_t)TC_A_BYTES + 3 * x_piece : 2 * x_piece;
      for (int i = 0; i < iters; i++) {
        const int b = i % XS;
        if (i >= XS) mbar_wait(&x_empty[b], ((i / XS) - 1) & 1, a.err);
        uint8_t* xb = xring + (size_t)b * x_stage;
        mbar_expect_tx(&x_full[b], bytes);
        const int k = k_begin + i * TC_BK;
        if (WB) {
          tc_tma_load(xb, &wmap, k, r0, &x_full[b]);
#pragma unroll
          for (int p = 0; p < 3; p++) tc_tma_load(xb + TC_A_BYTES + p * x_piece, &xmap, k, p * a.n_pad + t0, &x_full[b]);
        } else {
          tc_tma_load(xb, &xmap, k, t0, &x_full[b]);
          tc_tma_load(xb + x_piece, &xmap, k, a.n_pad + t0, &x_full[b]);
        }
      }
    }
  } else if (warp == TC_MMA_WARP) {
    // ---- MMA issue (one thread): 4 K16 steps x (Wh.Xh, Wh.Xl, Wl.Xh) per stage
    if (lane == 0) {
      const uint32_t idesc = tc_idesc(NT, WB);
      bool first0 = true, first1 = true;
      for (int i = 0; i < iters; i++) {
        const int xb = i % XS, wb = i % WS;
        mbar_wait(&x_full[xb], (i / XS) & 1, a.err);
        if (!WB) mbar_wait(&w_full[wb], (i / WS) & 1, a.err);
        tc_fence_after();
        const int k = k_begin + i * TC_BK;
        const bool second = two_acc && k >= a.k_split;
        const uint32_t d = tmem + (second ? TC_MAXN : 0);
        bool& first = second ? first1 : first0;
        const uint32_t sx = smem_u32(xring + (size_t)xb * x_stage);
        const uint32_t sa = WB ? sx : smem_u32(wring + (size_t)wb * w_stage);
#pragma unroll
        for (int kk = 0; kk < TC_BK / 16; kk++) {
          const uint32_t off = kk * 32;  // 16 columns of 2 bytes
          if (WB) {
            const uint64_t w = tc_smem_desc(sa + off);
#pragma unroll
            for (int p = 0; p < 3; p++) {
              tc_mma(d, w, tc_smem_desc(sx + TC_A_BYTES + p * x_piece + off), idesc, first ? 0u : 1u);
              first = false;
            }
          } else {
            // Q8_0: Wh.Xh + Wh.Xl + Wl.Xh; K-quants: W1.Xh + W1.Xl + W2.Xh + W2.Xl + W3.Xh.
            const uint64_t wh = tc_smem_desc(sa + off);
            const uint64_t xh = tc_smem_desc(sx + off), xl = tc_smem_desc(sx + x_piece + off);
            tc_mma(d, wh, xh, idesc, first ? 0u : 1u);
            first = false;
            tc_mma(d, wh, xl, idesc, 1u);
#pragma unroll
            for (int p = 1; p < NP; p++) tc_mma(d, tc_smem_desc(sa + p * TC_A_BYTES + off), xh, idesc, 1u);
            if (WM == TCW_KQ) tc_mma(d, tc_smem_desc(sa + TC_A_BYTES + off), xl, idesc, 1u);
          }
        }
        tc_commit(&x_empty[xb]);
        if (DEEP && !WB) tc_commit(&w_empty[wb]);
      }
      tc_commit(acc_full);
    }
  } else {
    // ---- weight tiles (warps 0-15): 4 threads per row, 16 bytes each
    const int tid = threadIdx.x;  // 0..511
    const int kc = (tid & 3) * 16;
    const float wscale = tc_pow2(a.sw);
    // Q6_K: each thread builds one row's 16 values per stage and loads the
    // next stage's raw bytes first.
    const bool q6 = WM == TCW_KQ && a.W.fmt == FMT_Q6_K;
    Q6Raw nxt{};
    if (q6 && iters > 0) nxt = tc_q6k_load(a.W, r0 + (tid >> 2), k_begin + kc, r0 + (tid >> 2) < R && k_begin + kc < k_end);
    for (int i = 0; i < (WB ? 0 : iters); i++) {
      const int b = i % WS;
      const int k0 = k_begin + i * TC_BK + kc;
      Q6Raw cur{};
      if (q6) {
        cur = nxt;
        const int kn = k0 + TC_BK;
        if (i + 1 < iters) nxt = tc_q6k_load(a.W, r0 + (tid >> 2), kn, r0 + (tid >> 2) < R && kn < k_end);
      }
      if (i >= WS) mbar_wait(&w_empty[b], ((i / WS) - 1) & 1, a.err);
      uint8_t* aw = wring + (size_t)b * w_stage;
      for (int rr = tid >> 2; rr < TC_BM; rr += TC_DQW * 8) {
        uint4 pc[NP][2];
        if constexpr (WM == TCW_KQ) {
          if (q6)
            tc_q6k_build(cur, k0, wscale, pc);
          else
            tc_weight_pieces<WM>(a.W, r0 + rr, k0, k_end, wscale, pc);
        } else {
          tc_weight_pieces<WM>(a.W, r0 + rr, k0, k_end, wscale, pc);
        }
#pragma unroll
        for (int p = 0; p < NP; p++) {
          *reinterpret_cast<uint4*>(aw + p * TC_A_BYTES + tc_sw128(rr, kc)) = pc[p][0];
          *reinterpret_cast<uint4*>(aw + p * TC_A_BYTES + tc_sw128(rr, kc + 8)) = pc[p][1];
        }
      }
      // Generic writes must be visible to the tensor core (async proxy).
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&w_full[b]);
    }
    // ---- epilogue: warp w reads TMEM lanes 32(w % 4).. (weight rows),
    // column chunks w / 4, w / 4 + TC_DQW / 4, ...
    mbar_wait(acc_full, 0, a.err);
    tc_fence_after();
    const int quad = warp & 3;
    const int rr = quad * 32 + lane, r = r0 + rr;
    const float wunscale = tc_pow2(-a.sw);
    for (int c0 = (warp >> 2) * 16; c0 < NT; c0 += 16 * (TC_DQW / 4)) {
      float v[16], v2[16];
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + c0;
      tc_ld16(taddr, v);
      if (two_acc) tc_ld16(taddr + TC_MAXN, v2);
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const int t = t0 + c0 + j;
        const bool ok = t < a.n && r < R;
        const float sc = ok ? wunscale * tc_pow2(-a.sx[t]) : 0.f;
        const float lo = v[j] * sc;
        if (a.part) {
          if (ok) a.part[((size_t)blockIdx.z * a.n + t) * R + r] = lo;
          continue;
        }
        if constexpr (EPI == EPI_STORE) {
          if (ok) a.out[(size_t)t * a.out_stride + r] = lo;
        } else if constexpr (EPI == EPI_GLU) {
          const float up = __shfl_xor_sync(0xffffffffu, lo, 1);
          if (ok) {
            if (r < a.n_plain)
              a.out[(size_t)t * a.out_stride + r] = lo;
            else if (((r - a.n_plain) & 1) == 0)
              a.glu_out[(size_t)t * a.glu_stride + ((r - a.n_plain) >> 1)] =
                  a.glu_act ? silu_mul_llama(lo, up) : silu_mul_stablelm(lo, up);
          }
        } else if constexpr (EPI == EPI_RESID1) {
          if (ok) {
            float* x = a.resid + (size_t)t * a.resid_stride + r;
            *x = __fadd_rn(*x, lo);
          }
        } else if constexpr (EPI == EPI_RESID2) {
          if (ok) {
            float* x = a.resid + (size_t)t * a.resid_stride + r;
            *x = __fadd_rn(__fadd_rn(*x, lo), v2[j] * sc);
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == TC_MMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols));
  }
}

// Exact binary16 split of activation rows for the tensor-core GEMM: per
// token t, sx(t) = 13 - exponent of max|X[t]| (a power of two), then
// Xh = fp16(X * 2^sx), Xl = fp16(X * 2^sx - Xh). out: [2][n_pad][K] binary16
// (rows >= n are left as they are; the TMA loads zeros past the map).
__global__ void k_split_f16(const float* X, int ldx, int n, int K, int n_pad, __half* out, int* sx) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  const float* x = X + (size_t)t * ldx;
  float mx = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(x[k]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) {
      int e = 0;
      if (m > 0.f) frexpf(m, &e);  // m in [2^(e-1), 2^e)
      red[0] = (float)(m > 0.f ? 13 - e : 0);
    }
  }
  __syncthreads();
  const int s = (int)red[0];
  if (threadIdx.x == 0) sx[t] = s;
  const float scale = tc_pow2(s);
  __half* hi = out + (size_t)t * K;
  __half* lo = out + ((size_t)n_pad + t) * K;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = x[k] * scale;
    const __half h = __float2half_rn(v);
    hi[k] = h;
    lo[k] = __float2half_rn(v - __half2float(h));
  }
}

// Exact bfloat16 split of activation rows: per token t the power of two sx(t)
// as in k_split_f16, then X' = X * 2^sx = X0 + X1 + X2 with each piece the
// bfloat16 rounding of what the previous pieces leave (both differences are
// exact in float32). out: [3][n_pad][K] bfloat16.
__global__ void k_split_bf16(const float* X, int ldx, int n, int K, int n_pad, __nv_bfloat16* out, int* sx) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  const float* x = X + (size_t)t * ldx;
  float mx = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(x[k]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) {
      int e = 0;
      if (m > 0.f) frexpf(m, &e);
      red[0] = (float)(m > 0.f ? 13 - e : 0);
    }
  }
  __syncthreads();
  const int s = (int)red[0];
  if (threadIdx.x == 0) sx[t] = s;
  const float scale = tc_pow2(s);
  __nv_bfloat16* p0 = out + (size_t)t * K;
  __nv_bfloat16* p1 = out + ((size_t)n_pad + t) * K;
  __nv_bfloat16* p2 = out + ((size_t)2 * n_pad + t) * K;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = x[k] * scale;
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(h);
    const __nv_bfloat16 m1 = __float2bfloat16_rn(r1);
    p0[k] = h;
    p1[k] = m1;
    p2[k] = __float2bfloat16_rn(r1 - __bfloat162float(m1));
  }
}

// Largest |scale| of a Q8_0 scale plane (rows x nb valid blocks), as the
// bits of a non-negative float (their unsigned order is the float order).
__global__ void k_scale_absmax(const __half* s, int rows, int sstride, int nb, unsigned* out) {
  unsigned m = 0;
  const size_t total = (size_t)rows * nb;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const float v = fabsf(__half2float(s[(i / nb) * sstride + i % nb]));
    if (v == v) m = max(m, __float_as_uint(v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, m);
}

// Upper bound of |value| over a Q6_K or Q5_K matrix (nblocks super-blocks),
// as the bits of a non-negative float: Q6_K |d| * max|scale| * 32, Q5_K
// max(|d| * 63 * 31, |dmin| * 63).
__global__ void k_kquant_absmax(const uint8_t* w, size_t nblocks, int fmt, unsigned* out) {
  unsigned m = 0;
  for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblocks; b += (size_t)gridDim.x * blockDim.x) {
    float v;
    if (fmt == FMT_Q6_K) {
      const uint8_t* blk = w + b * 224;
      int ms = 0;
      for (int g = 0; g < 16; g++) ms = max(ms, abs((int)(int8_t)blk[192 + g]));
      v = fabsf(__half2float(__ushort_as_half((unsigned short)(blk[208] | (blk[209] << 8))))) * (float)ms * 32.f;
    } else {
      const uint8_t* blk = w + b * 176;
      const float d = fabsf(__half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8)))));
      const float dm = fabsf(__half2float(__ushort_as_half((unsigned short)(blk[2] | (blk[3] << 8)))));
      v = fmaxf(d * 63.f * 31.f, dm * 63.f);
    }
    if (v == v) m = max(m, __float_as_uint(v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, m);
}

// Split-K reduction of the out/down rows with the parallel residual
// (stablelm.go:365-377): slices [0, z_lo) cover the attention columns, the
// rest the SwiGLU columns; x = (x + lo) + hi, each sum in slice order.
__global__ void k_splitk_resid(const float* part, int z_lo, int z_n, int n, int R, float* resid, int stride) {
  const size_t total = (size_t)n * R;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / R), r = (int)(i % R);
    float lo = 0.f, hi = 0.f;
    for (int z = 0; z < z_lo; z++) lo += part[(size_t)z * total + i];
    for (int z = z_lo; z < z_n; z++) hi += part[(size_t)z * total + i];
    float* x = resid + (size_t)t * stride + r;
    *x = z_lo < z_n ? __fadd_rn(__fadd_rn(*x, lo), hi) : __fadd_rn(*x, lo);
  }
}

// Split-K sum for the GLU and STORE epilogues: part [z][n][R] is summed in
// slice order from 0, then stored (STORE rows, GLU rows below n_plain) or
// paired into act(gate) * up (GLU rows n_plain + 2j and n_plain + 2j + 1),
// as the single-pass epilogue of k_gemm_tc does.
template <int EPI>
__global__ void k_splitk_epi(const float* part, int z_n, int n, int R, float* out, int out_stride, int n_plain,
                             float* glu_out, int glu_stride, int glu_act) {
  const size_t total = (size_t)n * R;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / R), r = (int)(i % R);
    if (EPI == EPI_GLU && r >= n_plain && ((r - n_plain) & 1)) continue;
    float v = 0.f;
    for (int z = 0; z < z_n; z++) v += part[(size_t)z * total + i];
    if (EPI == EPI_STORE || r < n_plain) {
      out[(size_t)t * out_stride + r] = v;
      continue;
    }
    float up = 0.f;
    for (int z = 0; z < z_n; z++) up += part[(size_t)z * total + i + 1];
    glu_out[(size_t)t * glu_stride + ((r - n_plain) >> 1)] = glu_act ? silu_mul_llama(v, up) : silu_mul_stablelm(v, up);
  }
}

}  // namespace tcu
