// Shared-prefix attention on the 5th-generation tensor cores (binary16 KV).
//
// Branches of one prefix (mlx_branches.go:98-114) all read the prefix's KV
// pages. k_attn_shared_tc computes, for every query row of the branch batch,
// each whole 64-position split of that prefix: the per-split partial
// (sum_t exp(s_t - m) v_t, m, sum_t exp(s_t - m)) that k_attn_shared writes
// on CUDA cores, in the same place, for the per-row kernels to merge.
//
// One CTA per (run of splits, KV head, tile of 128 query rows). Query row qi
// is head g * G + qi % G of batch row qi / G, rotated at that row's position
// (the reference's RoPE operations, stablelm.go:309-326). Per split:
//   S = Q K^T      tcgen05.mma M = 128 rows, N = 64 positions, K = hd.
//                  The binary16 keys are exact operands; each float32 query
//                  row is scaled by 2^sx (sx = 13 - exponent of its max) and
//                  split into an exact binary16 pair Qh + Ql (22 of its 24
//                  bits), so S = Qh.K + Ql.K is accumulated in float32.
//   s = S 2^-sx / sqrt(hd) (correctly rounded division), per row the
//       split's max m, p_t = expf(s_t - m), l = sum_t p_t in position order
//       (one thread per row, scores read from TMEM).
//   O = P V        M = 128 rows, N = hd, K = 64 positions; P in [0, 1]
//                  split into a binary16 pair Ph + Pl (absolute error below
//                  2^-24 per weight), V exact.
// The dropped terms are ~2^-22 of each product, the accumulation order is
// the tensor core's: results agree with the float32 CUDA-core kernel to
// ~1e-6 relative, not bit for bit.
//
// Shared-memory operands use the no-swizzle K-major / MN-major layouts of
// 8-row x 16-byte core matrices. A K or V tile is stored [hd/8 chunks][64
// positions][8 values], so chunk c of position t is at c * 1024 + t * 16:
// as the B operand of S (K-major over hd) core matrices step 128 bytes over
// positions and 1024 over hd; as the B operand of O (MN-major: N = hd
// contiguous) they step 1024 bytes over hd and 128 over positions. Q and P
// tiles are [chunks][128 rows][8 values] (K-major A, 2048 bytes per chunk).
// cp.async brings the K/V tile of the next split while the current one is
// computed. All copies read this GPU's own memory into this CTA's shared
// memory; every mbarrier wait is bounded.
#pragma once
#include "attention.cuh"
#include "gemm_tc.cuh"

namespace tcu {

constexpr int AT_ROWS = 128;    // query rows per CTA (MMA M)
constexpr int AT_KEYS = 64;     // positions per split
constexpr int AT_THREADS = 128;  // one thread per query row / TMEM lane
constexpr uint32_t AT_TMEM_COLS = 256;  // scores at column 0, outputs at 128

// Dynamic shared memory for head size hd (multiple of 16, at most 256):
// Q pieces 2 x 128 x hd, K/V 2 stages x 2 x 64 x hd, P pieces 2 x 128 x 64
// (binary16), barrier and TMEM slot. At least 80 KB, so that at most two
// CTAs (2 x 256 TMEM columns) share an SM.
__host__ __device__ inline size_t at_smem_bytes(int hd) {
  const size_t b = (size_t)4 * AT_ROWS * hd + (size_t)8 * AT_KEYS * hd + (size_t)4 * AT_ROWS * AT_KEYS + 64;
  return b < 80 * 1024 ? 80 * 1024 : b;
}

// Shared-memory descriptor of a no-swizzle operand: lbo = byte distance of
// core matrices along K, sbo = along M / N.
__device__ __forceinline__ uint64_t at_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version; layout type 0 (no swizzle)
  return d;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Sixteen TMEM columns of this thread's lane, without waiting.
__device__ __forceinline__ void at_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void at_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Element k of head vector x after RoPE at pos: the value rope_pair leaves
// there (same operations, same rounding).
__device__ __forceinline__ float rope_elem(const float* x, int k, const Rope& r, int pos) {
  if (r.mode == 0) {
    if (k >= 2 * r.pairs) return x[k];
    const int i = k < r.pairs ? k : k - r.pairs;
    const float2 cs = r.table[(size_t)pos * r.pairs + i];
    const float a = x[i], b = x[i + r.pairs];
    return k < r.pairs ? __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y)) : __fadd_rn(__fmul_rn(b, cs.x), __fmul_rn(a, cs.y));
  }
  const int i = k >> 1;
  if (i >= r.pairs) return x[k];
  const float2 cs = r.table[(size_t)pos * r.pairs + i];
  const float v0 = x[2 * i], v1 = x[2 * i + 1];
  return (k & 1) ? __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x)) : __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
}

// Binary16 pair (h, l) of two floats: h = fp16(v), l = fp16(v - h).
__device__ __forceinline__ void at_split2(float v0, float v1, uint32_t& h, uint32_t& l) {
  const __half2 hh = __floats2half2_rn(v0, v1);
  const float2 hf = __half22float2(hh);
  const __half2 ll = __floats2half2_rn(__fsub_rn(v0, hf.x), __fsub_rn(v1, hf.y));
  h = *reinterpret_cast<const uint32_t*>(&hh);
  l = *reinterpret_cast<const uint32_t*>(&ll);
}

// Shared memory of the attention kernels: P pieces first, then Q pieces,
// then the two K/V stages (the order keeps every operand read inside the
// allocation), then the barrier and the TMEM slot.
struct AtSmem {
  uint8_t* ps;   // [2 pieces][8 chunks][128 rows][16 B]
  uint8_t* qs;   // [2 pieces][hd/8 chunks][128 rows][16 B]
  uint8_t* kvs;  // [2 stages][K, V][hd/8 chunks][64 positions][16 B]
  uint64_t* bar;
  uint32_t* tslot;
  uint32_t q_piece, kv_tile, p_piece;  // bytes of one Q piece, one K (or V) tile, one P piece
};

__device__ __forceinline__ AtSmem at_carve(uint8_t* base, int hd) {
  AtSmem m;
  m.ps = base;
  m.qs = m.ps + 4 * AT_ROWS * AT_KEYS;
  m.kvs = m.qs + 4 * AT_ROWS * hd;
  m.bar = reinterpret_cast<uint64_t*>(m.kvs + 8 * AT_KEYS * hd);
  m.tslot = reinterpret_cast<uint32_t*>(m.bar + 1);
  m.q_piece = 2 * AT_ROWS * hd;
  m.kv_tile = 2 * AT_KEYS * hd;
  m.p_piece = 2 * AT_ROWS * AT_KEYS;
  return m;
}

// Barrier init (thread 0) and the TMEM allocation (warp 0).
__device__ __forceinline__ void at_begin(const AtSmem& sm) {
  if (threadIdx.x == 0) {
    mbar_init(sm.bar, 1);
    fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(sm.tslot)), "r"(AT_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
}

__device__ __forceinline__ void at_end(const AtSmem& sm, uint32_t tmem) {
  cp_async_wait<0>();
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AT_TMEM_COLS));
  }
}

// This thread's query row x (float32, hd values; rotated at pos first when
// ROPE) as the binary16 pair of x * 2^sx into the Q tiles; returns sx.
template <bool ROPE>
__device__ __forceinline__ int at_q_pieces(const AtSmem& sm, const float* x, bool valid, int hd, const Rope& rope, int pos) {
  auto val = [&](int k) { return !valid ? 0.f : ROPE ? rope_elem(x, k, rope, pos) : x[k]; };
  float mx = 0.f;
  for (int k = 0; k < hd; k++) mx = fmaxf(mx, fabsf(val(k)));
  int ex = 0;
  if (mx > 0.f) frexpf(mx, &ex);
  const int sx = mx > 0.f ? 13 - ex : 0;
  const float qscale = tc_pow2(sx);
  for (int c = 0; c < hd / 8; c++) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; j++) at_split2(val(8 * c + 2 * j) * qscale, val(8 * c + 2 * j + 1) * qscale, h[j], l[j]);
    *reinterpret_cast<uint4*>(sm.qs + c * (AT_ROWS * 16) + threadIdx.x * 16) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(sm.qs + sm.q_piece + c * (AT_ROWS * 16) + threadIdx.x * 16) = make_uint4(l[0], l[1], l[2], l[3]);
  }
  return sx;
}

// Keys and values of positions [t0, t0 + 64) of KV head g into stage st
// (chunk c of position t at c * 1024 + t * 16); positions past last are
// zero (their weights are zero, and 0 * 0 keeps the products finite).
__device__ __forceinline__ void at_load_kv(const AtSmem& sm, int st, const KVView& kv, int layer, const int* page_table, int g, int t0,
                                           int last, int hd) {
  uint8_t* kb = sm.kvs + (size_t)st * 2 * sm.kv_tile;
  uint8_t* vb = kb + sm.kv_tile;
  const int cpr = hd / 8;
  for (int e = threadIdx.x; e < AT_KEYS * cpr; e += AT_THREADS) {
    const int t = e % AT_KEYS, c = e / AT_KEYS, ta = t0 + t;
    const int so = c * (AT_KEYS * 16) + t * 16;
    if (ta <= last) {
      const size_t off = kv.off(layer, page_table[ta / kv.P], g, ta % kv.P) + 8 * c;
      cp_async16(kb + so, reinterpret_cast<const __half*>(kv.k) + off);
      cp_async16(vb + so, reinterpret_cast<const __half*>(kv.v) + off);
    } else {
      *reinterpret_cast<uint4*>(kb + so) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(vb + so) = make_uint4(0, 0, 0, 0);
    }
  }
  cp_async_commit();
}

// Waits for the tensor core's last commit; true on every thread if any
// thread's wait ran out (all threads then leave together).
__device__ __forceinline__ bool at_wait_mma(const AtSmem& sm, uint32_t& phase, int* err) {
  const bool failed = __syncthreads_or(!mbar_wait(sm.bar, phase, err));
  phase ^= 1;
  tc_fence_after();
  return failed;
}

// Makes this thread's shared-memory writes (copies, P tiles) visible to the
// tensor core, then synchronises the CTA.
__device__ __forceinline__ void at_publish() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// S = Qh.K + Ql.K into TMEM columns [0, 64) (thread 0 issues, then commits).
__device__ __forceinline__ void at_issue_scores(const AtSmem& sm, uint32_t tmem, int st, int hd) {
  const uint32_t idesc = (1u << 4) | ((uint32_t)(AT_KEYS >> 3) << 17) | ((uint32_t)(AT_ROWS >> 4) << 24);
  const uint32_t qb = smem_u32(sm.qs), kb = smem_u32(sm.kvs + (size_t)st * 2 * sm.kv_tile);
  for (int kk = 0; kk < hd / 16; kk++) {
    const uint64_t kd = at_desc(kb + kk * 2 * (AT_KEYS * 16), AT_KEYS * 16, 128);
    tc_mma(tmem, at_desc(qb + kk * 2 * (AT_ROWS * 16), AT_ROWS * 16, 128), kd, idesc, kk > 0 ? 1u : 0u);
    tc_mma(tmem, at_desc(qb + sm.q_piece + kk * 2 * (AT_ROWS * 16), AT_ROWS * 16, 128), kd, idesc, 1u);
  }
  tc_commit(sm.bar);
}

// O = Ph.V + Pl.V into TMEM columns [128, 128 + hd) (V as the MN-major B).
__device__ __forceinline__ void at_issue_values(const AtSmem& sm, uint32_t tmem, int st, int hd) {
  const uint32_t idesc = (1u << 4) | (1u << 16) | ((uint32_t)(hd >> 3) << 17) | ((uint32_t)(AT_ROWS >> 4) << 24);
  const uint32_t pb = smem_u32(sm.ps), vb = smem_u32(sm.kvs + (size_t)st * 2 * sm.kv_tile) + sm.kv_tile;
  for (int kk = 0; kk < AT_KEYS / 16; kk++) {
    const uint64_t vd = at_desc(vb + kk * 2 * 128, 128, AT_KEYS * 16);
    tc_mma(tmem + 128, at_desc(pb + kk * 2 * (AT_ROWS * 16), AT_ROWS * 16, 128), vd, idesc, kk > 0 ? 1u : 0u);
    tc_mma(tmem + 128, at_desc(pb + sm.p_piece + kk * 2 * (AT_ROWS * 16), AT_ROWS * 16, 128), vd, idesc, 1u);
  }
  tc_commit(sm.bar);
}

// This thread's 64 scores from TMEM (its warp's lanes).
__device__ __forceinline__ void at_ld_scores(uint32_t tmem, float (&sc)[AT_KEYS]) {
  const uint32_t lane_base = (uint32_t)((threadIdx.x >> 5) * 32) << 16;
#pragma unroll
  for (int j = 0; j < AT_KEYS / 16; j++) {
    uint32_t r[16];
    at_ld16(tmem + lane_base + j * 16, r);
    at_wait_ld();
#pragma unroll
    for (int i = 0; i < 16; i++) sc[j * 16 + i] = __uint_as_float(r[i]);
  }
}

// This thread's softmax weights as the binary16 pair of its P row.
__device__ __forceinline__ void at_write_p(const AtSmem& sm, const float (&p)[AT_KEYS]) {
#pragma unroll
  for (int c = 0; c < AT_KEYS / 8; c++) {
    uint32_t h[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; j++) at_split2(p[8 * c + 2 * j], p[8 * c + 2 * j + 1], h[j], lo[j]);
    *reinterpret_cast<uint4*>(sm.ps + c * (AT_ROWS * 16) + threadIdx.x * 16) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(sm.ps + sm.p_piece + c * (AT_ROWS * 16) + threadIdx.x * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// grid: (ceil(nshared / per), KVH, ceil(M * G / 128)); AT_THREADS threads.
// Splits [blockIdx.x * per, min(nshared, +per)) of KV head blockIdx.y.
// Requires a.kv.half, a.hd % 16 == 0, a.hd <= 256, a.split == AT_KEYS.
__global__ void __launch_bounds__(AT_THREADS) k_attn_shared_tc(DecodeAttnArgs a, int nshared, int per, int* err) {
  extern __shared__ __align__(128) uint8_t at_smem[];
  const int hd = a.hd, g = blockIdx.y, G = a.H / a.KVH, nrow = a.M * G;
  const int q0 = blockIdx.z * AT_ROWS;
  const int s_lo = blockIdx.x * per, s_hi = min(nshared, s_lo + per);
  const int tid = threadIdx.x;
  if (s_lo >= s_hi) return;
  const AtSmem sm = at_carve(at_smem, hd);
  at_begin(sm);

  // Query rows: float32 staging in the K/V buffers (128 x hd floats fill
  // them exactly), then RoPE at the row's position and the binary16 pair.
  float* qf = reinterpret_cast<float*>(sm.kvs);
  for (int e = tid; e < AT_ROWS * hd; e += AT_THREADS) {
    const int qi = e / hd, i = e % hd, row = q0 + qi;
    qf[e] = row < nrow ? a.qkv[(size_t)(row / G) * a.qkv_stride + (g * G + row % G) * hd + i] : 0.f;
  }
  __syncthreads();
  const int row = q0 + tid;
  const bool valid = row < nrow;
  const int sx = at_q_pieces<true>(sm, qf + tid * hd, valid, hd, a.rope, valid ? a.pos[row / G] : 0);
  const float unscale = tc_pow2(-sx);
  tc_fence_before();
  __syncthreads();  // staging read; the K/V buffers are free
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm.tslot);
  const int last = nshared * AT_KEYS - 1;
  at_load_kv(sm, 0, a.kv, a.layer, a.page_table, g, s_lo * AT_KEYS, last, hd);

  uint32_t phase = 0;
  for (int s = s_lo; s < s_hi; s++) {
    const int st = (s - s_lo) & 1;
    if (s + 1 < s_hi) {
      at_load_kv(sm, st ^ 1, a.kv, a.layer, a.page_table, g, (s + 1) * AT_KEYS, last, hd);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    at_publish();
    if (tid == 0) at_issue_scores(sm, tmem, st, hd);
    if (at_wait_mma(sm, phase, err)) break;
    float sc[AT_KEYS];
    at_ld_scores(tmem, sc);
    float m = -INFINITY;
#pragma unroll
    for (int t = 0; t < AT_KEYS; t++) {
      sc[t] = __fdiv_rn(sc[t] * unscale, a.scale);
      m = fmaxf(m, sc[t]);
    }
    float l = 0.f;
#pragma unroll
    for (int t = 0; t < AT_KEYS; t++) {
      sc[t] = expf(sc[t] - m);
      l += sc[t];
    }
    at_write_p(sm, sc);
    at_publish();
    if (tid == 0) at_issue_values(sm, tmem, st, hd);
    if (at_wait_mma(sm, phase, err)) break;
    float* part = valid ? a.part + (((size_t)(row / G) * a.H + g * G + row % G) * a.max_splits + s) * (hd + 2) : nullptr;
    const uint32_t lane_base = (uint32_t)((tid >> 5) * 32) << 16;
    for (int c0 = 0; c0 < hd; c0 += 16) {
      uint32_t r[16];
      at_ld16(tmem + lane_base + 128 + c0, r);
      at_wait_ld();
      if (valid) {
#pragma unroll
        for (int i = 0; i < 16; i += 2) *reinterpret_cast<float2*>(part + c0 + i) = make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1]));
      }
    }
    if (valid) *reinterpret_cast<float2*>(part + hd) = make_float2(m, l);
  }
  at_end(sm, tmem);
}

// Causal attention of a prefill chunk (attention.go:6-45: query i at
// position start + i attends to positions [0, start + i]; q already
// rotated) on the tensor cores, binary16 KV. One CTA per (tile of 128
// queries, query head); 64-position key blocks in order with the online
// softmax of k_attn_prefill: per block s = S 2^-sx / sqrt(hd), masked past
// the query's position, m' = max(m, block max), alpha = expf(m - m'),
// p = expf(s - m'), l = l alpha + sum p, o = o alpha + P V (the block's
// P V from TMEM), out = o / l. NC = hd / 16.
template <int NC>
__global__ void __launch_bounds__(AT_THREADS) k_attn_prefill_tc(PrefillAttnArgs a, int* err) {
  extern __shared__ __align__(128) uint8_t at_smem[];
  constexpr int HD = 16 * NC;
  const int h = blockIdx.y, g = h / (a.H / a.KVH);
  const int q0 = blockIdx.x * AT_ROWS, nq = min(AT_ROWS, a.n - q0);
  const int tid = threadIdx.x;
  const AtSmem sm = at_carve(at_smem, HD);
  at_begin(sm);
  float* qf = reinterpret_cast<float*>(sm.kvs);
  for (int e = tid; e < AT_ROWS * HD; e += AT_THREADS) {
    const int qi = e / HD, i = e % HD;
    qf[e] = qi < nq ? a.qkv[(size_t)(q0 + qi) * a.qkv_stride + h * HD + i] : 0.f;
  }
  __syncthreads();
  const bool valid = tid < nq;
  const int sx = at_q_pieces<false>(sm, qf + tid * HD, valid, HD, Rope{}, 0);
  const float unscale = tc_pow2(-sx);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm.tslot);
  const int last = a.start + q0 + nq - 1;
  const int qpos = valid ? a.start + q0 + tid : last;  // rows past the chunk copy the last row's mask
  const int nblk = last / AT_KEYS + 1;
  at_load_kv(sm, 0, a.kv, a.layer, a.page_table, g, 0, last, HD);

  float o[HD];
#pragma unroll
  for (int c = 0; c < HD; c++) o[c] = 0.f;
  float m = -INFINITY, l = 0.f;
  uint32_t phase = 0;
  const uint32_t lane_base = (uint32_t)((tid >> 5) * 32) << 16;
  for (int j = 0; j < nblk; j++) {
    const int st = j & 1, t0 = j * AT_KEYS;
    if (j + 1 < nblk) {
      at_load_kv(sm, st ^ 1, a.kv, a.layer, a.page_table, g, t0 + AT_KEYS, last, HD);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    at_publish();
    if (tid == 0) at_issue_scores(sm, tmem, st, HD);
    if (at_wait_mma(sm, phase, err)) break;
    float sc[AT_KEYS];
    at_ld_scores(tmem, sc);
    float mb = -INFINITY;
#pragma unroll
    for (int t = 0; t < AT_KEYS; t++) {
      sc[t] = t0 + t <= qpos ? __fdiv_rn(sc[t] * unscale, a.scale) : -INFINITY;
      mb = fmaxf(mb, sc[t]);
    }
    const float mnew = fmaxf(m, mb);
    const float alpha = m == -INFINITY ? 0.f : expf(m - mnew);
    float ls = 0.f;
#pragma unroll
    for (int t = 0; t < AT_KEYS; t++) {
      sc[t] = sc[t] == -INFINITY ? 0.f : expf(sc[t] - mnew);
      ls += sc[t];
    }
    l = l * alpha + ls;
    m = mnew;
    at_write_p(sm, sc);
    at_publish();
    if (tid == 0) at_issue_values(sm, tmem, st, HD);
    if (at_wait_mma(sm, phase, err)) break;
#pragma unroll
    for (int c0 = 0; c0 < HD; c0 += 16) {
      uint32_t r[16];
      at_ld16(tmem + lane_base + 128 + c0, r);
      at_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; i++) o[c0 + i] = __fadd_rn(__fmul_rn(o[c0 + i], alpha), __uint_as_float(r[i]));
    }
  }
  if (valid) {
    float* out = a.out + (size_t)(q0 + tid) * a.out_stride + h * HD;
#pragma unroll
    for (int c = 0; c < HD; c++) out[c] = __fdiv_rn(o[c], l);
  }
  at_end(sm, tmem);
}

}  // namespace tcu
