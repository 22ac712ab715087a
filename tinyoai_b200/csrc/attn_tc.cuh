// Attention on the 5th-generation tensor cores (binary16 KV).
//
// k_attn_shared_tc: branches of one prefix (mlx_branches.go:98-114) all read
// the prefix's KV pages. For every query row of the branch batch it attends
// to a run of whole 64-position splits of that prefix and writes the run's
// partial (sum_t exp(s_t - m) v_t, m, sum_t exp(s_t - m)) for the per-row
// kernels to merge with the rest of the row's history.
//
// k_attn_prefill_tc: causal attention of a prefill chunk (attention.go:6-45).
//
// Both take 128 query rows per CTA as the MMA's M. Per 64-position block:
//   S = Q K^T      tcgen05.mma M = 128, N = 64, K = hd. The binary16 keys
//                  are exact operands; each float32 query row is scaled by
//                  2^sx (sx = 13 - exponent of its max) and split into an
//                  exact binary16 pair Qh + Ql (22 of its 24 bits), so
//                  S = Qh.K + Ql.K is accumulated in float32.
//   s = S * (2^-sx / sqrt(hd)), m' = max(m, block max),
//   p = 2^((s - m') log2 e) (ex2.approx), alpha = 2^((m - m') log2 e),
//   l = l alpha + sum p in position order (one thread per query row, scores
//   read from TMEM).
//   O = P V        M = 128, N = hd, K = 64 positions; P split into a
//                  binary16 pair Ph + Pl, V exact; o = o alpha + O in
//                  registers.
// Scaling by the reciprocal, ex2.approx and the dropped 2^-22 terms put the
// results ~1e-6 (relative) from the float32 CUDA-core kernels, not bit for
// bit.
//
// Work is done by groups of four warps (128 threads, one per query row and
// TMEM lane). A group owns a P tile, two K/V stages, an mbarrier, a named
// barrier and 256 TMEM columns (scores at 0, block outputs at 128); one
// thread of the group issues its MMAs. cp.async brings the group's next K/V
// block while the current one is computed. The prefill kernel runs two
// groups on alternate key blocks (when shared memory allows) and merges
// their states at the end; the shared kernel runs one group, two CTAs per
// SM.
//
// Shared-memory operands use the no-swizzle K-major / MN-major layouts of
// 8-row x 16-byte core matrices. A K or V tile is stored [hd/8 chunks][64
// positions][8 values], so chunk c of position t is at c * 1024 + t * 16:
// as the B operand of S (K-major over hd) core matrices step 128 bytes over
// positions and 1024 over hd; as the B operand of O (MN-major: N = hd
// contiguous) they step 1024 bytes over hd and 128 over positions. Q and P
// tiles are [chunks][128 rows][8 values] (K-major A, 2048 bytes per chunk).
// The regions are ordered P, Q, K/V, so that every operand read stays inside
// the CTA's allocation under either reading of the two descriptor strides.
// All copies read this GPU's own memory into this CTA's shared memory;
// every mbarrier wait is bounded.
#pragma once
#include <climits>

#include "attention.cuh"
#include "gemm_tc.cuh"

namespace tcu {

constexpr int AT_ROWS = 128;   // query rows per CTA (MMA M)
constexpr int AT_KEYS = 64;    // positions per block (one split)
constexpr int AT_GROUP = 128;  // threads per group: one per query row / TMEM lane
constexpr float AT_LOG2E = 1.4426950408889634f;
// Page ids a CTA copies into shared memory up front (192: two shared-prefix
// CTAs at hd = 80 still fit one SM's 228 KB with their 1 KB reserves).
constexpr int AT_PAGE_CACHE = 192;

// Dynamic shared memory for head size hd (multiple of 16) and ng groups:
// P tiles ng x 2 x 128 x 64, Q pieces 2 x 128 x hd, K/V ng x 2 stages x 2 x
// 64 x hd (binary16), the mbarriers, the TMEM slot and a copy of the page
// ids the CTA reads. At least 80 KB, so that at most two CTAs (2 x 256 TMEM
// columns) share an SM.
__host__ __device__ inline size_t at_smem_bytes(int hd, int ng) {
  const size_t b = (size_t)ng * 4 * AT_ROWS * AT_KEYS + (size_t)4 * AT_ROWS * hd + (size_t)ng * 8 * AT_KEYS * hd + 64 + 4 * AT_PAGE_CACHE;
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

// 2^x (PTX ex2.approx; 2^-inf = +0).
__device__ __forceinline__ float at_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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

// Binary16 pair (h, l) of two floats: h = fp16(v), l = fp16(v - h).
__device__ __forceinline__ void at_split2(float v0, float v1, uint32_t& h, uint32_t& l) {
  const __half2 hh = __floats2half2_rn(v0, v1);
  const float2 hf = __half22float2(hh);
  const __half2 ll = __floats2half2_rn(__fsub_rn(v0, hf.x), __fsub_rn(v1, hf.y));
  h = *reinterpret_cast<const uint32_t*>(&hh);
  l = *reinterpret_cast<const uint32_t*>(&ll);
}

// The CTA's shared regions: the Q tiles (one copy for all groups), the
// mbarriers and the TMEM slot.
struct AtSmem {
  uint8_t* qs;  // [2 pieces][hd/8 chunks][128 rows][16 B]
  uint32_t q_piece;
  uint64_t* bars;  // one per group
  uint32_t* tslot;
  int* pages;      // [AT_PAGE_CACHE]
  int hd;
};

// One group's resources.
struct AtGroup {
  uint8_t* ps;   // [2 pieces][8 chunks][128 rows][16 B]
  uint8_t* kvs;  // [2 stages][K, V][hd/8 chunks][64 positions][16 B]
  uint64_t* bar;
  uint32_t tmem;  // this group's 256 columns
  int id;         // named barrier of the group: 1 + group index
  int tid;        // thread within the group (query row / TMEM lane)
};

__device__ __forceinline__ AtSmem at_carve(uint8_t* base, int hd, int ng) {
  AtSmem m;
  m.qs = base + (size_t)ng * 4 * AT_ROWS * AT_KEYS;
  m.q_piece = 2 * AT_ROWS * hd;
  m.bars = reinterpret_cast<uint64_t*>(m.qs + 4 * AT_ROWS * hd + (size_t)ng * 8 * AT_KEYS * hd);
  m.tslot = reinterpret_cast<uint32_t*>(m.bars + ng);
  m.pages = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(m.bars) + 64);
  m.hd = hd;
  return m;
}

__device__ __forceinline__ AtGroup at_group(uint8_t* base, const AtSmem& sm, int g) {
  AtGroup G;
  G.ps = base + (size_t)g * 4 * AT_ROWS * AT_KEYS;
  G.kvs = sm.qs + 4 * AT_ROWS * sm.hd + (size_t)g * 8 * AT_KEYS * sm.hd;
  G.bar = sm.bars + g;
  G.tmem = 0;
  G.id = 1 + g;
  G.tid = threadIdx.x - g * AT_GROUP;
  return G;
}

// Barrier init (thread 0) and the TMEM allocation, 256 columns per group
// (warp 0).
__device__ __forceinline__ void at_begin(const AtSmem& sm, int ng) {
  if (threadIdx.x == 0) {
    for (int g = 0; g < ng; g++) mbar_init(sm.bars + g, 1);
    fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(sm.tslot)), "r"(256u * ng));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
}

__device__ __forceinline__ void at_end(uint32_t tmem, int ng) {
  cp_async_wait<0>();
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256u * ng));
  }
}

// The power of two sx of query row x (float32, hd values, already rotated):
// 13 - exponent of its largest magnitude.
__device__ __forceinline__ int at_q_sx(const float* x, bool valid, int hd) {
  float mx = 0.f;
  if (valid)
    for (int k = 0; k < hd; k++) mx = fmaxf(mx, fabsf(x[k]));
  int ex = 0;
  if (mx > 0.f) frexpf(mx, &ex);
  return mx > 0.f ? 13 - ex : 0;
}

// That row as the binary16 pair of x * 2^sx into row `row` of the Q tiles.
__device__ __forceinline__ void at_q_write(const AtSmem& sm, int row, const float* x, bool valid, int sx) {
  const float qscale = tc_pow2(sx);
  for (int c = 0; c < sm.hd / 8; c++) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int k = 8 * c + 2 * j;
      const float v0 = valid ? x[k] : 0.f;
      const float v1 = valid ? x[k + 1] : 0.f;
      at_split2(v0 * qscale, v1 * qscale, h[j], l[j]);
    }
    *reinterpret_cast<uint4*>(sm.qs + c * (AT_ROWS * 16) + row * 16) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(sm.qs + sm.q_piece + c * (AT_ROWS * 16) + row * 16) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// Where a CTA reads page ids: page index i is pt[i - base] (a copy of the
// CTA's range in shared memory, or the page table itself).
struct AtPages {
  const int* pt;
  int base;
};

// Copies page ids [first, first + count) into shared memory when they fit
// (every thread of the CTA calls this; a CTA barrier must follow).
__device__ __forceinline__ AtPages at_cache_pages(const AtSmem& sm, const int* page_table, int first, int count) {
  if (count > AT_PAGE_CACHE) return AtPages{page_table, 0};
  for (int i = threadIdx.x; i < count; i += blockDim.x) sm.pages[i] = page_table[first + i];
  return AtPages{sm.pages, first};
}

// Keys and values of positions [t0, t0 + 64) of KV head g into the group's
// stage st (chunk c of position t at c * 1024 + t * 16); positions past
// `last` are zero (their weights are zero, and zero values keep the
// products finite). Each thread looks up one position's page.
__device__ __forceinline__ void at_load_kv(const AtGroup& G, int hd, int st, const KVView& kv, int layer, AtPages pages, int g,
                                           int t0, int last) {
  uint8_t* kb = G.kvs + (size_t)st * 4 * AT_KEYS * hd;
  uint8_t* vb = kb + 2 * AT_KEYS * hd;
  const int t = G.tid % AT_KEYS, ta = t0 + t;
  const bool ok = ta <= last;
  size_t base = 0;
  if (ok) base = kv.off(layer, pages.pt[ta / kv.P - pages.base], g, ta % kv.P);
  for (int c = G.tid / AT_KEYS; c < hd / 8; c += AT_GROUP / AT_KEYS) {
    const int so = c * (AT_KEYS * 16) + t * 16;
    if (ok) {
      cp_async16(kb + so, reinterpret_cast<const __half*>(kv.k) + base + 8 * c);
      cp_async16(vb + so, reinterpret_cast<const __half*>(kv.v) + base + 8 * c);
    } else {
      *reinterpret_cast<uint4*>(kb + so) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(vb + so) = make_uint4(0, 0, 0, 0);
    }
  }
  cp_async_commit();
}

// Makes this thread's shared-memory writes (copies, P tiles) visible to the
// tensor core, then synchronises the group.
__device__ __forceinline__ void at_publish(const AtGroup& G) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  named_bar_sync(G.id, AT_GROUP);
  tc_fence_after();
}

// Waits for the group's last MMA commit; true on every thread of the group
// if any thread's wait ran out (the group then leaves its loop together).
__device__ __forceinline__ bool at_wait_mma(const AtGroup& G, uint32_t& phase, int* err) {
  const int ok = mbar_wait(G.bar, phase, err) ? 1 : 0;
  int all;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.b32 p, %1, 0;\n barrier.red.and.pred q, %2, %3, p;\n selp.b32 %0, 1, 0, q;\n}\n"
      : "=r"(all)
      : "r"(ok), "r"(G.id), "r"(AT_GROUP)
      : "memory");
  phase ^= 1;
  tc_fence_after();
  return all == 0;
}

// S = Qh.K + Ql.K into the group's TMEM columns [0, 64).
__device__ __forceinline__ void at_issue_scores(const AtSmem& sm, const AtGroup& G, int st) {
  const int hd = sm.hd;
  const uint32_t idesc = (1u << 4) | ((uint32_t)(AT_KEYS >> 3) << 17) | ((uint32_t)(AT_ROWS >> 4) << 24);
  const uint32_t qb = smem_u32(sm.qs), kb = smem_u32(G.kvs + (size_t)st * 4 * AT_KEYS * hd);
  for (int kk = 0; kk < hd / 16; kk++) {
    const uint64_t kd = at_desc(kb + kk * 2 * (AT_KEYS * 16), AT_KEYS * 16, 128);
    tc_mma(G.tmem, at_desc(qb + kk * 2 * (AT_ROWS * 16), AT_ROWS * 16, 128), kd, idesc, kk > 0 ? 1u : 0u);
    tc_mma(G.tmem, at_desc(qb + sm.q_piece + kk * 2 * (AT_ROWS * 16), AT_ROWS * 16, 128), kd, idesc, 1u);
  }
  tc_commit(G.bar);
}

// O = Ph.V + Pl.V into the group's TMEM columns [128, 128 + hd) (V as the
// MN-major B operand).
__device__ __forceinline__ void at_issue_values(const AtSmem& sm, const AtGroup& G, int st) {
  const int hd = sm.hd;
  const uint32_t idesc = (1u << 4) | (1u << 16) | ((uint32_t)(hd >> 3) << 17) | ((uint32_t)(AT_ROWS >> 4) << 24);
  const uint32_t pb = smem_u32(G.ps), vb = smem_u32(G.kvs + (size_t)st * 4 * AT_KEYS * hd) + 2 * AT_KEYS * hd;
  const uint32_t p_piece = 2 * AT_ROWS * AT_KEYS;
  for (int kk = 0; kk < AT_KEYS / 16; kk++) {
    const uint64_t vd = at_desc(vb + kk * 2 * 128, 128, AT_KEYS * 16);
    tc_mma(G.tmem + 128, at_desc(pb + kk * 2 * (AT_ROWS * 16), AT_ROWS * 16, 128), vd, idesc, kk > 0 ? 1u : 0u);
    tc_mma(G.tmem + 128, at_desc(pb + p_piece + kk * 2 * (AT_ROWS * 16), AT_ROWS * 16, 128), vd, idesc, 1u);
  }
  tc_commit(G.bar);
}

// This thread's 64 scores from TMEM, times k.
__device__ __forceinline__ void at_ld_scores(const AtGroup& G, float k, float (&sc)[AT_KEYS]) {
  const uint32_t lane_base = (uint32_t)((G.tid >> 5) * 32) << 16;
  uint32_t r[AT_KEYS / 16][16];
#pragma unroll
  for (int j = 0; j < AT_KEYS / 16; j++) at_ld16(G.tmem + lane_base + j * 16, r[j]);
  at_wait_ld();
#pragma unroll
  for (int j = 0; j < AT_KEYS / 16; j++)
#pragma unroll
    for (int i = 0; i < 16; i++) sc[j * 16 + i] = __uint_as_float(r[j][i]) * k;
}

// This thread's softmax weights as the binary16 pair of its P row.
__device__ __forceinline__ void at_write_p(const AtGroup& G, const float (&p)[AT_KEYS]) {
  const uint32_t p_piece = 2 * AT_ROWS * AT_KEYS;
#pragma unroll
  for (int c = 0; c < AT_KEYS / 8; c++) {
    uint32_t h[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; j++) at_split2(p[8 * c + 2 * j], p[8 * c + 2 * j + 1], h[j], lo[j]);
    *reinterpret_cast<uint4*>(G.ps + c * (AT_ROWS * 16) + G.tid * 16) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(G.ps + p_piece + c * (AT_ROWS * 16) + G.tid * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// The online softmax of one block (scores in natural units, -inf where
// masked): updates the running (m, l), turns sc into the block's weights
// and returns alpha, the factor for the running outputs. A row that has seen
// no visible position yet (a group's first blocks past its causal limit)
// keeps m = -inf, l = 0 and gets zero weights.
__device__ __forceinline__ float at_softmax(float (&sc)[AT_KEYS], float& m, float& l) {
  float mb = m;
#pragma unroll
  for (int t = 0; t < AT_KEYS; t++) mb = fmaxf(mb, sc[t]);
  const float alpha = m == -INFINITY ? 0.f : at_ex2((m - mb) * AT_LOG2E);
  const float mref = mb == -INFINITY ? 0.f : mb;  // -inf - -inf would be NaN
  float ls = 0.f;
#pragma unroll
  for (int t = 0; t < AT_KEYS; t++) {
    sc[t] = at_ex2((sc[t] - mref) * AT_LOG2E);
    ls += sc[t];
  }
  l = l * alpha + ls;
  m = mb;
  return alpha;
}

// o = o alpha + (the block's P V from TMEM; all columns loaded, then one wait).
template <int HD>
__device__ __forceinline__ void at_acc_values(const AtGroup& G, float alpha, float (&o)[HD]) {
  const uint32_t lane_base = (uint32_t)((G.tid >> 5) * 32) << 16;
  uint32_t r[HD / 16][16];
#pragma unroll
  for (int c = 0; c < HD / 16; c++) at_ld16(G.tmem + lane_base + 128 + 16 * c, r[c]);
  at_wait_ld();
#pragma unroll
  for (int c = 0; c < HD / 16; c++)
#pragma unroll
    for (int i = 0; i < 16; i++) o[16 * c + i] = fmaf(o[16 * c + i], alpha, __uint_as_float(r[c][i]));
}

// One group's pass over key blocks j = j0, j0 + step, ... < nblk of KV head
// kvh: the online softmax state (o, m, l) of the group's query rows. qpos:
// this row's last visible position (causal mask), or INT_MAX.
template <int HD>
__device__ __forceinline__ void at_blocks(const AtSmem& sm, const AtGroup& G, const KVView& kv, int layer, AtPages pages, int kvh,
                                          int j0, int step, int nblk, int last, int qpos, float k, int* err, float (&o)[HD], float& m,
                                          float& l) {
#pragma unroll
  for (int c = 0; c < HD; c++) o[c] = 0.f;
  m = -INFINITY;
  l = 0.f;
  if (j0 >= nblk) return;
  uint32_t phase = 0;
  at_load_kv(G, HD, 0, kv, layer, pages, kvh, j0 * AT_KEYS, last);
  for (int j = j0, it = 0; j < nblk; j += step, it++) {
    const int st = it & 1, t0 = j * AT_KEYS;
    if (j + step < nblk) {
      at_load_kv(G, HD, st ^ 1, kv, layer, pages, kvh, t0 + step * AT_KEYS, last);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    at_publish(G);
    if (G.tid == 0) at_issue_scores(sm, G, st);
    if (at_wait_mma(G, phase, err)) break;
    float sc[AT_KEYS];
    at_ld_scores(G, k, sc);
    if (qpos < t0 + AT_KEYS - 1) {
#pragma unroll
      for (int t = 0; t < AT_KEYS; t++)
        if (t0 + t > qpos) sc[t] = -INFINITY;
    }
    const float alpha = at_softmax(sc, m, l);
    at_write_p(G, sc);
    at_publish(G);
    if (G.tid == 0) at_issue_values(sm, G, st);
    if (at_wait_mma(G, phase, err)) break;
    at_acc_values<HD>(G, alpha, o);
  }
}

// grid: (runs, KVH, ceil(M * G / 128)); 128 threads (one group); HD = hd.
// Run r covers splits [r * per, min(nshared, (r + 1) * per)) of KV head
// blockIdx.y and writes its partial into slot r of each row's partials.
// Requires a.kv.half and a.split == AT_KEYS.
template <int HD>
__global__ void __launch_bounds__(AT_GROUP) k_attn_shared_tc(DecodeAttnArgs a, int nshared, int per, int* err) {
  extern __shared__ __align__(128) uint8_t at_smem[];
  const int kvh = blockIdx.y, Gq = a.H / a.KVH, nrow = a.M * Gq;
  const int q0 = blockIdx.z * AT_ROWS;
  const int s_lo = blockIdx.x * per, s_hi = min(nshared, s_lo + per);
  const int tid = threadIdx.x;
  if (s_lo >= s_hi) return;
  const AtSmem sm = at_carve(at_smem, HD, 1);
  AtGroup G = at_group(at_smem, sm, 0);
  at_begin(sm, 1);

  // Query rows: float32 staging in the K/V buffers (128 x hd floats fill
  // them exactly), rotated in place at each row's position (one rotary pair
  // per thread and step, as rope_pair does it), then the binary16 pair.
  float* qf = reinterpret_cast<float*>(G.kvs);
  constexpr int C4 = HD / 4;
#pragma unroll 4
  for (int e = tid; e < AT_ROWS * C4; e += AT_GROUP) {
    const int qi = e / C4, c = e % C4, row = q0 + qi;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < nrow) v = *reinterpret_cast<const float4*>(a.qkv + (size_t)(row / Gq) * a.qkv_stride + (kvh * Gq + row % Gq) * HD + 4 * c);
    reinterpret_cast<float4*>(qf)[e] = v;
  }
  const int first_page = s_lo * AT_KEYS / a.kv.P;
  const AtPages pages = at_cache_pages(sm, a.page_table, first_page, (s_hi * AT_KEYS - 1) / a.kv.P - first_page + 1);
  __syncthreads();
  const int nq = min(AT_ROWS, nrow - q0);
  for (int e = tid; e < nq * a.rope.pairs; e += AT_GROUP) {
    const int qi = e / a.rope.pairs;
    rope_pair(qf + qi * HD, e % a.rope.pairs, a.rope, a.pos[(q0 + qi) / Gq]);
  }
  __syncthreads();
  const int row = q0 + tid;
  const bool valid = row < nrow;
  const int sx = at_q_sx(qf + tid * HD, valid, HD);
  at_q_write(sm, tid, qf + tid * HD, valid, sx);
  const float k = tc_pow2(-sx) * (1.f / a.scale);
  tc_fence_before();
  __syncthreads();  // staging read; the K/V buffers are free
  tc_fence_after();
  G.tmem = *reinterpret_cast<volatile uint32_t*>(sm.tslot);

  float o[HD], m, l;
  at_blocks<HD>(sm, G, a.kv, a.layer, pages, kvh, s_lo, 1, s_hi, nshared * AT_KEYS - 1, INT_MAX, k, err, o, m, l);
  if (valid) {
    float* part = a.part + (((size_t)(row / Gq) * a.H + kvh * Gq + row % Gq) * a.max_splits + blockIdx.x) * (HD + 2);
#pragma unroll
    for (int c = 0; c < HD; c += 2) *reinterpret_cast<float2*>(part + c) = make_float2(o[c], o[c + 1]);
    *reinterpret_cast<float2*>(part + HD) = make_float2(m, l);
  }
  at_end(G.tmem, 1);
}

// Causal attention of a prefill chunk (attention.go:6-45: query i at
// position start + i attends to positions [0, start + i]; q already
// rotated). grid: (ceil(n / 128), H); NG groups of 128 threads take
// alternate 64-position key blocks; group 0 merges their states and writes
// out = o / l. HD = hd.
template <int HD, int NG>
__global__ void __launch_bounds__(AT_GROUP * NG) k_attn_prefill_tc(PrefillAttnArgs a, int* err) {
  extern __shared__ __align__(128) uint8_t at_smem[];
  const int h = blockIdx.y, kvh = h / (a.H / a.KVH);
  const int q0 = blockIdx.x * AT_ROWS, nq = min(AT_ROWS, a.n - q0);
  const int tid = threadIdx.x;
  const AtSmem sm = at_carve(at_smem, HD, NG);
  AtGroup G = at_group(at_smem, sm, tid / AT_GROUP);
  at_begin(sm, NG);
  float* qf = reinterpret_cast<float*>(sm.qs + 4 * AT_ROWS * HD);  // group 0's K/V stages
  constexpr int C4 = HD / 4;
#pragma unroll 4
  for (int e = tid; e < AT_ROWS * C4; e += AT_GROUP * NG) {
    const int qi = e / C4, c = e % C4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (qi < nq) v = *reinterpret_cast<const float4*>(a.qkv + (size_t)(q0 + qi) * a.qkv_stride + h * HD + 4 * c);
    reinterpret_cast<float4*>(qf)[e] = v;
  }
  const AtPages pages = at_cache_pages(sm, a.page_table, 0, (a.start + q0 + nq - 1) / a.kv.P + 1);
  __syncthreads();
  const int r = G.tid;
  const bool valid = r < nq;
  const int sx = at_q_sx(qf + r * HD, valid, HD);
  if (G.id == 1) at_q_write(sm, r, qf + r * HD, valid, sx);
  const float k = tc_pow2(-sx) * (1.f / a.scale);
  tc_fence_before();
  __syncthreads();  // staging read; the K/V buffers are free
  tc_fence_after();
  const uint32_t tmem0 = *reinterpret_cast<volatile uint32_t*>(sm.tslot);
  G.tmem = tmem0 + 256u * (G.id - 1);
  const int last = a.start + q0 + nq - 1;
  const int qpos = valid ? a.start + q0 + r : last;  // rows past the chunk copy the last row's mask
  const int nblk = last / AT_KEYS + 1;

  float o[HD], m, l;
  at_blocks<HD>(sm, G, a.kv, a.layer, pages, kvh, G.id - 1, NG, nblk, last, qpos, k, err, o, m, l);
  if (NG > 1) {
    // Group 1 hands (o, m, l) to group 0 through the Q and K/V buffers
    // ([HD + 2][128] floats), after every group's copies and MMAs are done.
    cp_async_wait<0>();
    tc_fence_before();
    __syncthreads();
    float* xs = reinterpret_cast<float*>(sm.qs);
    if (G.id == 2) {
#pragma unroll
      for (int c = 0; c < HD; c++) xs[c * AT_ROWS + r] = o[c];
      xs[HD * AT_ROWS + r] = m;
      xs[(HD + 1) * AT_ROWS + r] = l;
    }
    __syncthreads();
    if (G.id == 1) {
      const float m1 = xs[HD * AT_ROWS + r], l1 = xs[(HD + 1) * AT_ROWS + r];
      const float mm = fmaxf(m, m1);
      const float a0 = m == -INFINITY ? 0.f : at_ex2((m - mm) * AT_LOG2E);
      const float a1 = m1 == -INFINITY ? 0.f : at_ex2((m1 - mm) * AT_LOG2E);
      l = l * a0 + l1 * a1;
#pragma unroll
      for (int c = 0; c < HD; c++) o[c] = o[c] * a0 + xs[c * AT_ROWS + r] * a1;
    }
  }
  if (G.id == 1 && valid) {
    float* out = a.out + (size_t)(q0 + r) * a.out_stride + h * HD;
    const float inv = 1.f / l;
#pragma unroll
    for (int c = 0; c < HD; c++) out[c] = o[c] * inv;
  }
  at_end(tmem0, NG);
}

}  // namespace tcu
