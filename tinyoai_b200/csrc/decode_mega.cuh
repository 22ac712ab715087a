// Persistent decode step for one StableLM sequence with Q8_0 weights: the
// whole forward of one token (stablelm.go:332-387) in a single cooperative
// launch.
//
// Grid = one CTA per SM. Warp 8 lane 0 is the producer: it walks the CTA's
// fixed schedule for the step -- per layer its share of the fused
// q/k/v/gate/up rows, its attention units' KV page tiles, its share of the
// fused out/down rows; then its share of the lm_head rows -- and streams each
// piece into a shared-memory ring of slots with cp.async.bulk, running ahead
// across phase boundaries. Warps 0..7 consume in the same order. Phases that
// need every CTA's results are separated by a grid barrier (bounded spin);
// the producer keeps prefetching through it.
//
// Matrix-vector products use exact integer dot products (dp4a): the input
// vector is quantised per 16-value block to 24-bit fixed point relative to the
// block's largest magnitude (absolute error at most half an ulp of that
// value) and split into three byte digits, so every block sum of int8 weight
// x digit is exact in int32; the digit sums are recombined in float32 and
// scaled by the weight and input block scales (dot.go:31-40 computes the
// weight-block sums in float64). LayerNorm, RoPE, attention and the parallel
// residual follow the reference arithmetic as the separate kernels do.
//
// The input of the out/down rows ([attention | SwiGLU]) is quantised once,
// by the CTA that produces each block (the attention merge, the SwiGLU rows),
// and published as digits; every CTA then copies the digits in with one bulk
// copy instead of quantising the whole vector itself.
#pragma once
#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "tma.cuh"

namespace tcu {

constexpr int MG_CW = 8;                      // consumer warps
constexpr int MG_THREADS = (MG_CW + 1) * 32;  // + producer warp
constexpr int MG_CT = MG_CW * 32;
constexpr int MG_MAX_SLOTS = 6;
constexpr int MG_W1_RS = 16;  // rows per stage, q/k/v/gate/up and head
constexpr int MG_W2_RS = 4;   // rows per stage, out/down (4 K chunks x 2 row groups)
constexpr int MG_NJ = 5;      // 16-value vectors per lane (K chunk <= 2560)
constexpr int MG_MAXK = 10240;
constexpr int MG_CPART_ROWS = 32;  // out/down rows per CTA (hidden <= 2 * 32 * grid)

struct MegaLayer {
  const int8_t* w1;  // [n_plain + 2ff][d] quants
  const __half* s1;  // [..][s1_stride]
  const int8_t* w2;  // [d][d+ff]
  const __half* s2;
  const float* nw;
  const float* nb;
};

struct MegaArgs {
  int L, d, ff, V, H, KVH, hd;
  int s1_stride, s2_stride, sh_stride, se_stride;
  double eps;
  const MegaLayer* layers;
  const int8_t* head_w;
  const __half* head_s;
  const int8_t* emb_w;
  const __half* emb_s;
  const float* fnw;
  const float* fnb;
  Rope rope;
  KVView kv;
  const int* page_table;
  int split, max_splits;
  float scale;  // float32(sqrt(hd))
  // per-step state
  int* pos;
  unsigned long long* keys;  // [2], indexed by step parity
  int* step;
  int* out_tokens;
  int* out_count;
  float* logits;  // optional
  // scratch
  float* x_buf;  // [d]
  float* qkv;    // [d + 2 kvw]
  float* ah;     // [d + ff] (SwiGLU part used)
  uint32_t* adig;  // [(d + ff) / 16][12] digits of [attention | SwiGLU]
  float* asx;      // [(d + ff) / 16] their block scales
  int* bcnt;       // [ff / 16] SwiGLU block arrivals (zero between steps)
  uint32_t dig_bytes, sx_bytes;  // phase C staging sizes (multiples of 16)
  float* part;   // [H][max_splits][hd+2]
  int* counters;  // [KVH]
  unsigned* bar;  // [2]: arrival count, generation
  int* err;
  uint32_t slot_bytes;
  int nslots;  // ring depth (<= MG_MAX_SLOTS)
  uint32_t off_x, off_dig, off_sx, off_part, off_slots;
};

__device__ __forceinline__ int dp4a_su(uint32_t a_signed, uint32_t b_unsigned, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_signed), "r"(b_unsigned), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// 16 int8 weights . 16 digit-encoded inputs -> value in units of the input
// block scale.
__device__ __forceinline__ float dot16_dp4a(const uint4& w, const uint32_t* dg) {
  int t0 = 0, t1 = 0, t2 = 0;
  const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int q = 0; q < 4; q++) {
    t0 = dp4a_su(ww[q], dg[q * 3 + 0], t0);
    t1 = dp4a_su(ww[q], dg[q * 3 + 1], t1);
    t2 = dp4a_ss(ww[q], dg[q * 3 + 2], t2);
  }
  return fmaf((float)t2, 65536.f, (float)(t1 * 256 + t0));
}

// Grid-wide barrier among the consumer warps of all CTAs (the producer warps
// never take part). Sense reversal on a generation word; bounded spin.
__device__ void mg_grid_sync(const MegaArgs& a) {
  named_bar_sync(1, MG_CT);
  if (threadIdx.x == 0) {
    volatile unsigned* gen = a.bar + 1;
    const unsigned g = *gen;
    __threadfence();
    if (atomicAdd(a.bar, 1u) == gridDim.x - 1) {
      atomicExch(a.bar, 0u);
      __threadfence();
      atomicAdd(a.bar + 1, 1u);
    } else {
      const unsigned long long t0 = global_ns();
      uint32_t i = 0;
      while (*gen == g) {
        if ((++i & 63) == 0) {
          if (*(volatile int*)a.err) break;
          if (global_ns() - t0 > TCU_WAIT_NS) {
            atomicExch(a.err, 2);
            break;
          }
        }
      }
    }
    __threadfence();
  }
  named_bar_sync(1, MG_CT);
}

// LayerNorm of xs[0..K) (stablelm.go:288-305) fused with the digit
// quantisation of the normalised values: float64 mean and variance
// (two passes), float32 affine, then warp-per-block digits.
__device__ void mg_ln_digits(const float* xs, int K, const float* nw, const float* nb, double eps, uint32_t* dig, float* sx);

// One thread quantises the 16 values v into 12 digit words (word 3q + k holds
// digit k of values 4q..4q+3) and the block scale.
__device__ __forceinline__ void mg_quant16(const float (&v)[16], uint32_t* dig12, float* sc) {
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 16; i++) mx = fmaxf(mx, fabsf(v[i]));
  const float inv = mx > 0.f ? __fdiv_rn(8388607.f, mx) : 0.f;
  uint32_t w[12];
#pragma unroll
  for (int q = 0; q < 4; q++) {
    uint32_t b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      int xi = __float2int_rn(v[4 * q + k] * inv);
      xi = max(-8388607, min(8388607, xi));
      const uint32_t u = (uint32_t)xi & 0xFFFFFFu;
      b0 |= (u & 0xFFu) << (8 * k);
      b1 |= ((u >> 8) & 0xFFu) << (8 * k);
      b2 |= (u >> 16) << (8 * k);
    }
    w[3 * q] = b0;
    w[3 * q + 1] = b1;
    w[3 * q + 2] = b2;
  }
  uint4* o = reinterpret_cast<uint4*>(dig12);
  o[0] = make_uint4(w[0], w[1], w[2], w[3]);
  o[1] = make_uint4(w[4], w[5], w[6], w[7]);
  o[2] = make_uint4(w[8], w[9], w[10], w[11]);
  *sc = mx > 0.f ? __fdiv_rn(mx, 8388607.f) : 0.f;
}

__device__ void mg_ln_digits(const float* xs, int K, const float* nw, const float* nb, double eps, uint32_t* dig, float* sx) {
  __shared__ double red[2][MG_CW];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Thread t normalises and quantises block t (K / 16 <= MG_CT); its weight
  // and bias are fetched before the reductions.
  const int b = threadIdx.x;
  const bool has_blk = b < K / 16;
  float4 wv[4], bv[4];
  if (has_blk) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
      wv[q] = __ldg(reinterpret_cast<const float4*>(nw + 16 * b) + q);
      bv[q] = __ldg(reinterpret_cast<const float4*>(nb + 16 * b) + q);
    }
  }
  double s = 0;
  for (int i = threadIdx.x; i < K; i += MG_CT) s += (double)xs[i];
  s = warp_sum_d(s);
  if (lane == 0) red[0][warp] = s;
  named_bar_sync(1, MG_CT);
  double tot = 0;
#pragma unroll
  for (int w = 0; w < MG_CW; w++) tot += red[0][w];
  const double mean = tot / (double)K;
  double v = 0;
  for (int i = threadIdx.x; i < K; i += MG_CT) {
    const double d = (double)xs[i] - mean;
    v += d * d;
  }
  v = warp_sum_d(v);
  if (lane == 0) red[1][warp] = v;
  named_bar_sync(1, MG_CT);
  double var = 0;
#pragma unroll
  for (int w = 0; w < MG_CW; w++) var += red[1][w];
  const float inv = (float)(1.0 / sqrt(var / (double)K + eps));
  const float mf = (float)mean;
  if (has_blk) {
    float v[16];
    const float* wf = reinterpret_cast<const float*>(wv);
    const float* bf = reinterpret_cast<const float*>(bv);
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const float4 x4 = reinterpret_cast<const float4*>(xs + 16 * b)[q];
      const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int i = 4 * q + k;
        v[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv[k], mf), inv), wf[i]), bf[i]);
      }
    }
    mg_quant16(v, dig + 12 * b, sx + b);
  }
  named_bar_sync(1, MG_CT);
}

// Balanced share [rb, re) of R rows in pairs for CTA c of G.
__device__ __forceinline__ void mg_rows(int R, int c, int G, int& rb, int& re) {
  const int pairs = (R + 1) >> 1;
  rb = min(R, 2 * (int)(((long long)pairs * c) / G));
  re = min(R, 2 * (int)(((long long)pairs * (c + 1)) / G));
}

struct MgRing {
  uint64_t* full;
  uint64_t* empty;
  uint8_t* slots;
  uint32_t slot_bytes;
  int n;  // slots
  int i;  // running stage index
};

// Producer side: next slot, ready for writing (waits until consumers released it).
__device__ __forceinline__ uint8_t* mg_produce(MgRing& r, uint32_t bytes, int* err) {
  const int slot = r.i % r.n;
  if (r.i >= r.n) mbar_wait(&r.empty[slot], ((r.i / r.n) - 1) & 1, err);
  mbar_expect_tx(&r.full[slot], bytes);
  return r.slots + (size_t)slot * r.slot_bytes;
}
__device__ __forceinline__ uint64_t* mg_full(MgRing& r) { return &r.full[r.i % r.n]; }

// Consumer side.
__device__ __forceinline__ const uint8_t* mg_consume(MgRing& r, int* err) {
  const int slot = r.i % r.n;
  mbar_wait(&r.full[slot], (r.i / r.n) & 1, err);
  return r.slots + (size_t)slot * r.slot_bytes;
}
__device__ __forceinline__ void mg_release(MgRing& r) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&r.empty[r.i % r.n]);
  r.i++;
}

// Attention units of a layer: (kv head g, chunk s) for chunks of the history.
__device__ __forceinline__ int mg_units(const MegaArgs& a, int T) { return a.KVH * ((T + a.split - 1) / a.split); }

__global__ void __launch_bounds__(MG_THREADS, 1) k_decode_mega(MegaArgs a) {
  extern __shared__ __align__(128) uint8_t mg_smem[];
  MgRing ring;
  ring.full = reinterpret_cast<uint64_t*>(mg_smem);
  ring.empty = ring.full + MG_MAX_SLOTS;
  uint64_t* inbar = ring.full + 2 * MG_MAX_SLOTS;  // phase inputs staged by bulk copy
  uint32_t in_phase = 0;
  ring.slots = mg_smem + a.off_slots;
  ring.slot_bytes = a.slot_bytes;
  ring.n = a.nslots;
  ring.i = 0;
  float* xs = reinterpret_cast<float*>(mg_smem + a.off_x);
  uint32_t* dig = reinterpret_cast<uint32_t*>(mg_smem + a.off_dig);
  float* sx = reinterpret_cast<float*>(mg_smem + a.off_sx);
  float* cpart = reinterpret_cast<float*>(mg_smem + a.off_part);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, c = blockIdx.x;
  const int d = a.d, ff = a.ff, hd = a.hd, kvw = a.KVH * hd;
  const int n_plain = d + 2 * kvw;
  const int R1 = n_plain + 2 * ff, K2 = d + ff;
  const size_t row2 = (size_t)K2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ring.n; i++) {
      mbar_init(&ring.full[i], 1);
      mbar_init(&ring.empty[i], MG_CW);
    }
    mbar_init(inbar, 1);
    fence_barrier_init();
  }
  __syncthreads();

  const int pos = *(volatile int*)a.pos;
  const int T = pos + 1;
  const int nsplit = (T + a.split - 1) / a.split;
  const int units = mg_units(a, T);
  int rb1, re1, rb2, re2, rbh, reh;
  mg_rows(R1, c, G, rb1, re1);
  mg_rows(d, c, G, rb2, re2);
  mg_rows(a.V, c, G, rbh, reh);
  const int es = a.kv.half ? 2 : 4;
  const uint32_t page_bytes = (uint32_t)(a.kv.P * hd * es);
  const int pages_per_split = a.split / a.kv.P;

  // ------------------------------------------------------------------ producer
  if (warp == MG_CW) {
    if (lane == 0) {
      for (int l = 0; l < a.L; l++) {
        const MegaLayer& ly = a.layers[l];
        for (int r0 = rb1; r0 < re1; r0 += MG_W1_RS) {
          const int nr = min(MG_W1_RS, re1 - r0);
          const uint32_t qb = (uint32_t)(nr * d), sb = (uint32_t)(nr * a.s1_stride * 2);
          uint8_t* dst = mg_produce(ring, qb + sb, a.err);
          bulk_g2s(dst, ly.w1 + (size_t)r0 * d, qb, mg_full(ring));
          bulk_g2s(dst + (size_t)MG_W1_RS * d, ly.s1 + (size_t)r0 * a.s1_stride, sb, mg_full(ring));
          ring.i++;
        }
        for (int u = c; u < units; u += G) {
          const int g = u / nsplit, s = u % nsplit;
          const int t0 = s * a.split;
          const int nt = min(T, t0 + a.split) - t0;
          const int n_hist = (s == nsplit - 1) ? nt - 1 : nt;
          const int np = (n_hist + a.kv.P - 1) / a.kv.P;
          uint8_t* dst = mg_produce(ring, 2u * np * page_bytes, a.err);
          for (int j = 0; j < np; j++) {
            const int page = a.page_table[t0 / a.kv.P + j];
            const size_t o = a.kv.off(l, page, g, 0) * es;
            bulk_g2s(dst + (size_t)j * page_bytes, reinterpret_cast<const uint8_t*>(a.kv.k) + o, page_bytes, mg_full(ring));
            bulk_g2s(dst + (size_t)(pages_per_split + j) * page_bytes, reinterpret_cast<const uint8_t*>(a.kv.v) + o, page_bytes,
                     mg_full(ring));
          }
          ring.i++;
        }
        for (int r0 = rb2; r0 < re2; r0 += MG_W2_RS) {
          const int nr = min(MG_W2_RS, re2 - r0);
          const uint32_t qb = (uint32_t)(nr * row2), sb = (uint32_t)(nr * a.s2_stride * 2);
          uint8_t* dst = mg_produce(ring, qb + sb, a.err);
          bulk_g2s(dst, ly.w2 + (size_t)r0 * row2, qb, mg_full(ring));
          bulk_g2s(dst + (size_t)MG_W2_RS * row2, ly.s2 + (size_t)r0 * a.s2_stride, sb, mg_full(ring));
          ring.i++;
        }
      }
      for (int r0 = rbh; r0 < reh; r0 += MG_W1_RS) {
        const int nr = min(MG_W1_RS, reh - r0);
        const uint32_t qb = (uint32_t)(nr * d), sb = (uint32_t)(nr * a.sh_stride * 2);
        uint8_t* dst = mg_produce(ring, qb + sb, a.err);
        bulk_g2s(dst, a.head_w + (size_t)r0 * d, qb, mg_full(ring));
        bulk_g2s(dst + (size_t)MG_W1_RS * d, a.head_s + (size_t)r0 * a.sh_stride, sb, mg_full(ring));
        ring.i++;
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int step = *(volatile int*)a.step;
  const unsigned long long key_in = *(volatile unsigned long long*)(a.keys + (step & 1));
  int token = argmax_index(key_in);
  token = (token >= 0 && token < a.V) ? token : 0;
  if (c == 0 && threadIdx.x == 0) {
    a.keys[(step + 1) & 1] = 0ull;
    const int cnt = a.out_count[0];
    a.out_tokens[cnt] = token;
    a.out_count[0] = cnt + 1;
  }
  // Embedding row (Q8_0 decode, matmul.go:24-34), computed by every CTA.
  for (int i = threadIdx.x; i < d; i += MG_CT)
    xs[i] = __fmul_rn(__half2float(a.emb_s[(size_t)token * a.se_stride + i / 32]), (float)a.emb_w[(size_t)token * d + i]);
  named_bar_sync(1, MG_CT);
  if (c == 0)
    for (int i = threadIdx.x; i < d; i += MG_CT) a.x_buf[i] = xs[i];

  uint32_t dr[MG_NJ][12];
  float sxr[MG_NJ];
  unsigned long long best = 0ull;

  // Copies n floats (n * 4 a multiple of 16) from global memory into xs with
  // one bulk copy issued by consumer thread 0, and waits for it. The fence
  // and barrier order every consumer's earlier generic accesses to xs, and
  // the other CTAs' stores to src seen through the grid barrier, before the
  // copy (async proxy).
  auto stage_in = [&](const float* src, int n) {
    fence_proxy_async();
    named_bar_sync(1, MG_CT);
    if (threadIdx.x == 0) {
      mbar_expect_tx(inbar, (uint32_t)n * 4u);
      bulk_g2s(xs, src, (uint32_t)n * 4u, inbar);
    }
    mbar_wait(inbar, in_phase & 1, a.err);
    in_phase++;
  };

  // Loads this warp's digit registers for vectors [vb, ve) of the input.
  auto load_regs = [&](int vb, int ve) {
#pragma unroll
    for (int j = 0; j < MG_NJ; j++) {
      const int v = vb + lane + 32 * j;
      uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0, q2 = q0;
      if (v < ve) {
        const uint4* p = reinterpret_cast<const uint4*>(dig + v * 12);
        q0 = p[0];
        q1 = p[1];
        q2 = p[2];
      }
      dr[j][0] = q0.x, dr[j][1] = q0.y, dr[j][2] = q0.z, dr[j][3] = q0.w;
      dr[j][4] = q1.x, dr[j][5] = q1.y, dr[j][6] = q1.z, dr[j][7] = q1.w;
      dr[j][8] = q2.x, dr[j][9] = q2.y, dr[j][10] = q2.z, dr[j][11] = q2.w;
      sxr[j] = v < ve ? sx[v] : 0.f;
    }
  };

  for (int l = 0; l < a.L; l++) {
    const MegaLayer& ly = a.layers[l];
    // Phase A: LayerNorm, then q/k/v rows and SwiGLU of (gate, up) pairs.
    if (l > 0) stage_in(a.x_buf, d);
    mg_ln_digits(xs, d, ly.nw, ly.nb, a.eps, dig, sx);
    load_regs(0, d / 16);
    for (int r0 = rb1; r0 < re1; r0 += MG_W1_RS) {
      const int nr = min(MG_W1_RS, re1 - r0);
      const uint8_t* st = mg_consume(ring, a.err);
      const __half* ss = reinterpret_cast<const __half*>(st + (size_t)MG_W1_RS * d);
      float acc[2];
#pragma unroll
      for (int t = 0; t < 2; t++) {
        const int lr = 2 * warp + t;
        float s = 0.f;
        if (lr < nr) {
#pragma unroll
          for (int j = 0; j < MG_NJ; j++) {
            const int v = lane + 32 * j;
            if (v < d / 16) {
              const uint4 w = *reinterpret_cast<const uint4*>(st + (size_t)lr * d + (size_t)v * 16);
              s = fmaf(dot16_dp4a(w, dr[j]), __half2float(ss[(size_t)lr * a.s1_stride + (v >> 1)]) * sxr[j], s);
            }
          }
        }
        acc[t] = warp_sum(s);
      }
      mg_release(ring);
      if (lane == 0 && 2 * warp < nr) {
        const int r = r0 + 2 * warp;
        if (r < n_plain) {
          a.qkv[r] = acc[0];
          if (2 * warp + 1 < nr) a.qkv[r + 1] = acc[1];
        } else {
          a.ah[d + ((r - n_plain) >> 1)] = silu_mul_stablelm(acc[0], acc[1]);
        }
      }
    }
    // Digits of this CTA's SwiGLU outputs j in [j0, j1): a 16-value block is
    // quantised by whichever CTA completes it (blocks at the edge of a CTA's
    // rows are shared with its neighbour).
    {
      const int j0 = max(0, rb1 - n_plain) >> 1, j1 = max(0, re1 - n_plain) >> 1;
      if (j1 > j0) {
        __threadfence();
        named_bar_sync(1, MG_CT);
        for (int b = j0 / 16 + threadIdx.x; b < (j1 + 15) / 16; b += MG_CT) {
          const int cnt = min(j1, 16 * b + 16) - max(j0, 16 * b);
          bool last = cnt == 16;
          if (!last) last = atomicAdd(a.bcnt + b, cnt) + cnt == 16;
          if (last) {
            __threadfence();
            if (cnt != 16) a.bcnt[b] = 0;
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = __ldcg(a.ah + d + 16 * b + i);
            mg_quant16(v, a.adig + (size_t)(d / 16 + b) * 12, a.asx + d / 16 + b);
          }
        }
      }
    }
    mg_grid_sync(a);

    // Phase B: attention units (stablelm.go:401-427), split over the history.
    {
      const int G_q = a.H / a.KVH;
      float* qs = xs;                         // [G_q][hd]
      float* cur = xs + G_q * hd;             // [2][hd]
      float* sc = cur + 2 * hd;               // [G_q][split]
      __shared__ int is_last;
      __shared__ float mloc[32], lloc[32];
      for (int u = c; u < units; u += G) {
        const int g = u / nsplit, s = u % nsplit;
        const int t0 = s * a.split;
        const int nt = min(T, t0 + a.split) - t0;
        const bool has_cur = (s == nsplit - 1);
        const int n_hist = has_cur ? nt - 1 : nt;
        for (int e = threadIdx.x; e < G_q * hd; e += MG_CT) qs[e] = __ldcg(a.qkv + (g * G_q) * hd + e);
        if (has_cur)
          for (int e = threadIdx.x; e < hd; e += MG_CT) {
            cur[e] = __ldcg(a.qkv + a.H * hd + g * hd + e);
            cur[hd + e] = __ldcg(a.qkv + (a.H + a.KVH) * hd + g * hd + e);
          }
        named_bar_sync(1, MG_CT);
        for (int e = threadIdx.x; e < G_q * a.rope.pairs; e += MG_CT) rope_pair(qs + (e / a.rope.pairs) * hd, e % a.rope.pairs, a.rope, pos);
        if (has_cur)
          for (int e = threadIdx.x; e < a.rope.pairs; e += MG_CT) rope_pair(cur, e, a.rope, pos);
        named_bar_sync(1, MG_CT);
        if (has_cur) {
          for (int e = threadIdx.x; e < 2 * hd; e += MG_CT) cur[e] = kv_round(cur[e], a.kv.half);
          named_bar_sync(1, MG_CT);
          const int page = a.page_table[pos / a.kv.P], row = pos % a.kv.P;
          const size_t o = a.kv.off(l, page, g, row);
          for (int e = threadIdx.x; e < hd; e += MG_CT) {
            kv_store(a.kv, a.kv.k, o + e, cur[e]);
            kv_store(a.kv, a.kv.v, o + e, cur[hd + e]);
          }
        }
        const uint8_t* st = mg_consume(ring, a.err);
        const uint8_t* ktile = st;
        const uint8_t* vtile = st + (size_t)pages_per_split * page_bytes;
        for (int e = threadIdx.x; e < G_q * a.split; e += MG_CT) {
          const int hh = e / a.split, t = e % a.split;
          if (t < nt) {
            const float* q = qs + hh * hd;
            float acc = 0.f;
            const int i0 = t % hd;
            if (has_cur && t == nt - 1) {
              for (int i = 0; i < hd; i++) {
                int ii = i0 + i;
                ii -= ii >= hd ? hd : 0;
                acc = fmaf(q[ii], cur[ii], acc);
              }
            } else {
              for (int i = 0; i < hd; i++) {
                int ii = i0 + i;
                ii -= ii >= hd ? hd : 0;
                acc = fmaf(q[ii], kv_ld(ktile, a.kv.half, (size_t)t * hd + ii), acc);
              }
            }
            sc[hh * a.split + t] = __fdiv_rn(acc, a.scale);
          }
        }
        named_bar_sync(1, MG_CT);
        for (int hh = warp; hh < G_q; hh += MG_CW) {
          float mx = -INFINITY;
          for (int t = lane; t < nt; t += 32) mx = fmaxf(mx, sc[hh * a.split + t]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          float lsum = 0.f;
          for (int t = lane; t < nt; t += 32) {
            const float p = expf(sc[hh * a.split + t] - mx);
            sc[hh * a.split + t] = p;
            lsum += p;
          }
          lsum = warp_sum(lsum);
          if (lane == 0) {
            mloc[hh] = mx;
            lloc[hh] = lsum;
          }
        }
        named_bar_sync(1, MG_CT);
        float* pg = a.part + (size_t)(g * G_q) * a.max_splits * (hd + 2);
        for (int e = threadIdx.x; e < G_q * hd; e += MG_CT) {
          const int hh = e / hd, i = e % hd;
          float o = 0.f;
          for (int t = 0; t < n_hist; t++) o = fmaf(sc[hh * a.split + t], kv_ld(vtile, a.kv.half, (size_t)t * hd + i), o);
          if (has_cur) o = fmaf(sc[hh * a.split + nt - 1], cur[hd + i], o);
          pg[((size_t)hh * a.max_splits + s) * (hd + 2) + i] = o;
        }
        if (threadIdx.x < G_q) {
          pg[((size_t)threadIdx.x * a.max_splits + s) * (hd + 2) + hd] = mloc[threadIdx.x];
          pg[((size_t)threadIdx.x * a.max_splits + s) * (hd + 2) + hd + 1] = lloc[threadIdx.x];
        }
        mg_release(ring);
        __threadfence();
        named_bar_sync(1, MG_CT);
        if (threadIdx.x == 0) is_last = (atomicAdd(a.counters + g, 1) == nsplit - 1);
        named_bar_sync(1, MG_CT);
        if (is_last) {
          __threadfence();
          // Merged head outputs go to qs (no longer read), then their digits
          // to adig: G_q * hd is a multiple of 16.
          for (int e = threadIdx.x; e < G_q * hd; e += MG_CT) {
            const int hh = e / hd, i = e % hd;
            const float* ph = pg + (size_t)hh * a.max_splits * (hd + 2);
            float mx = -INFINITY;
            for (int j = 0; j < nsplit; j++) mx = fmaxf(mx, __ldcg(ph + (size_t)j * (hd + 2) + hd));
            float lsum = 0.f, o = 0.f;
            for (int j = 0; j < nsplit; j++) {
              const float* pj = ph + (size_t)j * (hd + 2);
              const float w = expf(__ldcg(pj + hd) - mx);
              lsum = fmaf(__ldcg(pj + hd + 1), w, lsum);
              o = fmaf(__ldcg(pj + i), w, o);
            }
            qs[e] = __fdiv_rn(o, lsum);
          }
          named_bar_sync(1, MG_CT);
          const int nb16 = G_q * hd / 16;
          for (int b = threadIdx.x; b < nb16; b += MG_CT) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = qs[16 * b + i];
            mg_quant16(v, a.adig + (size_t)(g * nb16 + b) * 12, a.asx + g * nb16 + b);
          }
          if (threadIdx.x == 0) a.counters[g] = 0;
        }
        named_bar_sync(1, MG_CT);
      }
    }
    mg_grid_sync(a);

    // Phase C: out/down rows over [attention | SwiGLU], parallel residual
    // (stablelm.go:365-377). K chunks: [0, d) then down split in three.
    // The digits of [attention | SwiGLU] were published by their producers.
    fence_proxy_async();
    named_bar_sync(1, MG_CT);
    if (threadIdx.x == 0) {
      mbar_expect_tx(inbar, a.dig_bytes + a.sx_bytes);
      bulk_g2s(dig, a.adig, a.dig_bytes, inbar);
      bulk_g2s(sx, a.asx, a.sx_bytes, inbar);
    }
    mbar_wait(inbar, in_phase & 1, a.err);
    in_phase++;
    {
      const int chunk = warp & 3, sub = warp >> 2;
      const int nvd = ff / 16;
      int vb, ve;
      if (chunk == 0) {
        vb = 0;
        ve = d / 16;
      } else {
        vb = d / 16 + (nvd * (chunk - 1)) / 3;
        ve = d / 16 + (nvd * chunk) / 3;
      }
      load_regs(vb, ve);
      for (int r0 = rb2; r0 < re2; r0 += MG_W2_RS) {
        const int nr = min(MG_W2_RS, re2 - r0);
        const uint8_t* st = mg_consume(ring, a.err);
        const __half* ss = reinterpret_cast<const __half*>(st + (size_t)MG_W2_RS * row2);
        float acc[2];
#pragma unroll
        for (int t = 0; t < 2; t++) {
          const int lr = 2 * sub + t;
          float s = 0.f;
          if (lr < nr) {
#pragma unroll
            for (int j = 0; j < MG_NJ; j++) {
              const int v = vb + lane + 32 * j;
              if (v < ve) {
                const uint4 w = *reinterpret_cast<const uint4*>(st + (size_t)lr * row2 + (size_t)v * 16);
                s = fmaf(dot16_dp4a(w, dr[j]), __half2float(ss[(size_t)lr * a.s2_stride + (v >> 1)]) * sxr[j], s);
              }
            }
          }
          acc[t] = warp_sum(s);
        }
        mg_release(ring);
        // Chunk partials of each row stay in shared memory until the phase
        // ends; one fixed-order reduction per row follows the loop.
        if (lane == 0) {
#pragma unroll
          for (int t = 0; t < 2; t++)
            if (2 * sub + t < nr) cpart[(r0 - rb2 + 2 * sub + t) * 4 + chunk] = acc[t];
        }
      }
      named_bar_sync(1, MG_CT);
      for (int l = threadIdx.x; l < re2 - rb2; l += MG_CT) {
        const float lo = cpart[l * 4 + 0];
        const float hi = (cpart[l * 4 + 1] + cpart[l * 4 + 2]) + cpart[l * 4 + 3];
        const int r = rb2 + l;
        a.x_buf[r] = __fadd_rn(__fadd_rn(__ldcg(a.x_buf + r), lo), hi);
      }
    }
    mg_grid_sync(a);
  }

  // Final LayerNorm and lm_head with argmax (stablelm.go:380-385, model.go:622-630).
  stage_in(a.x_buf, d);
  mg_ln_digits(xs, d, a.fnw, a.fnb, a.eps, dig, sx);
  load_regs(0, d / 16);
  for (int r0 = rbh; r0 < reh; r0 += MG_W1_RS) {
    const int nr = min(MG_W1_RS, reh - r0);
    const uint8_t* st = mg_consume(ring, a.err);
    const __half* ss = reinterpret_cast<const __half*>(st + (size_t)MG_W1_RS * d);
    float acc[2];
#pragma unroll
    for (int t = 0; t < 2; t++) {
      const int lr = 2 * warp + t;
      float s = 0.f;
      if (lr < nr) {
#pragma unroll
        for (int j = 0; j < MG_NJ; j++) {
          const int v = lane + 32 * j;
          if (v < d / 16) {
            const uint4 w = *reinterpret_cast<const uint4*>(st + (size_t)lr * d + (size_t)v * 16);
            s = fmaf(dot16_dp4a(w, dr[j]), __half2float(ss[(size_t)lr * a.sh_stride + (v >> 1)]) * sxr[j], s);
          }
        }
      }
      acc[t] = warp_sum(s);
    }
    mg_release(ring);
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < 2; t++) {
        const int lr = 2 * warp + t;
        if (lr < nr) {
          const int r = r0 + lr;
          if (a.logits) a.logits[r] = acc[t];
          const unsigned long long k = argmax_pack(acc[t], r);
          best = k > best ? k : best;
        }
      }
    }
  }
  __shared__ unsigned long long bred[MG_CW];
  if (lane == 0) bred[warp] = best;
  named_bar_sync(1, MG_CT);
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < MG_CW; w++) b = bred[w] > b ? bred[w] : b;
    atomicMax(a.keys + ((step + 1) & 1), b);
  }
  // The next launch reads pos and step after this one completes.
  if (c == 0 && threadIdx.x == 0) {
    *a.pos = pos + 1;
    *a.step = step + 1;
  }
}

// Logs the argmax of the last step (the final generated token).
__global__ void k_finish_mega(const unsigned long long* keys, const int* step, int* out_tokens, int* out_count) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const int c = out_count[0];
    out_tokens[c] = argmax_index(keys[step[0] & 1]);
    out_count[0] = c + 1;
  }
}

}  // namespace tcu
