// Persistent decode step for one StableLM sequence with Q8_0 weights: the
// whole forward of one token (stablelm.go:332-387) in a single cooperative
// launch.
//
// Grid = one CTA per SM. Warp 8 lane 0 is the producer, warps 0..7 consume,
// warp 9 of CTA g merges the history splits of KV head g (g < KV heads).
// Work is handed out dynamically: for each layer the producer takes items
// from global counters -- tiles of the fused q/k/v/gate/up rows, attention
// units (KV head x history split), tiles of the down-projection rows (the
// SwiGLU columns of the fused out/down matrix), tiles of the out-projection
// rows (its attention columns); then tiles of the lm_head rows -- and streams
// each item's weights or KV pages into a shared-memory ring of slots with
// cp.async.bulk, tagging the slot with the item. SMs that stream faster take
// more items, so the phases end together. A phase's input is awaited only
// where it is read:
//   - attention needs every q/k/v row (a count of finished q/k/v tiles);
//   - the down rows need every SwiGLU block, so they run while attention
//     does; the out rows need every merged attention head;
//   - a residual row needs its down sum; the next layer needs every row.
// Each wait is a bounded poll of one counter. Per-layer x and digit buffers
// mean no CTA overwrites what a slower CTA may still be reading.
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
// Failure: every wait is bounded (%globaltimer). A wait that gives up sets the
// error word and ends the item loop it is in. Loops over row tiles contain no
// CTA-wide barrier (warps meet through shared-memory arrival counters), and
// attention items are dispatched CTA-uniformly, so the kernel always ends.
#pragma once
#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "tma.cuh"

namespace tcu {

constexpr int MG_CW = 8;                      // consumer warps
constexpr int MG_THREADS = (MG_CW + 2) * 32;  // + producer warp + merge warp
constexpr int MG_MW = MG_CW + 1;              // the merge warp
// Register bound: 10 warps put 3 on two of the four SM sub-partitions, whose
// register files hold 16,384 each, so a thread may use at most 170.
constexpr int MG_REG_THREADS = 384;
constexpr int MG_CT = MG_CW * 32;
constexpr int MG_MAX_SLOTS = 6;
constexpr int MG_W1_RS = 16;  // rows per stage, q/k/v/gate/up and head
constexpr int MG_DN_RS = 4;   // rows per stage, down projection (4 K chunks x 2 row groups)
constexpr int MG_O_RS = 16;   // rows per stage, out projection (2 rows per warp)
constexpr int MG_NJ = 5;      // 16-value vectors per lane (K chunk <= 2560)
constexpr int MG_MAXK = 10240;
// Control words per (launch parity, layer). grab: 0 q/k/v/gate/up tiles,
// 1 attention units, 2 down tiles, 3 out tiles; grab[L][0]: lm_head tiles.
// done: 0 q/k/v rows, 1 gate/up tiles, 2 residual rows, 3 merged heads,
// 4 down rows; done[L][3] counts the CTAs that finished the launch.
constexpr int MG_CTL = 8;
constexpr int MG_HDR = 256;   // shared-memory header: mbarriers and slot tags
constexpr int MG_SEQ = 8;     // in-flight tiles tracked by the arrival counters
constexpr int MG_SWT = 24;    // W1 tiles per CTA and layer (gate/up values kept for quantisation after the loop)

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
  int dn_sstride;  // scale halves per row in a down tile (staged segment)
  int dn_soff;     // first scale of the down segment within that staged run
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
  float* xl;       // [L + 1][d]: input of layer l (xl[L]: input of the final norm)
  float* xdn;      // [L][d]: down-projection sums of layer l
  float* qkv;      // [d + 2 kvw]
  uint32_t* adig;  // [L][(d + ff) / 16][12] digits of [attention | SwiGLU]
  float* asx;      // [L][asx_stride] their block scales
  int asx_stride;  // floats per layer (multiple of 4)
  int att_warp;    // floats of attention scratch per consumer warp
  float* part;     // [H][max_splits][hd+2]
  int* counters;   // [KVH] split arrivals per KV head (zero between layers)
  int* grab;       // [2][L + 1][MG_CTL] work counters by launch parity
  int* done;       // [2][L + 1][MG_CTL] completion counters by launch parity
  int* err;
  // Failure-detection test hook (-1: off). In the launch whose step counter is
  // 0, the merge warp of KV head 0 in layer hold_layer does not publish its
  // head, so every CTA's wait for the merged heads runs out (TCU_WAIT_NS),
  // sets the error word, and the launch still ends. Set from the host only by
  // the TCU_TEST_HOLD_ARRIVAL environment variable.
  int hold_layer;
  uint32_t slot_bytes;
  int nslots;  // ring depth (<= MG_MAX_SLOTS)
  uint32_t off_x, off_att, off_dig, off_sx, off_slots;
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

// One thread quantises the 16 values v into 12 digit words (word 3q + k holds
// digit k of values 4q..4q+3) and the block scale: scale = max|v| / (2^23 - 1),
// digits = low, middle and signed high byte of round(v / scale).
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

// The same quantisation by a warp: lanes 0-15 hold the 16 values (lanes
// 16-31 take part in the shuffles only); lanes 0, 4, 8, 12 write the words.
__device__ __forceinline__ void mg_quant16_warp(float v, uint32_t* dig12, float* sc) {
  const int lane = threadIdx.x & 31;
  float mx = fabsf(v);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float inv = mx > 0.f ? __fdiv_rn(8388607.f, mx) : 0.f;
  int xi = __float2int_rn(v * inv);
  xi = max(-8388607, min(8388607, xi));
  const uint32_t u = (uint32_t)xi & 0xFFFFFFu;
  const uint32_t u1 = __shfl_down_sync(0xffffffffu, u, 1);
  const uint32_t u2 = __shfl_down_sync(0xffffffffu, u, 2);
  const uint32_t u3 = __shfl_down_sync(0xffffffffu, u, 3);
  if (lane < 16 && (lane & 3) == 0) {
    uint32_t* w = dig12 + 3 * (lane >> 2);
    w[0] = (u & 0xFF) | (u1 & 0xFF) << 8 | (u2 & 0xFF) << 16 | (u3 & 0xFF) << 24;
    w[1] = ((u >> 8) & 0xFF) | ((u1 >> 8) & 0xFF) << 8 | ((u2 >> 8) & 0xFF) << 16 | ((u3 >> 8) & 0xFF) << 24;
    w[2] = (u >> 16) | (u1 >> 16) << 8 | (u2 >> 16) << 16 | (u3 >> 16) << 24;
  }
  if (lane == 0) *sc = mx > 0.f ? __fdiv_rn(mx, 8388607.f) : 0.f;
}

// Dot products of two rows (lr0, lr0 + 1) of a stage with the lane's digit
// registers, over vectors v = vb + lane + 32 j (j < MG_NJ). All shared-memory
// loads are issued before the arithmetic and nothing is branched on: a lane
// past the input's end (ve) reads the row's last vector and adds exactly zero
// (its digits and scale are zero); a row past nr repeats row nr - 1 and its
// result is not used.
__device__ __forceinline__ void mg_dot2(const uint8_t* st, size_t pitch, const __half* ss, int sstride, int lr0, int nr, int vb,
                                        int ve, const uint32_t (&dr)[MG_NJ][12], const float (&sxr)[MG_NJ], float (&acc)[2]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int t = 0; t < 2; t++) {
    const int lr = min(lr0 + t, nr - 1);
    uint4 w[MG_NJ];
    float sc[MG_NJ];
#pragma unroll
    for (int j = 0; j < MG_NJ; j++) {
      const int v = min(vb + lane + 32 * j, ve - 1);
      w[j] = *reinterpret_cast<const uint4*>(st + (size_t)lr * pitch + (size_t)v * 16);
      sc[j] = __half2float(ss[lr * sstride + (v >> 1)]);
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < MG_NJ; j++) s = fmaf(dot16_dp4a(w[j], dr[j]), sc[j] * sxr[j], s);
    acc[t] = warp_sum(s);
  }
}

// LayerNorm of xs[0..K) (stablelm.go:288-305) fused with the digit
// quantisation of the normalised values: float64 mean and variance (two
// passes), float32 affine; thread t normalises and quantises block t
// (K / 16 <= MG_CT), with its weight and bias fetched before the reductions.
__device__ void mg_ln_digits(const float* xs, int K, const float* nw, const float* nb, double eps, uint32_t* dig, float* sx) {
  __shared__ double red[2][MG_CW];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
    float y[16];
    const float* wf = reinterpret_cast<const float*>(wv);
    const float* bf = reinterpret_cast<const float*>(bv);
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const float4 x4 = reinterpret_cast<const float4*>(xs + 16 * b)[q];
      const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int i = 4 * q + k;
        y[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv[k], mf), inv), wf[i]), bf[i]);
      }
    }
    mg_quant16(y, dig + 12 * b, sx + b);
  }
  named_bar_sync(1, MG_CT);
}

// Bounded wait until *ctr >= target (acquire). Called by one thread; returns
// false (and sets *err) if it gives up or another thread already did.
__device__ bool mg_wait_count(const int* ctr, int target, int* err) {
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 0;; i++) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if ((i & 31) == 31) {
      if (*(volatile int*)err) return false;
      if (global_ns() - t0 > TCU_WAIT_NS) {
        atomicExch(err, 2);
        return false;
      }
    }
  }
}

// Release / acquire-release atomics at GPU scope: the release orders every
// write this thread has made or observed (including a warp's or CTA's writes
// it synchronised with) before the update.
__device__ __forceinline__ int mg_atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void mg_red_add_release(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits (bounded, without touching the error word) for the phase with the
// given parity of bar to complete: the copies of a stage landing.
__device__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > TCU_WAIT_NS) return;
}

struct MgRing {
  uint64_t* full;
  uint64_t* empty;
  int* tag;
  uint8_t* slots;
  uint32_t slot_bytes;
  int n;  // slots
  int i;  // running stage index
};

// Producer: takes the next slot (waiting until the consumers released it),
// tags it and arms its barrier for `bytes` of copies (0: a bare tag).
// Returns nullptr if the wait failed: the producer then stops.
__device__ __forceinline__ uint8_t* mg_produce(MgRing& r, int tag, uint32_t bytes, int* err) {
  const int slot = r.i % r.n;
  if (r.i >= r.n && !mbar_wait(&r.empty[slot], ((r.i / r.n) - 1) & 1, err)) return nullptr;
  r.tag[slot] = tag;
  mbar_expect_tx(&r.full[slot], bytes);
  return r.slots + (size_t)slot * r.slot_bytes;
}
__device__ __forceinline__ uint64_t* mg_full(MgRing& r) { return &r.full[r.i % r.n]; }

// Consumer warp: waits for the next slot; returns its tag (-1: end of the
// phase), or -2 if the wait failed. Warp-uniform.
__device__ __forceinline__ int mg_next_warp(MgRing& r, const uint8_t** st, int* err) {
  const int slot = r.i % r.n;
  const bool ok = __all_sync(0xffffffffu, mbar_wait(&r.full[slot], (r.i / r.n) & 1, err));
  *st = r.slots + (size_t)slot * r.slot_bytes;
  return ok ? r.tag[slot] : -2;
}
__device__ __forceinline__ void mg_release(MgRing& r) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&r.empty[r.i % r.n]);
  r.i++;
}

// Publishes n finished items of this CTA on a completion counter, after
// every consumer thread's global writes (the barrier, then a release).
__device__ __forceinline__ void mg_publish(int* ctr, int n) {
  named_bar_sync(1, MG_CT);
  if (threadIdx.x == 0 && n > 0) mg_red_add_release(ctr, n);
}

// Waits, CTA-uniformly, until *ctr >= target. The result of a failed wait is
// garbage but the kernel keeps going to its end.
__device__ __forceinline__ void mg_await(const int* ctr, int target, int* err) {
  if (threadIdx.x == 0) {
    mg_wait_count(ctr, target, err);
    fence_proxy_async();  // later bulk copies read what the counter covers
  }
  named_bar_sync(1, MG_CT);
}

// Merges the nsplit partials (rows of hd outputs, max, sum) of each of the
// G_q query heads of one KV head into wo[G_q][hd], by one warp: the fp32
// maximum over the splits, weights expf(max_j - max), then the sum and the
// outputs accumulated in split order. Lane j holds split j's max, sum and
// weight; output rows are loaded 8 splits at a time before any is used, so
// the merge costs a few L2 round trips rather than one per split.
__device__ __forceinline__ void mg_merge_head(const float* pg, int max_splits, int hd, int G_q, int nsplit, int lane, float* wo) {
  const int rs = hd + 2;
  if (nsplit <= 32 && hd <= 128) {
    // Up to 32 splits (lane j holds split j's max, sum, weight): the output
    // rows load 16 splits at a time, every load of a batch before any use.
    for (int hh = 0; hh < G_q; hh++) {
      const float* ph = pg + (size_t)hh * max_splits * rs;
      const float mj = lane < nsplit ? __ldcg(ph + (size_t)lane * rs + hd) : -INFINITY;
      const float sj = lane < nsplit ? __ldcg(ph + (size_t)lane * rs + hd + 1) : 0.f;
      float o4[4] = {0.f, 0.f, 0.f, 0.f}, lsum = 0.f, wj = 0.f;
      for (int jb = 0; jb < nsplit; jb += 16) {
        float pv[16][4];
#pragma unroll
        for (int j = 0; j < 16; j++)
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const int i = lane + 32 * k;
            pv[j][k] = (jb + j < nsplit && i < hd) ? __ldcg(ph + (size_t)(jb + j) * rs + i) : 0.f;
          }
        if (jb == 0) {
          float mx = mj;
#pragma unroll
          for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          wj = lane < nsplit ? expf(mj - mx) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const float w = __shfl_sync(0xffffffffu, wj, (jb + j) & 31);
          const float sv = __shfl_sync(0xffffffffu, sj, (jb + j) & 31);
          if (jb + j < nsplit) {
            lsum = fmaf(sv, w, lsum);
#pragma unroll
            for (int k = 0; k < 4; k++) o4[k] = fmaf(pv[j][k], w, o4[k]);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int i = lane + 32 * k;
        if (i < hd) wo[hh * hd + i] = __fdiv_rn(o4[k], lsum);
      }
    }
    return;
  }
  for (int hh = 0; hh < G_q; hh++) {
    const float* ph = pg + (size_t)hh * max_splits * rs;
    float mx = -INFINITY;
    for (int jb = 0; jb < nsplit; jb += 32)
      if (jb + lane < nsplit) mx = fmaxf(mx, __ldcg(ph + (size_t)(jb + lane) * rs + hd));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int ib = 0; ib < hd; ib += 128) {
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      float lsum = 0.f;
      for (int jb = 0; jb < nsplit; jb += 32) {
        const int jl = jb + lane, n = min(32, nsplit - jb);
        float wj = 0.f, sj = 0.f;
        if (jl < nsplit) {
          wj = expf(__ldcg(ph + (size_t)jl * rs + hd) - mx);
          sj = __ldcg(ph + (size_t)jl * rs + hd + 1);
        }
        for (int j8 = 0; j8 < n; j8 += 8) {
          float pv[8][4];
#pragma unroll
          for (int jj = 0; jj < 8; jj++)
#pragma unroll
            for (int k = 0; k < 4; k++) {
              const int i = ib + lane + 32 * k;
              pv[jj][k] = (j8 + jj < n && i < hd) ? __ldcg(ph + (size_t)(jb + j8 + jj) * rs + i) : 0.f;
            }
#pragma unroll
          for (int jj = 0; jj < 8; jj++) {
            const float w = __shfl_sync(0xffffffffu, wj, (j8 + jj) & 31);
            const float sv = __shfl_sync(0xffffffffu, sj, (j8 + jj) & 31);
            if (j8 + jj < n) {
              lsum = fmaf(sv, w, lsum);
#pragma unroll
              for (int k = 0; k < 4; k++) o[k] = fmaf(pv[jj][k], w, o[k]);
            }
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int i = ib + lane + 32 * k;
        if (i < hd) wo[hh * hd + i] = __fdiv_rn(o[k], lsum);
      }
    }
  }
}

// Scores, softmax and weighted values of one attention unit, by one warp
// (stablelm.go:401-427 with the history split): K and V tiles of n_hist
// tokens in shared memory (float32 or binary16 rows of hd values), this
// position's k, v (float32, already rounded to the KV precision) in cur.
// Writes the unit's partial (hd outputs, max, sum) per query head to pg.
// Scores: a lane per token reads its K row in 16-byte chunks from a
// token-dependent starting chunk (conflict-free); values: a lane per chunk
// of dimensions with one accumulator per dimension.
template <bool HALF>
__device__ __forceinline__ void mg_unit_core(const MegaArgs& a, const uint8_t* ktile, uint32_t vofs, const float* wq, const float* cur,
                                             float* sc, int G_q, int hd, int n_hist, int nt, bool has_cur, float* pg, int s) {
  constexpr int CE = HALF ? 8 : 4;  // values per 16-byte chunk
  const int lane = threadIdx.x & 31;
  const int nch = hd / CE;
  const size_t row_bytes = (size_t)hd * (HALF ? 2 : 4);
  const uint8_t* vtile = ktile + vofs;
  for (int t = lane; t < n_hist; t += 32) {
    const uint8_t* krow = ktile + (size_t)t * row_bytes;
    for (int hh = 0; hh < G_q; hh++) {
      const float* q = wq + hh * hd;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      int c = t % nch;
      for (int j = 0; j < nch; j++) {
        const uint4 raw = *reinterpret_cast<const uint4*>(krow + (size_t)c * 16);
        if (HALF) {
          const __half2* h = reinterpret_cast<const __half2*>(&raw);
          const float4 q0 = *reinterpret_cast<const float4*>(q + 8 * c);
          const float4 q1 = *reinterpret_cast<const float4*>(q + 8 * c + 4);
          const float2 k0 = __half22float2(h[0]), k1 = __half22float2(h[1]), k2 = __half22float2(h[2]), k3 = __half22float2(h[3]);
          a0 = fmaf(q0.x, k0.x, a0);
          a1 = fmaf(q0.y, k0.y, a1);
          a2 = fmaf(q0.z, k1.x, a2);
          a3 = fmaf(q0.w, k1.y, a3);
          a0 = fmaf(q1.x, k2.x, a0);
          a1 = fmaf(q1.y, k2.y, a1);
          a2 = fmaf(q1.z, k3.x, a2);
          a3 = fmaf(q1.w, k3.y, a3);
        } else {
          const float4 k4 = *reinterpret_cast<const float4*>(&raw);
          const float4 q4 = *reinterpret_cast<const float4*>(q + 4 * c);
          a0 = fmaf(q4.x, k4.x, a0);
          a1 = fmaf(q4.y, k4.y, a1);
          a2 = fmaf(q4.z, k4.z, a2);
          a3 = fmaf(q4.w, k4.w, a3);
        }
        c = c + 1 == nch ? 0 : c + 1;
      }
      sc[hh * a.split + t] = __fdiv_rn((a0 + a1) + (a2 + a3), a.scale);
    }
  }
  if (has_cur)
    for (int hh = 0; hh < G_q; hh++) {
      float acc = 0.f;
      for (int i = lane; i < hd; i += 32) acc = fmaf(wq[hh * hd + i], cur[i], acc);
      acc = warp_sum(acc);
      if (lane == 0) sc[hh * a.split + nt - 1] = __fdiv_rn(acc, a.scale);
    }
  __syncwarp();
  float mloc = 0.f, lloc = 0.f;  // lane hh holds head hh's max and sum
  for (int hh = 0; hh < G_q; hh++) {
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
    if (lane == hh) {
      mloc = mx;
      lloc = lsum;
    }
  }
  __syncwarp();
  for (int hh = 0; hh < G_q; hh++) {
    const float* p = sc + hh * a.split;
    float* po = pg + ((size_t)hh * a.max_splits + s) * (hd + 2);
    for (int c = lane; c < nch; c += 32) {
      float acc[CE];
#pragma unroll
      for (int k = 0; k < CE; k++) acc[k] = 0.f;
      for (int t = 0; t < n_hist; t++) {
        const uint4 raw = *reinterpret_cast<const uint4*>(vtile + (size_t)t * row_bytes + (size_t)c * 16);
        const float pt = p[t];
        if (HALF) {
          const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const float2 v2 = __half22float2(h[k]);
            acc[2 * k] = fmaf(pt, v2.x, acc[2 * k]);
            acc[2 * k + 1] = fmaf(pt, v2.y, acc[2 * k + 1]);
          }
        } else {
          const float4 v4 = *reinterpret_cast<const float4*>(&raw);
          acc[0] = fmaf(pt, v4.x, acc[0]);
          acc[1] = fmaf(pt, v4.y, acc[1]);
          acc[2] = fmaf(pt, v4.z, acc[2]);
          acc[3] = fmaf(pt, v4.w, acc[3]);
        }
      }
      if (has_cur) {
        const float pt = p[nt - 1];
#pragma unroll
        for (int k = 0; k < CE; k++) acc[k] = fmaf(pt, cur[hd + c * CE + k], acc[k]);
      }
#pragma unroll
      for (int k = 0; k < CE; k++) po[c * CE + k] = acc[k];
    }
    if (lane == hh) {
      po[hd] = mloc;
      po[hd + 1] = lloc;
    }
  }
}

__global__ void __launch_bounds__(MG_REG_THREADS, 1) k_decode_mega(MegaArgs a) {
  extern __shared__ __align__(128) uint8_t mg_smem[];
  __shared__ float swg[MG_SWT][16], swu[MG_SWT][16];  // gate / up of this layer's gate/up tiles
  __shared__ int swtile[MG_SWT];
  float(*cpart)[16] = swg;  // out/down chunk partials of this layer's tiles (phase C)
  MgRing ring;
  ring.full = reinterpret_cast<uint64_t*>(mg_smem);
  ring.empty = ring.full + MG_MAX_SLOTS;
  uint64_t* inbar = ring.full + 2 * MG_MAX_SLOTS;  // phase inputs staged by bulk copy
  ring.tag = reinterpret_cast<int*>(mg_smem + 128);
  uint32_t in_phase = 0;
  ring.slots = mg_smem + a.off_slots;
  ring.slot_bytes = a.slot_bytes;
  ring.n = a.nslots;
  ring.i = 0;
  float* xs = reinterpret_cast<float*>(mg_smem + a.off_x);
  float* att = reinterpret_cast<float*>(mg_smem + a.off_att);
  uint32_t* dig = reinterpret_cast<uint32_t*>(mg_smem + a.off_dig);
  float* sx = reinterpret_cast<float*>(mg_smem + a.off_sx);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, c = blockIdx.x;
  const int d = a.d, ff = a.ff, hd = a.hd, kvw = a.KVH * hd;
  const int n_plain = d + 2 * kvw;
  const int K2 = d + ff;
  const size_t row2 = (size_t)K2;
  const int n_pt = n_plain / MG_W1_RS;     // q/k/v tiles (16 rows)
  const int n_w1t = n_pt + ff / 16;        // + gate/up tiles (32 rows: 16 SwiGLU values)
  const int n_dnt = (d + MG_DN_RS - 1) / MG_DN_RS;
  const int n_ot = (d + MG_O_RS - 1) / MG_O_RS;
  const int osc = (d / 32 + 7) / 8 * 8;  // scale halves per row in an out tile
  const int n_ht = (a.V + MG_W1_RS - 1) / MG_W1_RS;
  const int G_q = a.H / a.KVH;

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
  const int step = *(volatile int*)a.step;
  const int par = step & 1;
  int* grab = a.grab + (size_t)par * (a.L + 1) * MG_CTL;
  int* done = a.done + (size_t)par * (a.L + 1) * MG_CTL;
  const int T = pos + 1;
  const int nsplit = (T + a.split - 1) / a.split;
  const int units = a.KVH * nsplit;
  const int es = a.kv.half ? 2 : 4;
  const uint32_t page_bytes = (uint32_t)(a.kv.P * hd * es);
  const int pages_per_split = a.split / a.kv.P;

  // ------------------------------------------------------------------ producer
  if (warp == MG_CW) {
    if (lane == 0) {
      bool stop = false;
      // Ends a phase for the consumers with a bare tag.
      auto end_phase = [&]() {
        if (!mg_produce(ring, -1, 0, a.err))
          stop = true;
        else
          ring.i++;
      };
      for (int l = 0; l < a.L && !stop; l++) {
        // Kept in registers: the grab atomics would otherwise force reloads.
        const int8_t* const w1p = a.layers[l].w1;
        const __half* const s1p = a.layers[l].s1;
        const int8_t* const w2p = a.layers[l].w2;
        const __half* const s2p = a.layers[l].s2;
        int* gl = grab + l * MG_CTL;
        // Two grabs stay in flight, so the atomic's round trip overlaps the copies.
        // At most MG_SWT tiles per layer (the row warps keep their gate/up
        // values in shared memory until the phase ends); others take the rest.
        int q0 = atomicAdd(gl + 0, 1), q1 = atomicAdd(gl + 0, 1), grabs = 2;
        while (!stop) {
          const int t = q0;
          q0 = q1;
          if (t >= n_w1t) {
            end_phase();
            break;
          }
          if (grabs < MG_SWT) {
            q1 = atomicAdd(gl + 0, 1);
            grabs++;
          } else {
            q1 = n_w1t;
          }
          const int nst = t < n_pt ? 1 : 2;
          const int rbase = t < n_pt ? t * MG_W1_RS : n_plain + (t - n_pt) * 2 * MG_W1_RS;
          for (int sub = 0; sub < nst && !stop; sub++) {
            const int r0 = rbase + sub * MG_W1_RS;
            const uint32_t qb = (uint32_t)(MG_W1_RS * d), sb = (uint32_t)(MG_W1_RS * a.s1_stride * 2);
            uint8_t* dst = mg_produce(ring, (t << 1) | sub, qb + sb, a.err);
            if (!dst) {
              stop = true;
              break;
            }
            bulk_g2s(dst, w1p + (size_t)r0 * d, qb, mg_full(ring));
            bulk_g2s(dst + (size_t)MG_W1_RS * d, s1p + (size_t)r0 * a.s1_stride, sb, mg_full(ring));
            ring.i++;
          }
        }
        q0 = atomicAdd(gl + 1, 1);
        q1 = atomicAdd(gl + 1, 1);
        while (!stop) {
          const int u = q0;
          q0 = q1;
          if (u >= units) {
            end_phase();
            break;
          }
          q1 = atomicAdd(gl + 1, 1);
          const int g = u / nsplit, s = u % nsplit;
          const int t0 = s * a.split;
          const int nt = min(T, t0 + a.split) - t0;
          const int n_hist = (s == nsplit - 1) ? nt - 1 : nt;
          const int np = (n_hist + a.kv.P - 1) / a.kv.P;
          uint8_t* dst = mg_produce(ring, u, 2u * np * page_bytes, a.err);
          if (!dst) {
            stop = true;
            break;
          }
          for (int j = 0; j < np; j++) {
            const int page = a.page_table[t0 / a.kv.P + j];
            const size_t o = a.kv.off(l, page, g, 0) * es;
            bulk_g2s(dst + (size_t)j * page_bytes, reinterpret_cast<const uint8_t*>(a.kv.k) + o, page_bytes, mg_full(ring));
            bulk_g2s(dst + (size_t)(pages_per_split + j) * page_bytes, reinterpret_cast<const uint8_t*>(a.kv.v) + o, page_bytes,
                     mg_full(ring));
          }
          ring.i++;
        }
        // Down tiles, then out tiles: at most MG_SWT of each per layer, as for
        // the W1 tiles. Each row's segment of the fused matrix is one copy
        // (quants), plus one for its scales.
        for (int ph = 0; ph < 2 && !stop; ph++) {
          const int nt = ph == 0 ? n_dnt : n_ot;
          const int rs = ph == 0 ? MG_DN_RS : MG_O_RS;
          const int qoff = ph == 0 ? d : 0, qlen = ph == 0 ? ff : d;
          const int soff = ph == 0 ? d / 32 - a.dn_soff : 0, slen = ph == 0 ? a.dn_sstride : osc;
          int* gc = gl + 2 + ph;
          // A fair share per CTA (one more for down tiles): producers grab
          // ahead of their consumers, so an uncapped early CTA would take
          // tiles that later CTAs could start sooner. G * cap covers nt.
          const int cap = min(MG_SWT, max(2, (nt + G - 1) / G + (ph == 0 ? 1 : 0)));
          q0 = atomicAdd(gc, 1);
          q1 = atomicAdd(gc, 1);
          grabs = 2;
          while (!stop) {
            const int t = q0;
            q0 = q1;
            if (t >= nt) {
              end_phase();
              break;
            }
            if (grabs < cap) {
              q1 = atomicAdd(gc, 1);
              grabs++;
            } else {
              q1 = nt;
            }
            const int r0 = t * rs, nr = min(rs, d - r0);
            uint8_t* dst = mg_produce(ring, t, (uint32_t)nr * (qlen + 2 * slen), a.err);
            if (!dst) {
              stop = true;
              break;
            }
            for (int lr = 0; lr < nr; lr++) {
              const size_t r = (size_t)(r0 + lr);
              bulk_g2s(dst + (size_t)lr * qlen, w2p + r * row2 + qoff, (uint32_t)qlen, mg_full(ring));
              bulk_g2s(dst + (size_t)rs * qlen + (size_t)lr * slen * 2, s2p + r * a.s2_stride + soff, (uint32_t)slen * 2u,
                       mg_full(ring));
            }
            ring.i++;
          }
        }
      }
      int* gh = grab + a.L * MG_CTL;
      int h0 = stop ? 0 : atomicAdd(gh, 1), h1 = stop ? 0 : atomicAdd(gh, 1);
      while (!stop) {
        const int t = h0;
        h0 = h1;
        if (t >= n_ht) {
          end_phase();
          break;
        }
        h1 = atomicAdd(gh, 1);
        const int r0 = t * MG_W1_RS, nr = min(MG_W1_RS, a.V - r0);
        const uint32_t qb = (uint32_t)(nr * d), sb = (uint32_t)(nr * a.sh_stride * 2);
        uint8_t* dst = mg_produce(ring, t, qb + sb, a.err);
        if (!dst) {
          stop = true;
          break;
        }
        bulk_g2s(dst, a.head_w + (size_t)r0 * d, qb, mg_full(ring));
        bulk_g2s(dst + (size_t)MG_W1_RS * d, a.head_s + (size_t)r0 * a.sh_stride, sb, mg_full(ring));
        ring.i++;
      }
      // No copy may still be landing in this CTA's shared memory when it exits.
      for (int k = 0; k < ring.n && k < ring.i; k++) {
        const int last = ring.i - 1 - ((ring.i - 1 - k) % ring.n);
        mbar_drain(&ring.full[k], (last / ring.n) & 1);
      }
    }
    return;
  }

  // ------------------------------------------------------------ merge warp
  // Waits until every split of its KV heads has written its partial, merges
  // them (fp32 max / sum) and publishes the digits of the heads' outputs.
  if (warp == MG_MW) {
    float* wo = att + (size_t)MG_CW * a.att_warp;  // [G_q][hd], after the consumer warps' scratch
    const int ghd = G_q * hd, nb16 = ghd / 16;
    for (int l = 0; l < a.L; l++) {
      int* dl = done + l * MG_CTL;
      uint32_t* adig_l = a.adig + (size_t)l * (K2 / 16) * 12;
      float* asx_l = a.asx + (size_t)l * a.asx_stride;
      for (int g = c; g < a.KVH; g += G) {
        int ok = 1;
        if (lane == 0) ok = mg_wait_count(a.counters + g, nsplit, a.err);
        if (!__shfl_sync(0xffffffffu, ok, 0)) return;
        const float* pg = a.part + (size_t)(g * G_q) * a.max_splits * (hd + 2);
        mg_merge_head(pg, a.max_splits, hd, G_q, nsplit, lane, wo);
        __syncwarp();
        for (int b = lane; b < nb16; b += 32) {
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; i++) v[i] = wo[16 * b + i];
          mg_quant16(v, adig_l + (size_t)(g * nb16 + b) * 12, asx_l + g * nb16 + b);
        }
        __syncwarp();
        if (lane == 0) {
          a.counters[g] = 0;  // the next layer's splits count from zero
          if (!(l == a.hold_layer && g == 0 && step == 0)) mg_red_add_release(dl + 3, 1);
        }
        __syncwarp();
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  if (c == 0) {
    // Control words of the next launch (the other parity) start at zero.
    const int n = (a.L + 1) * MG_CTL;
    int* g2 = a.grab + (size_t)(par ^ 1) * n;
    int* d2 = a.done + (size_t)(par ^ 1) * n;
    for (int i = threadIdx.x; i < n; i += MG_CT) {
      g2[i] = 0;
      d2[i] = 0;
    }
  }
  // This position's RoPE row (cos, sin per pair) and KV page, for every layer.
  __shared__ float2 rope_cs[64];
  for (int i = threadIdx.x; i < a.rope.pairs; i += MG_CT) rope_cs[i] = a.rope.table[(size_t)pos * a.rope.pairs + i];
  const int page_cur = a.page_table[pos / a.kv.P];
  const unsigned long long key_in = *(volatile unsigned long long*)(a.keys + par);
  int token = argmax_index(key_in);
  token = (token >= 0 && token < a.V) ? token : 0;
  // Embedding row (Q8_0 decode, matmul.go:24-34), computed by every CTA.
  for (int i = threadIdx.x; i < d; i += MG_CT)
    xs[i] = __fmul_rn(__half2float(a.emb_s[(size_t)token * a.se_stride + i / 32]), (float)a.emb_w[(size_t)token * d + i]);
  named_bar_sync(1, MG_CT);

  uint32_t dr[MG_NJ][12];
  float sxr[MG_NJ];
  unsigned long long best = 0ull;
  int sw_seq = 0, cp_seq = 0;  // local sequence numbers of gate/up and out/down tiles

  // Copies n bytes from global memory into shared memory at dst with one bulk
  // copy issued by consumer thread 0, and waits for it (all consumers).
  auto stage_in = [&](void* dst, const void* src, uint32_t n, void* dst2, const void* src2, uint32_t n2) {
    fence_proxy_async();
    named_bar_sync(1, MG_CT);
    if (threadIdx.x == 0) {
      mbar_expect_tx(inbar, n + n2);
      bulk_g2s(dst, src, n, inbar);
      if (n2) bulk_g2s(dst2, src2, n2, inbar);
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

  // Two dot products of one 16-row stage: rows 2w and 2w+1 against the
  // digit registers (vectors [0, d/16)).
  auto rows16 = [&](const uint8_t* st, int nr, int sstride, float (&acc)[2]) {
    mg_dot2(st, (size_t)d, reinterpret_cast<const __half*>(st + (size_t)MG_W1_RS * d), sstride, 2 * warp, nr, 0, d / 16, dr, sxr,
            acc);
  };

  for (int l = 0; l < a.L; l++) {
    const MegaLayer& ly = a.layers[l];
    int* dl = done + l * MG_CTL;
    uint32_t* adig_l = a.adig + (size_t)l * (K2 / 16) * 12;
    float* asx_l = a.asx + (size_t)l * a.asx_stride;

    // ---- Phase A: LayerNorm, then q/k/v tiles and gate/up tiles (SwiGLU).
    if (l > 0) {
      mg_await(done + (l - 1) * MG_CTL + 2, d, a.err);
      stage_in(xs, a.xl + (size_t)l * d, (uint32_t)d * 4u, nullptr, nullptr, 0);
    }
    mg_ln_digits(xs, d, ly.nw, ly.nb, a.eps, dig, sx);
    load_regs(0, d / 16);
    {
      int n_plain_done = 0;
      bool plain_open = true;
      for (;;) {
        const uint8_t* st;
        const int tag = mg_next_warp(ring, &st, a.err);
        if (tag == -2) break;
        const bool is_plain = tag >= 0 && (tag >> 1) < n_pt;
        if (!is_plain && plain_open) {
          // This warp's q/k/v rows are written (by its lane 0): publish them.
          plain_open = false;
          if (lane == 0 && n_plain_done > 0) mg_red_add_release(dl + 0, 2 * n_plain_done);
        }
        if (tag == -1) {
          mg_release(ring);
          break;
        }
        const int t = tag >> 1, sub = tag & 1;
        float acc[2];
        rows16(st, MG_W1_RS, a.s1_stride, acc);
        mg_release(ring);
        if (is_plain) {
          if (lane == 0) {
            a.qkv[t * MG_W1_RS + 2 * warp] = acc[0];
            a.qkv[t * MG_W1_RS + 2 * warp + 1] = acc[1];
          }
          n_plain_done++;
        } else {
          // Gate/up pair j = 16 (t - n_pt) + 8 sub + warp; its tile is
          // quantised after the loop (kept off the streaming path).
          // (The producer takes at most MG_SWT W1 tiles per layer.)
          if (lane == 0) {
            swg[sw_seq][8 * sub + warp] = acc[0];
            swu[sw_seq][8 * sub + warp] = acc[1];
            if (warp == 0 && sub == 1) swtile[sw_seq] = t;
          }
          if (sub == 1) sw_seq++;
        }
      }
      // SwiGLU values and digits of this layer's gate/up tiles: warp w takes
      // tiles w, w + 8, ... (lane i: value i); read in phase C only.
      named_bar_sync(1, MG_CT);
      for (int q = warp; q < sw_seq; q += MG_CW) {
        const float v = lane < 16 ? silu_mul_stablelm_f32(swg[q][lane], swu[q][lane]) : 0.f;
        const int b = d / 16 + (swtile[q] - n_pt);
        mg_quant16_warp(v, adig_l + (size_t)b * 12, asx_l + b);
      }
      mg_publish(dl + 1, threadIdx.x == 0 ? sw_seq : 0);
      sw_seq = 0;
    }

    // ---- Phase B: attention units (stablelm.go:401-427), split over the
    // history. The k-th unit this CTA receives goes to warp k % 8, so up to
    // one unit per ring slot runs at once; the other warps release its slot.
    // Each unit writes its partial (outputs, max, sum); the merge warp of the
    // KV head's CTA combines them.
    {
      const int ghd = G_q * hd;
      float* wq = att + (size_t)warp * a.att_warp;  // [G_q][hd] rotated queries
      float* cur = wq + ghd;                         // [2][hd] this position's k, v
      float* sc = cur + 2 * hd;                      // [G_q][split] scores / weights
      float* wo = sc + G_q * a.split;                // [G_q][hd] merged outputs
      bool s1 = false;
      int k_unit = 0;
      for (;;) {
        const uint8_t* st;
        const int u = mg_next_warp(ring, &st, a.err);
        if (u < 0) {
          if (u == -1) mg_release(ring);
          break;
        }
        const bool mine = (k_unit % MG_CW) == warp;
        k_unit++;
        if (!mine) {
          mg_release(ring);
          continue;
        }
        if (!s1) {
          if (lane == 0) mg_wait_count(dl + 0, n_plain, a.err);
          __syncwarp();
          s1 = true;
        }
        const int g = u / nsplit, s = u % nsplit;
        const int t0 = s * a.split;
        const int nt = min(T, t0 + a.split) - t0;
        const bool has_cur = (s == nsplit - 1);
        const int n_hist = has_cur ? nt - 1 : nt;
        const int pairs = a.rope.pairs;
        for (int e = lane; e < ghd; e += 32) wq[e] = __ldcg(a.qkv + (g * G_q) * hd + e);
        if (has_cur)
          for (int e = lane; e < hd; e += 32) {
            cur[e] = __ldcg(a.qkv + a.H * hd + g * hd + e);
            cur[hd + e] = __ldcg(a.qkv + (a.H + a.KVH) * hd + g * hd + e);
          }
        __syncwarp();
        // Split-half RoPE (stablelm.go:309-326) with this position's row.
        for (int e = lane; e < (G_q + (has_cur ? 1 : 0)) * pairs; e += 32) {
          const int hh = e / pairs, i = e % pairs;
          float* x = hh < G_q ? wq + hh * hd : cur;
          const float2 cs = rope_cs[i];
          const float x0 = x[i], x1 = x[i + pairs];
          x[i] = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
          x[i + pairs] = __fadd_rn(__fmul_rn(x1, cs.x), __fmul_rn(x0, cs.y));
        }
        __syncwarp();
        if (has_cur) {
          for (int e = lane; e < 2 * hd; e += 32) cur[e] = kv_round(cur[e], a.kv.half);
          __syncwarp();
          const size_t o = a.kv.off(l, page_cur, g, pos % a.kv.P);
          for (int e = lane; e < hd; e += 32) {
            kv_store(a.kv, a.kv.k, o + e, cur[e]);
            kv_store(a.kv, a.kv.v, o + e, cur[hd + e]);
          }
        }
        float* pg = a.part + (size_t)(g * G_q) * a.max_splits * (hd + 2);
        if (a.kv.half)
          mg_unit_core<true>(a, st, pages_per_split * page_bytes, wq, cur, sc, G_q, hd, n_hist, nt, has_cur, pg, s);
        else
          mg_unit_core<false>(a, st, pages_per_split * page_bytes, wq, cur, sc, G_q, hd, n_hist, nt, has_cur, pg, s);
        mg_release(ring);
        __syncwarp();
        // This split's partial is written: count it for the merge warp.
        if (lane == 0) mg_red_add_release(a.counters + g, 1);
        __syncwarp();
      }
    }

    // ---- Phase C: down-projection rows over the SwiGLU blocks (4 K chunks x
    // 2 row pairs per tile); their sums go to xdn for the residual.
    mg_await(dl + 1, ff / 16, a.err);
    {
      const int sb = (d / 16) & ~3, se = (K2 / 16 + 3) & ~3;  // sx staged in 16-byte units
      stage_in(dig + (d / 16) * 12, adig_l + (size_t)(d / 16) * 12, (uint32_t)(ff / 16) * 48u, sx + sb, asx_l + sb,
               (uint32_t)(se - sb) * 4u);
      const int chunk = warp & 3, sub = warp >> 2;
      const int nvd = ff / 16;
      const int vb = d / 16 + (nvd * chunk) / 4, ve = d / 16 + (nvd * (chunk + 1)) / 4;
      load_regs(vb, ve);
      for (;;) {
        const uint8_t* st;
        const int tag = mg_next_warp(ring, &st, a.err);
        if (tag < 0) {
          if (tag == -1) mg_release(ring);
          break;
        }
        const int nr = min(MG_DN_RS, d - tag * MG_DN_RS);
        float acc[2];
        mg_dot2(st, (size_t)ff, reinterpret_cast<const __half*>(st + (size_t)MG_DN_RS * ff) + a.dn_soff, a.dn_sstride, 2 * sub, nr,
                vb - d / 16, ve - d / 16, dr, sxr, acc);
        mg_release(ring);
        // Chunk partials wait in shared memory (the gate/up buffer, free in
        // this phase) until the loop ends. (The producer takes at most MG_SWT
        // down tiles per layer.)
        if (lane == 0) {
          cpart[cp_seq][(2 * sub) * 4 + chunk] = acc[0];
          cpart[cp_seq][(2 * sub + 1) * 4 + chunk] = acc[1];
          if (warp == 0) swtile[cp_seq] = tag;
        }
        cp_seq++;
      }
      // Down sums of this CTA's rows, chunk partials added in a fixed order.
      named_bar_sync(1, MG_CT);
      float* xd = a.xdn + (size_t)l * d;
      int rows = 0;
      for (int i = threadIdx.x; i < cp_seq * MG_DN_RS; i += MG_CT) {
        const int q = i / MG_DN_RS, lr = i % MG_DN_RS;
        const int r = swtile[q] * MG_DN_RS + lr;
        if (r < d) xd[r] = ((cpart[q][lr * 4 + 0] + cpart[q][lr * 4 + 1]) + cpart[q][lr * 4 + 2]) + cpart[q][lr * 4 + 3];
      }
      if (threadIdx.x == 0)
        for (int q = 0; q < cp_seq; q++) rows += min(MG_DN_RS, d - swtile[q] * MG_DN_RS);
      mg_publish(dl + 4, rows);
      cp_seq = 0;
    }

    // ---- Phase D: out-projection rows over the merged attention heads (2
    // rows per warp, all of K), then the parallel residual
    // x + attn_o + mlp_down in the reference's order (stablelm.go:365-377).
    mg_await(dl + 3, a.KVH, a.err);
    {
      stage_in(dig, adig_l, (uint32_t)(d / 16) * 48u, sx, asx_l, (uint32_t)((d / 16 + 3) & ~3) * 4u);
      load_regs(0, d / 16);
      for (;;) {
        const uint8_t* st;
        const int tag = mg_next_warp(ring, &st, a.err);
        if (tag < 0) {
          if (tag == -1) mg_release(ring);
          break;
        }
        const int nr = min(MG_O_RS, d - tag * MG_O_RS);
        float acc[2];
        mg_dot2(st, (size_t)d, reinterpret_cast<const __half*>(st + (size_t)MG_O_RS * d), osc, 2 * warp, nr, 0, d / 16, dr, sxr, acc);
        mg_release(ring);
        if (lane == 0) {
          cpart[cp_seq][2 * warp] = acc[0];
          cpart[cp_seq][2 * warp + 1] = acc[1];
          if (warp == 0) swtile[cp_seq] = tag;
        }
        cp_seq++;
      }
      // Every down sum is written (usually long before).
      mg_await(dl + 4, d, a.err);
      const float* xd = a.xdn + (size_t)l * d;
      float* xo = a.xl + (size_t)(l + 1) * d;
      int rows = 0;
      for (int i = threadIdx.x; i < cp_seq * MG_O_RS; i += MG_CT) {
        const int q = i / MG_O_RS, lr = i % MG_O_RS;
        const int r = swtile[q] * MG_O_RS + lr;
        if (r < d) xo[r] = __fadd_rn(__fadd_rn(xs[r], cpart[q][lr]), __ldcg(xd + r));
      }
      if (threadIdx.x == 0)
        for (int q = 0; q < cp_seq; q++) rows += min(MG_O_RS, d - swtile[q] * MG_O_RS);
      mg_publish(dl + 2, rows);
      cp_seq = 0;
    }
  }

  // ---- Final LayerNorm and lm_head with argmax (stablelm.go:380-385, model.go:622-630).
  mg_await(done + (a.L - 1) * MG_CTL + 2, d, a.err);
  stage_in(xs, a.xl + (size_t)a.L * d, (uint32_t)d * 4u, nullptr, nullptr, 0);
  mg_ln_digits(xs, d, a.fnw, a.fnb, a.eps, dig, sx);
  load_regs(0, d / 16);
  for (;;) {
    const uint8_t* st;
    const int tag = mg_next_warp(ring, &st, a.err);
    if (tag < 0) {
      if (tag == -1) mg_release(ring);
      break;
    }
    const int r0 = tag * MG_W1_RS, nr = min(MG_W1_RS, a.V - r0);
    float acc[2];
    rows16(st, nr, a.sh_stride, acc);
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
    if (b) atomicMax(a.keys + (par ^ 1), b);
    // The last CTA to finish logs the token this step consumed, clears its key
    // (the next step's argmax target) and advances the position; every CTA has
    // read pos, step and the key by then.
    __threadfence();
    if (atomicAdd(done + a.L * MG_CTL + 3, 1) == G - 1) {
      __threadfence();
      const int cnt = a.out_count[0];
      a.out_tokens[cnt] = token;
      a.out_count[0] = cnt + 1;
      a.keys[par] = 0ull;
      *a.pos = pos + 1;
      *a.step = step + 1;
    }
    if (in_phase > 0) mbar_drain(inbar, (in_phase - 1) & 1);
  }
}

// Logs the argmax of the last persistent step (keys[step & 1]).
__global__ void k_finish_mega(const unsigned long long* keys, const int* step, int* out_tokens, int* out_count) {
  if (threadIdx.x == 0) {
    const int cnt = out_count[0];
    out_tokens[cnt] = argmax_index(keys[step[0] & 1]);
    out_count[0] = cnt + 1;
  }
}

}  // namespace tcu
