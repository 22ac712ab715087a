// Decode matrix-vector product for one sequence, streaming the weights
// through shared memory with bulk copies (the hot loop of every decode step).
//
// Same contract as k_gemv (gemv.cuh) for M == 1; replaces mulRowsScalar
// (dot.go:14-70) / mulQ8Rows (dot_simd.go:169-212) on the decode path.
//
// One CTA per SM: warp 8 lane 0 is the producer, keeping NSTAGE row blocks of
// the CTA's contiguous row range in flight with cp.async.bulk (weights do not
// depend on the previous kernel, so it starts before griddepcontrol.wait);
// warps 0..7 consume. Each consumer warp owns one K chunk (KS chunks of at
// most 2560 values) and holds that chunk of the input vector in registers for
// the whole kernel, so shared memory only serves the weights. With KS == 1 a
// warp owns two adjacent rows of every stage (a gate/up pair for SwiGLU);
// with KS > 1 the chunk partials of a row are summed in a fixed order after a
// consumer barrier, so results do not depend on timing.
#pragma once
#include "gemv.cuh"
#include "tma.cuh"

namespace tcu {

constexpr int GS_CONSUMERS = 8;
constexpr int GS_THREADS = (GS_CONSUMERS + 1) * 32;
constexpr int GS_MAX_KS = 4;
constexpr int GS_CHUNK = 2560;  // max K chunk per warp (values held in registers)
constexpr int GS_MAX_STAGES = 8;

struct GemvStreamArgs {
  GemvArgs g;                // M must be 1
  int rs;                    // rows per stage (multiple of 2 * GS_CONSUMERS / KS)
  int nstage;                // pipeline depth (<= GS_MAX_STAGES)
  int kc[GS_MAX_KS + 1];     // chunk boundaries (values), multiples of the vector width
  int lo_chunks;             // EPI_RESID2: chunks [0, lo_chunks) form the first term
  uint32_t stage_bytes;      // bytes per stage buffer (multiple of 128)
  uint32_t off_x, off_part, off_stage;  // shared-memory layout
  int* err;                  // device error word (bounded waits)
};

template <int FMT>
__device__ __forceinline__ float vec_dot_reg(const uint4& w, const float* x) {
  float acc = 0.f;
  if constexpr (FMT == FMT_Q8_0) {
    const uint32_t ww[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
#pragma unroll
    for (int p = 0; p < 4; p++) {
      acc = fmaf(i8f(ww[p], 0), x[4 * p + 0], acc);
      acc = fmaf(i8f(ww[p], 1), x[4 * p + 1], acc);
      acc = fmaf(i8f(ww[p], 2), x[4 * p + 2], acc);
      acc = fmaf(i8f(ww[p], 3), x[4 * p + 3], acc);
    }
  } else if constexpr (FMT == FMT_BF16) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int p = 0; p < 4; p++) {
      acc = fmaf(__uint_as_float(ww[p] << 16), x[2 * p], acc);
      acc = fmaf(__uint_as_float(ww[p] & 0xffff0000u), x[2 * p + 1], acc);
    }
  } else if constexpr (FMT == FMT_F16) {
    const __half2* hh = reinterpret_cast<const __half2*>(&w);
#pragma unroll
    for (int p = 0; p < 4; p++) {
      float2 f = __half22float2(hh[p]);
      acc = fmaf(f.x, x[2 * p], acc);
      acc = fmaf(f.y, x[2 * p + 1], acc);
    }
  } else {
    acc = fmaf(__uint_as_float(w.x), x[0], acc);
    acc = fmaf(__uint_as_float(w.y), x[1], acc);
    acc = fmaf(__uint_as_float(w.z), x[2], acc);
    acc = fmaf(__uint_as_float(w.w), x[3], acc);
  }
  return acc;
}

template <int FMT, int PRO, int EPI, int KS>
__global__ void __launch_bounds__(GS_THREADS, 1) k_gemv_stream(GemvStreamArgs sa) {
  constexpr int E = VecTraits<FMT>::E;
  constexpr int BYTES = VecTraits<FMT>::BYTES;
  constexpr int NJ = GS_CHUNK / 32 / E;  // vectors per lane per row
  constexpr int SUBG = GS_CONSUMERS / KS;
  const GemvArgs& a = sa.g;
  const int K = a.W.cols, R = a.W.rows;
  const size_t row_bytes = (size_t)K * BYTES;
  extern __shared__ __align__(128) uint8_t gs_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(gs_smem);
  uint64_t* empty = full + GS_MAX_STAGES;
  float* xs = reinterpret_cast<float*>(gs_smem + sa.off_x);
  float* part = reinterpret_cast<float*>(gs_smem + sa.off_part);
  uint8_t* stages = gs_smem + sa.off_stage;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = sa.nstage, rs = sa.rs;

  // This CTA's rows: a balanced share of the row pairs.
  const int pairs = (R + 1) >> 1;
  const int rb = min(R, 2 * (int)(((long long)pairs * blockIdx.x) / gridDim.x));
  const int re = min(R, 2 * (int)(((long long)pairs * (blockIdx.x + 1)) / gridDim.x));
  const int nst = (re - rb + rs - 1) / rs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ns; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], GS_CONSUMERS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == GS_CONSUMERS) {
    // Producer: weights are independent of the previous kernel.
    if (lane == 0) {
      for (int i = 0; i < nst; i++) {
        const int slot = i % ns;
        if (i >= ns && !mbar_wait(&empty[slot], ((i / ns) - 1) & 1, sa.err)) break;
        const int r0 = rb + i * rs, nr = min(rs, re - r0);
        const uint32_t qb = (uint32_t)(nr * row_bytes);
        const uint32_t sb = (FMT == FMT_Q8_0) ? (uint32_t)(nr * a.W.sstride * 2) : 0u;
        uint8_t* dst = stages + (size_t)slot * sa.stage_bytes;
        mbar_expect_tx(&full[slot], qb + sb);
        bulk_g2s(dst, a.W.w + (size_t)r0 * row_bytes, qb, &full[slot]);
        if (FMT == FMT_Q8_0) bulk_g2s(dst + (size_t)rs * row_bytes, a.W.s + (size_t)r0 * a.W.sstride, sb, &full[slot]);
      }
    }
    return;
  }

  // Consumers: input vector (depends on the previous kernel).
  pdl_wait();
  const float* in = a.in;
  if constexpr (PRO == PRO_COPY) {
    for (int k = threadIdx.x; k < K; k += GS_CONSUMERS * 32) xs[k] = in[k];
  } else if constexpr (PRO == PRO_LN) {
    __shared__ double red[GS_CONSUMERS];
    double s = 0;
    for (int k = threadIdx.x; k < K; k += GS_CONSUMERS * 32) s += (double)in[k];
    s = warp_sum_d(s);
    if (lane == 0) red[warp] = s;
    named_bar_sync(1, GS_CONSUMERS * 32);
    double tot = 0;
    for (int w = 0; w < GS_CONSUMERS; w++) tot += red[w];
    const double mean = tot / (double)K;
    named_bar_sync(1, GS_CONSUMERS * 32);
    double v = 0;
    for (int k = threadIdx.x; k < K; k += GS_CONSUMERS * 32) {
      double d = (double)in[k] - mean;
      v += d * d;
    }
    v = warp_sum_d(v);
    if (lane == 0) red[warp] = v;
    named_bar_sync(1, GS_CONSUMERS * 32);
    double var = 0;
    for (int w = 0; w < GS_CONSUMERS; w++) var += red[w];
    const float inv = (float)(1.0 / sqrt(var / (double)K + a.eps));
    const float mf = (float)mean;
    for (int k = threadIdx.x; k < K; k += GS_CONSUMERS * 32)
      xs[k] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(in[k], mf), inv), a.nw[k]), a.nb[k]);
  } else {
    __shared__ float inv_s;
    if (threadIdx.x == 0) {
      float ss = 0.f;
      for (int k = 0; k < K; k++) ss = __fadd_rn(ss, __fmul_rn(in[k], in[k]));
      inv_s = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(__fdiv_rn(ss, (float)K), 1e-5f)));
    }
    named_bar_sync(1, GS_CONSUMERS * 32);
    for (int k = threadIdx.x; k < K; k += GS_CONSUMERS * 32) xs[k] = __fmul_rn(a.nw[k], __fmul_rn(inv_s, in[k]));
  }
  named_bar_sync(1, GS_CONSUMERS * 32);

  // This warp's K chunk of the input, in registers.
  const int chunk = warp % KS, sub = warp / KS;
  const int v_begin = sa.kc[chunk] / E, v_end = sa.kc[chunk + 1] / E;
  float xr[NJ * E];
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int v = v_begin + lane + 32 * j;
#pragma unroll
    for (int e = 0; e < E; e += 4) {
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (v < v_end) f = *reinterpret_cast<const float4*>(xs + (size_t)v * E + e);
      xr[j * E + e] = f.x;
      xr[j * E + e + 1] = f.y;
      xr[j * E + e + 2] = f.z;
      xr[j * E + e + 3] = f.w;
    }
  }

  const int rpw = rs / SUBG;  // rows per warp per stage (2 when KS == 1)
  unsigned long long best = 0ull;
  for (int i = 0; i < nst; i++) {
    const int slot = i % ns;
    // A timed-out wait flags sa.err and the warp carries on (with stale data)
    // so that every consumer still reaches the same barriers; the host
    // reports the error. Every issued stage is waited for exactly once.
    mbar_wait(&full[slot], (i / ns) & 1, sa.err);
    const int r0 = rb + i * rs, nr = min(rs, re - r0);
    const uint8_t* wst = stages + (size_t)slot * sa.stage_bytes;
    const __half* sst = reinterpret_cast<const __half*>(wst + (size_t)rs * row_bytes);
    float acc[4];
#pragma unroll
    for (int t = 0; t < 4; t++) acc[t] = 0.f;
#pragma unroll
    for (int t = 0; t < 4; t++) {
      if (t < rpw) {
        const int lr = sub * rpw + t;
        if (lr < nr) {
          const uint8_t* wrow = wst + (size_t)lr * row_bytes;
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < NJ; j++) {
            const int v = v_begin + lane + 32 * j;
            if (v < v_end) {
              const uint4 w = *reinterpret_cast<const uint4*>(wrow + (size_t)v * 16);
              float p = vec_dot_reg<FMT>(w, xr + j * E);
              if constexpr (FMT == FMT_Q8_0) p *= __half2float(sst[(size_t)lr * a.W.sstride + (v >> 1)]);
              s += p;
            }
          }
          acc[t] = warp_sum(s);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);  // this warp is done with the stage's weights

    if constexpr (KS == 1) {
      if (lane == 0) {
        const int lr0 = sub * rpw;
        if (lr0 < nr) {
          const int r = r0 + lr0;
          const bool has1 = lr0 + 1 < nr;
          if constexpr (EPI == EPI_GLU) {
            if (r < a.n_plain) {
              a.out[r] = acc[0];
              if (has1) a.out[r + 1] = acc[1];
            } else {
              a.glu_out[(r - a.n_plain) >> 1] = a.glu_act ? silu_mul_llama(acc[0], acc[1]) : silu_mul_stablelm(acc[0], acc[1]);
            }
          } else if constexpr (EPI == EPI_STORE) {
            a.out[r] = acc[0];
            if (has1) a.out[r + 1] = acc[1];
          } else if constexpr (EPI == EPI_RESID1) {
            a.resid[r] = __fadd_rn(a.resid[r], acc[0]);
            if (has1) a.resid[r + 1] = __fadd_rn(a.resid[r + 1], acc[1]);
          } else if constexpr (EPI == EPI_HEAD) {
            if (a.logits) {
              a.logits[r] = acc[0];
              if (has1) a.logits[r + 1] = acc[1];
            }
            unsigned long long k0 = argmax_pack(acc[0], r);
            best = k0 > best ? k0 : best;
            if (has1) {
              unsigned long long k1 = argmax_pack(acc[1], r + 1);
              best = k1 > best ? k1 : best;
            }
          }
        }
      }
    } else {
      float* ps = part + (size_t)slot * rs * KS;
      if (lane == 0) {
#pragma unroll
        for (int t = 0; t < 4; t++)
          if (t < rpw) ps[(sub * rpw + t) * KS + chunk] = acc[t];
      }
      named_bar_sync(1, GS_CONSUMERS * 32);
      if (warp == 0 && lane < nr) {
        float lo = 0.f, hi = 0.f;
#pragma unroll
        for (int c = 0; c < KS; c++) {
          if (c < sa.lo_chunks)
            lo += ps[lane * KS + c];
          else
            hi += ps[lane * KS + c];
        }
        const int r = r0 + lane;
        if constexpr (EPI == EPI_RESID2) {
          a.resid[r] = __fadd_rn(__fadd_rn(a.resid[r], lo), hi);
        } else if constexpr (EPI == EPI_RESID1) {
          a.resid[r] = __fadd_rn(a.resid[r], lo + hi);
        } else if constexpr (EPI == EPI_STORE) {
          a.out[r] = lo + hi;
        }
      }
    }
  }
  if constexpr (EPI == EPI_HEAD) {
    __shared__ unsigned long long bred[GS_CONSUMERS];
    if (lane == 0) bred[warp] = best;
    named_bar_sync(1, GS_CONSUMERS * 32);
    if (threadIdx.x == 0) {
      unsigned long long b = 0;
      for (int w = 0; w < GS_CONSUMERS; w++) b = bred[w] > b ? bred[w] : b;
      atomicMax(a.argmax, b);
    }
  }
}

}  // namespace tcu
