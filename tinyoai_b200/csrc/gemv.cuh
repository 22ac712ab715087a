// Decode matrix-vector kernels: y = W x for M <= 4 input vectors, streaming
// the weights once from HBM with 16-byte coalesced loads.
//
// Replaces weightTensor.mulScratch -> mulRows -> mulRowsScalar
// (safetensors.go:275-280, dot.go:14-70) and the MLX quantized matmul of the
// decode step (internal/mlx/mlx.go:423-429). The prologue fuses the LayerNorm
// (stablelm.go:288-305) or RMSNorm (model.go:591-600) that feeds the product;
// the epilogues fuse SwiGLU (stablelm.go:369-374), the parallel residual
// (stablelm.go:375-377), the llama residual (model.go:465,476) and the
// lm_head argmax (model.go:622-630).
#pragma once
#include "common.cuh"

namespace tcu {

enum Pro : int { PRO_COPY = 0, PRO_LN = 1, PRO_RMS = 2 };
enum Epi : int { EPI_STORE = 0, EPI_GLU = 1, EPI_RESID2 = 2, EPI_RESID1 = 3, EPI_HEAD = 4 };

constexpr int GEMV_MAX_M = 4;
constexpr int GEMV_WARPS = 8;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;
constexpr int GEMV_UNROLL = 4;

struct GemvArgs {
  DMat W;
  int M;
  // prologue input: in[m * in_stride + k], k < W.cols
  const float* in;
  int in_stride;
  const float* nw;  // norm weight (float32, decoded at load)
  const float* nb;  // norm bias (LayerNorm only)
  double eps;
  // EPI_STORE / EPI_GLU plain rows: out[m * out_stride + r], r < n_plain
  float* out;
  int out_stride;
  int n_plain;
  // EPI_GLU interleaved (gate, up) row pairs -> glu_out[m * glu_stride + p]
  float* glu_out;
  int glu_stride;
  int glu_act;  // 0: StableLM, 1: llama2.c
  // EPI_RESID*: resid[m * resid_stride + r] updated in place
  float* resid;
  int resid_stride;
  int k_split;  // EPI_RESID2: columns [0, k_split) feed the first term
  // EPI_HEAD
  unsigned long long* argmax;  // [M], max-reduced
  float* logits;               // optional [M][logits_stride]
  int logits_stride;
};

template <int FMT>
struct VecTraits;
template <>
struct VecTraits<FMT_Q8_0> {
  static constexpr int E = 16;
  static constexpr int BYTES = 1;
};
template <>
struct VecTraits<FMT_BF16> {
  static constexpr int E = 8;
  static constexpr int BYTES = 2;
};
template <>
struct VecTraits<FMT_F16> {
  static constexpr int E = 8;
  static constexpr int BYTES = 2;
};
template <>
struct VecTraits<FMT_F32> {
  static constexpr int E = 4;
  static constexpr int BYTES = 4;
};

// Shared-memory position of element k in a vector of K values: elements are
// split into E/4 planes so that lane l reading vector v hits consecutive
// 16-byte words (no bank conflicts). With E == 4 this is the identity, for
// any K.
template <int E>
__device__ __forceinline__ int swz(int k, int K) {
  int c = k / E, r = k % E;
  return (r >> 2) * ((K / E) * 4) + c * 4 + (r & 3);
}

// int8 -> float exactly: byte b (after xor 0x80) placed in the mantissa of
// 2^23, then 2^23 + 128 subtracted.
__device__ __forceinline__ float i8f(uint32_t wx, int k) {
  return __uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7440u | (uint32_t)k)) - 8388736.0f;
}

template <int FMT>
__device__ __forceinline__ float vec_dot(const uint4& w, const float* xs, int v, int K) {
  const float4* xp = reinterpret_cast<const float4*>(xs);
  float acc = 0.f;
  if constexpr (FMT == FMT_Q8_0) {
    const uint32_t ww[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
#pragma unroll
    for (int p = 0; p < 4; p++) {
      float4 x = xp[p * (K >> 4) + v];
      acc = fmaf(i8f(ww[p], 0), x.x, acc);
      acc = fmaf(i8f(ww[p], 1), x.y, acc);
      acc = fmaf(i8f(ww[p], 2), x.z, acc);
      acc = fmaf(i8f(ww[p], 3), x.w, acc);
    }
  } else if constexpr (FMT == FMT_BF16) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int p = 0; p < 2; p++) {
      float4 x = xp[p * (K >> 3) + v];
      acc = fmaf(__uint_as_float(ww[2 * p] << 16), x.x, acc);
      acc = fmaf(__uint_as_float(ww[2 * p] & 0xffff0000u), x.y, acc);
      acc = fmaf(__uint_as_float(ww[2 * p + 1] << 16), x.z, acc);
      acc = fmaf(__uint_as_float(ww[2 * p + 1] & 0xffff0000u), x.w, acc);
    }
  } else if constexpr (FMT == FMT_F16) {
    const __half2* hh = reinterpret_cast<const __half2*>(&w);
#pragma unroll
    for (int p = 0; p < 2; p++) {
      float4 x = xp[p * (K >> 3) + v];
      float2 a = __half22float2(hh[2 * p]);
      float2 b = __half22float2(hh[2 * p + 1]);
      acc = fmaf(a.x, x.x, acc);
      acc = fmaf(a.y, x.y, acc);
      acc = fmaf(b.x, x.z, acc);
      acc = fmaf(b.y, x.w, acc);
    }
  } else {  // F32
    float4 x = xp[v];
    acc = fmaf(__uint_as_float(w.x), x.x, acc);
    acc = fmaf(__uint_as_float(w.y), x.y, acc);
    acc = fmaf(__uint_as_float(w.z), x.z, acc);
    acc = fmaf(__uint_as_float(w.w), x.w, acc);
  }
  return acc;
}

__device__ __forceinline__ double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0;
  for (int i = 0; i < nw; i++) t += red[i];
  return t;
}

// Fills xs[m][.] (swizzled with plane width E) from the prologue input.
template <int PRO, int E>
__device__ void gemv_prologue(const GemvArgs& a, float* xs, int K, double* red) {
  for (int m = 0; m < a.M; m++) {
    const float* in = a.in + (size_t)m * a.in_stride;
    float* dst = xs + (size_t)m * K;
    if constexpr (PRO == PRO_COPY) {
      for (int k = threadIdx.x; k < K; k += blockDim.x) dst[swz<E>(k, K)] = in[k];
    } else if constexpr (PRO == PRO_LN) {
      // stablelm.go:292-303: float64 mean and variance, float32 affine.
      double s = 0;
      for (int k = threadIdx.x; k < K; k += blockDim.x) s += (double)in[k];
      double mean = block_sum_d(s, red) / (double)K;
      double v = 0;
      for (int k = threadIdx.x; k < K; k += blockDim.x) {
        double d = (double)in[k] - mean;
        v += d * d;
      }
      double var = block_sum_d(v, red);
      float inv = (float)(1.0 / sqrt(var / (double)K + a.eps));
      float mf = (float)mean;
      for (int k = threadIdx.x; k < K; k += blockDim.x) {
        float t = __fmul_rn(__fmul_rn(__fsub_rn(in[k], mf), inv), a.nw[k]);
        dst[swz<E>(k, K)] = __fadd_rn(t, a.nb[k]);
      }
    } else {
      // model.go:591-600: sequential float32 sum of squares.
      __shared__ float inv_s;
      if (threadIdx.x == 0) {
        float ss = 0.f;
        for (int k = 0; k < K; k++) ss = __fadd_rn(ss, __fmul_rn(in[k], in[k]));
        float mean = __fadd_rn(__fdiv_rn(ss, (float)K), 1e-5f);
        inv_s = __fdiv_rn(1.0f, (float)sqrt((double)mean));
      }
      __syncthreads();
      float inv = inv_s;
      for (int k = threadIdx.x; k < K; k += blockDim.x) dst[swz<E>(k, K)] = __fmul_rn(a.nw[k], __fmul_rn(inv, in[k]));
      __syncthreads();
    }
  }
  __syncthreads();
}

template <int EPI, int M>
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, int r0, bool has1, float (&lo)[M][2], float (&hi)[M][2],
                                              unsigned long long (&best)[M]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int m = 0; m < M; m++) {
    float y0 = lo[m][0], y1 = lo[m][1];
    if constexpr (EPI == EPI_STORE) {
      if (lane == 0) {
        a.out[(size_t)m * a.out_stride + r0] = y0;
        if (has1) a.out[(size_t)m * a.out_stride + r0 + 1] = y1;
      }
    } else if constexpr (EPI == EPI_GLU) {
      if (lane == 0) {
        if (r0 < a.n_plain) {
          a.out[(size_t)m * a.out_stride + r0] = y0;
          if (has1) a.out[(size_t)m * a.out_stride + r0 + 1] = y1;
        } else {
          int p = (r0 - a.n_plain) >> 1;
          float h = a.glu_act ? silu_mul_llama(y0, y1) : silu_mul_stablelm(y0, y1);
          a.glu_out[(size_t)m * a.glu_stride + p] = h;
        }
      }
    } else if constexpr (EPI == EPI_RESID2) {
      if (lane == 0) {
        float* x = a.resid + (size_t)m * a.resid_stride;
        x[r0] = __fadd_rn(__fadd_rn(x[r0], y0), hi[m][0]);
        if (has1) x[r0 + 1] = __fadd_rn(__fadd_rn(x[r0 + 1], y1), hi[m][1]);
      }
    } else if constexpr (EPI == EPI_RESID1) {
      if (lane == 0) {
        float* x = a.resid + (size_t)m * a.resid_stride;
        x[r0] = __fadd_rn(x[r0], y0);
        if (has1) x[r0 + 1] = __fadd_rn(x[r0 + 1], y1);
      }
    } else {  // EPI_HEAD
      if (lane == 0 && a.logits) {
        a.logits[(size_t)m * a.logits_stride + r0] = y0;
        if (has1) a.logits[(size_t)m * a.logits_stride + r0 + 1] = y1;
      }
      unsigned long long k0 = argmax_pack(y0, r0);
      if (k0 > best[m]) best[m] = k0;
      if (has1) {
        unsigned long long k1 = argmax_pack(y1, r0 + 1);
        if (k1 > best[m]) best[m] = k1;
      }
    }
  }
}

// Vectorised kernel: one warp computes two adjacent rows at a time over the
// whole reduction; lanes stride over 16-byte weight vectors.
template <int FMT, int M, int PRO, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(GemvArgs a) {
  extern __shared__ __align__(16) float gemv_smem[];
  __shared__ double red[GEMV_WARPS];
  constexpr int E = VecTraits<FMT>::E;
  const int K = a.W.cols, R = a.W.rows;
  float* xs = gemv_smem;
  gemv_prologue<PRO, E>(a, xs, K, red);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = K / E;
  const int npairs = (R + 1) >> 1;
  const size_t row_bytes = (size_t)K * VecTraits<FMT>::BYTES;
  const int vsplit = (EPI == EPI_RESID2) ? a.k_split / E : nvec;
  unsigned long long best[M];
#pragma unroll
  for (int m = 0; m < M; m++) best[m] = 0ull;

  for (int pr = blockIdx.x * GEMV_WARPS + warp; pr < npairs; pr += gridDim.x * GEMV_WARPS) {
    const int r0 = 2 * pr;
    const bool has1 = r0 + 1 < R;
    const uint8_t* w0 = a.W.w + (size_t)r0 * row_bytes;
    const uint8_t* w1 = has1 ? w0 + row_bytes : w0;
    const __half* s0 = (FMT == FMT_Q8_0) ? a.W.s + (size_t)r0 * a.W.sstride : nullptr;
    const __half* s1 = (FMT == FMT_Q8_0) ? (has1 ? s0 + a.W.sstride : s0) : nullptr;
    float lo[M][2], hi[M][2];
#pragma unroll
    for (int m = 0; m < M; m++) lo[m][0] = lo[m][1] = hi[m][0] = hi[m][1] = 0.f;

    for (int v0 = lane; v0 < nvec; v0 += 32 * GEMV_UNROLL) {
      uint4 wa[GEMV_UNROLL], wb[GEMV_UNROLL];
      float sa[GEMV_UNROLL], sb[GEMV_UNROLL];
#pragma unroll
      for (int u = 0; u < GEMV_UNROLL; u++) {
        const int v = v0 + 32 * u;
        if (v < nvec) {
          wa[u] = ld_stream16(w0 + (size_t)v * 16);
          wb[u] = ld_stream16(w1 + (size_t)v * 16);
          if constexpr (FMT == FMT_Q8_0) {
            sa[u] = __half2float(s0[v >> 1]);
            sb[u] = __half2float(s1[v >> 1]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < GEMV_UNROLL; u++) {
        const int v = v0 + 32 * u;
        if (v < nvec) {
#pragma unroll
          for (int m = 0; m < M; m++) {
            const float* xm = xs + (size_t)m * K;
            float p0 = vec_dot<FMT>(wa[u], xm, v, K);
            float p1 = vec_dot<FMT>(wb[u], xm, v, K);
            if constexpr (FMT == FMT_Q8_0) {
              p0 *= sa[u];
              p1 *= sb[u];
            }
            if (EPI == EPI_RESID2 && v >= vsplit) {
              hi[m][0] += p0;
              hi[m][1] += p1;
            } else {
              lo[m][0] += p0;
              lo[m][1] += p1;
            }
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; m++) {
      lo[m][0] = warp_sum(lo[m][0]);
      lo[m][1] = warp_sum(lo[m][1]);
      if constexpr (EPI == EPI_RESID2) {
        hi[m][0] = warp_sum(hi[m][0]);
        hi[m][1] = warp_sum(hi[m][1]);
      }
    }
    gemv_epilogue<EPI, M>(a, r0, has1, lo, hi, best);
  }
  if constexpr (EPI == EPI_HEAD) {
    __shared__ unsigned long long bred[GEMV_WARPS][GEMV_MAX_M];
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < M; m++) bred[warp][m] = best[m];
    }
    __syncthreads();
    if (threadIdx.x < M) {
      unsigned long long b = 0;
      for (int w = 0; w < GEMV_WARPS; w++) b = bred[w][threadIdx.x] > b ? bred[w][threadIdx.x] : b;
      atomicMax(a.argmax + threadIdx.x, b);
    }
  }
}

// Generic kernel for every format and shape (K-quant blocks, odd widths):
// elements are decoded one at a time exactly as the reference decoder does.
template <int M, int PRO, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv_generic(GemvArgs a) {
  extern __shared__ __align__(16) float gemv_smem[];
  __shared__ double red[GEMV_WARPS];
  const int K = a.W.cols, R = a.W.rows;
  float* xs = gemv_smem;
  gemv_prologue<PRO, 4>(a, xs, K, red);  // E == 4: linear layout
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int npairs = (R + 1) >> 1;
  unsigned long long best[M];
#pragma unroll
  for (int m = 0; m < M; m++) best[m] = 0ull;
  for (int pr = blockIdx.x * GEMV_WARPS + warp; pr < npairs; pr += gridDim.x * GEMV_WARPS) {
    const int r0 = 2 * pr;
    const bool has1 = r0 + 1 < R;
    float lo[M][2], hi[M][2];
#pragma unroll
    for (int m = 0; m < M; m++) lo[m][0] = lo[m][1] = hi[m][0] = hi[m][1] = 0.f;
    if ((a.W.fmt == FMT_Q6_K || a.W.fmt == FMT_Q5_K) && (K & 255) == 0 && (EPI != EPI_RESID2 || (a.k_split & 7) == 0)) {
      // K-quant rows of whole super-blocks: a lane takes 8 values of one
      // scale group per step (the block address and scale once).
      for (int k0 = lane * 8; k0 < K; k0 += 256) {
        float w0[8], w1[8];
        kquant_decode8(a.W, r0, k0, w0);
        if (has1)
          kquant_decode8(a.W, r0 + 1, k0, w1);
        else
#pragma unroll
          for (int i = 0; i < 8; i++) w1[i] = 0.f;
        const bool second = EPI == EPI_RESID2 && k0 >= a.k_split;
#pragma unroll
        for (int m = 0; m < M; m++) {
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const float x = xs[(size_t)m * K + k0 + i];
            if (second) {
              hi[m][0] = fmaf(w0[i], x, hi[m][0]);
              hi[m][1] = fmaf(w1[i], x, hi[m][1]);
            } else {
              lo[m][0] = fmaf(w0[i], x, lo[m][0]);
              lo[m][1] = fmaf(w1[i], x, lo[m][1]);
            }
          }
        }
      }
    } else
    for (int k = lane; k < K; k += 32) {
      float w0 = dmat_at(a.W, r0, k);
      float w1 = has1 ? dmat_at(a.W, r0 + 1, k) : 0.f;
#pragma unroll
      for (int m = 0; m < M; m++) {
        float x = xs[(size_t)m * K + k];
        if (EPI == EPI_RESID2 && k >= a.k_split) {
          hi[m][0] = fmaf(w0, x, hi[m][0]);
          hi[m][1] = fmaf(w1, x, hi[m][1]);
        } else {
          lo[m][0] = fmaf(w0, x, lo[m][0]);
          lo[m][1] = fmaf(w1, x, lo[m][1]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; m++) {
      lo[m][0] = warp_sum(lo[m][0]);
      lo[m][1] = warp_sum(lo[m][1]);
      hi[m][0] = warp_sum(hi[m][0]);
      hi[m][1] = warp_sum(hi[m][1]);
    }
    gemv_epilogue<EPI, M>(a, r0, has1, lo, hi, best);
  }
  if constexpr (EPI == EPI_HEAD) {
    __shared__ unsigned long long bred[GEMV_WARPS][GEMV_MAX_M];
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < M; m++) bred[warp][m] = best[m];
    }
    __syncthreads();
    if (threadIdx.x < M) {
      unsigned long long b = 0;
      for (int w = 0; w < GEMV_WARPS; w++) b = bred[w][threadIdx.x] > b ? bred[w][threadIdx.x] : b;
      atomicMax(a.argmax + threadIdx.x, b);
    }
  }
}

}  // namespace tcu
