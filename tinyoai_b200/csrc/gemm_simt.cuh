// Prefill / batched projection on CUDA cores: out[n][R] = A[n][K] * W[R][K]^T
// with W dequantized into shared memory tile by tile.
//
// Replaces weightTensor.mulBatch (matmul.go:55-95) for prompt chunks and
// branch batches, with the epilogues of the decode kernels (gemv.cuh). This
// is the portable float32 path; the tensor-core path lives in gemm_tc.cuh.
#pragma once
#include "common.cuh"
#include "gemv.cuh"

namespace tcu {

constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 32, SG_THREADS = 256;

struct GemmArgs {
  DMat W;
  int n;           // rows of A (tokens)
  const float* A;  // [n][lda]
  int lda;
  // epilogue, as GemvArgs but indexed by token
  float* out;
  int out_stride;
  int n_plain;
  float* glu_out;
  int glu_stride;
  int glu_act;
  float* resid;
  int resid_stride;
  int k_split;
  // Split K (out/down rows with few row tiles): slice blockIdx.z covers
  // columns [z * k_per_z, (z + 1) * k_per_z) and writes its sums to
  // part[z][n][rows] instead of applying the epilogue (nullptr: no split).
  float* part;
  int k_per_z;
};

// Decodes W[r][k0 .. k0+8) into dst (zeros outside the matrix).
__device__ __forceinline__ void decode8(const DMat& W, int r, int k0, float* dst) {
  if (r >= W.rows) {
#pragma unroll
    for (int i = 0; i < 8; i++) dst[i] = 0.f;
    return;
  }
  const int K = W.cols;
  if (W.fmt == FMT_Q8_0 && k0 + 8 <= K) {
    const float s = __half2float(W.s[(size_t)r * W.sstride + k0 / 32]);
    const uint2 q = *reinterpret_cast<const uint2*>(W.w + (size_t)r * K + k0);
    const uint32_t a = q.x ^ 0x80808080u, b = q.y ^ 0x80808080u;
#pragma unroll
    for (int i = 0; i < 4; i++) dst[i] = __fmul_rn(s, i8f(a, i));
#pragma unroll
    for (int i = 0; i < 4; i++) dst[4 + i] = __fmul_rn(s, i8f(b, i));
    return;
  }
  if (W.fmt == FMT_BF16 && k0 + 8 <= K && (K & 7) == 0) {
    const uint4 q = *reinterpret_cast<const uint4*>(W.w + ((size_t)r * K + k0) * 2);
    const uint32_t ww[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      dst[2 * i] = __uint_as_float(ww[i] << 16);
      dst[2 * i + 1] = __uint_as_float(ww[i] & 0xffff0000u);
    }
    return;
  }
  if ((W.fmt == FMT_Q6_K || W.fmt == FMT_Q5_K) && (K & 255) == 0 && k0 + 8 <= K) {
    kquant_decode8(W, r, k0, dst);
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; i++) dst[i] = (k0 + i < K) ? dmat_at(W, r, k0 + i) : 0.f;
}

template <int EPI>
__global__ void __launch_bounds__(SG_THREADS) k_gemm_simt(GemmArgs a) {
  __shared__ float As[SG_BK][SG_BM + 4];
  __shared__ float Ws[SG_BK][SG_BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;  // rows tx*4.., tokens ty*4..
  const int m0 = blockIdx.y * SG_BM, r0 = blockIdx.x * SG_BN;
  const int K = a.W.cols;
  float lo[4][4], hi[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) lo[i][j] = hi[i][j] = 0.f;
  const int lr = tid / 4, lk = (tid % 4) * 8;  // loader: row/token lr, columns lk..lk+7
  const int k_begin = a.part ? blockIdx.z * a.k_per_z : 0;
  const int k_end = a.part ? min(K, k_begin + a.k_per_z) : K;
  for (int k0 = k_begin; k0 < k_end; k0 += SG_BK) {
    {
      const int tok = m0 + lr;
      const float* ap = a.A + (size_t)tok * a.lda + k0 + lk;
#pragma unroll
      for (int i = 0; i < 8; i++) As[lk + i][lr] = (tok < a.n && k0 + lk + i < K) ? ap[i] : 0.f;
      float w8[8];
      decode8(a.W, r0 + lr, k0 + lk, w8);
#pragma unroll
      for (int i = 0; i < 8; i++) Ws[lk + i][lr] = w8[i];
    }
    __syncthreads();
    const int kmax = min(SG_BK, K - k0);
    for (int kk = 0; kk < kmax; kk++) {
      const float4 av = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 wv = *reinterpret_cast<const float4*>(&Ws[kk][tx * 4]);
      const float ar[4] = {av.x, av.y, av.z, av.w};
      const float wr[4] = {wv.x, wv.y, wv.z, wv.w};
      if (EPI == EPI_RESID2 && k0 + kk >= a.k_split) {
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int j = 0; j < 4; j++) hi[i][j] = fmaf(ar[i], wr[j], hi[i][j]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int j = 0; j < 4; j++) lo[i][j] = fmaf(ar[i], wr[j], lo[i][j]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int tok = m0 + ty * 4 + i;
    if (tok >= a.n) continue;
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      const int r = r0 + tx * 4 + j;
      if (r >= a.W.rows) continue;
      const bool has1 = r + 1 < a.W.rows;
      if (a.part) {  // a slice lies wholly before or after k_split: one of lo, hi is zero
        float* pp = a.part + ((size_t)blockIdx.z * a.n + tok) * a.W.rows + r;
        pp[0] = lo[i][j] + hi[i][j];
        if (has1) pp[1] = lo[i][j + 1] + hi[i][j + 1];
        continue;
      }
      if constexpr (EPI == EPI_STORE) {
        a.out[(size_t)tok * a.out_stride + r] = lo[i][j];
        if (has1) a.out[(size_t)tok * a.out_stride + r + 1] = lo[i][j + 1];
      } else if constexpr (EPI == EPI_GLU) {
        if (r < a.n_plain) {
          a.out[(size_t)tok * a.out_stride + r] = lo[i][j];
          if (has1) a.out[(size_t)tok * a.out_stride + r + 1] = lo[i][j + 1];
        } else {
          const int p = (r - a.n_plain) >> 1;
          a.glu_out[(size_t)tok * a.glu_stride + p] =
              a.glu_act ? silu_mul_llama(lo[i][j], lo[i][j + 1]) : silu_mul_stablelm(lo[i][j], lo[i][j + 1]);
        }
      } else if constexpr (EPI == EPI_RESID2) {
        float* x = a.resid + (size_t)tok * a.resid_stride;
        x[r] = __fadd_rn(__fadd_rn(x[r], lo[i][j]), hi[i][j]);
        if (has1) x[r + 1] = __fadd_rn(__fadd_rn(x[r + 1], lo[i][j + 1]), hi[i][j + 1]);
      } else if constexpr (EPI == EPI_RESID1) {
        float* x = a.resid + (size_t)tok * a.resid_stride;
        x[r] = __fadd_rn(x[r], lo[i][j]);
        if (has1) x[r + 1] = __fadd_rn(x[r + 1], lo[i][j + 1]);
      }
    }
  }
}

// Row-wise LayerNorm / RMSNorm for prefill chunks (stablelm.go:288-305,
// model.go:591-600): out[j] = norm(in[j]) for j < n.
struct NormRowsArgs {
  int n, K;
  const float* in;
  int in_stride;
  float* out;
  int out_stride;
  const float* nw;
  const float* nb;
  double eps;
  int rms;
};

__global__ void k_norm_rows(NormRowsArgs a) {
  __shared__ double red[32];
  const int j = blockIdx.x;
  const float* in = a.in + (size_t)j * a.in_stride;
  float* out = a.out + (size_t)j * a.out_stride;
  if (!a.rms) {
    double s = 0;
    for (int k = threadIdx.x; k < a.K; k += blockDim.x) s += (double)in[k];
    double mean = block_sum_d(s, red) / (double)a.K;
    double v = 0;
    for (int k = threadIdx.x; k < a.K; k += blockDim.x) {
      double d = (double)in[k] - mean;
      v += d * d;
    }
    double var = block_sum_d(v, red);
    float inv = (float)(1.0 / sqrt(var / (double)a.K + a.eps));
    float mf = (float)mean;
    for (int k = threadIdx.x; k < a.K; k += blockDim.x)
      out[k] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(in[k], mf), inv), a.nw[k]), a.nb[k]);
  } else {
    __shared__ float inv_s;
    if (threadIdx.x == 0) {
      float ss = 0.f;
      for (int k = 0; k < a.K; k++) ss = __fadd_rn(ss, __fmul_rn(in[k], in[k]));
      float mean = __fadd_rn(__fdiv_rn(ss, (float)a.K), 1e-5f);
      inv_s = __fdiv_rn(1.0f, (float)sqrt((double)mean));
    }
    __syncthreads();
    for (int k = threadIdx.x; k < a.K; k += blockDim.x) out[k] = __fmul_rn(a.nw[k], __fmul_rn(inv_s, in[k]));
  }
}

}  // namespace tcu
