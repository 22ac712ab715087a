// weightTensor.readValues (matmul.go:12-50) on the device, through each of
// the library's weight decoders, so that a host can check every decoder the
// kernels use against the reference's float32 values bit for bit
// (quant_k_test.go:14-48 does this for the Go decoder).
#pragma once
#include "common.cuh"
#include "gemm_tc.cuh"

namespace tcu {

// Decoders, as TCU_DECODE_* of include/tinyoai_cuda.h.
enum ReadDecoder : int { RD_ELEMENT = 0, RD_GROUP8 = 1, RD_TC = 2 };

// Value j (0..15) of a group of sixteen tensor-core operand pieces, summed
// back in float32 in piece order (each partial sum is exact: the pieces hold
// disjoint bits of a value of at most 24 significant bits). Zero pieces
// after the first are skipped, so a -0 weight reads back as -0.
template <int NP>
__device__ __forceinline__ float tc_pieces_value(const uint4 (&p)[NP][2], int j) {
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < NP; k++) {
    const uint4 q = p[k][j >> 3];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    const uint32_t word = w[(j & 7) >> 1];
    const float v = __half2float(__ushort_as_half((unsigned short)((j & 1) ? (word >> 16) : (word & 0xffffu))));
    s = k == 0 ? v : (v != 0.f ? __fadd_rn(s, v) : s);
  }
  return s;
}

// out[i] = element offset + i (row-major) of W, for i < n.
__global__ void k_read_values(DMat W, long long offset, long long n, int decoder, float* out) {
  const float wscale = tc_pow2(W.tc_sw), wunscale = tc_pow2(-W.tc_sw);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long e = offset + i;
    const int r = (int)(e / W.cols), c = (int)(e % W.cols);
    float v;
    if (decoder == RD_GROUP8) {
      float g[8];
      kquant_decode8(W, r, c & ~7, g);
      v = g[c & 7];
    } else if (decoder == RD_TC) {
      if (W.fmt == FMT_Q8_0) {
        uint4 p[tc_pieces(TCW_Q8)][2];
        tc_weight_pieces<TCW_Q8>(W, r, c & ~15, W.cols, wscale, p);
        v = __fmul_rn(tc_pieces_value(p, c & 15), wunscale);
      } else {
        uint4 p[tc_pieces(TCW_KQ)][2];
        tc_weight_pieces<TCW_KQ>(W, r, c & ~15, W.cols, wscale, p);
        v = __fmul_rn(tc_pieces_value(p, c & 15), wunscale);
      }
    } else {
      v = dmat_at(W, r, c);
    }
    out[i] = v;
  }
}

}  // namespace tcu
