// Shared device helpers for the tinyoai B200 kernels (sm_100a).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tcu {

// Weight formats use GGUF type codes (gguf.go:177-205).
enum Fmt : int { FMT_F32 = 0, FMT_F16 = 1, FMT_Q5_1 = 7, FMT_Q8_0 = 8, FMT_Q5_K = 13, FMT_Q6_K = 14, FMT_BF16 = 30 };

// A weight matrix in device layout, row-major [rows][cols].
//  Q8_0: w = int8 quants [rows][cols], s = binary16 block scales
//        [rows][sstride] with sstride = cols/32 rounded up to 8 (the 34-byte
//        GGUF block split into two planes whose rows start on 16 bytes).
//  F32 / F16 / BF16: w = the raw elements.
//  Q6_K / Q5_K / Q5_1: w = the GGUF blocks as stored (row-major blocks).
struct DMat {
  int fmt;
  int rows, cols;
  const uint8_t* w;
  const __half* s;
  int sstride;    // Q8_0 scale row stride in halves
  int tc_sw = 0;  // Q8_0: power of two applied before the tensor-core split (gemm_tc.cuh)
};

__device__ __forceinline__ float bf16_bits_to_float(uint32_t b) { return __uint_as_float(b << 16); }

// Order-preserving map of a float to uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_order_key(float v) {
  uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float float_from_order_key(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}
// argmax packing: max over (value, -index) so that ties keep the earliest
// index, as the strict comparison of model.go:622-630 does.
__device__ __forceinline__ unsigned long long argmax_pack(float v, int idx) {
  return ((unsigned long long)float_order_key(v) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}
__device__ __forceinline__ int argmax_index(unsigned long long key) { return (int)(0xffffffffu - (uint32_t)(key & 0xffffffffu)); }

// Streaming 16-byte load that bypasses L1 (weights are read once per token).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// SwiGLU of the StableLM MLP (stablelm.go:371-373): v/(1+exp(-v)) * up with a
// float64 exponential rounded to float32 and separately rounded float32 ops.
__device__ __forceinline__ float silu_mul_stablelm(float v, float up) {
  float e = (float)exp(-(double)v);
  float den = __fadd_rn(1.0f, e);
  float s = __fdiv_rn(v, den);
  return __fmul_rn(s, up);
}
// The same with exp evaluated in float32 (expf, within 2 ulp of the rounded
// float64 value): for the persistent decode step, where the float64 exp sits
// on the critical path of every gate/up tile.
__device__ __forceinline__ float silu_mul_stablelm_f32(float v, float up) {
  float e = expf(-v);
  float den = __fadd_rn(1.0f, e);
  float s = __fdiv_rn(v, den);
  return __fmul_rn(s, up);
}
// SwiGLU of the llama2.c MLP (model.go:470-473): v * (1/(1+exp(-v))) * up.
__device__ __forceinline__ float silu_mul_llama(float v, float up) {
  float e = (float)exp(-(double)v);
  float den = __fadd_rn(1.0f, e);
  float r = __fdiv_rn(1.0f, den);
  return __fmul_rn(__fmul_rn(v, r), up);
}

// Decodes one GGUF K-quant / Q5_1 block element (quant_k.go:31-86), with the
// same separately rounded float32 operations as the reference decoder.
__device__ __forceinline__ float kquant_at(const uint8_t* block, int i, int fmt) {
  if (fmt == FMT_Q5_1) {
    float d = __half2float(__ushort_as_half((unsigned short)(block[0] | (block[1] << 8))));
    float mn = __half2float(__ushort_as_half((unsigned short)(block[2] | (block[3] << 8))));
    uint32_t high = (uint32_t)block[4] | ((uint32_t)block[5] << 8) | ((uint32_t)block[6] << 16) | ((uint32_t)block[7] << 24);
    uint32_t low = (block[8 + i % 16] >> (i / 16 * 4)) & 15;
    uint32_t q = low | (((high >> i) & 1) << 4);
    return __fadd_rn(__fmul_rn(d, (float)q), mn);
  }
  if (fmt == FMT_Q6_K) {
    float d = __half2float(__ushort_as_half((unsigned short)(block[208] | (block[209] << 8))));
    int group = i / 16;
    float scale = __fmul_rn(d, (float)(int8_t)block[192 + group]);
    int low = (block[(i / 128) * 64 + i % 64] >> ((i % 128) / 64 * 4)) & 15;
    int high = (block[128 + (i / 128) * 32 + i % 32] >> ((i % 128) / 32 * 2)) & 3;
    return __fmul_rn(scale, (float)((low | high << 4) - 32));
  }
  // Q5_K
  float d = __half2float(__ushort_as_half((unsigned short)(block[0] | (block[1] << 8))));
  float dmin = __half2float(__ushort_as_half((unsigned short)(block[2] | (block[3] << 8))));
  const uint8_t* sc = block + 4;
  int group = i / 32, j = i % 32;
  int scale, minimum;
  if (group < 4) {
    scale = sc[group] & 63;
    minimum = sc[group + 4] & 63;
  } else {
    scale = (sc[group + 4] & 15) | ((sc[group - 4] >> 6) << 4);
    minimum = (sc[group + 4] >> 4) | ((sc[group] >> 6) << 4);
  }
  float ds = __fmul_rn(d, (float)scale), dm = __fmul_rn(dmin, (float)minimum);
  int low = (block[48 + (group / 2) * 32 + j] >> (group % 2 * 4)) & 15;
  int high = (block[16 + j] >> group) & 1;
  return __fsub_rn(__fmul_rn(ds, (float)(low | high << 4)), dm);
}

__host__ __device__ inline int kquant_block_bytes(int fmt) { return fmt == FMT_Q5_1 ? 24 : fmt == FMT_Q6_K ? 210 : 176; }
// Bytes between super-blocks in device memory: a Q6_K block (210 bytes in
// the file) is padded to 224, so that its ql, qh and scale sections start on
// 16-byte boundaries; Q5_K (176) and Q5_1 keep the file's size.
__host__ __device__ inline int kquant_dev_bytes(int fmt) { return fmt == FMT_Q6_K ? 224 : kquant_block_bytes(fmt); }
__host__ __device__ inline int kquant_block_width(int fmt) { return fmt == FMT_Q5_1 ? 32 : 256; }

// Eight values W[r][k0 .. k0 + 8) of a Q6_K or Q5_K matrix whose rows are
// whole super-blocks (cols % 256 == 0, k0 % 8 == 0, so the eight share one
// scale group): the block address and the group's scale are computed once,
// each value exactly as kquant_at computes it (quant_k.go:47-85).
__device__ __forceinline__ void kquant_decode8(const DMat& W, int r, int k0, float* dst) {
  const int K = W.cols;
  const int i0 = k0 & 255;
  const uint8_t* blk = W.w + ((size_t)r * (K >> 8) + (k0 >> 8)) * (W.fmt == FMT_Q6_K ? 224 : 176);
  if (W.fmt == FMT_Q6_K) {
    const float d = __half2float(__ushort_as_half((unsigned short)(blk[208] | (blk[209] << 8))));
    const float scale = __fmul_rn(d, (float)(int8_t)blk[192 + i0 / 16]);
    const uint8_t* ql = blk + (i0 / 128) * 64 + i0 % 64;
    const uint8_t* qh = blk + 128 + (i0 / 128) * 32 + i0 % 32;
    const int ls = (i0 % 128) / 64 * 4, hs = (i0 % 128) / 32 * 2;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int q = ((ql[i] >> ls) & 15) | (((qh[i] >> hs) & 3) << 4);
      dst[i] = __fmul_rn(scale, (float)(q - 32));
    }
  } else {
    const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(blk[2] | (blk[3] << 8))));
    const uint8_t* sc = blk + 4;
    const int group = i0 / 32, j0 = i0 % 32;
    int scale, minimum;
    if (group < 4) {
      scale = sc[group] & 63;
      minimum = sc[group + 4] & 63;
    } else {
      scale = (sc[group + 4] & 15) | ((sc[group - 4] >> 6) << 4);
      minimum = (sc[group + 4] >> 4) | ((sc[group] >> 6) << 4);
    }
    const float ds = __fmul_rn(d, (float)scale), dm = __fmul_rn(dmin, (float)minimum);
    const uint8_t* qs = blk + 48 + (group / 2) * 32 + j0;
    const uint8_t* qh = blk + 16 + j0;
    const int ls = group % 2 * 4;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int q = ((qs[i] >> ls) & 15) | (((qh[i] >> group) & 1) << 4);
      dst[i] = __fsub_rn(__fmul_rn(ds, (float)q), dm);
    }
  }
}

// Element (r, c) of a device matrix, decoded exactly as the reference does.
__device__ __forceinline__ float dmat_at(const DMat& m, int r, int c) {
  switch (m.fmt) {
    case FMT_Q8_0:
      return __fmul_rn(__half2float(m.s[(size_t)r * m.sstride + c / 32]), (float)((const int8_t*)m.w)[(size_t)r * m.cols + c]);
    case FMT_F32:
      return ((const float*)m.w)[(size_t)r * m.cols + c];
    case FMT_F16:
      return __half2float(((const __half*)m.w)[(size_t)r * m.cols + c]);
    case FMT_BF16:
      return bf16_bits_to_float(((const uint16_t*)m.w)[(size_t)r * m.cols + c]);
    default: {
      int width = kquant_block_width(m.fmt), bytes = kquant_dev_bytes(m.fmt);
      size_t index = (size_t)r * m.cols + c;
      return kquant_at(m.w + index / width * bytes, (int)(index % width), m.fmt);
    }
  }
}

}  // namespace tcu
