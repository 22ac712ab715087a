// Load-time repacking, KV page copy-on-write and the sampling shortlist.
#pragma once
#include "common.cuh"

namespace tcu {

// Copies a checkpoint tensor (file encoding) into a device matrix at
// (row0 + i*row_step, col0), splitting Q8_0 blocks (gguf.go:186-189: 2-byte
// binary16 scale + 32 int8) into the quant and scale planes and padding Q6_K
// super-blocks to their device size (kquant_dev_bytes).
struct RepackArgs {
  const uint8_t* raw;
  int fmt;
  int rows, cols;  // source shape
  DMat dst;        // destination (dst.w / dst.s writable)
  int row0, row_step, col0;
};

__global__ void k_repack(RepackArgs a) {
  const int K2 = a.dst.cols;
  uint8_t* dw = const_cast<uint8_t*>(a.dst.w);
  if (a.fmt == FMT_Q8_0) {
    const int nb = a.cols / 32;
    const size_t total = (size_t)a.rows * nb;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
      const int r = (int)(idx / nb), b = (int)(idx % nb);
      const uint8_t* blk = a.raw + idx * 34;
      const int dr = a.row0 + r * a.row_step;
      __half* ds = const_cast<__half*>(a.dst.s);
      ds[(size_t)dr * a.dst.sstride + a.col0 / 32 + b] = __ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8)));
      uint8_t* q = dw + (size_t)dr * K2 + a.col0 + b * 32;
#pragma unroll
      for (int i = 0; i < 32; i++) q[i] = blk[2 + i];
    }
  } else if (a.fmt == FMT_F32 || a.fmt == FMT_F16 || a.fmt == FMT_BF16) {
    const int es = a.fmt == FMT_F32 ? 4 : 2;
    const size_t total = (size_t)a.rows * a.cols;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
      const int r = (int)(idx / a.cols), c = (int)(idx % a.cols);
      const int dr = a.row0 + r * a.row_step;
      uint8_t* d = dw + ((size_t)dr * K2 + a.col0 + c) * es;
      const uint8_t* s = a.raw + idx * es;
      for (int i = 0; i < es; i++) d[i] = s[i];
    }
  } else {
    const int width = kquant_block_width(a.fmt), bytes = kquant_block_bytes(a.fmt), dbytes = kquant_dev_bytes(a.fmt);
    const int nb = a.cols / width;
    const size_t total = (size_t)a.rows * nb;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
      const int r = (int)(idx / nb), b = (int)(idx % nb);
      const int dr = a.row0 + r * a.row_step;
      uint8_t* d = dw + ((size_t)dr * (K2 / width) + a.col0 / width + b) * dbytes;
      const uint8_t* s = a.raw + idx * bytes;
      for (int i = 0; i < bytes; i++) d[i] = s[i];
      for (int i = bytes; i < dbytes; i++) d[i] = 0;
    }
  }
}

// Copy-on-write of one KV page (all layers, all kv heads): the
// partially-filled tail page a fork or a branch writes into.
__global__ void k_copy_page(uint4* k, uint4* v, size_t page_vec, int num_pages, int src, int dst, int layers) {
  // page_vec: 16-byte vectors per page per layer (kvh * P * hd * elem / 16)
  const size_t total = page_vec * layers;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t l = i / page_vec, e = i % page_vec;
    const size_t so = (l * num_pages + src) * page_vec + e, dO = (l * num_pages + dst) * page_vec + e;
    k[dO] = k[so];
    v[dO] = v[so];
  }
}

// Sampling shortlist over one logits row (sampling.go:112-143 ordering:
// descending value, ties by ascending id) and the full-vocabulary
// log-sum-exp in float64 (logprobs.go:67-90). One CTA; k <= 256.
__global__ void __launch_bounds__(1024) k_shortlist(const float* logits, int V, int k, int* ids, float* vals, double* lse) {
  extern __shared__ uint32_t taken[];  // V bits
  __shared__ double red_d[32];
  __shared__ unsigned long long red_k[32];
  __shared__ float mx_s;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int i = threadIdx.x; i < (V + 31) / 32; i += blockDim.x) taken[i] = 0;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, logits[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red_d[warp] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    for (int w = 0; w < nw; w++) m = fmaxf(m, (float)red_d[w]);
    mx_s = m;
  }
  __syncthreads();
  const double best = (double)mx_s;
  double s = 0;
  for (int i = threadIdx.x; i < V; i += blockDim.x) s += exp((double)logits[i] - best);
  s = warp_sum_d(s);
  __syncthreads();
  if (lane == 0) red_d[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0;
    for (int w = 0; w < nw; w++) t += red_d[w];
    *lse = best + log(t);
  }
  for (int j = 0; j < k; j++) {
    unsigned long long b = 0;
    for (int i = threadIdx.x; i < V; i += blockDim.x)
      if (!((taken[i >> 5] >> (i & 31)) & 1u)) {
        unsigned long long key = argmax_pack(logits[i], i);
        b = key > b ? key : b;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
      b = t > b ? t : b;
    }
    __syncthreads();
    if (lane == 0) red_k[warp] = b;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long t = 0;
      for (int w = 0; w < nw; w++) t = red_k[w] > t ? red_k[w] : t;
      const int id = argmax_index(t);
      ids[j] = id;
      vals[j] = logits[id];
      taken[id >> 5] |= 1u << (id & 31);
    }
    __syncthreads();
  }
}

// Per-row argmax of a logits matrix (batched branch steps).
__global__ void k_argmax_rows(const float* logits, int V, int stride, unsigned long long* out) {
  // One CTA per row; each thread keeps four loads in flight. The packed
  // (value, index) maximum does not depend on the visiting order.
  const int r = blockIdx.x, nt = blockDim.x;
  const float* row = logits + (size_t)r * stride;
  unsigned long long b = 0;
  for (int i0 = threadIdx.x; i0 < V; i0 += 4 * nt) {
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; u++) v[u] = i0 + u * nt < V ? row[i0 + u * nt] : 0.f;
#pragma unroll
    for (int u = 0; u < 4; u++) {
      if (i0 + u * nt < V) {
        const unsigned long long key = argmax_pack(v[u], i0 + u * nt);
        b = key > b ? key : b;
      }
    }
  }
  __shared__ unsigned long long red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
    b = t > b ? t : b;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = b;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) t = red[w] > t ? red[w] : t;
    out[r] = t;
  }
}

}  // namespace tcu

namespace tcu {

// Keeps the better of two (score, id) pairs: higher score, then lower id
// (id < 0: empty).
__device__ __forceinline__ void cand_better(double& bv, int& bi, double v, int i) {
  if (i >= 0 && (bi < 0 || v > bv || (v == bv && i < bi))) {
    bv = v;
    bi = i;
  }
}

// The block's best (score, id) pair; every thread returns it. red_v / red_i:
// one slot per warp.
__device__ __forceinline__ void cand_block_best(double& bv, int& bi, double* red_v, int* red_i) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double v = __shfl_xor_sync(0xffffffffu, bv, o);
    const int i = __shfl_xor_sync(0xffffffffu, bi, o);
    cand_better(bv, bi, v, i);
  }
  __syncthreads();
  if (lane == 0) {
    red_v[warp] = bv;
    red_i[warp] = bi;
  }
  __syncthreads();
  bv = red_v[0];
  bi = red_i[0];
  for (int w = 1; w < nw; w++) cand_better(bv, bi, red_v[w], red_i[w]);
}

// summarizeLogits (logprobs.go:64-95) for row r = blockIdx.x of a logits
// matrix: z = best + log(sum exp(v - best)) in float64 over the whole row,
// then logits[targets[r]] - z and the `count` largest logits (descending,
// ties by lower id) as (id, logit - z). One CTA per row, count <= 256.
__global__ void __launch_bounds__(1024) k_logprob_rows(const float* logits, int V, int stride, const int* targets, int count,
                                                       double* chosen, int* top_ids, double* top_vals) {
  extern __shared__ uint32_t lp_taken[];  // V bits
  __shared__ double red_v[32];
  __shared__ int red_i[32];
  __shared__ double z_s;
  const int r = blockIdx.x;
  const float* row = logits + (size_t)r * stride;
  for (int i = threadIdx.x; i < (V + 31) / 32; i += blockDim.x) lp_taken[i] = 0;
  double bv = 0.0;
  int bi = -1;
  for (int i = threadIdx.x; i < V; i += blockDim.x) cand_better(bv, bi, (double)row[i], i);
  cand_block_best(bv, bi, red_v, red_i);
  const double best = bv;
  double s = 0.0;
  for (int i = threadIdx.x; i < V; i += blockDim.x) s += exp((double)row[i] - best);
  s = warp_sum_d(s);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red_v[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red_v[w];
    z_s = best + log(t);
    chosen[r] = (double)row[targets[r]] - z_s;
  }
  __syncthreads();
  const double z = z_s;
  for (int j = 0; j < count; j++) {
    double v = 0.0;
    int id = -1;
    for (int i = threadIdx.x; i < V; i += blockDim.x)
      if (!((lp_taken[i >> 5] >> (i & 31)) & 1u)) cand_better(v, id, (double)row[i], i);
    cand_block_best(v, id, red_v, red_i);
    if (threadIdx.x == 0) {
      top_ids[(size_t)r * count + j] = id;
      top_vals[(size_t)r * count + j] = id >= 0 ? (double)row[id] - z : 0.0;
      if (id >= 0) lp_taken[id >> 5] |= 1u << (id & 31);
    }
    __syncthreads();
  }
}

// Penalised scores of several rows, grouped by id on the host: row r has
// the distinct ids ids[row_off[r] .. row_off[r + 1]) in ascending order, and
// id j's float64 score is (double)logit - terms[term_off[j]] - ... -
// terms[term_off[j + 1] - 1], subtracted in that order (the order
// penalizedLogits applies them, sampling.go:76-101).
struct PenaltyRows {
  const int* row_off;
  const int* ids;
  const int* term_off;
  const double* terms;
};

// samplingCandidates(penalizedLogits(row), k) (sampling.go:76-143) for row
// r = blockIdx.x: the k largest float64 scores, descending, ties by lower id.
// Dynamic shared memory: two V-bit maps, then the row's penalised ids and
// scores (max_ids each).
__global__ void __launch_bounds__(1024) k_candidates_rows(const float* logits, int V, int stride, PenaltyRows pr, int max_ids, int k,
                                                          int* out_ids, double* out_vals) {
  extern __shared__ __align__(8) uint8_t cand_smem[];
  const int nwords = (V + 31) / 32;
  double* pv = reinterpret_cast<double*>(cand_smem);
  int* pid = reinterpret_cast<int*>(pv + max_ids);
  uint32_t* taken = reinterpret_cast<uint32_t*>(pid + max_ids);
  uint32_t* pen = taken + nwords;
  __shared__ double red_v[32];
  __shared__ int red_i[32];
  const int r = blockIdx.x;
  const float* row = logits + (size_t)r * stride;
  for (int i = threadIdx.x; i < nwords; i += blockDim.x) taken[i] = pen[i] = 0;
  __syncthreads();
  const int j0 = pr.row_off[r], nd = pr.row_off[r + 1] - j0;
  for (int j = threadIdx.x; j < nd; j += blockDim.x) {
    const int id = pr.ids[j0 + j];
    double v = (double)row[id];
    for (int t = pr.term_off[j0 + j]; t < pr.term_off[j0 + j + 1]; t++) v = __dsub_rn(v, pr.terms[t]);
    pv[j] = v;
    pid[j] = id;
    atomicOr(&pen[id >> 5], 1u << (id & 31));
  }
  __syncthreads();
  for (int j = 0; j < k; j++) {
    double bv = 0.0;
    int bi = -1;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const uint32_t bit = 1u << (i & 31);
      if (taken[i >> 5] & bit) continue;
      double v;
      if (pen[i >> 5] & bit) {
        int lo = 0, hi = nd - 1;  // ids ascending: binary search
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (pid[mid] < i)
            lo = mid + 1;
          else
            hi = mid;
        }
        v = pv[lo];
      } else {
        v = (double)row[i];
      }
      cand_better(bv, bi, v, i);
    }
    cand_block_best(bv, bi, red_v, red_i);
    if (threadIdx.x == 0) {
      out_ids[(size_t)r * k + j] = bi;
      out_vals[(size_t)r * k + j] = bv;
      if (bi >= 0) taken[bi >> 5] |= 1u << (bi & 31);
    }
    __syncthreads();
  }
}

}  // namespace tcu

namespace tcu {

// x[i] += p[i] over n values: the residual update of a tensor-parallel layer
// after the all-reduce of the ranks' out + down partial sums
// (stablelm.go:365-377 with the two products summed across ranks).
__global__ void k_add_rows(float* x, const float* p, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) x[i] = __fadd_rn(x[i], p[i]);
}

}  // namespace tcu
