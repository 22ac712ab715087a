// The per-layer exchange of head-parallel tensor parallelism over NVLink
// peer memory: one kernel sums the ranks' out + down partials and adds the
// sum to the residual rows (stablelm.go:365-377 gives the parallel residual
// x + attn_out + mlp_down that the sum reassembles).
//
// Every rank owns an exchange buffer (cudaMalloc, shared with the other
// ranks through CUDA IPC): flags [2 parities][TPX_MAX_CTAS][TPX_MAX_RANKS]
// uint32 and data [2 parities][TPX_MAX_RANKS][max_count] float. Call k
// (seq = k + 1) uses parity seq & 1. The call count lives in device memory
// (read by every CTA at its start, advanced by the last CTA to finish), so a
// captured CUDA graph replays the exchange correctly. CTA c owns elements
// [c chunk, (c + 1) chunk):
//   1. it stores its rank's partial of those elements into slot `rank` of
//      every rank's data (plain stores through the peer mappings);
//   2. after a CTA barrier, thread p sets flag [c][rank] of rank p to seq
//      (system-scope fence, then a release store);
//   3. thread j waits (bounded, acquire loads) until its own flag [c][j]
//      reads seq, then the CTA sums slots 0, 1, ..., world - 1 in that order
//      (the same order on every rank, so every rank gets the same sums) and
//      adds the sum to x.
// CTA c of one rank waits only for CTA c of the others, and the launch has
// at most one CTA per SM, so all CTAs are resident together. Two parities
// suffice: a rank can write parity p again only after every rank raised its
// flags of the call in between, which each does after its own reads of
// parity p. Every wait gives up after ~TCU_WAIT_NS and sets the error word.
#pragma once
#include <stdint.h>

#include "tma.cuh"

namespace tcu {

constexpr int TPX_MAX_RANKS = 8;
constexpr int TPX_MAX_CTAS = 256;
constexpr int TPX_THREADS = 256;
constexpr int TPX_PEER_ROWS = 64;  // exchanges of up to this many rows use the peer path
constexpr size_t TPX_FLAG_BYTES = 2 * TPX_MAX_CTAS * TPX_MAX_RANKS * sizeof(uint32_t);

__host__ __device__ inline size_t tpx_bytes(size_t max_count) {
  return TPX_FLAG_BYTES + 2 * (size_t)TPX_MAX_RANKS * max_count * sizeof(float);
}

struct TpxArgs {
  float* x;             // residual rows (count values)
  const float* part;    // this rank's partial
  long long count;      // values
  long long max_count;  // data slot size of the exchange buffers
  int chunk;            // values per CTA (multiple of 4)
  int world, rank;
  uint32_t* seq;               // [0]: exchanges completed by this rank, [1]: CTAs finished in this call
  uint8_t* ex[TPX_MAX_RANKS];  // every rank's exchange buffer as mapped here (own included)
  int* err;
};

__device__ __forceinline__ uint32_t* tpx_flag(uint8_t* ex, int par, int c, int r) {
  return reinterpret_cast<uint32_t*>(ex) + ((size_t)par * TPX_MAX_CTAS + c) * TPX_MAX_RANKS + r;
}
__device__ __forceinline__ float* tpx_data(uint8_t* ex, int par, int r, long long max_count) {
  return reinterpret_cast<float*>(ex + TPX_FLAG_BYTES) + ((size_t)par * TPX_MAX_RANKS + r) * max_count;
}

__device__ __forceinline__ void tpx_store_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t tpx_load_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(TPX_THREADS) k_tp_exchange_add(TpxArgs a) {
  __shared__ uint32_t seq_s;
  if (threadIdx.x == 0) seq_s = *reinterpret_cast<volatile uint32_t*>(a.seq) + 1;
  __syncthreads();
  const uint32_t seq = seq_s;
  const int c = blockIdx.x, par = seq & 1;
  const long long lo = (long long)c * a.chunk, hi = min(a.count, lo + a.chunk);
  // 1. This rank's partial into slot `rank` of every rank.
  for (int p = 0; p < a.world; p++) {
    float* dst = tpx_data(a.ex[p], par, a.rank, a.max_count);
    long long i = lo + 4 * (long long)threadIdx.x;
    for (; i + 3 < hi; i += 4 * TPX_THREADS)
      *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(a.part + i);
    if (i < hi)
      for (; i < hi; i++) dst[i] = a.part[i];
  }
  __syncthreads();
  // 2. Flags: every rank's [c][rank] = seq.
  if (threadIdx.x < a.world) {
    __threadfence_system();
    tpx_store_release(tpx_flag(a.ex[threadIdx.x], par, c, a.rank), seq);
  }
  // 3. Wait for every rank's slot of this chunk, then sum in rank order.
  int ok = 1;
  if (threadIdx.x < a.world) {
    const uint32_t* f = tpx_flag(a.ex[a.rank], par, c, threadIdx.x);
    if (tpx_load_acquire(f) != seq) {
      const unsigned long long t0 = global_ns();
      for (uint32_t it = 1;; it++) {
        if (tpx_load_acquire(f) == seq) break;
        if ((it & 255) == 0) {
          if (*(volatile int*)a.err || global_ns() - t0 > TCU_WAIT_NS) {
            atomicExch(a.err, TCU_DEV_TIMEOUT);
            ok = 0;
            break;
          }
        }
      }
    }
  }
  if (__syncthreads_and(ok)) {
    const float* own[TPX_MAX_RANKS];
#pragma unroll
    for (int j = 0; j < TPX_MAX_RANKS; j++) own[j] = tpx_data(a.ex[a.rank], par, j < a.world ? j : 0, a.max_count);
    for (long long i = lo + threadIdx.x; i < hi; i += TPX_THREADS) {
      float s = __ldcg(own[0] + i);
      for (int j = 1; j < a.world; j++) s = __fadd_rn(s, __ldcg(own[j] + i));
      a.x[i] = __fadd_rn(a.x[i], s);
    }
  }
  // Every CTA has read the call count by now; the last one advances it.
  if (threadIdx.x == 0 && atomicAdd(a.seq + 1, 1u) == gridDim.x - 1) {
    a.seq[1] = 0;
    a.seq[0] = seq;
  }
}

}  // namespace tcu
