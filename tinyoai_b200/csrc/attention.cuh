// Attention over the paged KV pool, RoPE, KV append and embedding gather.
//
// KV pool layout (one pool per KV dtype, shared by every session of a model):
//   K, V: [layer][page][kv_head][P][head_dim]   (float32 or binary16)
// A sequence's page table maps logical page i (positions i*P .. i*P+P-1) to a
// physical page. Full pages may be shared by several sequences (fork,
// branches); a sequence only ever writes pages it owns alone.
#pragma once
#include "common.cuh"
#include "tma.cuh"

namespace tcu {

struct KVView {
  void* k;
  void* v;
  int half;       // 1: binary16 storage (kv_cache.go:27-65), 0: float32
  int P;          // positions per page
  int num_pages;  // pages in the pool
  int kvh, hd;
  __device__ __forceinline__ size_t off(int layer, int page, int g, int row) const {
    return ((((size_t)layer * num_pages + page) * kvh + g) * P + row) * hd;
  }
};

// RoPE tables. StableLM (stablelm.go:309-326): cos/sin of the float32 angle
// float32(pos) * (1 / float32(theta^(2i/rotary))) evaluated in float64 and
// rounded, tabulated on the host per (pos, i < rotary/2). llama2.c
// (model.go:611-618): the checkpoint's freq_cis_real/imag rows per (pos, i < hd/2).
struct Rope {
  const float2* table;  // [max_pos][pairs] (cos, sin)
  int pairs;
  int mode;  // 0: StableLM split-half over the first 2*pairs dims; 1: llama adjacent pairs
};

// Rotates one head vector x[hd] in place for position pos (split-half) or
// (adjacent pairs); operations are separately rounded as in the reference.
__device__ __forceinline__ void rope_pair(float* x, int i, const Rope& r, int pos) {
  float2 cs = r.table[(size_t)pos * r.pairs + i];
  if (r.mode == 0) {
    int j = i + r.pairs;
    float a = x[i], b = x[j];
    x[i] = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
    x[j] = __fadd_rn(__fmul_rn(b, cs.x), __fmul_rn(a, cs.y));
  } else {
    int j = 2 * i;
    float v0 = x[j], v1 = x[j + 1];
    x[j] = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
    x[j + 1] = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
  }
}

__device__ __forceinline__ float kv_round(float v, int half) { return half ? __half2float(__float2half_rn(v)) : v; }

__device__ __forceinline__ void kv_store(const KVView& kv, void* base, size_t off, float v) {
  if (kv.half)
    reinterpret_cast<__half*>(base)[off] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(base)[off] = v;
}

// Loads rows [0, n) of one page (kv head g) into smem with row stride hd+1.
__device__ __forceinline__ void load_page_rows(const KVView& kv, const void* base, int layer, int page, int g, int n,
                                               float* dst, int dst_row0) {
  const int hd = kv.hd;
  const size_t o = kv.off(layer, page, g, 0);
  if (kv.half) {
    const __half* src = reinterpret_cast<const __half*>(base) + o;
    for (int e = threadIdx.x; e < n * hd; e += blockDim.x) {
      int r = e / hd, c = e % hd;
      dst[(dst_row0 + r) * (hd + 1) + c] = __half2float(src[e]);
    }
  } else {
    const float* src = reinterpret_cast<const float*>(base) + o;
    if ((hd & 3) == 0) {
      const float4* s4 = reinterpret_cast<const float4*>(src);
      for (int e = threadIdx.x; e < n * hd / 4; e += blockDim.x) {
        float4 f = s4[e];
        int r = (e * 4) / hd, c = (e * 4) % hd;
        float* d = dst + (dst_row0 + r) * (hd + 1) + c;
        d[0] = f.x;
        d[1] = f.y;
        d[2] = f.z;
        d[3] = f.w;
      }
    } else {
      for (int e = threadIdx.x; e < n * hd; e += blockDim.x) {
        int r = e / hd, c = e % hd;
        dst[(dst_row0 + r) * (hd + 1) + c] = src[e];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Decode attention: one token per sequence, split over the history.
//
// Restates attendHeads (stablelm.go:401-427) / model.go:443-462: scores are
// float32 q.k / float32(sqrt(hd)), softmax subtracts the maximum, and the
// output is the probability-weighted sum of values. The history is split into
// chunks of `split` positions handled by separate CTAs; the last CTA of each
// (sequence, kv head) merges the partial softmax states. This CTA also
// rotates q/k at the sequence's position and appends k/v to the KV page.

struct DecodeAttnArgs {
  int M, H, KVH, hd;
  Rope rope;
  const float* qkv;  // q at [m*qkv_stride + h*hd], k after H*hd, v after (H+KVH)*hd
  int qkv_stride;
  KVView kv;
  int layer;
  const int* page_table;  // [M][pt_stride]
  int pt_stride;
  const int* pos;  // [M]: position of the new token
  int split;       // positions per CTA (multiple of P)
  int max_splits;
  float* part;    // [M][H][max_splits][hd + 2]
  int* counters;  // [M][KVH], zero between launches
  float* out;     // out[m*out_stride + h*hd + i]
  int out_stride;
  float scale;  // float32(sqrt(hd))
  int s_begin;  // splits below this are computed for all rows by k_attn_shared
  int s_runs;   // > 0: the shared splits left s_runs merged partials in slots [0, s_runs)
  int per;      // k_attn_decode_bulk: splits per CTA (1 elsewhere)
};

// Partial slots of a row's merge: the first `lo` slots (the shared splits'
// partials), then the row's own partials from slot lo + off on.
struct SplitSlots {
  int n, lo, off;
  __device__ __forceinline__ int operator()(int j) const { return j < lo ? j : j + off; }
};

// The row's own splits [s_begin, nsplit) leave one partial per run of `per`
// splits, in slots s_begin, s_begin + 1, ...; the shared splits below s_begin
// leave s_runs partials in slots [0, s_runs) (tensor cores) or one per split
// (s_runs = 0).
__device__ __forceinline__ SplitSlots split_slots(const DecodeAttnArgs& a, int nsplit) {
  const int per = a.per > 0 ? a.per : 1;
  const int nruns = (nsplit - a.s_begin + per - 1) / per;
  const int lo = a.s_runs > 0 && a.s_begin > 0 ? a.s_runs : a.s_begin;
  return SplitSlots{lo + nruns, lo, a.s_begin - lo};
}

// Merges the sl.n partials (hd outputs, max, sum; partial j in slot sl(j))
// of each of the G heads of one (row, KV head) into out[G][hd], by the whole
// CTA: fp32 maximum over
// the splits, weights expf(max_j - max), the sum and the outputs accumulated
// in split order. The splits' maxima and sums load in parallel into shared
// memory (wsm: cap floats, at least 2 * nsplit); each output loads its
// partials 16 splits at a time, so the merge costs a few L2 round trips
// rather than one per split. Longer merges (2 * nsplit > cap) read the
// partials one split at a time.
__device__ void attn_merge_splits(const float* part, int max_splits, int hd, int G, SplitSlots sl, float* wsm, int cap, float* out) {
  const int rs = hd + 2, nsplit = sl.n;
  for (int hh = 0; hh < G; hh++) {
    const float* ph = part + (size_t)hh * max_splits * rs;
    if (2 * nsplit > cap) {
      for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float mx = -INFINITY;
        for (int j = 0; j < nsplit; j++) mx = fmaxf(mx, __ldcg(ph + (size_t)sl(j) * rs + hd));
        float l = 0.f, o = 0.f;
        for (int j = 0; j < nsplit; j++) {
          const float* pj = ph + (size_t)sl(j) * rs;
          const float w = expf(__ldcg(pj + hd) - mx);
          l = fmaf(__ldcg(pj + hd + 1), w, l);
          o = fmaf(__ldcg(pj + i), w, o);
        }
        out[hh * hd + i] = __fdiv_rn(o, l);
      }
      continue;
    }
    __syncthreads();  // wsm is free (previous head or the attention tiles)
    for (int j = threadIdx.x; j < nsplit; j += blockDim.x) {
      wsm[j] = __ldcg(ph + (size_t)sl(j) * rs + hd);
      wsm[nsplit + j] = __ldcg(ph + (size_t)sl(j) * rs + hd + 1);
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int j = 0; j < nsplit; j++) mx = fmaxf(mx, wsm[j]);
    __syncthreads();
    for (int j = threadIdx.x; j < nsplit; j += blockDim.x) wsm[j] = expf(wsm[j] - mx);
    __syncthreads();
    float l = 0.f;
    for (int j = 0; j < nsplit; j++) l = fmaf(wsm[nsplit + j], wsm[j], l);
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
      float o = 0.f;
      for (int j0 = 0; j0 < nsplit; j0 += 16) {
        float pv[16];
#pragma unroll
        for (int jj = 0; jj < 16; jj++) pv[jj] = j0 + jj < nsplit ? __ldcg(ph + (size_t)sl(j0 + jj) * rs + i) : 0.f;
#pragma unroll
        for (int jj = 0; jj < 16; jj++)
          if (j0 + jj < nsplit) o = fmaf(pv[jj], wsm[j0 + jj], o);
      }
      out[hh * hd + i] = __fdiv_rn(o, l);
    }
  }
}

__global__ void __launch_bounds__(128) k_attn_decode(DecodeAttnArgs a) {
  extern __shared__ __align__(16) float att_smem[];
  const int s = blockIdx.x + a.s_begin, g = blockIdx.y, m = blockIdx.z;
  const int hd = a.hd, G = a.H / a.KVH, split = a.split;
  const int pos = a.pos[m];
  const int T = pos + 1;
  const int nsplit = (T + split - 1) / split;
  if (s >= nsplit) return;
  const int t0 = s * split;
  const int nt = min(T, t0 + split) - t0;
  const bool has_cur = (s == nsplit - 1);  // this chunk holds position pos

  float* qs = att_smem;                   // [G][hd]
  float* ks = qs + G * hd;                // [split][hd+1]
  float* vs = ks + split * (hd + 1);      // [split][hd+1]
  float* sc = vs + split * (hd + 1);      // [G][split]
  float* cur = sc + G * split;            // [2][hd]
  __shared__ int is_last;

  const float* q_in = a.qkv + (size_t)m * a.qkv_stride;
  for (int e = threadIdx.x; e < G * hd; e += blockDim.x) qs[e] = q_in[(g * G) * hd + e];
  if (has_cur) {
    for (int e = threadIdx.x; e < hd; e += blockDim.x) {
      cur[e] = q_in[a.H * hd + g * hd + e];
      cur[hd + e] = q_in[(a.H + a.KVH) * hd + g * hd + e];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * a.rope.pairs; e += blockDim.x) rope_pair(qs + (e / a.rope.pairs) * hd, e % a.rope.pairs, a.rope, pos);
  if (has_cur)
    for (int e = threadIdx.x; e < a.rope.pairs; e += blockDim.x) rope_pair(cur, e, a.rope, pos);
  __syncthreads();
  const int* pt = a.page_table + (size_t)m * a.pt_stride;
  if (has_cur) {
    // Round to the KV storage precision: attention reads stored values
    // (kv_cache.go:71-86), and the new position is appended here.
    for (int e = threadIdx.x; e < 2 * hd; e += blockDim.x) cur[e] = kv_round(cur[e], a.kv.half);
    __syncthreads();
    const int page = pt[pos / a.kv.P], row = pos % a.kv.P;
    const size_t o = a.kv.off(a.layer, page, g, row);
    for (int e = threadIdx.x; e < hd; e += blockDim.x) {
      kv_store(a.kv, a.kv.k, o + e, cur[e]);
      kv_store(a.kv, a.kv.v, o + e, cur[hd + e]);
    }
  }
  // Stage the chunk's history (positions < pos) page by page.
  const int n_hist = has_cur ? nt - 1 : nt;
  for (int t = 0; t < n_hist;) {
    const int ta = t0 + t;
    const int page = pt[ta / a.kv.P], row = ta % a.kv.P;
    const int n = min(n_hist - t, a.kv.P - row);
    // rows [row, row+n) of this page
    {
      const size_t o = a.kv.off(a.layer, page, g, row);
      for (int e = threadIdx.x; e < n * hd; e += blockDim.x) {
        int r = e / hd, c = e % hd;
        float kvk, kvv;
        if (a.kv.half) {
          kvk = __half2float(reinterpret_cast<const __half*>(a.kv.k)[o + e]);
          kvv = __half2float(reinterpret_cast<const __half*>(a.kv.v)[o + e]);
        } else {
          kvk = reinterpret_cast<const float*>(a.kv.k)[o + e];
          kvv = reinterpret_cast<const float*>(a.kv.v)[o + e];
        }
        ks[(t + r) * (hd + 1) + c] = kvk;
        vs[(t + r) * (hd + 1) + c] = kvv;
      }
    }
    t += n;
  }
  if (has_cur) {
    for (int e = threadIdx.x; e < hd; e += blockDim.x) {
      ks[(nt - 1) * (hd + 1) + e] = cur[e];
      vs[(nt - 1) * (hd + 1) + e] = cur[hd + e];
    }
  }
  __syncthreads();
  // Scores.
  for (int e = threadIdx.x; e < G * split; e += blockDim.x) {
    const int hh = e / split, t = e % split;
    if (t < nt) {
      const float* q = qs + hh * hd;
      const float* k = ks + t * (hd + 1);
      float d = 0.f;
      for (int i = 0; i < hd; i++) d = fmaf(q[i], k[i], d);
      sc[hh * split + t] = __fdiv_rn(d, a.scale);
    }
  }
  __syncthreads();
  // Per-head local softmax state.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  __shared__ float mloc[32], lloc[32];
  for (int hh = warp; hh < G; hh += nwarps) {
    float mx = -INFINITY;
    for (int t = lane; t < nt; t += 32) mx = fmaxf(mx, sc[hh * split + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float l = 0.f;
    for (int t = lane; t < nt; t += 32) {
      float p = expf(sc[hh * split + t] - mx);
      sc[hh * split + t] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      mloc[hh] = mx;
      lloc[hh] = l;
    }
  }
  __syncthreads();
  float* part = a.part + ((size_t)m * a.H + g * G) * a.max_splits * (hd + 2);
  for (int e = threadIdx.x; e < G * hd; e += blockDim.x) {
    const int hh = e / hd, i = e % hd;
    float o = 0.f;
    for (int t = 0; t < nt; t++) o = fmaf(sc[hh * split + t], vs[t * (hd + 1) + i], o);
    part[((size_t)hh * a.max_splits + s) * (hd + 2) + i] = o;
  }
  if (threadIdx.x < G) {
    part[((size_t)threadIdx.x * a.max_splits + s) * (hd + 2) + hd] = mloc[threadIdx.x];
    part[((size_t)threadIdx.x * a.max_splits + s) * (hd + 2) + hd + 1] = lloc[threadIdx.x];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int prev = atomicAdd(a.counters + m * a.KVH + g, 1);
    is_last = (prev == nsplit - a.s_begin - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // Merge the nsplit partial states of each head in the group.
  attn_merge_splits(part, a.max_splits, hd, G, split_slots(a, nsplit), ks, split * (hd + 1), a.out + (size_t)m * a.out_stride + g * G * hd);
  if (threadIdx.x == 0) a.counters[m * a.KVH + g] = 0;
}

// ---------------------------------------------------------------------------
// Prefill: rotate q/k of n new tokens (positions start..start+n-1) in place
// and append k/v to the pages (prefill.go:74-84).
struct RopeStoreArgs {
  int n, H, KVH, hd, start;
  Rope rope;
  float* qkv;
  int qkv_stride;
  KVView kv;
  int layer;
  const int* page_table;
};

__global__ void k_rope_store(RopeStoreArgs a) {
  const int j = blockIdx.x;
  const int pos = a.start + j;
  float* row = a.qkv + (size_t)j * a.qkv_stride;
  const int hd = a.hd, pairs = a.rope.pairs;
  // q and k heads: rotate (each pair touched by exactly one thread).
  for (int e = threadIdx.x; e < (a.H + a.KVH) * pairs; e += blockDim.x) rope_pair(row + (e / pairs) * hd, e % pairs, a.rope, pos);
  __syncthreads();
  const int page = a.page_table[pos / a.kv.P], r = pos % a.kv.P;
  for (int e = threadIdx.x; e < a.KVH * hd; e += blockDim.x) {
    const int g = e / hd, i = e % hd;
    const size_t o = a.kv.off(a.layer, page, g, r) + i;
    kv_store(a.kv, a.kv.k, o, row[a.H * hd + e]);
    kv_store(a.kv, a.kv.v, o, row[(a.H + a.KVH) * hd + e]);
  }
}

// Causal attention of n queries (positions start..start+n-1, already rotated)
// over positions [0, start+n) of one sequence (attention.go:6-45, scalar build:
// every query attends to its exact causal prefix).
struct PrefillAttnArgs {
  int n, H, KVH, hd, start;
  const float* qkv;
  int qkv_stride;
  KVView kv;
  int layer;
  const int* page_table;
  float* out;
  int out_stride;
  float scale;
};

constexpr int PA_QT = 64;       // queries per CTA
constexpr int PA_KT = 64;       // keys per tile
constexpr int PA_THREADS = 256;  // 16 row groups (4 queries) x 16 column groups
constexpr int PA_KTS = PA_KT + 4;  // row stride of the transposed key tile (floats)

// Dynamic shared memory of k_attn_prefill for head size hd.
__host__ __device__ inline size_t pa_smem_bytes(int hd) {
  return sizeof(float) * ((size_t)hd * PA_QT + (size_t)hd * PA_KTS + (size_t)PA_KT * hd + (size_t)PA_KT * PA_QT);
}

// Dynamic shared memory of k_attn_shared: its softmax weights reuse the key
// tile once the scores are done (61 KB at hd = 80: three CTAs per SM).
__host__ __device__ inline size_t pa_shared_smem_bytes(int hd) {
  const size_t kt = (size_t)hd * PA_KTS, ps = (size_t)PA_KT * PA_QT;
  return sizeof(float) * ((size_t)hd * PA_QT + (kt > ps ? kt : ps) + (size_t)PA_KT * hd);
}

// Causal attention of a prefill chunk (attention.go:6-45 semantics: every
// query attends to the history and to the chunk up to itself), flash style on
// CUDA cores. One CTA per (64-query tile, query head). Thread (rg, cg) holds
// the scores of queries 4rg..4rg+3 against keys 4cg..4cg+3 of the current
// 64-key tile, each a float32 dot product in dimension order divided by
// sqrt(hd) (stablelm.go:401-431), and the outputs of the same four queries
// at dimensions cg, cg + 16, ... . Queries and keys sit transposed in shared
// memory, so each step of a dot product is two float4 loads and 16 FMAs. The
// softmax runs online over the key tiles (fp32 max, expf, sum), the weighted
// values accumulate in key order. The next tile's keys and values are loaded
// into registers (4 values per load) while the current tile is computed.
// NC = ceil(hd / 16): output columns and 4-value load chunks per thread.
template <int NC>
__global__ void __launch_bounds__(PA_THREADS, NC <= 5 ? 2 : 1) k_attn_prefill(PrefillAttnArgs a) {
  extern __shared__ __align__(16) float pa_smem[];
  const int hd = a.hd, h = blockIdx.y, g = h / (a.H / a.KVH);
  const int q0 = blockIdx.x * PA_QT;
  const int nq = min(PA_QT, a.n - q0);
  float* qT = pa_smem;               // [hd][QT]
  float* kT = qT + hd * PA_QT;       // [hd][KTS]
  float* vs = kT + hd * PA_KTS;      // [KT][hd]
  float* ps = vs + PA_KT * hd;       // [KT][QT] softmax weights
  const int tid = threadIdx.x, rg = tid >> 4, cg = tid & 15;
  for (int e = tid; e < PA_QT * hd; e += PA_THREADS) {
    const int qi = e / hd, i = e % hd;
    qT[i * PA_QT + qi] = qi < nq ? a.qkv[(size_t)(q0 + qi) * a.qkv_stride + h * hd + i] : 0.f;
  }
  constexpr int MAXC = NC;
  const int ncol = (hd + 15) / 16;
  float o[4][MAXC];
#pragma unroll
  for (int r = 0; r < 4; r++)
#pragma unroll
    for (int j = 0; j < MAXC; j++) o[r][j] = 0.f;
  float m[4], l[4];
#pragma unroll
  for (int r = 0; r < 4; r++) {
    m[r] = -INFINITY;
    l[r] = 0.f;
  }
  const int last_pos = a.start + q0 + nq - 1;
  // Chunk e = tid + PA_THREADS * j of a tile: key e / (hd/4), values
  // 4 (e % (hd/4)) .. +3 (hd % 4 == 0; a tile is 64 * hd / 4 <= 256 * NC chunks).
  const int cpk = hd / 4;
  float4 kr[NC], vr[NC];
  auto fetch = [&](int t0) {
    const int nt = min(PA_KT, last_pos + 1 - t0);
#pragma unroll
    for (int j = 0; j < NC; j++) {
      const int e = tid + PA_THREADS * j, r = e / cpk, c4 = e % cpk;
      kr[j] = vr[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < nt) {
        const int ta = t0 + r;
        const size_t off = a.kv.off(a.layer, a.page_table[ta / a.kv.P], g, ta % a.kv.P) + 4 * c4;
        if (a.kv.half) {
          const uint2 kb = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(a.kv.k) + off);
          const uint2 vb = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(a.kv.v) + off);
          const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&kb.x)), k1 = __half22float2(*reinterpret_cast<const __half2*>(&kb.y));
          const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&vb.x)), v1 = __half22float2(*reinterpret_cast<const __half2*>(&vb.y));
          kr[j] = make_float4(k0.x, k0.y, k1.x, k1.y);
          vr[j] = make_float4(v0.x, v0.y, v1.x, v1.y);
        } else {
          kr[j] = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.kv.k) + off);
          vr[j] = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.kv.v) + off);
        }
      }
    }
  };
  fetch(0);
  for (int t0 = 0; t0 <= last_pos; t0 += PA_KT) {
    const int nt = min(PA_KT, last_pos + 1 - t0);
    __syncthreads();  // the previous tile's keys, values and weights are read
#pragma unroll
    for (int j = 0; j < NC; j++) {
      const int e = tid + PA_THREADS * j, r = e / cpk, c4 = e % cpk;
      if (r < PA_KT) {
        kT[(4 * c4 + 0) * PA_KTS + r] = kr[j].x;
        kT[(4 * c4 + 1) * PA_KTS + r] = kr[j].y;
        kT[(4 * c4 + 2) * PA_KTS + r] = kr[j].z;
        kT[(4 * c4 + 3) * PA_KTS + r] = kr[j].w;
        *reinterpret_cast<float4*>(vs + r * hd + 4 * c4) = vr[j];
      }
    }
    __syncthreads();
    if (t0 + PA_KT <= last_pos) fetch(t0 + PA_KT);
    // Scores of 4 queries x 4 keys.
    float sc[4][4];
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int c = 0; c < 4; c++) sc[r][c] = 0.f;
    for (int i = 0; i < hd; i++) {
      const float4 qv = *reinterpret_cast<const float4*>(qT + i * PA_QT + 4 * rg);
      const float4 kv = *reinterpret_cast<const float4*>(kT + i * PA_KTS + 4 * cg);
      const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) sc[r][c] = fmaf(qa[r], ka[c], sc[r][c]);
    }
    float alpha[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int qi = 4 * rg + r;
      const int qpos = a.start + q0 + qi;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const int t = 4 * cg + c;
        const bool ok = qi < nq && t < nt && t0 + t <= qpos;
        sc[r][c] = ok ? __fdiv_rn(sc[r][c], a.scale) : -INFINITY;
        mx = fmaxf(mx, sc[r][c]);
      }
#pragma unroll
      for (int x = 1; x < 16; x <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, x));
      const float mnew = fmaxf(m[r], mx);
      float ls = 0.f;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const float p = sc[r][c] == -INFINITY ? 0.f : expf(sc[r][c] - mnew);
        sc[r][c] = p;
        ls += p;
      }
#pragma unroll
      for (int x = 1; x < 16; x <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, x);
      alpha[r] = m[r] == -INFINITY ? 0.f : expf(m[r] - mnew);
      l[r] = l[r] * alpha[r] + ls;
      m[r] = mnew;
    }
#pragma unroll
    for (int c = 0; c < 4; c++)
      *reinterpret_cast<float4*>(ps + (4 * cg + c) * PA_QT + 4 * rg) = make_float4(sc[0][c], sc[1][c], sc[2][c], sc[3][c]);
    __syncthreads();
    // Outputs of the same 4 queries at dimensions cg + 16 j, keys in order.
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int j = 0; j < MAXC; j++) o[r][j] *= alpha[r];
    for (int t = 0; t < nt; t++) {
      const float4 pv = *reinterpret_cast<const float4*>(ps + t * PA_QT + 4 * rg);
      const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
      const float* vr = vs + t * hd;
#pragma unroll
      for (int j = 0; j < MAXC; j++) {
        const int c = cg + 16 * j;
        if (j < ncol && c < hd) {
          const float vv = vr[c];
#pragma unroll
          for (int r = 0; r < 4; r++) o[r][j] = fmaf(pa[r], vv, o[r][j]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int qi = 4 * rg + r;
    if (qi >= nq) continue;
#pragma unroll
    for (int j = 0; j < MAXC; j++) {
      const int c = cg + 16 * j;
      if (j < ncol && c < hd) a.out[(size_t)(q0 + qi) * a.out_stride + h * hd + c] = __fdiv_rn(o[r][j], l[r]);
    }
  }
}

// Attention over history splits that every row shares (branches of one
// prefix: mlx_branches.go:98-114 reads the prefix read-only for all of them).
// One CTA per (shared split of 64 positions, KV head, tile of 64 query rows):
// the split's keys and values are loaded once for all rows, query qi is head
// g * G + qi % G of row qi / G, rotated at that row's position. Scores,
// softmax and weighted values as in k_attn_prefill (no causal mask: every
// position precedes every row's own). Writes each row's split partial
// (sum_t exp(s_t - m) v_t, m, sum_t exp(s_t - m)) where the per-row kernels
// expect it; they handle the later splits and merge all of them.
template <int NC>
__global__ void __launch_bounds__(PA_THREADS, NC <= 5 ? 2 : 1) k_attn_shared(DecodeAttnArgs a) {
  extern __shared__ __align__(16) float pa_smem[];
  const int hd = a.hd, s = blockIdx.x, g = blockIdx.y, G = a.H / a.KVH;
  const int nrow = a.M * G;
  const int q0 = blockIdx.z * PA_QT;
  const int nq = min(PA_QT, nrow - q0);
  float* qT = pa_smem;                                       // [hd][QT]
  float* kT = qT + hd * PA_QT;                               // [hd][KTS]
  float* vs = kT + max(hd * PA_KTS, PA_KT * PA_QT);          // [KT][hd]; first holds the query rows for RoPE
  float* ps = kT;                                            // [KT][QT], over the key tile after the scores
  const int tid = threadIdx.x, rg = tid >> 4, cg = tid & 15;
  for (int e = tid; e < PA_QT * hd; e += PA_THREADS) {
    const int qi = e / hd, i = e % hd, row = q0 + qi;
    vs[e] = qi < nq ? a.qkv[(size_t)(row / G) * a.qkv_stride + (g * G + row % G) * hd + i] : 0.f;
  }
  __syncthreads();
  for (int e = tid; e < nq * a.rope.pairs; e += PA_THREADS) {
    const int qi = e / a.rope.pairs;
    rope_pair(vs + qi * hd, e % a.rope.pairs, a.rope, a.pos[(q0 + qi) / G]);
  }
  __syncthreads();
  for (int e = tid; e < PA_QT * hd; e += PA_THREADS) qT[(e % hd) * PA_QT + e / hd] = vs[e];
  __syncthreads();
  // Keys and values of the split (pages of row 0's table: shared by all rows).
  const int t0 = s * PA_KT;
  for (int t = 0; t < PA_KT;) {
    const int ta = t0 + t;
    const int page = a.page_table[ta / a.kv.P], row = ta % a.kv.P;
    const int n = min(PA_KT - t, a.kv.P - row);
    const size_t off = a.kv.off(a.layer, page, g, row);
    for (int e = tid; e < n * hd; e += PA_THREADS) {
      const int r = e / hd, c = e % hd;
      float kk, vv;
      if (a.kv.half) {
        kk = __half2float(reinterpret_cast<const __half*>(a.kv.k)[off + e]);
        vv = __half2float(reinterpret_cast<const __half*>(a.kv.v)[off + e]);
      } else {
        kk = reinterpret_cast<const float*>(a.kv.k)[off + e];
        vv = reinterpret_cast<const float*>(a.kv.v)[off + e];
      }
      kT[c * PA_KTS + t + r] = kk;
      vs[(t + r) * hd + c] = vv;
    }
    t += n;
  }
  __syncthreads();
  float sc[4][4];
#pragma unroll
  for (int r = 0; r < 4; r++)
#pragma unroll
    for (int c = 0; c < 4; c++) sc[r][c] = 0.f;
  for (int i = 0; i < hd; i++) {
    const float4 qv = *reinterpret_cast<const float4*>(qT + i * PA_QT + 4 * rg);
    const float4 kv = *reinterpret_cast<const float4*>(kT + i * PA_KTS + 4 * cg);
    const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int c = 0; c < 4; c++) sc[r][c] = fmaf(qa[r], ka[c], sc[r][c]);
  }
  float mrow[4], lrow[4];
#pragma unroll
  for (int r = 0; r < 4; r++) {
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      sc[r][c] = __fdiv_rn(sc[r][c], a.scale);
      mx = fmaxf(mx, sc[r][c]);
    }
#pragma unroll
    for (int x = 1; x < 16; x <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, x));
    float ls = 0.f;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      sc[r][c] = expf(sc[r][c] - mx);
      ls += sc[r][c];
    }
#pragma unroll
    for (int x = 1; x < 16; x <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, x);
    mrow[r] = mx;
    lrow[r] = ls;
  }
  __syncthreads();  // every thread's reads of the key tile are done
#pragma unroll
  for (int c = 0; c < 4; c++)
    *reinterpret_cast<float4*>(ps + (4 * cg + c) * PA_QT + 4 * rg) = make_float4(sc[0][c], sc[1][c], sc[2][c], sc[3][c]);
  __syncthreads();
  const int ncol = (hd + 15) / 16;
  float o[4][NC];
#pragma unroll
  for (int r = 0; r < 4; r++)
#pragma unroll
    for (int j = 0; j < NC; j++) o[r][j] = 0.f;
  for (int t = 0; t < PA_KT; t++) {
    const float4 pv = *reinterpret_cast<const float4*>(ps + t * PA_QT + 4 * rg);
    const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
    const float* vr = vs + t * hd;
#pragma unroll
    for (int j = 0; j < NC; j++) {
      const int c = cg + 16 * j;
      if (j < ncol && c < hd) {
        const float vv = vr[c];
#pragma unroll
        for (int r = 0; r < 4; r++) o[r][j] = fmaf(pa[r], vv, o[r][j]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int qi = 4 * rg + r;
    if (qi >= nq) continue;
    const int row = q0 + qi, m = row / G;
    float* part = a.part + (((size_t)m * a.H + g * G + row % G) * a.max_splits + s) * (hd + 2);
#pragma unroll
    for (int j = 0; j < NC; j++) {
      const int c = cg + 16 * j;
      if (j < ncol && c < hd) part[c] = o[r][j];
    }
    if (cg == 0) {
      part[hd] = mrow[r];
      part[hd + 1] = lrow[r];
    }
  }
}

// ---------------------------------------------------------------------------
// Embedding rows (stablelm.go:338, prefill.go:58-60, model.go:419). In step
// mode the token of sequence m is the argmax of the previous step
// (greedy decoding kept on the device), and the step bookkeeping advances.
struct EmbedArgs {
  DMat E;
  int n;
  const int* tokens;  // [n] (token mode)
  // step mode (tokens == nullptr)
  unsigned long long* argmax;  // [n], consumed and cleared
  int* pos;                    // [n], advanced by one
  int* out_tokens;             // [n][out_stride] token log
  int out_stride;
  int* out_count;              // [n]
  float* x;
  int x_stride;
};

__global__ void k_embed(EmbedArgs a) {
  const int m = blockIdx.x;
  __shared__ int tok;
  if (threadIdx.x == 0) {
    int t;
    if (a.tokens) {
      t = a.tokens[m];
    } else {
      t = argmax_index(a.argmax[m]);
      a.argmax[m] = 0ull;
      a.pos[m] += 1;
      int c = a.out_count[m];
      a.out_tokens[(size_t)m * a.out_stride + c] = t;
      a.out_count[m] = c + 1;
    }
    tok = (t >= 0 && t < a.E.rows) ? t : 0;
  }
  __syncthreads();
  const int d = a.E.cols;
  for (int i = threadIdx.x; i < d; i += blockDim.x) a.x[(size_t)m * a.x_stride + i] = dmat_at(a.E, tok, i);
}

// Writes the final greedy token (the argmax of the last evaluated step).
__global__ void k_finish_greedy(const unsigned long long* argmax, int* out_tokens, int out_stride, int* out_count, int n) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m < n) {
    int c = out_count[m];
    out_tokens[(size_t)m * out_stride + c] = argmax_index(argmax[m]);
    out_count[m] = c + 1;
  }
}



// ---------------------------------------------------------------------------
// Decode attention with the history staged by bulk copies: CTA r of (row m,
// KV head g) takes the run of splits [s_begin + r per, s_begin + (r + 1) per)
// and copies each split's K and V page tiles ([P][hd], contiguous per page and
// kv head) into shared memory with cp.async.bulk, the next split's while the
// current one is computed (two stages). Per split the arithmetic of
// k_attn_decode (scores as float32 dot products in dimension order divided
// by sqrt(hd), the split's max, expf weights, position-order sums); the run
// keeps the online merge of its splits (o = o expf(m - m') + o_split expf(m_s
// - m')) and writes one partial into slot s_begin + r. The run holding the
// last split rotates and stores the new token's k and v. The last CTA of the
// row and KV head merges every partial (attn_merge_splits).

__device__ __forceinline__ float kv_ld(const void* base, int half, size_t i) {
  return half ? __half2float(reinterpret_cast<const __half*>(base)[i]) : reinterpret_cast<const float*>(base)[i];
}

struct DecodeAttn2Extra {
  int* err;
};

// Key / value elements of a staged tile as float32 (binary16 or float32 KV).
template <bool HALF>
__device__ __forceinline__ float kv_ld1(const uint8_t* tile, size_t i) {
  if constexpr (HALF)
    return __half2float(reinterpret_cast<const __half*>(tile)[i]);
  else
    return reinterpret_cast<const float*>(tile)[i];
}
template <bool HALF>
__device__ __forceinline__ float2 kv_ld2(const uint8_t* tile, size_t i) {
  if constexpr (HALF)
    return __half22float2(*reinterpret_cast<const __half2*>(tile + 2 * i));
  else
    return *reinterpret_cast<const float2*>(tile + 4 * i);
}
template <bool HALF>
__device__ __forceinline__ float4 kv_ld4(const uint8_t* tile, size_t i) {
  if constexpr (HALF) {
    const uint2 b = *reinterpret_cast<const uint2*>(tile + 2 * i);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&b.x)), c = __half22float2(*reinterpret_cast<const __half2*>(&b.y));
    return make_float4(a.x, a.y, c.x, c.y);
  } else {
    return *reinterpret_cast<const float4*>(tile + 4 * i);
  }
}

// Scores of one split for the G heads: two threads per (head, position), each
// a float32 dot product over half the head dimension in dimension order, the
// halves added by a shuffle, then divided by sqrt(hd).
template <bool HALF>
__device__ __forceinline__ void bulk_scores(const uint8_t* ktile, const float* qs, float* sc, int G, int split, int nt, int hd,
                                            float scale) {
  const int h2 = hd / 2;
  const bool vec = (hd & 7) == 0;
  for (int e = threadIdx.x; e < G * split * 2; e += blockDim.x) {
    const int half = e & 1, r = e >> 1, hh = r / split, t = r % split;
    float d = 0.f;
    if (t < nt) {
      const float* q = qs + hh * hd + half * h2;
      const size_t row = (size_t)t * hd + half * h2;
      int k = 0;
      if (vec)
        for (; k + 4 <= h2; k += 4) {
          const float4 kv = kv_ld4<HALF>(ktile, row + k);
          d = fmaf(q[k], kv.x, d);
          d = fmaf(q[k + 1], kv.y, d);
          d = fmaf(q[k + 2], kv.z, d);
          d = fmaf(q[k + 3], kv.w, d);
        }
      for (; k < h2; k++) d = fmaf(q[k], kv_ld1<HALF>(ktile, row + k), d);
    }
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    if (half == 0 && t < nt) sc[hh * split + t] = __fdiv_rn(d, scale);
  }
}

// The weighted values of one split merged into the run's outputs: two
// threads per (head, pair of dimensions), each over half the positions in
// position order, the halves added by a shuffle; then
// orun = orun * alpha + o * beta with the run's and the split's maxima.
template <bool HALF>
__device__ __forceinline__ void bulk_values(const uint8_t* vtile, const float* sc, int G, int split, int nt, int hd, const float* mrun,
                                            const float* mloc, float* orun) {
  const int hp = hd / 2, tasks = G * hp * 2, th = (nt + 1) / 2;
  for (int e = threadIdx.x; e < (tasks + 31) / 32 * 32; e += blockDim.x) {  // whole warps: every lane reaches the shuffles
    const bool ok = e < tasks;
    const int ph = e & 1, pr = e >> 1, hh = pr / hp, dp = pr % hp;
    float o0 = 0.f, o1 = 0.f;
    if (ok) {
      const float* p = sc + hh * split;
      for (int t = ph * th, t1 = min(nt, ph * th + th); t < t1; t++) {
        const float2 v = kv_ld2<HALF>(vtile, (size_t)t * hd + 2 * dp);
        o0 = fmaf(p[t], v.x, o0);
        o1 = fmaf(p[t], v.y, o1);
      }
    }
    o0 += __shfl_xor_sync(0xffffffffu, o0, 1);
    o1 += __shfl_xor_sync(0xffffffffu, o1, 1);
    if (ok && ph == 0) {
      const float mo = mrun[hh], mn = fmaxf(mo, mloc[hh]);
      const float alpha = mo == -INFINITY ? 0.f : expf(mo - mn), beta = expf(mloc[hh] - mn);
      float* o = orun + hh * hd + 2 * dp;
      o[0] = o[0] * alpha + o0 * beta;
      o[1] = o[1] * alpha + o1 * beta;
    }
  }
}

// Dynamic shared memory of k_attn_decode_bulk: barriers, two stages of K and V
// tiles, q, scores, the new k/v and the run's outputs.
__host__ __device__ inline size_t attn_bulk_smem(int G, int split, int hd, int es) {
  return 128 + 4 * (size_t)split * hd * es + sizeof(float) * (2 * (size_t)G * hd + (size_t)G * split + 2 * (size_t)hd);
}

__global__ void __launch_bounds__(128) k_attn_decode_bulk(DecodeAttnArgs a, DecodeAttn2Extra x) {
  extern __shared__ __align__(128) uint8_t ab_smem[];
  const int r = blockIdx.x, g = blockIdx.y, m = blockIdx.z;
  const int hd = a.hd, G = a.H / a.KVH, split = a.split, P = a.kv.P, per = a.per;
  const int es = a.kv.half ? 2 : 4;
  pdl_launch_dependents();
  pdl_wait();
  const int pos = a.pos[m];
  const int T = pos + 1;
  const int nsplit = (T + split - 1) / split;
  const int s_first = a.s_begin + r * per;
  if (s_first >= nsplit) return;
  const int s_last = min(nsplit, s_first + per) - 1;
  const bool has_cur = s_last == nsplit - 1;
  const size_t tile = (size_t)split * hd * es;

  uint64_t* bar = reinterpret_cast<uint64_t*>(ab_smem);  // [2]
  uint8_t* stages = ab_smem + 128;                        // [2][K tile, V tile]
  float* qs = reinterpret_cast<float*>(stages + 4 * tile);
  float* sc = qs + G * hd;
  float* cur = sc + G * split;
  float* orun = cur + 2 * hd;
  __shared__ int is_last;
  __shared__ float mloc[32], lloc[32], mrun[32], lrun[32];

  const int* pt = a.page_table + (size_t)m * a.pt_stride;
  // Thread 0: the bulk copies of split s's history pages into stage st.
  auto issue = [&](int s, int st) {
    const int t0 = s * split;
    const int nt = min(T, t0 + split) - t0;
    const int n_hist = s == nsplit - 1 ? nt - 1 : nt;
    const int npages = (n_hist + P - 1) / P;
    const uint32_t pbytes = (uint32_t)(P * hd * es);
    uint8_t* kt = stages + (size_t)st * 2 * tile;
    mbar_expect_tx(bar + st, 2u * npages * pbytes);  // no pages: the phase completes at once
    for (int j = 0; j < npages; j++) {
      const int page = pt[t0 / P + j];
      const size_t o = a.kv.off(a.layer, page, g, 0) * es;
      bulk_g2s(kt + (size_t)j * pbytes, reinterpret_cast<const uint8_t*>(a.kv.k) + o, pbytes, bar + st);
      bulk_g2s(kt + tile + (size_t)j * pbytes, reinterpret_cast<const uint8_t*>(a.kv.v) + o, pbytes, bar + st);
    }
  };
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 1);
    fence_barrier_init();
  }
  if (threadIdx.x < G) {
    mrun[threadIdx.x] = -INFINITY;
    lrun[threadIdx.x] = 0.f;
  }
  for (int e = threadIdx.x; e < G * hd; e += blockDim.x) orun[e] = 0.f;
  __syncthreads();
  if (threadIdx.x == 0) issue(s_first, 0);
  // While the copies fly: q of the group and, for the last split, the new k/v.
  const float* q_in = a.qkv + (size_t)m * a.qkv_stride;
  for (int e = threadIdx.x; e < G * hd; e += blockDim.x) qs[e] = q_in[(g * G) * hd + e];
  if (has_cur) {
    for (int e = threadIdx.x; e < hd; e += blockDim.x) {
      cur[e] = q_in[a.H * hd + g * hd + e];
      cur[hd + e] = q_in[(a.H + a.KVH) * hd + g * hd + e];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * a.rope.pairs; e += blockDim.x) rope_pair(qs + (e / a.rope.pairs) * hd, e % a.rope.pairs, a.rope, pos);
  if (has_cur)
    for (int e = threadIdx.x; e < a.rope.pairs; e += blockDim.x) rope_pair(cur, e, a.rope, pos);
  __syncthreads();
  if (has_cur) {
    for (int e = threadIdx.x; e < 2 * hd; e += blockDim.x) cur[e] = kv_round(cur[e], a.kv.half);
    __syncthreads();
    const int page = pt[pos / P], row = pos % P;
    const size_t o = a.kv.off(a.layer, page, g, row);
    for (int e = threadIdx.x; e < hd; e += blockDim.x) {
      kv_store(a.kv, a.kv.k, o + e, cur[e]);
      kv_store(a.kv, a.kv.v, o + e, cur[hd + e]);
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int s = s_first, i = 0; s <= s_last; s++, i++) {
    const int st = i & 1;
    if (threadIdx.x == 0 && s < s_last) {
      fence_proxy_async();  // the stage's earlier reads come before the copies into it
      issue(s + 1, st ^ 1);
    }
    const int t0 = s * split;
    const int nt = min(T, t0 + split) - t0;
    const bool cur_here = s == nsplit - 1;
    mbar_wait(bar + st, (i >> 1) & 1, x.err);
    const uint8_t* ktile = stages + (size_t)st * 2 * tile;
    const uint8_t* vtile = ktile + tile;
    // The new token's key and value (already rounded to the KV precision)
    // take their row of the staged tiles, so every position reads alike.
    if (cur_here) {
      uint8_t* kt = stages + (size_t)st * 2 * tile;
      for (int e = threadIdx.x; e < hd; e += blockDim.x) {
        const size_t o = (size_t)(nt - 1) * hd + e;
        if (a.kv.half) {
          reinterpret_cast<__half*>(kt)[o] = __float2half_rn(cur[e]);
          reinterpret_cast<__half*>(kt + tile)[o] = __float2half_rn(cur[hd + e]);
        } else {
          reinterpret_cast<float*>(kt)[o] = cur[e];
          reinterpret_cast<float*>(kt + tile)[o] = cur[hd + e];
        }
      }
      __syncthreads();
    }
    if (a.kv.half)
      bulk_scores<true>(ktile, qs, sc, G, split, nt, hd, a.scale);
    else
      bulk_scores<false>(ktile, qs, sc, G, split, nt, hd, a.scale);
    __syncthreads();
    for (int hh = warp; hh < G; hh += nwarps) {
      float mx = -INFINITY;
      for (int t = lane; t < nt; t += 32) mx = fmaxf(mx, sc[hh * split + t]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float l = 0.f;
      for (int t = lane; t < nt; t += 32) {
        float p = expf(sc[hh * split + t] - mx);
        sc[hh * split + t] = p;
        l += p;
      }
      l = warp_sum(l);
      if (lane == 0) {
        mloc[hh] = mx;
        lloc[hh] = l;
      }
    }
    __syncthreads();
    if (a.kv.half)
      bulk_values<true>(vtile, sc, G, split, nt, hd, mrun, mloc, orun);
    else
      bulk_values<false>(vtile, sc, G, split, nt, hd, mrun, mloc, orun);
    __syncthreads();
    if (threadIdx.x < G) {
      const float mo = mrun[threadIdx.x], mn = fmaxf(mo, mloc[threadIdx.x]);
      const float alpha = mo == -INFINITY ? 0.f : expf(mo - mn), beta = expf(mloc[threadIdx.x] - mn);
      lrun[threadIdx.x] = lrun[threadIdx.x] * alpha + lloc[threadIdx.x] * beta;
      mrun[threadIdx.x] = mn;
    }
    __syncthreads();
  }
  float* part = a.part + ((size_t)m * a.H + g * G) * a.max_splits * (hd + 2);
  const int slot = a.s_begin + r;
  for (int e = threadIdx.x; e < G * hd; e += blockDim.x)
    part[((size_t)(e / hd) * a.max_splits + slot) * (hd + 2) + e % hd] = orun[e];
  if (threadIdx.x < G) {
    part[((size_t)threadIdx.x * a.max_splits + slot) * (hd + 2) + hd] = mrun[threadIdx.x];
    part[((size_t)threadIdx.x * a.max_splits + slot) * (hd + 2) + hd + 1] = lrun[threadIdx.x];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int nruns = (nsplit - a.s_begin + per - 1) / per;
    int prev = atomicAdd(a.counters + m * a.KVH + g, 1);
    is_last = (prev == nruns - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // Merge every partial of each head in the group (the stages are free).
  attn_merge_splits(part, a.max_splits, hd, G, split_slots(a, nsplit), reinterpret_cast<float*>(stages), (int)(4 * tile / 4),
                    a.out + (size_t)m * a.out_stride + g * G * hd);
  if (threadIdx.x == 0) a.counters[m * a.KVH + g] = 0;
}

}  // namespace tcu
