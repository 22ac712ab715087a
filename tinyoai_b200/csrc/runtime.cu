// tinyoai B200 backend: model upload, paged KV pool, sessions, branches and
// the C ABI declared in include/tinyoai_cuda.h.
//
// The host side mirrors the reference's native-forwarder contract
// (mlx.go:45-57, branches.go:49-59, sessions.go:26-30, mlx_llama.go:27-35):
// a session holds a resident token prefix whose KV lives in pages of a
// per-model pool; Forward replaces the suffix after `prefix`; Fork and
// branches share full pages by reference count and copy only a page they
// write while it is shared.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/tinyoai_cuda.h"
#include "attention.cuh"
#include "common.cuh"
#include "gemm_simt.cuh"
#include "gemv.cuh"
#include "gemv_stream.cuh"
#include "decode_mega.cuh"
#include "gemm_tc.cuh"
#include <cudaTypedefs.h>
#include "misc.cuh"
#include "read_values.cuh"
#include "attn_tc.cuh"
#include "tp_exchange.cuh"
#include "gguf.h"
#include "kv_snapshot.h"

using namespace tcu;

static const int CHUNK = 512;      // prompt tokens per internal chunk (mlx.go:352-355)
static const int SPLIT_PAGES = 2;  // KV pages per decode attention unit
static const int LP_ROWS = 32;     // log-probability rows per head product (mlx_native.go's probabilityBatch)

// ---------------------------------------------------------------------------
// Errors: integer status + thread-local message (internal/mlx/bridge.c:13-33).
static thread_local std::string g_err;

static int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define CK(x)                                                                                   \
  do {                                                                                          \
    cudaError_t e_ = (x);                                                                       \
    if (e_ != cudaSuccess) return fail(TCU_ECUDA, "%s (%s:%d): %s", #x, __FILE__, __LINE__, cudaGetErrorString(e_)); \
  } while (0)
// First kernel launch or async call on this thread whose launch reported an
// error, named in the message of the call that fails.
static thread_local const char* g_err_site = nullptr;
static inline void note_launch(const char* site) {
  if (!g_err_site && cudaPeekAtLastError() != cudaSuccess) g_err_site = site;
}
#define NOTE(site) note_launch(site)

#define TRY(x)               \
  do {                       \
    int r_ = (x);            \
    if (r_ != TCU_OK) return r_; \
  } while (0)

// ---------------------------------------------------------------------------
// Model

enum Arch { ARCH_STABLELM = 0, ARCH_LLAMA = 1 };

struct Layer {
  DMat w1{}, w2{}, w3{}, w4{};
  float *n1w = nullptr, *n1b = nullptr, *n2w = nullptr;
};

struct KVPool {
  int half = 0, P = 32, L = 0, kvh = 0, hd = 0, num_pages = 0;
  void *k = nullptr, *v = nullptr;
  std::vector<int> ref;
  std::vector<int> free_list;
  size_t used() const { return (size_t)(num_pages - (int)free_list.size()); }
  size_t page_elems() const { return (size_t)kvh * P * hd; }
  size_t elem() const { return half ? 2 : 4; }
  KVView view() const {
    KVView w;
    w.k = k;
    w.v = v;
    w.half = half;
    w.P = P;
    w.num_pages = num_pages;
    w.kvh = kvh;
    w.hd = hd;
    return w;
  }
};

struct Work;

struct tcu_model {
  Arch arch = ARCH_STABLELM;
  int device = 0;
  int V = 0, d = 0, ff = 0, L = 0, H = 0, KVH = 0, hd = 0, max_pos = 0;
  int kvw = 0;  // KVH * hd
  int aw = 0;   // attention width H * hd: the hidden size, or this rank's heads under tensor parallelism
  double eps = 1e-5;
  Rope rope{};
  std::vector<Layer> layers;
  DMat embed{}, head{};
  float *fnw = nullptr, *fnb = nullptr;
  std::vector<void*> allocs;
  uint64_t weight_bytes = 0;
  int P = 32;
  int64_t pool_budget = 0;
  KVPool* pools[2] = {nullptr, nullptr};
  std::mutex mu;
  int sessions = 0;
  int sm_count = 148;
  int gemv_smem_optin = 0;
  bool disable_stream = false;  // TCU_DECODE_KERNELS=portable selects the non-TMA kernels
  bool use_tc = true;           // tensor-core prefill GEMM (TCU_GEMM=simt selects the CUDA-core one)
  bool use_tc_attn = true;      // tensor-core shared-prefix attention (TCU_ATTN=simt selects the CUDA-core one)
  unsigned* scratch_u32 = nullptr;
  // Persistent decode step (decode_mega.cuh): Q8_0 StableLM shapes that fit.
  bool mega = false;
  MegaLayer* mega_layers = nullptr;  // device array
  uint32_t mega_slot_bytes = 0, mega_off[5] = {0, 0, 0, 0, 0};
  int mega_slots = 0, mega_split = 0, mega_att_warp = 0;
  size_t mega_smem = 0;
  std::vector<Work*> work_pool;  // workspaces of closed handles (work_take / work_give), guarded by mu
  // Head-parallel tensor parallelism (tcu_stablelm_load_tp): this rank's
  // share of the heads and of the MLP, and the communicator of the per-layer
  // all-reduce of the out + down partial sums.
  int tp_world = 1, tp_rank = 0;
  ncclComm_t tp_comm = nullptr;
  // The exchange over NVLink peer memory (tp_exchange.cuh), once every rank
  // has opened the others' buffers (tcu_tp_exchange_open); NCCL otherwise.
  uint8_t* tp_ex = nullptr;
  uint8_t* tp_peer[TPX_MAX_RANKS] = {};
  long long tp_ex_count = 0;
  uint32_t* tp_seq = nullptr;  // device: exchanges completed, CTAs finished in the current one
  bool tp_ex_on = false;
};

static int dalloc(tcu_model* m, void** p, size_t n) {
  if (n == 0) n = 16;
  cudaError_t e = cudaMalloc(p, n);
  if (e != cudaSuccess) return fail(e == cudaErrorMemoryAllocation ? TCU_ENOMEM : TCU_ECUDA, "cudaMalloc(%zu): %s", n, cudaGetErrorString(e));
  m->allocs.push_back(*p);
  m->weight_bytes += n;
  return TCU_OK;
}

// NCCL, resolved at run time so that the library loads where NCCL is absent;
// only tensor-parallel models use it. If the process already holds a
// libnccl.so.2 (a framework's), dlopen returns that one.
struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};
static NcclApi g_nccl;
static std::once_flag g_nccl_once;

static const NcclApi* nccl_api() {
  std::call_once(g_nccl_once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    g_nccl.comm_init_rank = reinterpret_cast<decltype(g_nccl.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    g_nccl.all_reduce = reinterpret_cast<decltype(g_nccl.all_reduce)>(dlsym(h, "ncclAllReduce"));
    g_nccl.comm_destroy = reinterpret_cast<decltype(g_nccl.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    g_nccl.error_string = reinterpret_cast<decltype(g_nccl.error_string)>(dlsym(h, "ncclGetErrorString"));
    g_nccl.ok = g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.all_reduce && g_nccl.comm_destroy && g_nccl.error_string;
  });
  return g_nccl.ok ? &g_nccl : nullptr;
}

static void work_pool_free(tcu_model* m);

static void model_release(tcu_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  work_pool_free(m);
  if (m->tp_comm && nccl_api()) nccl_api()->comm_destroy(m->tp_comm);
  for (int p = 0; p < TPX_MAX_RANKS; p++)
    if (m->tp_peer[p] && m->tp_peer[p] != m->tp_ex) cudaIpcCloseMemHandle(m->tp_peer[p]);
  if (m->tp_ex) cudaFree(m->tp_ex);
  for (void* p : m->allocs) cudaFree(p);
  for (KVPool* p : m->pools)
    if (p) {
      cudaFree(p->k);
      cudaFree(p->v);
      delete p;
    }
  delete m;
}

static size_t fmt_row_bytes(int fmt, int cols) {
  switch (fmt) {
    case FMT_Q8_0:
      return (size_t)cols;  // quant plane; scales separate
    case FMT_F32:
      return (size_t)cols * 4;
    case FMT_F16:
    case FMT_BF16:
      return (size_t)cols * 2;
    default:
      return (size_t)cols / kquant_block_width(fmt) * kquant_dev_bytes(fmt);
  }
}

static size_t file_bytes(int fmt, int64_t rows, int64_t cols) {
  switch (fmt) {
    case FMT_Q8_0:
      return (size_t)(rows * cols / 32 * 34);
    case FMT_F32:
      return (size_t)(rows * cols * 4);
    case FMT_F16:
    case FMT_BF16:
      return (size_t)(rows * cols * 2);
    case FMT_Q5_1:
    case FMT_Q5_K:
    case FMT_Q6_K:
      return (size_t)(rows * cols / kquant_block_width(fmt) * kquant_block_bytes(fmt));
    default:
      return 0;
  }
}

static bool fmt_known(int f) {
  return f == FMT_F32 || f == FMT_F16 || f == FMT_BF16 || f == FMT_Q8_0 || f == FMT_Q5_1 || f == FMT_Q5_K || f == FMT_Q6_K;
}

static int alloc_dmat(tcu_model* m, DMat* out, int fmt, int rows, int cols) {
  DMat w{};
  w.fmt = fmt;
  w.rows = rows;
  w.cols = cols;
  void* p = nullptr;
  TRY(dalloc(m, &p, fmt_row_bytes(fmt, cols) * rows));
  w.w = (const uint8_t*)p;
  if (fmt == FMT_Q8_0) {
    w.sstride = (cols / 32 + 7) / 8 * 8;
    void* s = nullptr;
    TRY(dalloc(m, &s, (size_t)rows * w.sstride * 2));
    w.s = (const __half*)s;
  }
  *out = w;
  return TCU_OK;
}

// Staging: raw tensor bytes go to a device scratch buffer, then k_repack
// writes them into their place in the fused device matrix.
struct Stager {
  uint8_t* buf = nullptr;
  size_t cap = 0;
  ~Stager() {
    if (buf) cudaFree(buf);
  }
};

static int place(Stager& st, const void* data, size_t nbytes, int fmt, int rows, int cols, const DMat& dst, int row0, int row_step,
                 int col0) {
  if (nbytes > st.cap) {
    if (st.buf) cudaFree(st.buf);
    st.buf = nullptr;
    st.cap = 0;
    CK(cudaMalloc(&st.buf, nbytes));
    st.cap = nbytes;
  }
  CK(cudaMemcpy(st.buf, data, nbytes, cudaMemcpyHostToDevice));
  RepackArgs a{st.buf, fmt, rows, cols, dst, row0, row_step, col0};
  k_repack<<<1184, 256>>>(a);
  NOTE("k_repack");
  CK(cudaGetLastError());
  CK(cudaDeviceSynchronize());
  return TCU_OK;
}

static float host_half(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16, ex = (h >> 10) & 31, frac = h & 1023, u;
  if (ex == 0) {
    float v = (float)ldexp((double)frac, -24);
    return sign ? -v : v;
  }
  if (ex == 31)
    u = sign | 0x7f800000u | frac << 13;
  else
    u = sign | (ex + 112) << 23 | frac << 13;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// Decodes a 1-D norm tensor to float32 (weightTensor.at, safetensors.go:230-246).
static int decode_vec(const tcu_tensor* t, int n, std::vector<float>& out) {
  out.resize(n);
  const uint8_t* p = (const uint8_t*)t->data;
  for (int i = 0; i < n; i++) {
    switch (t->dtype) {
      case TCU_F32:
        memcpy(&out[i], p + 4 * i, 4);
        break;
      case TCU_F16:
        out[i] = host_half((uint16_t)(p[2 * i] | (p[2 * i + 1] << 8)));
        break;
      case TCU_BF16: {
        uint32_t u = (uint32_t)(p[2 * i] | (p[2 * i + 1] << 8)) << 16;
        memcpy(&out[i], &u, 4);
        break;
      }
      default:
        return fail(TCU_EUNSUP, "tensor %s: unsupported dtype %d for a norm vector", t->name, t->dtype);
    }
  }
  return TCU_OK;
}

static int upload_floats(tcu_model* m, const std::vector<float>& v, float** out) {
  void* p = nullptr;
  TRY(dalloc(m, &p, v.size() * 4));
  CK(cudaMemcpy(p, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
  *out = (float*)p;
  return TCU_OK;
}

// Once per device (with it current): the largest dynamic shared memory of
// the one-CTA-per-row sampling kernels, whose need varies with the
// vocabulary. Set once, not per launch, so no other thread can lower it
// between another call's set and its launch.
static std::mutex g_attr_mu;
static bool g_attr_done[64] = {};
static int sampling_smem_attrs(int device) {
  std::lock_guard<std::mutex> g(g_attr_mu);
  if (device < 0 || device >= 64 || g_attr_done[device]) return TCU_OK;
  int optin = 0;
  CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  // Dynamic shared memory may take what the kernel's static arrays leave.
  auto set_max = [&](const void* f) -> int {
    cudaFuncAttributes fa;
    CK(cudaFuncGetAttributes(&fa, f));
    CK(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes));
    return TCU_OK;
  };
  TRY(set_max((const void*)k_shortlist));
  TRY(set_max((const void*)k_logprob_rows));
  TRY(set_max((const void*)k_candidates_rows));
  g_attr_done[device] = true;
  return TCU_OK;
}

static int check_device(int device) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return fail(TCU_ENODEV, "no CUDA device available");
  if (device < 0 || device >= n) return fail(TCU_ENODEV, "device %d out of range (%d devices)", device, n);
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) return fail(TCU_ENODEV, "device %d is sm_%d%d; this library is built for sm_100a", device, prop.major, prop.minor);
  CK(cudaSetDevice(device));
  return sampling_smem_attrs(device);
}

static void init_common(tcu_model* m, const tcu_load_options* o) {
  m->device = o ? o->device : 0;
  m->P = (o && o->kv_page_tokens > 0) ? o->kv_page_tokens : 32;
  m->pool_budget = o ? o->kv_pool_bytes : 0;
  cudaDeviceGetAttribute(&m->sm_count, cudaDevAttrMultiProcessorCount, m->device);
  cudaDeviceGetAttribute(&m->gemv_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device);
  const char* k = getenv("TCU_DECODE_KERNELS");
  m->disable_stream = k && strcmp(k, "portable") == 0;
  const char* g = getenv("TCU_GEMM");
  m->use_tc = !(g && strcmp(g, "simt") == 0);
  const char* at = getenv("TCU_ATTN");
  m->use_tc_attn = !(at && strcmp(at, "simt") == 0);
}

// StableLM rotary table (stablelm.go:309-326): per position and rotary pair,
// the float32 angle and its float64 sine/cosine rounded to float32.
static int build_stablelm_rope(tcu_model* m, double theta, int rotary) {
  const int pairs = rotary / 2;
  std::vector<float2> tab((size_t)m->max_pos * pairs);
  for (int i = 0; i < pairs; i++) {
    volatile float ftheta = (float)theta;
    volatile float expo = (float)(2 * i) / (float)rotary;
    volatile float power = (float)pow((double)ftheta, (double)expo);
    volatile float inv = 1.0f / power;
    for (int pos = 0; pos < m->max_pos; pos++) {
      volatile float angle = (float)pos * inv;
      tab[(size_t)pos * pairs + i] = make_float2((float)cos((double)angle), (float)sin((double)angle));
    }
  }
  void* p = nullptr;
  TRY(dalloc(m, &p, tab.size() * sizeof(float2)));
  CK(cudaMemcpy(p, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
  m->rope.table = (const float2*)p;
  m->rope.pairs = pairs;
  m->rope.mode = 0;
  return TCU_OK;
}

static const tcu_tensor* find_tensor(const tcu_tensor* t, int n, const std::string& name) {
  for (int i = 0; i < n; i++)
    if (t[i].name && name == t[i].name) return &t[i];
  return nullptr;
}

static int check_tensor(const tcu_tensor* t, const std::string& name, int64_t rows, int64_t cols) {
  if (!t) return fail(TCU_EINVAL, "missing tensor %s", name.c_str());
  if (!fmt_known(t->dtype)) return fail(TCU_EUNSUP, "tensor %s: unsupported dtype %d", name.c_str(), t->dtype);
  const int64_t want_rows = cols ? rows : 1, want_cols = cols ? cols : rows;
  const int64_t r = t->ndim == 2 ? t->shape[0] : 1, c = t->ndim == 2 ? t->shape[1] : t->shape[0];
  if ((cols && t->ndim != 2) || (!cols && t->ndim != 1) || r != want_rows || c != want_cols)
    return fail(TCU_EINVAL, "tensor %s: shape mismatch (want %lld x %lld)", name.c_str(), (long long)want_rows, (long long)want_cols);
  if ((t->dtype == FMT_Q8_0 || t->dtype == FMT_Q5_1) && c % 32)
    return fail(TCU_EINVAL, "tensor %s: %s rows must be divisible by 32", name.c_str(), t->dtype == FMT_Q8_0 ? "Q8_0" : "Q5_1");
  if ((t->dtype == FMT_Q5_K || t->dtype == FMT_Q6_K) && c % 256)
    return fail(TCU_EINVAL, "tensor %s: K-quant rows must be divisible by 256", name.c_str());
  if (t->nbytes != file_bytes(t->dtype, r, c)) return fail(TCU_EINVAL, "tensor %s: %llu bytes, want %zu", name.c_str(), (unsigned long long)t->nbytes, file_bytes(t->dtype, r, c));
  if (!t->data) return fail(TCU_EINVAL, "tensor %s: null data", name.c_str());
  return TCU_OK;
}

// Decides whether the persistent decode kernel serves this model and lays out
// its shared memory: Q8_0 weights everywhere, hidden <= 2560 (one register
// chunk per warp), intermediate <= 3 * 2560, head_dim such that an attention
// unit's K and V tiles fit one ring slot.
static int set_tc_shifts(tcu_model* m);

// Scale layout of a staged down-projection row: the scales of its SwiGLU
// columns alone when they start 16-byte aligned in the row, else the whole
// scale row with the down segment starting at *soff.
static void mega_dn_scales(const tcu_model* m, int* sstride, int* soff) {
  const bool aligned = (m->d / 32) % 8 == 0;
  *sstride = aligned ? (m->ff / 32 + 7) / 8 * 8 : m->layers[0].w2.sstride;
  *soff = aligned ? 0 : m->d / 32;
}

static int build_mega(tcu_model* m) {
  m->mega = false;
  if (m->disable_stream || m->arch != ARCH_STABLELM || m->tp_world > 1 || m->aw != m->d) return TCU_OK;
  if (m->embed.fmt != FMT_Q8_0 || m->head.fmt != FMT_Q8_0) return TCU_OK;
  for (const Layer& ly : m->layers)
    if (ly.w1.fmt != FMT_Q8_0 || ly.w2.fmt != FMT_Q8_0) return TCU_OK;
  const int d = m->d, ff = m->ff, K2 = d + ff;
  const int G_q = m->H / m->KVH, n_plain = d + 2 * m->kvw;
  if (d % 32 || ff % 32 || n_plain % MG_W1_RS || d / 16 > 32 * MG_NJ || (ff / 16 + 3) / 4 > 32 * MG_NJ || K2 > MG_MAXK) return TCU_OK;
  if (d / 16 > MG_CT || G_q > 32 || m->hd % 8 || (G_q * m->hd) % 16 || m->rope.pairs > 64 || m->rope.mode != 0) return TCU_OK;
  // Every W1 tile must fit under the per-CTA cap of the persistent step.
  if ((size_t)(n_plain / MG_W1_RS + ff / 16) > (size_t)m->sm_count * MG_SWT) return TCU_OK;
  if ((size_t)(d + MG_DN_RS - 1) / MG_DN_RS > (size_t)m->sm_count * MG_SWT) return TCU_OK;
  if ((size_t)(d + MG_O_RS - 1) / MG_O_RS > (size_t)m->sm_count * MG_SWT) return TCU_OK;
  cudaFuncAttributes fa;
  CK(cudaFuncGetAttributes(&fa, k_decode_mega));
  const size_t w1 = (size_t)MG_W1_RS * (d + m->layers[0].w1.sstride * 2);
  int dn_sstride = 0, dn_soff = 0;
  mega_dn_scales(m, &dn_sstride, &dn_soff);
  const size_t w2 = std::max((size_t)MG_DN_RS * (ff + dn_sstride * 2), (size_t)MG_O_RS * (d + (d / 32 + 7) / 8 * 8 * 2));
  const size_t hb = (size_t)MG_W1_RS * (d + m->head.sstride * 2);
  size_t slot = std::max(w1, std::max(w2, hb));
  int split = 2 * m->P;
  while (split > m->P && (size_t)2 * split * m->hd * 4 > slot) split -= m->P;
  slot = std::max(slot, (size_t)2 * split * m->hd * 4);  // f32 KV worst case
  slot = (slot + 127) / 128 * 128;
  const size_t ghd = (size_t)G_q * m->hd;
  const size_t att_warp = (2 * ghd + 2 * m->hd + (size_t)G_q * split + 3) / 4 * 4;  // q, k/v, scores, outputs
  const size_t att_floats = att_warp * MG_CW + (ghd + 3) / 4 * 4;  // consumer warps, then the merge warp's outputs
  auto r128 = [](size_t b) { return (uint32_t)((b + 127) / 128 * 128); };
  const uint32_t off_x = MG_HDR;
  const uint32_t off_att = off_x + r128((size_t)d * 4);
  const uint32_t off_dig = off_att + r128(att_floats * 4);
  const uint32_t off_sx = off_dig + r128((size_t)K2 / 16 * 48);
  const uint32_t off_slots = off_sx + r128((size_t)K2 / 16 * 4);
  const size_t limit = (size_t)m->gemv_smem_optin - fa.sharedSizeBytes;
  if (off_slots + 2 * slot > limit) return TCU_OK;
  const int nslots = (int)std::min<size_t>(MG_MAX_SLOTS, (limit - off_slots) / slot);
  std::vector<MegaLayer> hl(m->L);
  for (int l = 0; l < m->L; l++) {
    const Layer& ly = m->layers[l];
    hl[l] = MegaLayer{(const int8_t*)ly.w1.w, ly.w1.s, (const int8_t*)ly.w2.w, ly.w2.s, ly.n1w, ly.n1b};
  }
  void* p = nullptr;
  TRY(dalloc(m, &p, hl.size() * sizeof(MegaLayer)));
  CK(cudaMemcpy(p, hl.data(), hl.size() * sizeof(MegaLayer), cudaMemcpyHostToDevice));
  m->mega_layers = (MegaLayer*)p;
  m->mega_slot_bytes = (uint32_t)slot;
  m->mega_slots = nslots;
  m->mega_split = split;
  m->mega_att_warp = (int)att_warp;
  m->mega_off[0] = off_x;
  m->mega_off[1] = off_att;
  m->mega_off[2] = off_dig;
  m->mega_off[3] = off_sx;
  m->mega_off[4] = off_slots;
  m->mega_smem = off_slots + (size_t)nslots * slot;
  CK(cudaFuncSetAttribute(k_decode_mega, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->mega_smem));
  int occ = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_decode_mega, MG_THREADS, m->mega_smem));
  m->mega = occ >= 1;
  if (getenv("TCU_VERBOSE"))
    fprintf(stderr, "tinyoai_b200: persistent decode %s (blocks/SM %d, regs %d, static smem %zu, dynamic smem %zu, slots %d x %u, split %d)\n",
            m->mega ? "on" : "off", occ, fa.numRegs, (size_t)fa.sharedSizeBytes, m->mega_smem, nslots, (unsigned)slot, split);
  return TCU_OK;
}

// One rank's share of a StableLM under head-parallel tensor parallelism:
// contiguous blocks of query heads, KV heads and MLP rows. Query head h uses
// KV head h / (H / KVH), so rank r's query heads use exactly its KV heads.
struct TpSlice {
  int world = 1, rank = 0;
  int h0 = 0, nh = 0;    // query heads
  int kv0 = 0, nkv = 0;  // KV heads
  int f0 = 0, nf = 0;    // MLP rows (gate/up) = down columns
};

static int tp_slice(const tcu_stablelm_config* c, int world, int rank, TpSlice* out) {
  if (world < 1 || rank < 0 || rank >= world) return fail(TCU_EINVAL, "invalid rank %d of %d", rank, world);
  if (c->num_attention_heads % world || c->num_key_value_heads % world || c->intermediate_size % world)
    return fail(TCU_EINVAL, "%d ranks must divide the heads (%d), KV heads (%d) and MLP width (%d)", world, c->num_attention_heads,
                c->num_key_value_heads, c->intermediate_size);
  TpSlice t;
  t.world = world;
  t.rank = rank;
  t.nh = c->num_attention_heads / world;
  t.h0 = rank * t.nh;
  t.nkv = c->num_key_value_heads / world;
  t.kv0 = rank * t.nkv;
  t.nf = c->intermediate_size / world;
  t.f0 = rank * t.nf;
  *out = t;
  return TCU_OK;
}

// Bytes of `cols` values of one row in a format's file encoding.
static size_t file_row_bytes(int fmt, int64_t cols) { return file_bytes(fmt, 1, cols); }

// Columns [c0, c0 + nc) of every row of a file-encoded [rows x cols] tensor,
// gathered into one buffer (whole blocks: c0 and nc divisible by the block
// width of the format).
static void gather_cols(const tcu_tensor* t, int rows, int cols, int c0, int nc, std::vector<uint8_t>& out) {
  const size_t rb = file_row_bytes(t->dtype, cols), off = file_row_bytes(t->dtype, c0), nb = file_row_bytes(t->dtype, nc);
  out.resize((size_t)rows * nb);
  const uint8_t* src = (const uint8_t*)t->data;
  for (int r = 0; r < rows; r++) memcpy(out.data() + (size_t)r * nb, src + (size_t)r * rb + off, nb);
}

static int fmt_block_width(int fmt) {
  switch (fmt) {
    case FMT_Q8_0:
    case FMT_Q5_1:
      return 32;
    case FMT_Q5_K:
    case FMT_Q6_K:
      return 256;
    default:
      return 1;
  }
}

// tp == nullptr: the whole model. Otherwise this rank's share (the tensors
// are the whole checkpoint's; the load takes its rows and columns).
static int stablelm_load(const tcu_stablelm_config* c, const tcu_tensor* t, int n, const tcu_load_options* o, const TpSlice* tp,
                         tcu_model** out) {
  // stablelm.go:85-111 validate() (the structural flags are checked by the caller's config parser).
  if (!c || !out || (n > 0 && !t)) return fail(TCU_EINVAL, "null argument");
  if (c->hidden_size <= 0 || c->intermediate_size <= 0 || c->num_hidden_layers <= 0 || c->num_attention_heads <= 0 ||
      c->num_key_value_heads <= 0 || c->vocab_size <= 0 || c->max_position_embeddings <= 0 ||
      c->hidden_size % c->num_attention_heads != 0 || c->num_attention_heads % c->num_key_value_heads != 0)
    return fail(TCU_EINVAL, "invalid StableLM dimensions");
  const double rotary_f = (double)(c->hidden_size / c->num_attention_heads) * c->partial_rotary_factor;
  if (!(c->layer_norm_eps > 0) || std::isinf(c->layer_norm_eps) || !(c->rope_theta > 0) || std::isinf(c->rope_theta) ||
      !(c->partial_rotary_factor > 0) || c->partial_rotary_factor > 1 || rotary_f != std::trunc(rotary_f) || (int)rotary_f % 2 != 0 ||
      rotary_f < 2)
    return fail(TCU_EINVAL, "invalid LayerNorm or partial RoPE settings");
  if (c->bos_token_id < 0 || c->bos_token_id >= c->vocab_size || c->eos_token_id < 0 || c->eos_token_id >= c->vocab_size)
    return fail(TCU_EINVAL, "invalid BOS/EOS token IDs");
  TpSlice whole;
  if (!tp) TRY(tp_slice(c, 1, 0, &whole));
  const TpSlice& sl = tp ? *tp : whole;
  const int device = o ? o->device : 0;
  TRY(check_device(device));
  tcu_model* m = new tcu_model();
  init_common(m, o);
  m->arch = ARCH_STABLELM;
  m->V = c->vocab_size;
  m->d = c->hidden_size;
  m->L = c->num_hidden_layers;
  m->hd = m->d / c->num_attention_heads;
  m->H = sl.nh;
  m->KVH = sl.nkv;
  m->ff = sl.nf;
  m->kvw = m->hd * m->KVH;
  m->aw = m->hd * m->H;
  m->tp_world = sl.world;
  m->tp_rank = sl.rank;
  m->max_pos = c->max_position_embeddings;
  m->eps = c->layer_norm_eps;
  const int d = m->d, ff = m->ff, kvw = m->kvw, aw = m->aw, hd = m->hd;
  const int ffg = c->intermediate_size, kvg = hd * c->num_key_value_heads;  // whole-checkpoint widths
  auto bail = [&](int code) {
    model_release(m);
    return code;
  };
  // The prefill attention kernel holds up to 128 output dimensions per query.
  if (m->hd < 4 || m->hd > 128 || m->hd % 4) return bail(fail(TCU_EINVAL, "head size %d: a multiple of 4 in 4..128 is supported", m->hd));
  // Validate every tensor before allocating (loadStableWeights, stablelm.go:167-199).
  auto chk = [&](const std::string& name, int64_t r, int64_t cc) { return check_tensor(find_tensor(t, n, name), name, r, cc); };
  int rc;
  if ((rc = chk("model.embed_tokens.weight", m->V, d)) || (rc = chk("lm_head.weight", m->V, d)) || (rc = chk("model.norm.weight", d, 0)) ||
      (rc = chk("model.norm.bias", d, 0)))
    return bail(rc);
  for (int l = 0; l < m->L; l++) {
    std::string p = "model.layers." + std::to_string(l) + ".";
    if ((rc = chk(p + "input_layernorm.weight", d, 0)) || (rc = chk(p + "input_layernorm.bias", d, 0)) ||
        (rc = chk(p + "self_attn.q_proj.weight", d, d)) || (rc = chk(p + "self_attn.k_proj.weight", kvg, d)) ||
        (rc = chk(p + "self_attn.v_proj.weight", kvg, d)) || (rc = chk(p + "self_attn.o_proj.weight", d, d)) ||
        (rc = chk(p + "mlp.gate_proj.weight", ffg, d)) || (rc = chk(p + "mlp.up_proj.weight", ffg, d)) ||
        (rc = chk(p + "mlp.down_proj.weight", d, ffg)))
      return bail(rc);
    const int f1 = find_tensor(t, n, p + "self_attn.q_proj.weight")->dtype;
    for (const char* nm : {"self_attn.k_proj.weight", "self_attn.v_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight"})
      if (find_tensor(t, n, p + nm)->dtype != f1)
        return bail(fail(TCU_EUNSUP, "layer %d: q/k/v/gate/up must share one dtype (fused projection)", l));
    const int f2 = find_tensor(t, n, p + "self_attn.o_proj.weight")->dtype;
    if (find_tensor(t, n, p + "mlp.down_proj.weight")->dtype != f2)
      return bail(fail(TCU_EUNSUP, "layer %d: o_proj and down_proj must share one dtype (fused projection)", l));
    if ((f2 == FMT_Q5_K || f2 == FMT_Q6_K) && aw % 256) return bail(fail(TCU_EUNSUP, "layer %d: K-quant o|down fusion needs an attention width divisible by 256", l));
    const int bw = fmt_block_width(f2);
    if (sl.world > 1 && ((sl.h0 * hd) % bw || aw % bw || sl.f0 % bw || ff % bw))
      return bail(fail(TCU_EUNSUP, "layer %d: the o/down column slices of %d ranks split %s blocks", l, sl.world,
                       f2 == FMT_Q8_0 ? "Q8_0" : "quantised"));
  }
  if ((rc = build_stablelm_rope(m, c->rope_theta, (int)rotary_f))) return bail(rc);
  Stager st;
  m->layers.resize(m->L);
  const int n_plain = aw + 2 * kvw;
  std::vector<uint8_t> cols;
  for (int l = 0; l < m->L; l++) {
    std::string p = "model.layers." + std::to_string(l) + ".";
    Layer& ly = m->layers[l];
    auto T = [&](const char* nm) { return find_tensor(t, n, p + nm); };
    const tcu_tensor *q = T("self_attn.q_proj.weight"), *k = T("self_attn.k_proj.weight"), *v = T("self_attn.v_proj.weight");
    const tcu_tensor *o_ = T("self_attn.o_proj.weight"), *g = T("mlp.gate_proj.weight"), *u = T("mlp.up_proj.weight"),
                     *dn = T("mlp.down_proj.weight");
    // Row slices of q/k/v/gate/up start inside the file tensors; o and down
    // columns are gathered.
    auto rows_of = [&](const tcu_tensor* x, int r0) { return (const uint8_t*)x->data + (size_t)r0 * file_row_bytes(x->dtype, d); };
    const size_t rq = file_row_bytes(q->dtype, d);
    // W1 rows: [q | k | v | (gate_i, up_i) interleaved]; W2 columns: [o | down].
    if ((rc = alloc_dmat(m, &ly.w1, q->dtype, n_plain + 2 * ff, d)) || (rc = alloc_dmat(m, &ly.w2, o_->dtype, d, aw + ff)) ||
        (rc = place(st, rows_of(q, sl.h0 * hd), rq * aw, q->dtype, aw, d, ly.w1, 0, 1, 0)) ||
        (rc = place(st, rows_of(k, sl.kv0 * hd), rq * kvw, k->dtype, kvw, d, ly.w1, aw, 1, 0)) ||
        (rc = place(st, rows_of(v, sl.kv0 * hd), rq * kvw, v->dtype, kvw, d, ly.w1, aw + kvw, 1, 0)) ||
        (rc = place(st, rows_of(g, sl.f0), rq * ff, g->dtype, ff, d, ly.w1, n_plain, 2, 0)) ||
        (rc = place(st, rows_of(u, sl.f0), rq * ff, u->dtype, ff, d, ly.w1, n_plain + 1, 2, 0)))
      return bail(rc);
    if (sl.world == 1) {
      if ((rc = place(st, o_->data, o_->nbytes, o_->dtype, d, d, ly.w2, 0, 1, 0)) ||
          (rc = place(st, dn->data, dn->nbytes, dn->dtype, d, ff, ly.w2, 0, 1, d)))
        return bail(rc);
    } else {
      gather_cols(o_, d, d, sl.h0 * hd, aw, cols);
      if ((rc = place(st, cols.data(), cols.size(), o_->dtype, d, aw, ly.w2, 0, 1, 0))) return bail(rc);
      gather_cols(dn, d, ffg, sl.f0, ff, cols);
      if ((rc = place(st, cols.data(), cols.size(), dn->dtype, d, ff, ly.w2, 0, 1, aw))) return bail(rc);
    }
    std::vector<float> nw, nb;
    if ((rc = decode_vec(T("input_layernorm.weight"), d, nw)) || (rc = decode_vec(T("input_layernorm.bias"), d, nb)) ||
        (rc = upload_floats(m, nw, &ly.n1w)) || (rc = upload_floats(m, nb, &ly.n1b)))
      return bail(rc);
  }
  const tcu_tensor *e = find_tensor(t, n, "model.embed_tokens.weight"), *h = find_tensor(t, n, "lm_head.weight");
  if ((rc = alloc_dmat(m, &m->embed, e->dtype, m->V, d)) || (rc = place(st, e->data, e->nbytes, e->dtype, m->V, d, m->embed, 0, 1, 0)) ||
      (rc = alloc_dmat(m, &m->head, h->dtype, m->V, d)) || (rc = place(st, h->data, h->nbytes, h->dtype, m->V, d, m->head, 0, 1, 0)))
    return bail(rc);
  std::vector<float> fw, fb;
  if ((rc = decode_vec(find_tensor(t, n, "model.norm.weight"), d, fw)) || (rc = decode_vec(find_tensor(t, n, "model.norm.bias"), d, fb)) ||
      (rc = upload_floats(m, fw, &m->fnw)) || (rc = upload_floats(m, fb, &m->fnb)))
    return bail(rc);
  if ((rc = set_tc_shifts(m))) return bail(rc);
  if ((rc = build_mega(m))) return bail(rc);
  *out = m;
  return TCU_OK;
}

// llama2.c checkpoint (model.go:90-166): 7 int32 header fields, then float32
// tensors in the legacy order; the classifier is the embedding table.
static int llama_load(const void* ck, uint64_t nbytes, const tcu_load_options* o, tcu_model** out) {
  if (!ck || !out) return fail(TCU_EINVAL, "null argument");
  if (nbytes < 28) return fail(TCU_EINVAL, "read config header: truncated checkpoint");
  int32_t h[7];
  memcpy(h, ck, 28);
  if (h[0] <= 0 || h[1] <= 0 || h[2] <= 0 || h[3] <= 0 || h[4] <= 0 || h[3] % h[4] != 0 || h[5] < 2 || h[6] <= 0 || h[0] % h[3] != 0 ||
      (h[0] / h[3]) % 2 != 0)
    return fail(TCU_EINVAL, "invalid config header");
  const int64_t dim = h[0], hid = h[1], L = h[2], V = h[5], seq = h[6], hs = dim / h[3], kvd = hs * h[4];
  const int64_t sizes[13] = {V * dim, L * dim, L * dim * dim, L * dim * kvd, L * dim * kvd, L * dim * dim, L * dim,
                             L * hid * dim, L * dim * hid, L * hid * dim, dim, seq * hs / 2, seq * hs / 2};
  int64_t total = 0;
  for (int64_t s : sizes) total += s;
  if ((uint64_t)(28 + total * 4) != nbytes)
    return fail(TCU_EINVAL, "checkpoint has %lld bytes, weight layout needs %lld", (long long)nbytes, (long long)(28 + total * 4));
  const int device = o ? o->device : 0;
  TRY(check_device(device));
  tcu_model* m = new tcu_model();
  init_common(m, o);
  m->arch = ARCH_LLAMA;
  m->V = (int)V;
  m->d = (int)dim;
  m->ff = (int)hid;
  m->L = (int)L;
  m->H = h[3];
  m->KVH = h[4];
  m->hd = (int)hs;
  m->kvw = (int)kvd;
  m->aw = (int)dim;
  m->max_pos = (int)seq;
  auto bail = [&](int code) {
    model_release(m);
    return code;
  };
  // The prefill attention kernel holds up to 128 output dimensions per query.
  if (m->hd < 4 || m->hd > 128 || m->hd % 4) return bail(fail(TCU_EINVAL, "head size %d: a multiple of 4 in 4..128 is supported", m->hd));
  const float* f = (const float*)((const uint8_t*)ck + 28);
  const float* ptr[13];
  {
    const float* p = f;
    for (int i = 0; i < 13; i++) {
      ptr[i] = p;
      p += sizes[i];
    }
  }
  Stager st;
  int rc;
  m->layers.resize(m->L);
  for (int l = 0; l < m->L; l++) {
    Layer& ly = m->layers[l];
    const int64_t dd = dim * dim, dk = dim * kvd, dh = dim * hid;
    if ((rc = alloc_dmat(m, &ly.w1, FMT_F32, (int)(dim + 2 * kvd), (int)dim)) ||
        (rc = place(st, ptr[2] + l * dd, dd * 4, FMT_F32, (int)dim, (int)dim, ly.w1, 0, 1, 0)) ||
        (rc = place(st, ptr[3] + l * dk, dk * 4, FMT_F32, (int)kvd, (int)dim, ly.w1, (int)dim, 1, 0)) ||
        (rc = place(st, ptr[4] + l * dk, dk * 4, FMT_F32, (int)kvd, (int)dim, ly.w1, (int)(dim + kvd), 1, 0)) ||
        (rc = alloc_dmat(m, &ly.w2, FMT_F32, (int)dim, (int)dim)) ||
        (rc = place(st, ptr[5] + l * dd, dd * 4, FMT_F32, (int)dim, (int)dim, ly.w2, 0, 1, 0)) ||
        (rc = alloc_dmat(m, &ly.w3, FMT_F32, (int)(2 * hid), (int)dim)) ||
        (rc = place(st, ptr[7] + l * dh, dh * 4, FMT_F32, (int)hid, (int)dim, ly.w3, 0, 2, 0)) ||
        (rc = place(st, ptr[9] + l * dh, dh * 4, FMT_F32, (int)hid, (int)dim, ly.w3, 1, 2, 0)) ||
        (rc = alloc_dmat(m, &ly.w4, FMT_F32, (int)dim, (int)hid)) ||
        (rc = place(st, ptr[8] + l * dh, dh * 4, FMT_F32, (int)dim, (int)hid, ly.w4, 0, 1, 0)))
      return bail(rc);
    std::vector<float> a(ptr[1] + l * dim, ptr[1] + (l + 1) * dim), b(ptr[6] + l * dim, ptr[6] + (l + 1) * dim);
    if ((rc = upload_floats(m, a, &ly.n1w)) || (rc = upload_floats(m, b, &ly.n2w))) return bail(rc);
  }
  if ((rc = alloc_dmat(m, &m->embed, FMT_F32, (int)V, (int)dim)) ||
      (rc = place(st, ptr[0], V * dim * 4, FMT_F32, (int)V, (int)dim, m->embed, 0, 1, 0)))
    return bail(rc);
  m->head = m->embed;
  std::vector<float> fw(ptr[10], ptr[10] + dim);
  if ((rc = upload_floats(m, fw, &m->fnw))) return bail(rc);
  // Rotary tables from the checkpoint (freq_cis_real/imag [seq][hs/2]).
  std::vector<float2> tab((size_t)seq * (hs / 2));
  for (size_t i = 0; i < tab.size(); i++) tab[i] = make_float2(ptr[11][i], ptr[12][i]);
  void* p = nullptr;
  if ((rc = dalloc(m, &p, tab.size() * sizeof(float2)))) return bail(rc);
  if (cudaMemcpy(p, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess)
    return bail(fail(TCU_ECUDA, "rope table upload failed"));
  m->rope.table = (const float2*)p;
  m->rope.pairs = (int)(hs / 2);
  m->rope.mode = 1;
  if ((rc = set_tc_shifts(m))) return bail(rc);
  *out = m;
  return TCU_OK;
}

// ---------------------------------------------------------------------------
// KV pool

static int pool_get(tcu_model* m, int half, KVPool** out) {
  std::lock_guard<std::mutex> g(m->mu);
  if (m->pools[half]) {
    *out = m->pools[half];
    return TCU_OK;
  }
  KVPool* p = new KVPool();
  p->half = half;
  p->P = m->P;
  p->L = m->L;
  p->kvh = m->KVH;
  p->hd = m->hd;
  const size_t page_bytes = (size_t)m->L * p->page_elems() * p->elem() * 2;  // K + V, all layers
  int64_t budget = m->pool_budget;
  if (budget <= 0) {
    size_t fr = 0, tot = 0;
    cudaMemGetInfo(&fr, &tot);
    budget = (int64_t)(fr / 4);
  }
  int64_t pages = budget / (int64_t)page_bytes;
  // Never fewer pages than one full-context sequence.
  const int64_t min_pages = (m->max_pos + m->P - 1) / m->P + 1;
  pages = std::max<int64_t>(pages, min_pages);
  p->num_pages = (int)std::min<int64_t>(pages, 1 << 24);
  const size_t half_bytes = page_bytes / 2 * (size_t)p->num_pages;
  if (cudaMalloc(&p->k, half_bytes) != cudaSuccess || cudaMalloc(&p->v, half_bytes) != cudaSuccess) {
    if (p->k) cudaFree(p->k);
    delete p;
    cudaGetLastError();
    return fail(TCU_ENOMEM, "KV pool: cannot allocate %d pages (%zu bytes)", (int)pages, 2 * half_bytes);
  }
  // Zeroed on the legacy stream, which does not order with the sessions'
  // non-blocking streams: wait here so no session kernel can race it.
  cudaMemset(p->k, 0, half_bytes);
  cudaMemset(p->v, 0, half_bytes);
  if (cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p->k);
    cudaFree(p->v);
    delete p;
    return fail(TCU_ECUDA, "KV pool initialisation failed: %s", cudaGetErrorString(cudaGetLastError()));
  }
  p->ref.assign(p->num_pages, 0);
  p->free_list.reserve(p->num_pages);
  for (int i = p->num_pages - 1; i >= 0; i--) p->free_list.push_back(i);
  m->pools[half] = p;
  *out = p;
  return TCU_OK;
}

static int page_alloc(tcu_model* m, KVPool* p, int* page) {
  std::lock_guard<std::mutex> g(m->mu);
  if (p->free_list.empty()) return fail(TCU_ENOMEM, "KV pool exhausted (%d pages)", p->num_pages);
  *page = p->free_list.back();
  p->free_list.pop_back();
  p->ref[*page] = 1;
  return TCU_OK;
}
static void page_ref(tcu_model* m, KVPool* p, int page) {
  std::lock_guard<std::mutex> g(m->mu);
  p->ref[page]++;
}
static void page_unref(tcu_model* m, KVPool* p, int page) {
  std::lock_guard<std::mutex> g(m->mu);
  if (--p->ref[page] == 0) p->free_list.push_back(page);
}
static int page_refcount(tcu_model* m, KVPool* p, int page) {
  std::lock_guard<std::mutex> g(m->mu);
  return p->ref[page];
}

// ---------------------------------------------------------------------------
// Workspace for M concurrent sequences (a session: M = 1 decode or a prompt
// chunk of up to CHUNK tokens; branches: M = count).


struct Work {
  int rows = 0, seqs = 0, logits_rows = 0;
  float *x = nullptr, *xn = nullptr, *qkv = nullptr, *ah = nullptr, *logits = nullptr;
  int *tokens = nullptr, *pos = nullptr, *out_tokens = nullptr, *out_count = nullptr;
  unsigned long long* argmax = nullptr;
  float* part = nullptr;
  int* counters = nullptr;
  int* pt = nullptr;
  int pt_stride = 0, max_splits = 0, out_cap = 0;
  int* sl_ids = nullptr;
  float* sl_vals = nullptr;
  double* sl_lse = nullptr;
  int* err = nullptr;  // device error word of bounded waits (TCU_DEV_TIMEOUT)
  unsigned long long* keys = nullptr;  // persistent decode: argmax per step parity
  int* step = nullptr;
  // Persistent decode (decode_mega.cuh): per-layer inputs, published digits
  // of [attention | SwiGLU] and their scales, down-projection sums, work and
  // completion counters.
  float* xl = nullptr;
  float* xdn = nullptr;
  // Branch steps: leading history splits whose pages every row shares.
  int shared_splits = 0;
  uint32_t* adig = nullptr;
  float* asx = nullptr;
  int asx_stride = 0;
  int* grab = nullptr;
  int* done = nullptr;
  // Log-probability rows (k_logprob_rows), LP_ROWS rows at a time: targets,
  // chosen log probabilities, top ids and log probabilities (count <= 256).
  int* lp_targets = nullptr;
  double* lp_chosen = nullptr;
  int* lp_ids = nullptr;
  double* lp_vals = nullptr;
  // Sampling candidates (k_candidates_rows): [seqs][256] ids and scores, and
  // the penalty rows of one call (row offsets, ids, term offsets, terms),
  // grown when a call needs more.
  int* cd_ids = nullptr;
  double* cd_vals = nullptr;
  uint8_t* pen_buf = nullptr;
  size_t pen_cap = 0;
  // Tensor parallelism: this rank's out + down partial sums [rows][d], then
  // their sum over the ranks (in place).
  float* tp_part = nullptr;
  // Tensor-core GEMM workspace (allocated on first use): binary16 split of
  // the activations [2][tc_npad][tc_kmax], their shifts, split-K partials.
  __half* tc_split = nullptr;
  int* tc_sx = nullptr;
  float* tc_part = nullptr;
  int tc_npad = 0, tc_kmax = 0;
  size_t tc_part_floats = 0;
  std::vector<void*> allocs;
  ~Work() {
    for (void* p : allocs) cudaFree(p);
    if (pen_buf) cudaFree(pen_buf);
    if (tc_split) cudaFree(tc_split);
    if (tc_sx) cudaFree(tc_sx);
    if (tc_part) cudaFree(tc_part);
  }
  template <class T>
  int get(T** p, size_t n) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, std::max<size_t>(n * sizeof(T), 16));
    if (e != cudaSuccess) return fail(TCU_ENOMEM, "workspace: %s", cudaGetErrorString(e));
    cudaMemset(q, 0, std::max<size_t>(n * sizeof(T), 16));
    allocs.push_back(q);
    *p = (T*)q;
    return TCU_OK;
  }
};

static int work_init(tcu_model* m, Work* w, int rows, int seqs, int logits_rows, int out_cap) {
  w->rows = rows;
  w->seqs = seqs;
  w->logits_rows = logits_rows;
  w->pt_stride = (m->max_pos + m->P - 1) / m->P;
  // Room for the smallest history split (one page), which the persistent
  // decode step may use; the other kernels use SPLIT_PAGES pages.
  w->max_splits = (m->max_pos + m->P - 1) / m->P;
  w->out_cap = out_cap;
  const int qkvw = m->aw + 2 * m->kvw;
  TRY(w->get(&w->x, (size_t)rows * m->d));
  TRY(w->get(&w->xn, (size_t)rows * m->d));
  TRY(w->get(&w->qkv, (size_t)rows * qkvw));
  TRY(w->get(&w->ah, (size_t)rows * (m->aw + m->ff)));
  TRY(w->get(&w->logits, (size_t)logits_rows * m->V));
  TRY(w->get(&w->tokens, (size_t)std::max(rows, seqs)));
  TRY(w->get(&w->pos, (size_t)seqs));
  TRY(w->get(&w->out_tokens, (size_t)seqs * out_cap));
  TRY(w->get(&w->out_count, (size_t)seqs));
  TRY(w->get(&w->argmax, (size_t)seqs));
  TRY(w->get(&w->part, (size_t)seqs * m->H * w->max_splits * (m->hd + 2)));
  TRY(w->get(&w->counters, (size_t)seqs * m->KVH));
  TRY(w->get(&w->pt, (size_t)seqs * w->pt_stride));
  TRY(w->get(&w->sl_ids, 256));
  TRY(w->get(&w->sl_vals, 256));
  TRY(w->get(&w->sl_lse, 1));
  TRY(w->get(&w->err, 1));
  TRY(w->get(&w->keys, 2));
  TRY(w->get(&w->step, 1));
  TRY(w->get(&w->lp_targets, LP_ROWS));
  TRY(w->get(&w->lp_chosen, LP_ROWS));
  TRY(w->get(&w->lp_ids, (size_t)LP_ROWS * 256));
  TRY(w->get(&w->lp_vals, (size_t)LP_ROWS * 256));
  TRY(w->get(&w->cd_ids, (size_t)seqs * 256));
  TRY(w->get(&w->cd_vals, (size_t)seqs * 256));
  if (m->tp_world > 1) TRY(w->get(&w->tp_part, (size_t)rows * m->d));
  if (m->mega) {
    const size_t nb16 = (size_t)(m->d + m->ff) / 16;
    w->asx_stride = (int)((nb16 + 3) / 4 * 4);
    TRY(w->get(&w->xl, (size_t)(m->L + 1) * m->d));
    TRY(w->get(&w->xdn, (size_t)m->L * m->d));
    TRY(w->get(&w->adig, (size_t)m->L * nb16 * 12));
    TRY(w->get(&w->asx, (size_t)m->L * w->asx_stride));
    TRY(w->get(&w->grab, (size_t)2 * (m->L + 1) * MG_CTL));
    TRY(w->get(&w->done, (size_t)2 * (m->L + 1) * MG_CTL));
  }
  // The zeroing memsets ran on the legacy stream; wait for that stream only
  // (a device-wide synchronisation would stall the other sessions' streams).
  CK(cudaStreamSynchronize(cudaStreamLegacy));
  return TCU_OK;
}

// Workspaces of closed sessions, branch batches and batch runners are kept
// per model and handed to the next handle whose shape they cover, so opening
// and closing handles on a serving path neither allocates device memory nor
// frees it (cudaFree synchronises the whole device and would stall every
// other session). A reused workspace is in the state its last call left,
// the state a live session's next call also starts from.
static int work_take(tcu_model* m, Work** out, int rows, int seqs, int logits_rows, int out_cap) {
  *out = nullptr;
  {
    std::lock_guard<std::mutex> g(m->mu);
    int best = -1;
    for (int i = 0; i < (int)m->work_pool.size(); i++) {
      const Work* w = m->work_pool[i];
      if (w->rows < rows || w->seqs < seqs || w->logits_rows < logits_rows || w->out_cap < out_cap) continue;
      if (best < 0 || (size_t)w->rows * w->seqs < (size_t)m->work_pool[best]->rows * m->work_pool[best]->seqs) best = i;
    }
    if (best >= 0) {
      *out = m->work_pool[best];
      m->work_pool.erase(m->work_pool.begin() + best);
      return TCU_OK;
    }
  }
  Work* w = new Work();
  const int rc = work_init(m, w, rows, seqs, logits_rows, out_cap);
  if (rc != TCU_OK) {
    delete w;
    return rc;
  }
  *out = w;
  return TCU_OK;
}

// Returns a workspace to the model's pool; the caller has synchronised every
// stream that used it.
static void work_give(tcu_model* m, Work* w) {
  if (!w) return;
  w->shared_splits = 0;
  std::lock_guard<std::mutex> g(m->mu);
  m->work_pool.push_back(w);
}

static void work_pool_free(tcu_model* m) {
  for (Work* w : m->work_pool) delete w;
  m->work_pool.clear();
}

// ---------------------------------------------------------------------------
// Opt-in stage timing (the device counterpart of stableProfile,
// stablelm.go:229-250): CUDA events bracket every kernel of a stage; totals
// are accumulated after the stream is synchronised. With profiling off no
// event is recorded.

enum Stage { ST_EMBED = 0, ST_W1, ST_ATTN, ST_W2, ST_HEAD, ST_PF_GEMM, ST_PF_ATTN, ST_OTHER, ST_MEGA, ST_COMM, ST_COUNT };

struct Prof {
  bool on = false;
  std::vector<cudaEvent_t> ev;  // pairs
  std::vector<int> stage;
  size_t used = 0;
  int64_t launches[ST_COUNT] = {};
  double ms[ST_COUNT] = {};
  ~Prof() {
    for (cudaEvent_t e : ev) cudaEventDestroy(e);
  }
  void begin(int st, cudaStream_t s) {
    if (!on) return;
    if (2 * used + 2 > ev.size()) {
      cudaEvent_t a, b;
      cudaEventCreate(&a);
      cudaEventCreate(&b);
      ev.push_back(a);
      ev.push_back(b);
      stage.push_back(0);
    }
    stage[used] = st;
    record(ev[2 * used], s);
  }
  void end(cudaStream_t s) {
    if (!on) return;
    record(ev[2 * used + 1], s);
    used++;
  }
  // Under stream capture a plain cudaEventRecord only expresses a dependency;
  // cudaEventRecordExternal makes it an event-record node of the graph.
  static void record(cudaEvent_t e, cudaStream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &st);
    if (st == cudaStreamCaptureStatusActive)
      cudaEventRecordWithFlags(e, s, cudaEventRecordExternal);
    else
      cudaEventRecord(e, s);
  }
  // Call after the stream is synchronised.
  void collect(size_t n) {
    for (size_t i = 0; i < n; i++) {
      float t = 0;
      if (cudaEventElapsedTime(&t, ev[2 * i], ev[2 * i + 1]) == cudaSuccess) {
        ms[stage[i]] += t;
        launches[stage[i]]++;
      } else {
        cudaGetLastError();  // an unreadable pair is skipped, not reported by the next call
      }
    }
  }
};

static thread_local Prof* g_prof = nullptr;  // set while enqueueing for a profiled session
#define PROF_BEGIN(st, s) \
  if (g_prof) g_prof->begin(st, s)
#define PROF_END(s) \
  if (g_prof) g_prof->end(s)

// ---------------------------------------------------------------------------
// Kernel launch helpers

template <int FMT, int PRO, int EPI>
static void launch_gemv_fmt(const tcu_model* m, const GemvArgs& a, cudaStream_t s) {
  const int K = a.W.cols;
  const size_t smem = (size_t)a.M * K * sizeof(float);
  const int pairs = (a.W.rows + 1) / 2;
  int blocks = (pairs + GEMV_WARPS - 1) / GEMV_WARPS;
  blocks = std::min(blocks, m->sm_count * 2);
  switch (a.M) {
#define TCU_GEMV_CASE(MM)                                                                   \
  case MM: {                                                                                \
    auto kern = k_gemv<FMT, MM, PRO, EPI>;                                                  \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);     \
    NOTE("cudaFuncSetAttribute(k_gemv)");                                                   \
    kern<<<blocks, GEMV_THREADS, smem, s>>>(a);                                             \
    NOTE("k_gemv");                                                                         \
    break;                                                                                  \
  }
    TCU_GEMV_CASE(1)
    TCU_GEMV_CASE(2)
    TCU_GEMV_CASE(3)
    TCU_GEMV_CASE(4)
#undef TCU_GEMV_CASE
  }
}

// Launch with programmatic stream serialization: the kernel may start while
// the previous one drains and synchronises with griddepcontrol.wait.
template <typename Kern, typename Args>
static void launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, const Args& args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, args);
}

static const size_t GS_SMEM_LIMIT = 227 * 1024;

// Plans the streaming GEMV for W (M == 1): K chunks of at most GS_CHUNK
// values (for EPI_RESID2 the first chunk ends exactly at k_split), rows per
// stage and pipeline depth. Returns false when the shape does not fit.
static bool plan_gemv_stream(const DMat& W, int epi, int k_split, GemvStreamArgs* sa, int* ks_out) {
  int E;
  size_t esz;
  switch (W.fmt) {
    case FMT_Q8_0: E = 16; esz = 1; break;
    case FMT_BF16: case FMT_F16: E = 8; esz = 2; break;
    case FMT_F32: E = 4; esz = 4; break;
    default: return false;
  }
  const int K = W.cols;
  if (K % E || (W.fmt == FMT_Q8_0 && K % 32)) return false;
  int ks;
  if (epi == EPI_RESID2) {
    if (k_split <= 0 || k_split >= K || k_split % E || k_split > GS_CHUNK) return false;
    const int rest = K - k_split;
    int n = (rest + GS_CHUNK - 1) / GS_CHUNK;
    ks = n + 1 <= 2 ? 2 : 4;
    if (ks - 1 < n) return false;
    sa->kc[0] = 0;
    sa->kc[1] = k_split;
    const int nv = rest / E;
    for (int c = 1; c < ks; c++) sa->kc[c + 1] = k_split + (int)((long long)nv * c / (ks - 1)) * E;
    sa->lo_chunks = 1;
  } else {
    const int nv = K / E;
    ks = K <= GS_CHUNK ? 1 : (K <= 2 * GS_CHUNK ? 2 : 4);
    if (ks == 4 && K > 4 * GS_CHUNK) return false;
    for (int c = 0; c <= ks; c++) sa->kc[c] = (int)((long long)nv * c / ks) * E;
    sa->lo_chunks = ks;
    if (ks > 1 && epi != EPI_STORE && epi != EPI_RESID1) return false;  // GLU / head need whole rows per warp
  }
  for (int c = 0; c < ks; c++)
    if (sa->kc[c + 1] - sa->kc[c] > GS_CHUNK) return false;
  const int rs = 2 * (GS_CONSUMERS / ks);
  const size_t row_bytes = (size_t)K * esz;
  const size_t sbytes = W.fmt == FMT_Q8_0 ? (size_t)W.sstride * 2 : 0;
  const uint32_t stage = (uint32_t)(((size_t)rs * (row_bytes + sbytes) + 127) / 128 * 128);
  const uint32_t off_x = 128;
  const uint32_t off_part = off_x + (uint32_t)(((size_t)K * 4 + 127) / 128 * 128);
  const uint32_t off_stage = off_part + (uint32_t)(((size_t)GS_MAX_STAGES * rs * ks * 4 + 127) / 128 * 128);
  if (off_stage + 2 * (size_t)stage > GS_SMEM_LIMIT) return false;
  const int nstage = (int)std::min<size_t>(GS_MAX_STAGES, (GS_SMEM_LIMIT - off_stage) / stage);
  sa->rs = rs;
  sa->nstage = nstage;
  sa->stage_bytes = stage;
  sa->off_x = off_x;
  sa->off_part = off_part;
  sa->off_stage = off_stage;
  *ks_out = ks;
  return true;
}

template <int FMT, int PRO, int EPI, int KS>
static void launch_gemv_stream_k(const tcu_model* m, const GemvStreamArgs& sa, cudaStream_t s) {
  auto kern = k_gemv_stream<FMT, PRO, EPI, KS>;
  const size_t smem = sa.off_stage + (size_t)sa.nstage * sa.stage_bytes;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  NOTE("cudaFuncSetAttribute(k_gemv_stream)");
  const int pairs = (sa.g.W.rows + 1) / 2;
  const int grid = std::max(1, std::min(m->sm_count, pairs));
  launch_pdl(kern, dim3(grid), dim3(GS_THREADS), smem, s, sa);
  NOTE("k_gemv_stream");
}

template <int FMT, int PRO, int EPI>
static void launch_gemv_stream_fmt(const tcu_model* m, const GemvStreamArgs& sa, int ks, cudaStream_t s) {
  if constexpr (EPI == EPI_GLU || EPI == EPI_HEAD) {
    launch_gemv_stream_k<FMT, PRO, EPI, 1>(m, sa, s);
  } else {
    if (ks == 1)
      launch_gemv_stream_k<FMT, PRO, EPI, 1>(m, sa, s);
    else if (ks == 2)
      launch_gemv_stream_k<FMT, PRO, EPI, 2>(m, sa, s);
    else
      launch_gemv_stream_k<FMT, PRO, EPI, 4>(m, sa, s);
  }
}

// Returns true if the streaming kernel took the launch.
template <int PRO, int EPI>
static bool try_gemv_stream(const tcu_model* m, const GemvArgs& a, int* err, cudaStream_t s) {
  if (a.M != 1 || m->disable_stream) return false;
  if (EPI == EPI_RESID2 && m->arch != ARCH_STABLELM) return false;
  GemvStreamArgs sa{};
  sa.g = a;
  sa.err = err;
  int ks = 1;
  if (!plan_gemv_stream(a.W, EPI, a.k_split, &sa, &ks)) return false;
  if ((EPI == EPI_GLU || EPI == EPI_HEAD) && ks != 1) return false;
  switch (a.W.fmt) {
    case FMT_Q8_0: launch_gemv_stream_fmt<FMT_Q8_0, PRO, EPI>(m, sa, ks, s); return true;
    case FMT_BF16: launch_gemv_stream_fmt<FMT_BF16, PRO, EPI>(m, sa, ks, s); return true;
    case FMT_F16: launch_gemv_stream_fmt<FMT_F16, PRO, EPI>(m, sa, ks, s); return true;
    case FMT_F32: launch_gemv_stream_fmt<FMT_F32, PRO, EPI>(m, sa, ks, s); return true;
  }
  return false;
}

template <int PRO, int EPI>
static void launch_gemv_generic(const tcu_model* m, const GemvArgs& a, cudaStream_t s) {
  const int K = a.W.cols;
  const size_t smem = (size_t)a.M * K * sizeof(float);
  const int pairs = (a.W.rows + 1) / 2;
  int blocks = std::min((pairs + GEMV_WARPS - 1) / GEMV_WARPS, m->sm_count * 2);
  switch (a.M) {
#define TCU_GEMV_CASE(MM)                                                               \
  case MM: {                                                                            \
    auto kern = k_gemv_generic<MM, PRO, EPI>;                                           \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    kern<<<blocks, GEMV_THREADS, smem, s>>>(a);                                         \
    NOTE("k_gemv_generic");                                                             \
    break;                                                                              \
  }
    TCU_GEMV_CASE(1)
    TCU_GEMV_CASE(2)
    TCU_GEMV_CASE(3)
    TCU_GEMV_CASE(4)
#undef TCU_GEMV_CASE
  }
}

static bool gemv_vector_ok(const DMat& W) {
  switch (W.fmt) {
    case FMT_Q8_0:
      return W.cols % 32 == 0;
    case FMT_BF16:
    case FMT_F16:
      return W.cols % 8 == 0;
    case FMT_F32:
      return W.cols % 4 == 0;
    default:
      return false;
  }
}

static thread_local int g_stage = ST_OTHER;  // stage charged by the next launch helper

template <int PRO, int EPI>
static void launch_gemv_impl(const tcu_model* m, const GemvArgs& a, cudaStream_t s);

static thread_local int* g_err_word = nullptr;  // device error word of the enqueueing call

template <int PRO, int EPI>
static void launch_gemv(const tcu_model* m, const GemvArgs& a, cudaStream_t s) {
  PROF_BEGIN(g_stage, s);
  if (!try_gemv_stream<PRO, EPI>(m, a, g_err_word, s)) launch_gemv_impl<PRO, EPI>(m, a, s);
  PROF_END(s);
}

template <int PRO, int EPI>
static void launch_gemv_impl(const tcu_model* m, const GemvArgs& a, cudaStream_t s) {
  if (gemv_vector_ok(a.W)) {
    switch (a.W.fmt) {
      case FMT_Q8_0:
        return launch_gemv_fmt<FMT_Q8_0, PRO, EPI>(m, a, s);
      case FMT_BF16:
        return launch_gemv_fmt<FMT_BF16, PRO, EPI>(m, a, s);
      case FMT_F16:
        return launch_gemv_fmt<FMT_F16, PRO, EPI>(m, a, s);
      case FMT_F32:
        return launch_gemv_fmt<FMT_F32, PRO, EPI>(m, a, s);
    }
  }
  launch_gemv_generic<PRO, EPI>(m, a, s);
}

// ---------------------------------------------------------------------------
// Tensor-core GEMM (gemm_tc.cuh)

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library); nullptr if unavailable.
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    cudaGetLastError();
  });
  return g_encode;
}

// Power of two for the tensor-core split of a Q8_0 matrix: the largest
// |s * q| (q <= 128) scaled below 2^13.
// Power of two of a matrix's tensor-core split (Q8_0, Q6_K, Q5_K; others 0),
// from a bound on |value| reduced into *scratch (one device word).
static int tc_shift_of(DMat* W, unsigned* scratch, int sm_count) {
  const bool kq = (W->fmt == FMT_Q6_K || W->fmt == FMT_Q5_K) && W->cols % 256 == 0;
  if (W->fmt != FMT_Q8_0 && !kq) return TCU_OK;
  CK(cudaMemset(scratch, 0, sizeof(unsigned)));
  if (kq)
    k_kquant_absmax<<<sm_count * 4, 256>>>(W->w, (size_t)W->rows * (W->cols / 256), W->fmt, scratch);
  else
    k_scale_absmax<<<sm_count * 4, 256>>>(W->s, W->rows, W->sstride, W->cols / 32, scratch);
  CK(cudaGetLastError());
  unsigned bits = 0;
  CK(cudaMemcpy(&bits, scratch, sizeof(unsigned), cudaMemcpyDeviceToHost));
  float mx;
  memcpy(&mx, &bits, sizeof(mx));
  if (kq) mx /= 128.f;  // the bound below is for |scale| * 128
  int e = 0;
  if (mx > 0.f) frexpf(mx * 128.f, &e);
  W->tc_sw = mx > 0.f ? std::max(-100, std::min(100, 13 - e)) : 0;
  return TCU_OK;
}

static int set_tc_shift(tcu_model* m, DMat* W) {
  const bool kq = (W->fmt == FMT_Q6_K || W->fmt == FMT_Q5_K) && W->cols % 256 == 0;
  if (W->fmt != FMT_Q8_0 && !kq) return TCU_OK;
  if (!m->scratch_u32) TRY(dalloc(m, (void**)&m->scratch_u32, sizeof(unsigned)));
  return tc_shift_of(W, m->scratch_u32, m->sm_count);
}

static int set_tc_shifts(tcu_model* m) {
  for (Layer& ly : m->layers) {
    TRY(set_tc_shift(m, &ly.w1));
    TRY(set_tc_shift(m, &ly.w2));
    TRY(set_tc_shift(m, &ly.w3));
    TRY(set_tc_shift(m, &ly.w4));
  }
  TRY(set_tc_shift(m, &m->head));
  return TCU_OK;
}

static int work_reserve(void** p, size_t bytes) {
  if (cudaMalloc(p, bytes) != cudaSuccess) {
    cudaGetLastError();
    *p = nullptr;
    return TCU_ENOMEM;
  }
  cudaMemset(*p, 0, bytes);
  return TCU_OK;
}

// Enqueues a Q8_0 or BF16 product on the tensor cores; false if this shape
// or format takes the CUDA-core path.
template <int EPI>
static bool launch_gemm_tc(const tcu_model* m, Work* w, const GemmArgs& g, cudaStream_t s) {
  const DMat& W = g.W;
  const int K = W.cols, R = W.rows, n = g.n;
  const bool wb = W.fmt == FMT_BF16;
  const bool kq = W.fmt == FMT_Q6_K || W.fmt == FMT_Q5_K;
  if (!m->use_tc || !w || !(W.fmt == FMT_Q8_0 || wb || kq) || K % 16 || n < 1 || R < 1) return false;
  if (kq && (K % 256 || (EPI == EPI_RESID2 && g.k_split % 256))) return false;
  if (wb && ((uintptr_t)W.w % 16)) return false;
  if (EPI == EPI_RESID2 && g.k_split % TC_BK) return false;
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const int pieces = wb ? 3 : 2;  // activation split: bfloat16 x3 or binary16 x2
  const int n_tile = std::min(wb ? 128 : TC_MAXN, (n + 15) / 16 * 16);
  const int n_pad = (n + n_tile - 1) / n_tile * n_tile;
  const int row_tiles = (R + TC_BM - 1) / TC_BM;
  // Too few tiles to fill the GPU: split K into slices (out/down rows only).
  int z = 1, k_per_z = K, z_lo = 0;
  if (EPI == EPI_RESID2 && row_tiles * (n_pad / n_tile) < m->sm_count / 2) {
    k_per_z = TC_BK;
    for (int c = 20; c >= 1; c--)
      if (g.k_split % (c * TC_BK) == 0) {
        k_per_z = c * TC_BK;
        break;
      }
    z_lo = g.k_split / k_per_z;
    z = z_lo + (K - g.k_split + k_per_z - 1) / k_per_z;
  }
  // GLU and STORE products whose last wave is ragged (a 64-row branch batch's
  // W1: 168 tiles on 148 SMs) split K into z slices when the model
  // waves(z) * (stages per slice + 3) drops by 15 % or more. Slices are summed
  // in order by k_splitk_epi, which then runs the epilogue.
  if ((EPI == EPI_GLU || EPI == EPI_STORE) && n >= 16) {
    const int tiles = row_tiles * (n_pad / n_tile), sms = m->sm_count, iters = (K + TC_BK - 1) / TC_BK;
    auto cost = [&](int zz) { return (double)((tiles * zz + sms - 1) / sms) * ((iters + zz - 1) / zz + 3); };
    int best = 1;
    for (int zz = 2; zz <= 8; zz++)
      if (iters / zz >= 4 && cost(zz) < cost(best)) best = zz;
    if (best > 1 && cost(best) <= 0.85 * cost(1)) {
      k_per_z = (iters + best - 1) / best * TC_BK;
      z = (K + k_per_z - 1) / k_per_z;
    }
  }
  // Workspace: grows on first use (not during stream capture).
  if (n_pad > w->tc_npad || K > w->tc_kmax) {
    const int np = std::max(n_pad, w->tc_npad), kk = std::max(K, w->tc_kmax);
    if (w->tc_split) cudaFree(w->tc_split);
    if (w->tc_sx) cudaFree(w->tc_sx);
    w->tc_split = nullptr;
    w->tc_sx = nullptr;
    w->tc_npad = w->tc_kmax = 0;
    if (work_reserve((void**)&w->tc_split, (size_t)3 * np * kk * 2) || work_reserve((void**)&w->tc_sx, (size_t)np * 4)) return false;
    w->tc_npad = np;
    w->tc_kmax = kk;
  }
  if (z > 1 && (size_t)z * n * R > w->tc_part_floats) {
    if (w->tc_part) cudaFree(w->tc_part);
    w->tc_part = nullptr;
    w->tc_part_floats = 0;
    if (work_reserve((void**)&w->tc_part, (size_t)z * n * R * 4)) return false;
    w->tc_part_floats = (size_t)z * n * R;
  }
  const CUtensorMapDataType dt = wb ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap map, wmap;
  {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)(pieces * n_pad)};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)n_tile};
    cuuint32_t estr[2] = {1, 1};
    if (encode(&map, dt, 2, w->tc_split, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  wmap = map;
  if (wb) {
    // bfloat16 weights [R][K], tiles of 128 rows x 64 columns.
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)R};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)TC_BM};
    cuuint32_t estr[2] = {1, 1};
    if (encode(&wmap, dt, 2, const_cast<uint8_t*>(W.w), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  const int wm = wb ? TCW_BF16 : kq ? TCW_KQ : TCW_Q8;
  // Deep rings for BF16 and Q8_0 tiles of up to 128 tokens: activation and
  // weight stages are added in turn (up to TC_MAX_STAGES each) while they
  // fit. K-quant tiles and 256-token tiles keep two stages per ring.
  const bool deep = n_tile <= 128 && !kq;
  int ws = wb ? 0 : 2, xs = 2;
  if (deep)
    for (bool grew = true; grew;) {
      grew = false;
      if (xs < TC_MAX_STAGES && tc_smem_bytes(wm, n_tile, ws, xs + 1) <= TC_SMEM_LIMIT) {
        xs++;
        grew = true;
      }
      if (!wb && ws < TC_MAX_STAGES && tc_smem_bytes(wm, n_tile, ws + 1, xs) <= TC_SMEM_LIMIT) {
        ws++;
        grew = true;
      }
    }
  auto kern = wm == TCW_BF16 ? k_gemm_tc<EPI, TCW_BF16, true>
              : wm == TCW_KQ ? k_gemm_tc<EPI, TCW_KQ, false>
              : deep         ? k_gemm_tc<EPI, TCW_Q8, true>
                             : k_gemm_tc<EPI, TCW_Q8, false>;
  const int tc_smem = tc_smem_bytes(wm, n_tile, ws, xs);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  PROF_BEGIN(g_stage, s);
  if (wb) {
    k_split_bf16<<<n, 256, 0, s>>>(g.A, g.lda, n, K, n_pad, reinterpret_cast<__nv_bfloat16*>(w->tc_split), w->tc_sx);
    NOTE("k_split_bf16");
  } else {
    // One CTA per token row; 1024 threads keep a 64-row branch batch's split
    // from being bound by the latency of one CTA's two passes over its row.
    k_split_f16<<<n, 1024, 0, s>>>(g.A, g.lda, n, K, n_pad, w->tc_split, w->tc_sx);
    NOTE("k_split_f16");
  }
  TcArgs a{};
  a.W = W;
  a.n = n;
  a.n_tile = n_tile;
  a.n_pad = n_pad;
  a.sx = w->tc_sx;
  a.sw = wb ? 0 : W.tc_sw;
  a.out = g.out;
  a.out_stride = g.out_stride;
  a.n_plain = g.n_plain;
  a.glu_out = g.glu_out;
  a.glu_stride = g.glu_stride;
  a.glu_act = g.glu_act;
  a.resid = g.resid;
  a.resid_stride = g.resid_stride;
  a.k_split = g.k_split;
  a.part = z > 1 ? w->tc_part : nullptr;
  a.k_per_z = k_per_z;
  a.err = w->err;
  // BF16 and K-quant weights: the token tiles of a weight tile run together
  // (their weight reads hit L2). Q8_0 is bound by its dequantising warps and
  // measured faster with row tiles first.
  a.tok_fast = (wb || kq) ? 1 : 0;
  a.ws = ws;
  a.xs = xs;
  const dim3 grid = a.tok_fast ? dim3(n_pad / n_tile, row_tiles, z) : dim3(row_tiles, n_pad / n_tile, z);
  kern<<<grid, TC_THREADS, tc_smem, s>>>(map, wmap, a);
  NOTE("k_gemm_tc");
  if (z > 1) {
    if constexpr (EPI == EPI_RESID2) {
      k_splitk_resid<<<m->sm_count * 4, 256, 0, s>>>(w->tc_part, z_lo, z, n, R, g.resid, g.resid_stride);
      NOTE("k_splitk_resid");
    } else {
      k_splitk_epi<EPI><<<m->sm_count * 4, 256, 0, s>>>(w->tc_part, z, n, R, g.out, g.out_stride, g.n_plain, g.glu_out,
                                                         g.glu_stride, g.glu_act);
      NOTE("k_splitk_epi");
    }
  }
  PROF_END(s);
  return true;
}

template <int EPI>
static void launch_gemm(const tcu_model* m, Work* w, const GemmArgs& a, cudaStream_t s) {
  if (launch_gemm_tc<EPI>(m, w, a, s)) return;
  PROF_BEGIN(g_stage, s);
  dim3 grid((a.W.rows + SG_BN - 1) / SG_BN, (a.n + SG_BM - 1) / SG_BM);
  GemmArgs g = a;
  g.part = nullptr;
  g.k_per_z = a.W.cols;
  int z = 1, z_lo = 0;
  // Too few output tiles to fill the GPU (out/down rows of a branch batch):
  // split K into 256-column slices, reduced with the residual in slice order.
  if (EPI == EPI_RESID2 && w && (int)(grid.x * grid.y) < m->sm_count / 2 && a.k_split % 256 == 0) {
    const int kz = 256, K = a.W.cols;
    const int zz = a.k_split / kz + (K - a.k_split + kz - 1) / kz;
    if ((size_t)zz * a.n * a.W.rows > w->tc_part_floats) {
      if (w->tc_part) cudaFree(w->tc_part);
      w->tc_part = nullptr;
      w->tc_part_floats = 0;
      if (work_reserve((void**)&w->tc_part, (size_t)zz * a.n * a.W.rows * 4) == TCU_OK) w->tc_part_floats = (size_t)zz * a.n * a.W.rows;
    }
    if (w->tc_part) {
      z = zz;
      z_lo = a.k_split / kz;
      g.part = w->tc_part;
      g.k_per_z = kz;
      grid.z = z;
    }
  }
  k_gemm_simt<EPI><<<grid, SG_THREADS, 0, s>>>(g);
  NOTE("k_gemm_simt");
  if (z > 1) {
    k_splitk_resid<<<m->sm_count * 4, 256, 0, s>>>(w->tc_part, z_lo, z, a.n, a.W.rows, a.resid, a.resid_stride);
    NOTE("k_splitk_resid");
  }
  PROF_END(s);
}

static void launch_norm_rows(const tcu_model* m, const float* in, float* out, int n, const float* w, const float* b, cudaStream_t s) {
  PROF_BEGIN(ST_OTHER, s);
  NormRowsArgs a{n, m->d, in, m->d, out, m->d, w, b, m->eps, m->arch == ARCH_LLAMA};
  k_norm_rows<<<n, 1024, 0, s>>>(a);  // one CTA per row: 1024 threads hide a short batch's load latency
  NOTE("k_norm_rows");
  PROF_END(s);
}

static size_t attn_decode_smem(const tcu_model* m) {
  const int G = m->H / m->KVH, split = SPLIT_PAGES * m->P, hd = m->hd;
  return sizeof(float) * ((size_t)G * hd + 2 * (size_t)split * (hd + 1) + (size_t)G * split + 2 * hd);
}

static void launch_attn_decode(const tcu_model* m, KVPool* pool, Work* w, int M, int layer, int grid_splits, cudaStream_t s) {
  PROF_BEGIN(ST_ATTN, s);
  DecodeAttnArgs a;
  a.M = M;
  a.H = m->H;
  a.KVH = m->KVH;
  a.hd = m->hd;
  a.rope = m->rope;
  a.qkv = w->qkv;
  a.qkv_stride = m->aw + 2 * m->kvw;
  a.kv = pool->view();
  a.layer = layer;
  a.page_table = w->pt;
  a.pt_stride = w->pt_stride;
  a.pos = w->pos;
  a.split = SPLIT_PAGES * m->P;
  a.max_splits = w->max_splits;
  a.part = w->part;
  a.counters = w->counters;
  a.out = w->ah;
  a.out_stride = m->aw + m->ff;
  a.scale = (float)sqrt((double)m->hd);
  a.s_begin = 0;
  a.s_runs = 0;
  a.per = 1;
  const int es = pool->half ? 2 : 4;
  const int G = m->H / m->KVH;
  // Splits every row shares (branches): keys and values read once for all
  // rows; the per-row kernels start after them.
  const int hd16 = m->hd % 16 == 0 ? m->hd / 16 : 0;
  const bool tc_hd = hd16 == 4 || hd16 == 5 || hd16 == 6 || hd16 == 8;
  if (w->shared_splits > 0 && a.split == AT_KEYS && w->shared_splits < grid_splits && pool->half && m->use_tc_attn && tc_hd &&
      at_smem_bytes(m->hd, 1) <= (size_t)m->gemv_smem_optin) {
    // Tensor cores: one merged partial per run of splits, about two CTAs per SM.
    const int qt = (M * G + AT_ROWS - 1) / AT_ROWS;
    const int want = std::max(1, 2 * m->sm_count / (m->KVH * qt));
    const int per = (w->shared_splits + want - 1) / want;
    const int runs = (w->shared_splits + per - 1) / per;
    const size_t smem = at_smem_bytes(m->hd, 1);
    auto kern = hd16 == 4 ? k_attn_shared_tc<64> : hd16 == 5 ? k_attn_shared_tc<80> : hd16 == 6 ? k_attn_shared_tc<96> : k_attn_shared_tc<128>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    NOTE("cudaFuncSetAttribute(k_attn_shared_tc)");
    kern<<<dim3(runs, m->KVH, qt), AT_GROUP, smem, s>>>(a, w->shared_splits, per, w->err);
    NOTE("k_attn_shared_tc");
    a.s_begin = w->shared_splits;
    a.s_runs = runs;
  } else if (w->shared_splits > 0 && a.split == PA_KT && w->shared_splits < grid_splits) {
    const int nc = (m->hd + 15) / 16;
    auto kern = nc <= 2 ? k_attn_shared<2> : nc <= 4 ? k_attn_shared<4> : nc <= 5 ? k_attn_shared<5> : k_attn_shared<8>;
    const size_t smem = pa_shared_smem_bytes(m->hd);
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    NOTE("cudaFuncSetAttribute(k_attn_shared)");
    kern<<<dim3(w->shared_splits, m->KVH, (M * G + PA_QT - 1) / PA_QT), PA_THREADS, smem, s>>>(a);
    NOTE("k_attn_shared");
    a.s_begin = w->shared_splits;
  }
  const size_t bulk_smem = attn_bulk_smem(G, a.split, m->hd, es);
  if (!m->disable_stream && ((size_t)m->P * m->hd * es) % 16 == 0 && bulk_smem <= GS_SMEM_LIMIT && G <= 32) {
    // Long histories (16+ splits past the shared ones): runs of splits per
    // CTA, about five CTAs per SM, so the merge reads a partial per run.
    const int rest = grid_splits - a.s_begin;
    const int want = std::max(1, 5 * m->sm_count / (M * m->KVH));
    a.per = rest >= 16 && rest > want ? std::min(8, (rest + want - 1) / want) : 1;
    DecodeAttn2Extra x{w->err};
    cudaFuncSetAttribute(k_attn_decode_bulk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bulk_smem);
    NOTE("cudaFuncSetAttribute(k_attn_decode_bulk)");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rest + a.per - 1) / a.per, m->KVH, M);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = bulk_smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, k_attn_decode_bulk, a, x);
    NOTE("k_attn_decode_bulk");
  } else {
    const size_t smem = attn_decode_smem(m);
    cudaFuncSetAttribute(k_attn_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    NOTE("cudaFuncSetAttribute(k_attn_decode)");
    k_attn_decode<<<dim3(grid_splits - a.s_begin, m->KVH, M), 128, smem, s>>>(a);
    NOTE("k_attn_decode");
  }
  PROF_END(s);
}

// First failure of a collective on this thread (the enqueue paths report it
// after they return).
static thread_local std::string g_comm_err;

// The per-layer exchange of a tensor-parallel model: the ranks' out + down
// partial sums of n rows (w->tp_part) are summed in place by NCCL over
// NVLink, then added to the residual rows x (fp32, k_add_rows).
static void tp_reduce_add(const tcu_model* m, Work* w, int n, cudaStream_t s) {
  const size_t count = (size_t)n * m->d;
  if (m->tp_ex_on && (long long)count <= std::min<long long>(m->tp_ex_count, (long long)TPX_PEER_ROWS * m->d)) {
    // Decode-sized exchanges over peer memory: one kernel exchanges, sums
    // and adds to the residual (prefill chunks keep NCCL, faster at MBs).
    TpxArgs a{};
    a.x = w->x;
    a.part = w->tp_part;
    a.count = (long long)count;
    a.max_count = m->tp_ex_count;
    // The chunking depends on the count only, so every rank pairs CTA c with
    // the other ranks' CTA c; at most 128 CTAs, all resident at once.
    const int ctas = (int)std::min<long long>(128, (count + 1023) / 1024);
    a.chunk = (int)(((count + ctas - 1) / ctas + 3) / 4 * 4);
    a.world = m->tp_world;
    a.rank = m->tp_rank;
    a.seq = m->tp_seq;
    for (int p = 0; p < m->tp_world; p++) a.ex[p] = m->tp_peer[p];
    a.err = w->err;
    PROF_BEGIN(ST_COMM, s);
    k_tp_exchange_add<<<(int)((count + a.chunk - 1) / a.chunk), TPX_THREADS, 0, s>>>(a);
    NOTE("k_tp_exchange_add");
    PROF_END(s);
    return;
  }
  PROF_BEGIN(ST_COMM, s);
  const ncclResult_t r = nccl_api()->all_reduce(w->tp_part, w->tp_part, count, ncclFloat32, ncclSum, m->tp_comm, s);
  PROF_END(s);
  if (r != ncclSuccess && g_comm_err.empty()) g_comm_err = std::string("ncclAllReduce: ") + nccl_api()->error_string(r);
  PROF_BEGIN(ST_OTHER, s);
  k_add_rows<<<(int)std::min<size_t>((count + 255) / 256, (size_t)m->sm_count * 4), 256, 0, s>>>(w->x, w->tp_part, count);
  NOTE("k_add_rows");
  PROF_END(s);
}

// Reports (once) a collective that failed while work was being enqueued.
static int comm_check() {
  if (g_comm_err.empty()) return TCU_OK;
  std::string e = g_comm_err;
  g_comm_err.clear();
  return fail(TCU_ECUDA, "%s", e.c_str());
}

// One decode step for M sequences whose tokens are in w->tokens (token mode)
// or in w->argmax (step mode) and whose new positions are w->pos (token
// mode) / w->pos + 1 (step mode). Ends with the head: logits rows and argmax.
static void enqueue_decode(const tcu_model* m, KVPool* pool, Work* w, int M, bool step_mode, int grid_splits, bool write_logits,
                           cudaStream_t s) {
  const int d = m->d, ff = m->ff, aw = m->aw, qkvw = aw + 2 * m->kvw;
  EmbedArgs ea{};
  ea.E = m->embed;
  ea.n = M;
  ea.tokens = step_mode ? nullptr : w->tokens;
  ea.argmax = w->argmax;
  ea.pos = w->pos;
  ea.out_tokens = w->out_tokens;
  ea.out_stride = w->out_cap;
  ea.out_count = w->out_count;
  ea.x = w->x;
  ea.x_stride = d;
  PROF_BEGIN(ST_EMBED, s);
  k_embed<<<M, 256, 0, s>>>(ea);
  NOTE("k_embed");
  PROF_END(s);
  const bool gemv = M <= GEMV_MAX_M;
  for (int l = 0; l < m->L; l++) {
    const Layer& ly = m->layers[l];
    if (m->arch == ARCH_STABLELM) {
      g_stage = ST_W1;
      if (gemv) {
        GemvArgs a{};
        a.W = ly.w1;
        a.M = M;
        a.in = w->x;
        a.in_stride = d;
        a.nw = ly.n1w;
        a.nb = ly.n1b;
        a.eps = m->eps;
        a.out = w->qkv;
        a.out_stride = qkvw;
        a.n_plain = qkvw;
        a.glu_out = w->ah + aw;
        a.glu_stride = aw + ff;
        a.glu_act = 0;
        launch_gemv<PRO_LN, EPI_GLU>(m, a, s);
      } else {
        launch_norm_rows(m, w->x, w->xn, M, ly.n1w, ly.n1b, s);
        GemmArgs g{};
        g.W = ly.w1;
        g.n = M;
        g.A = w->xn;
        g.lda = d;
        g.out = w->qkv;
        g.out_stride = qkvw;
        g.n_plain = qkvw;
        g.glu_out = w->ah + aw;
        g.glu_stride = aw + ff;
        g.glu_act = 0;
        launch_gemm<EPI_GLU>(m, w, g, s);
      }
      launch_attn_decode(m, pool, w, M, l, grid_splits, s);
      g_stage = ST_W2;
      if (m->tp_world > 1) {
        // This rank's out + down partial of every row, summed over the ranks.
        if (gemv) {
          GemvArgs a{};
          a.W = ly.w2;
          a.M = M;
          a.in = w->ah;
          a.in_stride = aw + ff;
          a.out = w->tp_part;
          a.out_stride = d;
          launch_gemv<PRO_COPY, EPI_STORE>(m, a, s);
        } else {
          GemmArgs g{};
          g.W = ly.w2;
          g.n = M;
          g.A = w->ah;
          g.lda = aw + ff;
          g.out = w->tp_part;
          g.out_stride = d;
          launch_gemm<EPI_STORE>(m, w, g, s);
        }
        tp_reduce_add(m, w, M, s);
      } else if (gemv) {
        GemvArgs a{};
        a.W = ly.w2;
        a.M = M;
        a.in = w->ah;
        a.in_stride = aw + ff;
        a.resid = w->x;
        a.resid_stride = d;
        a.k_split = aw;
        launch_gemv<PRO_COPY, EPI_RESID2>(m, a, s);
      } else {
        GemmArgs g{};
        g.W = ly.w2;
        g.n = M;
        g.A = w->ah;
        g.lda = aw + ff;
        g.resid = w->x;
        g.resid_stride = d;
        g.k_split = aw;
        launch_gemm<EPI_RESID2>(m, w, g, s);
      }
    } else {
      g_stage = ST_W1;
      if (gemv) {
        GemvArgs a{};
        a.W = ly.w1;
        a.M = M;
        a.in = w->x;
        a.in_stride = d;
        a.nw = ly.n1w;
        a.out = w->qkv;
        a.out_stride = qkvw;
        launch_gemv<PRO_RMS, EPI_STORE>(m, a, s);
      } else {
        launch_norm_rows(m, w->x, w->xn, M, ly.n1w, nullptr, s);
        GemmArgs g{};
        g.W = ly.w1;
        g.n = M;
        g.A = w->xn;
        g.lda = d;
        g.out = w->qkv;
        g.out_stride = qkvw;
        launch_gemm<EPI_STORE>(m, w, g, s);
      }
      launch_attn_decode(m, pool, w, M, l, grid_splits, s);
      g_stage = ST_W2;
      if (gemv) {
        GemvArgs a{};
        a.W = ly.w2;
        a.M = M;
        a.in = w->ah;
        a.in_stride = aw + ff;
        a.resid = w->x;
        a.resid_stride = d;
        launch_gemv<PRO_COPY, EPI_RESID1>(m, a, s);
        GemvArgs b{};
        b.W = ly.w3;
        b.M = M;
        b.in = w->x;
        b.in_stride = d;
        b.nw = ly.n2w;
        b.n_plain = 0;
        b.glu_out = w->ah + aw;
        b.glu_stride = aw + ff;
        b.glu_act = 1;
        launch_gemv<PRO_RMS, EPI_GLU>(m, b, s);
        GemvArgs c{};
        c.W = ly.w4;
        c.M = M;
        c.in = w->ah + aw;
        c.in_stride = aw + ff;
        c.resid = w->x;
        c.resid_stride = d;
        launch_gemv<PRO_COPY, EPI_RESID1>(m, c, s);
      } else {
        GemmArgs g{};
        g.W = ly.w2;
        g.n = M;
        g.A = w->ah;
        g.lda = aw + ff;
        g.resid = w->x;
        g.resid_stride = d;
        launch_gemm<EPI_RESID1>(m, w, g, s);
        launch_norm_rows(m, w->x, w->xn, M, ly.n2w, nullptr, s);
        GemmArgs g3{};
        g3.W = ly.w3;
        g3.n = M;
        g3.A = w->xn;
        g3.lda = d;
        g3.n_plain = 0;
        g3.glu_out = w->ah + aw;
        g3.glu_stride = aw + ff;
        g3.glu_act = 1;
        launch_gemm<EPI_GLU>(m, w, g3, s);
        GemmArgs g4{};
        g4.W = ly.w4;
        g4.n = M;
        g4.A = w->ah + aw;
        g4.lda = aw + ff;
        g4.resid = w->x;
        g4.resid_stride = d;
        launch_gemm<EPI_RESID1>(m, w, g4, s);
      }
    }
  }
  // Final norm + head (stablelm.go:380-385, model.go:479-480).
  g_stage = ST_HEAD;
  if (gemv) {
    GemvArgs a{};
    a.W = m->head;
    a.M = M;
    a.in = w->x;
    a.in_stride = d;
    a.nw = m->fnw;
    a.nb = m->fnb;
    a.eps = m->eps;
    a.argmax = w->argmax;
    a.logits = write_logits ? w->logits : nullptr;
    a.logits_stride = m->V;
    if (m->arch == ARCH_STABLELM)
      launch_gemv<PRO_LN, EPI_HEAD>(m, a, s);
    else
      launch_gemv<PRO_RMS, EPI_HEAD>(m, a, s);
  } else {
    launch_norm_rows(m, w->x, w->xn, M, m->fnw, m->fnb, s);
    GemmArgs g{};
    g.W = m->head;
    g.n = M;
    g.A = w->xn;
    g.lda = d;
    g.out = w->logits;
    g.out_stride = m->V;
    launch_gemm<EPI_STORE>(m, w, g, s);
    PROF_BEGIN(ST_HEAD, s);
    k_argmax_rows<<<M, 1024, 0, s>>>(w->logits, m->V, m->V, w->argmax);
    NOTE("k_argmax_rows");
    PROF_END(s);
  }
}

// Prompt chunk of n tokens for one sequence at positions start..start+n-1
// (prefill.go:33-115 / mlx_native.go:324-495). Tokens are in w->tokens.
static void enqueue_prefill(const tcu_model* m, KVPool* pool, Work* w, int n, int start, cudaStream_t s) {
  const int d = m->d, ff = m->ff, aw = m->aw, qkvw = aw + 2 * m->kvw;
  EmbedArgs ea{};
  ea.E = m->embed;
  ea.n = n;
  ea.tokens = w->tokens;
  ea.x = w->x;
  ea.x_stride = d;
  PROF_BEGIN(ST_EMBED, s);
  k_embed<<<n, 256, 0, s>>>(ea);
  NOTE("k_embed");
  PROF_END(s);
  g_stage = ST_PF_GEMM;
  for (int l = 0; l < m->L; l++) {
    const Layer& ly = m->layers[l];
    launch_norm_rows(m, w->x, w->xn, n, ly.n1w, ly.n1b, s);
    GemmArgs g{};
    g.W = ly.w1;
    g.n = n;
    g.A = w->xn;
    g.lda = d;
    g.out = w->qkv;
    g.out_stride = qkvw;
    if (m->arch == ARCH_STABLELM) {
      g.n_plain = qkvw;
      g.glu_out = w->ah + aw;
      g.glu_stride = aw + ff;
      g.glu_act = 0;
      launch_gemm<EPI_GLU>(m, w, g, s);
    } else {
      launch_gemm<EPI_STORE>(m, w, g, s);
    }
    RopeStoreArgs r{};
    r.n = n;
    r.H = m->H;
    r.KVH = m->KVH;
    r.hd = m->hd;
    r.start = start;
    r.rope = m->rope;
    r.qkv = w->qkv;
    r.qkv_stride = qkvw;
    r.kv = pool->view();
    r.layer = l;
    r.page_table = w->pt;
    PROF_BEGIN(ST_OTHER, s);
    k_rope_store<<<n, 128, 0, s>>>(r);
    NOTE("k_rope_store");
    PROF_END(s);
    PrefillAttnArgs pa{};
    pa.n = n;
    pa.H = m->H;
    pa.KVH = m->KVH;
    pa.hd = m->hd;
    pa.start = start;
    pa.qkv = w->qkv;
    pa.qkv_stride = qkvw;
    pa.kv = pool->view();
    pa.layer = l;
    pa.page_table = w->pt;
    pa.out = w->ah;
    pa.out_stride = aw + ff;
    pa.scale = (float)sqrt((double)m->hd);
    const int hd16 = m->hd % 16 == 0 ? m->hd / 16 : 0;
    if (pool->half && m->use_tc_attn && (hd16 == 4 || hd16 == 5 || hd16 == 6 || hd16 == 8) &&
        at_smem_bytes(m->hd, 1) <= (size_t)m->gemv_smem_optin) {
      // Tensor cores (binary16 KV): one CTA per 128 queries and head; two
      // groups of four warps on alternate key blocks where shared memory
      // allows.
      auto pick = [&](int ng) -> void (*)(PrefillAttnArgs, int*) {
        if (ng == 2) return hd16 == 4 ? k_attn_prefill_tc<64, 2> : hd16 == 5 ? k_attn_prefill_tc<80, 2> : hd16 == 6 ? k_attn_prefill_tc<96, 2> : nullptr;
        return hd16 == 4 ? k_attn_prefill_tc<64, 1> : hd16 == 5 ? k_attn_prefill_tc<80, 1> : hd16 == 6 ? k_attn_prefill_tc<96, 1> : k_attn_prefill_tc<128, 1>;
      };
      const int ng = pick(2) && at_smem_bytes(m->hd, 2) <= (size_t)m->gemv_smem_optin ? 2 : 1;
      void (*kern)(PrefillAttnArgs, int*) = pick(ng);
      const size_t smem = at_smem_bytes(m->hd, ng);
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      NOTE("cudaFuncSetAttribute(k_attn_prefill_tc)");
      PROF_BEGIN(ST_PF_ATTN, s);
      kern<<<dim3((n + AT_ROWS - 1) / AT_ROWS, m->H), AT_GROUP * ng, smem, s>>>(pa, w->err);
      NOTE("k_attn_prefill_tc");
    } else {
      const size_t smem = pa_smem_bytes(m->hd);
      const int nc = (m->hd + 15) / 16;
      auto kern = nc <= 2 ? k_attn_prefill<2> : nc <= 4 ? k_attn_prefill<4> : nc <= 5 ? k_attn_prefill<5> : k_attn_prefill<8>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      NOTE("cudaFuncSetAttribute(k_attn_prefill)");
      PROF_BEGIN(ST_PF_ATTN, s);
      kern<<<dim3((n + PA_QT - 1) / PA_QT, m->H), PA_THREADS, smem, s>>>(pa);
      NOTE("k_attn_prefill");
    }
    PROF_END(s);
    if (m->arch == ARCH_STABLELM && m->tp_world > 1) {
      GemmArgs g2{};
      g2.W = ly.w2;
      g2.n = n;
      g2.A = w->ah;
      g2.lda = aw + ff;
      g2.out = w->tp_part;
      g2.out_stride = d;
      launch_gemm<EPI_STORE>(m, w, g2, s);
      tp_reduce_add(m, w, n, s);
    } else if (m->arch == ARCH_STABLELM) {
      GemmArgs g2{};
      g2.W = ly.w2;
      g2.n = n;
      g2.A = w->ah;
      g2.lda = aw + ff;
      g2.resid = w->x;
      g2.resid_stride = d;
      g2.k_split = aw;
      launch_gemm<EPI_RESID2>(m, w, g2, s);
    } else {
      GemmArgs g2{};
      g2.W = ly.w2;
      g2.n = n;
      g2.A = w->ah;
      g2.lda = aw + ff;
      g2.resid = w->x;
      g2.resid_stride = d;
      launch_gemm<EPI_RESID1>(m, w, g2, s);
      launch_norm_rows(m, w->x, w->xn, n, ly.n2w, nullptr, s);
      GemmArgs g3{};
      g3.W = ly.w3;
      g3.n = n;
      g3.A = w->xn;
      g3.lda = d;
      g3.n_plain = 0;
      g3.glu_out = w->ah + aw;
      g3.glu_stride = aw + ff;
      g3.glu_act = 1;
      launch_gemm<EPI_GLU>(m, w, g3, s);
      GemmArgs g4{};
      g4.W = ly.w4;
      g4.n = n;
      g4.A = w->ah + aw;
      g4.lda = aw + ff;
      g4.resid = w->x;
      g4.resid_stride = d;
      launch_gemm<EPI_RESID1>(m, w, g4, s);
    }
  }
}

// Head over the last row of a prefill chunk (prefill.go:103-109).
static void enqueue_head_row(const tcu_model* m, Work* w, int row, float* logits, cudaStream_t s) {
  cudaMemsetAsync(w->argmax, 0, sizeof(unsigned long long), s);
  NOTE("cudaMemsetAsync(w->argmax, 0, sizeof(uns");
  g_stage = ST_HEAD;
  GemvArgs a{};
  a.W = m->head;
  a.M = 1;
  a.in = w->x + (size_t)row * m->d;
  a.in_stride = m->d;
  a.nw = m->fnw;
  a.nb = m->fnb;
  a.eps = m->eps;
  a.argmax = w->argmax;
  a.logits = logits;
  a.logits_stride = m->V;
  if (m->arch == ARCH_STABLELM)
    launch_gemv<PRO_LN, EPI_HEAD>(m, a, s);
  else
    launch_gemv<PRO_RMS, EPI_HEAD>(m, a, s);
}

// ---------------------------------------------------------------------------
// Sessions

struct tcu_session {
  tcu_model* m = nullptr;
  KVPool* pool = nullptr;
  int half = 0;
  std::vector<int> pages;
  int length = 0;
  cudaStream_t stream = nullptr;
  Work* w = nullptr;  // from the model's workspace pool (work_take)
  bool closed = false;
  cudaStream_t own_stream = nullptr;  // created by the session; stream may be the caller's
  // cached decode-step graph (step mode, M = 1)
  cudaGraphExec_t graph = nullptr;
  int graph_splits = 0;
  bool graph_prof = false;
  size_t graph_events = 0;
  int branches_open = 0;
  Prof prof;
  int hold_layer = -1;  // failure-detection test hook of the persistent step (TCU_TEST_HOLD_ARRIVAL)
};

// Routes the launch helpers' stage events (when profiling) and bounded-wait
// error word to the session whose call is enqueueing work.
struct ProfScope {
  explicit ProfScope(tcu_session* s, int* err = nullptr) {
    g_prof = (s && s->prof.on) ? &s->prof : nullptr;
    g_err_word = err ? err : (s ? s->w->err : nullptr);
  }
  ~ProfScope() {
    g_prof = nullptr;
    g_err_word = nullptr;
  }
};

// Accumulates recorded stage events (the stream must be synchronised).
static void prof_collect(tcu_session* s) {
  if (!s->prof.on) return;
  s->prof.collect(s->prof.used);
  s->prof.used = 0;
}

struct tcu_branches {
  tcu_session* s = nullptr;
  int prefix = 0, count = 0, step = 0;
  std::vector<std::vector<int>> pages;
  Work* w = nullptr;  // from the model's workspace pool (work_take)
  bool closed = false;
};

static void release_pages(tcu_model* m, KVPool* pool, std::vector<int>& pages, size_t keep) {
  while (pages.size() > keep) {
    page_unref(m, pool, pages.back());
    pages.pop_back();
  }
}

// Makes positions [lo, hi) of a page list writable and allocated: pages past
// the end are allocated; shared pages in range are copied (copy-on-write).
static int prepare_pages(tcu_model* m, KVPool* pool, std::vector<int>& pages, int lo, int hi, cudaStream_t s) {
  const int P = pool->P;
  const size_t need = (size_t)(hi + P - 1) / P;
  while (pages.size() < need) {
    int pg;
    TRY(page_alloc(m, pool, &pg));
    pages.push_back(pg);
  }
  for (int i = lo / P; i < (int)need; i++) {
    if (page_refcount(m, pool, pages[i]) > 1) {
      int pg;
      TRY(page_alloc(m, pool, &pg));
      const size_t page_vec = pool->page_elems() * pool->elem() / 16;
      k_copy_page<<<592, 256, 0, s>>>((uint4*)pool->k, (uint4*)pool->v, page_vec, pool->num_pages, pages[i], pg, pool->L);
      NOTE("k_copy_page");
      CK(cudaGetLastError());
      page_unref(m, pool, pages[i]);
      pages[i] = pg;
    }
  }
  return TCU_OK;
}

static int sync_stream(cudaStream_t stream, int* err_word) {
  cudaError_t e = cudaStreamSynchronize(stream);
  const char* site = g_err_site ? g_err_site : "?";
  g_err_site = nullptr;
  if (e != cudaSuccess) return fail(TCU_ECUDA, "device execution failed: %s (first failing launch: %s)", cudaGetErrorString(e), site);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TCU_ECUDA, "launch failed: %s (at %s)", cudaGetErrorString(e), site);
  int flag = 0;
  if (cudaMemcpy(&flag, err_word, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && flag != 0) {
    const int zero = 0;
    cudaMemcpy(err_word, &zero, sizeof(int), cudaMemcpyHostToDevice);
    return fail(TCU_ETIMEOUT, "a bounded device wait expired (error word %d); results of this call are invalid", flag);
  }
  return TCU_OK;
}

static int session_sync(tcu_session* s) { return sync_stream(s->stream, s->w->err); }

static int upload_pt(tcu_session* s) {
  CK(cudaMemcpyAsync(s->w->pt, s->pages.data(), s->pages.size() * sizeof(int), cudaMemcpyHostToDevice, s->stream));
  return TCU_OK;
}

static int check_tokens(const tcu_model* m, const int32_t* tokens, int n) {
  if (n > 0 && !tokens) return fail(TCU_EINVAL, "null tokens");
  for (int i = 0; i < n; i++)
    if (tokens[i] < 0 || tokens[i] >= m->V) return fail(TCU_EINVAL, "invalid token %d", tokens[i]);
  return TCU_OK;
}

// Probability rows of a forward (ForwardWithLogprobs): per input position
// the target's log probability and `count` top (id, log probability).
struct LogprobReq {
  const int32_t* targets;
  int count;
  double* chosen;
  int32_t* top_ids;
  double* top_vals;
};

// summarizeLogits of `rows` logits rows at blk (stride V) for input
// positions i0 .. i0 + rows - 1: targets up, k_logprob_rows, results down
// into the caller's arrays (stream order keeps the device buffers of one
// block from being overwritten before their copies).
static int enqueue_logprob_block(const tcu_model* m, Work* w, const float* blk, int rows, int i0, const LogprobReq& lp, cudaStream_t s) {
  CK(cudaMemcpyAsync(w->lp_targets, lp.targets + i0, rows * sizeof(int), cudaMemcpyHostToDevice, s));
  const size_t smem = ((size_t)m->V + 31) / 32 * 4;
  k_logprob_rows<<<rows, 1024, smem, s>>>(blk, m->V, m->V, w->lp_targets, lp.count, w->lp_chosen, w->lp_ids, w->lp_vals);
  NOTE("k_logprob_rows");
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(lp.chosen + i0, w->lp_chosen, rows * sizeof(double), cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(lp.top_ids + (size_t)i0 * lp.count, w->lp_ids, (size_t)rows * lp.count * sizeof(int), cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(lp.top_vals + (size_t)i0 * lp.count, w->lp_vals, (size_t)rows * lp.count * sizeof(double), cudaMemcpyDeviceToHost,
                     s));
  return TCU_OK;
}

// Probability rows of the c positions of a prefill chunk (hidden rows in
// w->x): final norm, the head product over up to LP_ROWS rows at a time
// into the chunk's attention/SwiGLU buffer (free once the chunk's layers
// ran), then enqueue_logprob_block (mlx_native.go:436-478 in batches).
static int enqueue_logprob_chunk(const tcu_model* m, Work* w, int c, int i0, const LogprobReq& lp, cudaStream_t s) {
  const size_t cap_rows = (size_t)w->rows * (m->aw + m->ff) / (size_t)m->V;
  const int nb = (int)std::min<size_t>(LP_ROWS, cap_rows);
  if (nb < 1) return fail(TCU_EUNSUP, "vocabulary of %d is too large for the probability rows of this workspace", m->V);
  float* blk = w->ah;
  for (int j0 = 0; j0 < c; j0 += nb) {
    const int r = std::min(nb, c - j0);
    launch_norm_rows(m, w->x + (size_t)j0 * m->d, w->xn, r, m->fnw, m->fnb, s);
    GemmArgs g{};
    g.W = m->head;
    g.n = r;
    g.A = w->xn;
    g.lda = m->d;
    g.out = blk;
    g.out_stride = m->V;
    g_stage = ST_HEAD;
    launch_gemm<EPI_STORE>(m, w, g, s);
    TRY(enqueue_logprob_block(m, w, blk, r, i0 + j0, lp, s));
  }
  return TCU_OK;
}

// Runs tokens[0..n) at positions prefix.. and leaves the last row's argmax in
// w.argmax[0] and (if logits) its logits in w.logits; with lp, also every
// position's probability row.
static int session_run(tcu_session* s, int prefix, const int32_t* tokens, int n, float* all_logits, const LogprobReq* lp = nullptr) {
  tcu_model* m = s->m;
  TRY(prepare_pages(m, s->pool, s->pages, prefix, prefix + n, s->stream));
  TRY(upload_pt(s));
  if (n == 1 && !all_logits) {
    CK(cudaMemcpyAsync(s->w->tokens, tokens, sizeof(int), cudaMemcpyHostToDevice, s->stream));
    CK(cudaMemcpyAsync(s->w->pos, &prefix, sizeof(int), cudaMemcpyHostToDevice, s->stream));
    CK(cudaMemsetAsync(s->w->argmax, 0, sizeof(unsigned long long), s->stream));
    const int split = SPLIT_PAGES * m->P;
    enqueue_decode(m, s->pool, s->w, 1, false, (prefix + 1 + split - 1) / split, true, s->stream);
    CK(cudaGetLastError());
    TRY(comm_check());
    if (lp) TRY(enqueue_logprob_block(m, s->w, s->w->logits, 1, 0, *lp, s->stream));
    return TCU_OK;
  }
  for (int off = 0; off < n; off += CHUNK) {
    const int c = std::min(CHUNK, n - off);
    CK(cudaMemcpyAsync(s->w->tokens, tokens + off, c * sizeof(int), cudaMemcpyHostToDevice, s->stream));
    enqueue_prefill(m, s->pool, s->w, c, prefix + off, s->stream);
    CK(cudaGetLastError());
    TRY(comm_check());
    if (lp) TRY(enqueue_logprob_chunk(m, s->w, c, off, *lp, s->stream));
    if (all_logits) {
      for (int j = 0; j < c; j++) {
        enqueue_head_row(m, s->w, j, s->w->logits, s->stream);
        CK(cudaMemcpyAsync(all_logits + (size_t)(off + j) * m->V, s->w->logits, (size_t)m->V * 4, cudaMemcpyDeviceToHost, s->stream));
      }
    } else if (off + c == n) {
      enqueue_head_row(m, s->w, c - 1, s->w->logits, s->stream);
    }
    CK(cudaGetLastError());
  }
  return TCU_OK;
}

static int validate_forward(tcu_session* s, int prefix, const int32_t* tokens, int n) {
  if (!s) return fail(TCU_EINVAL, "null session");
  if (s->closed) return fail(TCU_ECLOSED, "session is closed");
  if (s->branches_open) return fail(TCU_EINVAL, "close the open branches first");
  // mlx_native.go:328-335
  if (prefix < 0 || prefix > s->length || n <= 0 || prefix + n > s->m->max_pos)
    return fail(TCU_EINVAL, "invalid cached prefix or context length (prefix %d, resident %d, tokens %d, limit %d)", prefix, s->length, n,
                s->m->max_pos);
  return check_tokens(s->m, tokens, n);
}

static void session_invalidate(tcu_session* s) {
  release_pages(s->m, s->pool, s->pages, 0);
  s->length = 0;
}

static int session_finish(tcu_session* s, int rc, int new_length) {
  if (rc == TCU_OK) rc = session_sync(s);
  if (rc == TCU_OK) prof_collect(s);
  s->prof.used = 0;
  if (rc != TCU_OK) {
    std::string msg = g_err;
    cudaStreamSynchronize(s->stream);
    session_invalidate(s);
    g_err = msg;
    return rc;
  }
  s->length = new_length;
  release_pages(s->m, s->pool, s->pages, (size_t)(new_length + s->pool->P - 1) / s->pool->P);
  return TCU_OK;
}

// Captures one greedy decode step (embed from argmax .. head) as a graph.
static int session_graph(tcu_session* s, int splits) {
  if (s->graph && s->graph_splits >= splits && s->graph_prof == s->prof.on) return TCU_OK;
  if (s->graph) {
    cudaGraphExecDestroy(s->graph);
    s->graph = nullptr;
  }
  cudaGraph_t g;
  s->prof.used = 0;
  CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeRelaxed));
  enqueue_decode(s->m, s->pool, s->w, 1, true, splits, true, s->stream);
  cudaError_t e = cudaStreamEndCapture(s->stream, &g);
  s->graph_events = s->prof.used;
  s->graph_prof = s->prof.on;
  s->prof.used = 0;
  if (e != cudaSuccess) return fail(TCU_ECUDA, "graph capture: %s", cudaGetErrorString(e));
  e = cudaGraphInstantiate(&s->graph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return fail(TCU_ECUDA, "graph instantiate: %s", cudaGetErrorString(e));
  s->graph_splits = splits;
  return TCU_OK;
}

// Releases the suffix pages of a branch batch (the shared prefix stays with
// its session); idempotent.
static void branches_release(tcu_branches* b) {
  if (b->closed) return;
  b->closed = true;
  tcu_session* s = b->s;
  cudaStreamSynchronize(s->stream);
  for (auto& pl : b->pages) release_pages(s->m, s->pool, pl, 0);
  s->branches_open--;
}

// ---------------------------------------------------------------------------
// Sampling penalties (sampling.go:45-101): the host turns each row's history
// into ordered float64 terms per penalised id; k_candidates_rows subtracts
// them on the device and ranks the row.

// SamplingOptions.Validate (sampling.go:45-58) for the penalty fields.
static int penalties_check(const tcu_penalties& p) {
  for (double v : {p.repetition_penalty, p.presence_penalty, p.frequency_penalty, p.repetition_slope})
    if (!std::isfinite(v)) return fail(TCU_EINVAL, "sampling values must be finite");
  if (p.repetition_penalty < 1 || p.repetition_range < 0 || p.repetition_slope < 0) return fail(TCU_EINVAL, "sampling value out of range");
  return TCU_OK;
}

// repetitionWeight (sampling.go:64-70).
static double repetition_weight(int age, int window, double slope) {
  if (slope == 0 || window <= 1) return 1;
  const double x = 1 - 2 * (double)age / (double)(window - 1);
  return 1 + slope * x / (1 + std::fabs(x) * (slope - 1));
}

// Rows of penalised ids, as k_candidates_rows reads them (PenaltyRows).
struct PenaltyHost {
  std::vector<int> row_off{0}, ids, term_off{0};
  std::vector<double> terms;
  int max_ids = 0;
};

// penalizedLogits (sampling.go:76-101) for one row as ordered terms: for the
// last `window` ids (most recent first), frequency * weight on every
// occurrence and (log(repetition) + presence) * weight on an id's most
// recent one; ids outside the vocabulary are skipped. Terms are grouped by id
// keeping their order, so each id's score is the same chain of float64
// subtractions the reference performs.
static void penalties_add_row(PenaltyHost& h, const int32_t* hist, int n_hist, const tcu_penalties& p, int V) {
  const int window = p.repetition_range == 0 ? n_hist : p.repetition_range;
  const int m = std::min(window, n_hist);
  std::vector<std::pair<int, double>> ops;
  ops.reserve((size_t)2 * m);
  std::vector<uint8_t> seen(m > 0 ? V : 0, 0);
  for (int age = 0; age < m; age++) {
    const int id = hist[n_hist - 1 - age];
    if (id < 0 || id >= V) continue;
    const double weight = repetition_weight(age, window, p.repetition_slope);
    ops.emplace_back(id, p.frequency_penalty * weight);
    if (!seen[id]) {
      ops.emplace_back(id, (std::log(p.repetition_penalty) + p.presence_penalty) * weight);
      seen[id] = 1;
    }
  }
  std::stable_sort(ops.begin(), ops.end(), [](const std::pair<int, double>& a, const std::pair<int, double>& b) { return a.first < b.first; });
  int nd = 0;
  for (size_t i = 0; i < ops.size(); i++) {
    if (i == 0 || ops[i].first != ops[i - 1].first) {
      if (i > 0) h.term_off.push_back((int)h.terms.size());
      h.ids.push_back(ops[i].first);
      nd++;
    }
    h.terms.push_back(ops[i].second);
  }
  if (nd > 0) h.term_off.push_back((int)h.terms.size());
  h.row_off.push_back((int)h.ids.size());
  h.max_ids = std::max(h.max_ids, nd);
}

static const int CAND_MAX_IDS = 16384;  // penalised ids per row (k_candidates_rows shared memory)

// Uploads the penalty rows and enqueues k_candidates_rows over `rows` logits
// rows; results in w->cd_ids / w->cd_vals ([rows][k]).
static int enqueue_candidates(const tcu_model* m, Work* w, const float* logits, int rows, const PenaltyHost& h, int k, cudaStream_t s) {
  if (h.max_ids > CAND_MAX_IDS) return fail(TCU_EINVAL, "%d distinct penalised ids in one row (at most %d)", h.max_ids, CAND_MAX_IDS);
  auto r16 = [](size_t b) { return (b + 15) / 16 * 16; };
  const size_t o_ids = r16(h.row_off.size() * 4), o_toff = o_ids + r16(std::max<size_t>(h.ids.size(), 1) * 4);
  const size_t o_terms = o_toff + r16(h.term_off.size() * 4), bytes = o_terms + std::max<size_t>(h.terms.size(), 1) * 8;
  if (bytes > w->pen_cap) {
    // Grows (rarely): synchronise the stream so no queued kernel still reads it.
    cudaStreamSynchronize(s);
    if (w->pen_buf) cudaFree(w->pen_buf);
    w->pen_buf = nullptr;
    w->pen_cap = 0;
    const size_t cap = std::max<size_t>(bytes * 2, 64 << 10);
    if (cudaMalloc(&w->pen_buf, cap) != cudaSuccess) {
      cudaGetLastError();
      return fail(TCU_ENOMEM, "penalty rows: cannot allocate %zu bytes", cap);
    }
    w->pen_cap = cap;
  }
  std::vector<uint8_t> stage(bytes, 0);
  memcpy(stage.data(), h.row_off.data(), h.row_off.size() * 4);
  if (!h.ids.empty()) memcpy(stage.data() + o_ids, h.ids.data(), h.ids.size() * 4);
  memcpy(stage.data() + o_toff, h.term_off.data(), h.term_off.size() * 4);
  if (!h.terms.empty()) memcpy(stage.data() + o_terms, h.terms.data(), h.terms.size() * 8);
  CK(cudaMemcpyAsync(w->pen_buf, stage.data(), bytes, cudaMemcpyHostToDevice, s));
  PenaltyRows pr{(const int*)w->pen_buf, (const int*)(w->pen_buf + o_ids), (const int*)(w->pen_buf + o_toff),
                 (const double*)(w->pen_buf + o_terms)};
  const int max_ids = std::max(1, h.max_ids);
  const size_t smem = (size_t)max_ids * 12 + ((size_t)m->V + 31) / 32 * 8;
  if (smem > 224 * 1024) return fail(TCU_EINVAL, "penalised ids and vocabulary exceed the candidates kernel's shared memory");
  k_candidates_rows<<<rows, 1024, smem, s>>>(logits, m->V, m->V, pr, max_ids, k, w->cd_ids, w->cd_vals);
  NOTE("k_candidates_rows");
  CK(cudaGetLastError());
  return TCU_OK;
}

// ---------------------------------------------------------------------------
// C ABI

extern "C" {

int tcu_abi_version(void) { return TCU_ABI_VERSION; }

const char* tcu_last_error(void) { return g_err.c_str(); }

int tcu_device_count(int32_t* count) {
  if (!count) return fail(TCU_EINVAL, "null count");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *count = 0;
    return TCU_OK;
  }
  *count = n;
  return TCU_OK;
}

int tcu_stablelm_load(const tcu_stablelm_config* config, const tcu_tensor* tensors, int32_t n_tensors, const tcu_load_options* options,
                      tcu_model** out) {
  return stablelm_load(config, tensors, n_tensors, options, nullptr, out);
}

int tcu_tp_unique_id(uint8_t* id) {
  if (!id) return fail(TCU_EINVAL, "null argument");
  const NcclApi* api = nccl_api();
  if (!api) return fail(TCU_EUNSUP, "tensor parallelism needs NCCL (libnccl.so.2 not found)");
  ncclUniqueId u;
  const ncclResult_t r = api->get_unique_id(&u);
  if (r != ncclSuccess) return fail(TCU_ECUDA, "ncclGetUniqueId: %s", api->error_string(r));
  memcpy(id, &u, sizeof u);
  return TCU_OK;
}

int tcu_tp_plan(const tcu_stablelm_config* config, int32_t world, int32_t rank, int32_t* out) {
  if (!config || !out) return fail(TCU_EINVAL, "null argument");
  TpSlice sl;
  TRY(tp_slice(config, world, rank, &sl));
  const int32_t v[6] = {sl.h0, sl.nh, sl.kv0, sl.nkv, sl.f0, sl.nf};
  memcpy(out, v, sizeof v);
  return TCU_OK;
}

int tcu_stablelm_load_tp(const tcu_stablelm_config* config, const tcu_tensor* tensors, int32_t n_tensors, const tcu_load_options* options,
                         const tcu_tp_options* tp, tcu_model** out) {
  if (!config || !tp || !out) return fail(TCU_EINVAL, "null argument");
  TpSlice sl;
  TRY(tp_slice(config, tp->world, tp->rank, &sl));
  const NcclApi* api = nullptr;
  if (tp->world > 1 && !(api = nccl_api())) return fail(TCU_EUNSUP, "tensor parallelism needs NCCL (libnccl.so.2 not found)");
  TRY(stablelm_load(config, tensors, n_tensors, options, &sl, out));
  if (tp->world > 1) {
    tcu_model* m = *out;
    ncclUniqueId u;
    memcpy(&u, tp->nccl_id, sizeof u);
    const ncclResult_t r = api->comm_init_rank(&m->tp_comm, tp->world, u, tp->rank);
    if (r != ncclSuccess) {
      m->tp_comm = nullptr;
      model_release(m);
      *out = nullptr;
      return fail(TCU_ECUDA, "ncclCommInitRank: %s", api->error_string(r));
    }
  }
  return TCU_OK;
}

int tcu_tp_exchange_handle(tcu_model* m, uint8_t* handle) {
  if (!m || !handle) return fail(TCU_EINVAL, "null argument");
  if (m->tp_world < 2) return fail(TCU_EINVAL, "not a tensor-parallel model");
  if (m->tp_world > TPX_MAX_RANKS) return fail(TCU_EUNSUP, "the peer exchange serves at most %d ranks", TPX_MAX_RANKS);
  CK(cudaSetDevice(m->device));
  std::lock_guard<std::mutex> lk(m->mu);
  if (!m->tp_ex) {
    const long long count = ((long long)CHUNK * m->d + 3) / 4 * 4;
    void* p = nullptr;
    CK(cudaMalloc(&p, tpx_bytes((size_t)count)));
    CK(cudaMemset(p, 0, TPX_FLAG_BYTES));
    m->tp_ex = (uint8_t*)p;
    m->tp_ex_count = count;
    TRY(dalloc(m, (void**)&m->tp_seq, 2 * sizeof(uint32_t)));
    CK(cudaMemset(m->tp_seq, 0, 2 * sizeof(uint32_t)));
  }
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, m->tp_ex));
  static_assert(sizeof(cudaIpcMemHandle_t) == TCU_TP_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof h);
  return TCU_OK;
}

int tcu_tp_exchange_open(tcu_model* m, const uint8_t* handles) {
  if (!m || !handles) return fail(TCU_EINVAL, "null argument");
  if (!m->tp_ex) return fail(TCU_EINVAL, "tcu_tp_exchange_handle first");
  if (m->tp_ex_on) return fail(TCU_EINVAL, "the peer exchange is already open");
  CK(cudaSetDevice(m->device));
  std::lock_guard<std::mutex> lk(m->mu);
  uint8_t* peer[TPX_MAX_RANKS] = {};
  for (int p = 0; p < m->tp_world; p++) {
    if (p == m->tp_rank) {
      peer[p] = m->tp_ex;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, handles + (size_t)p * TCU_TP_HANDLE_BYTES, sizeof h);
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < p; q++)
        if (peer[q] && q != m->tp_rank) cudaIpcCloseMemHandle(peer[q]);
      return fail(TCU_ECUDA, "cudaIpcOpenMemHandle(rank %d): %s", p, cudaGetErrorString(e));
    }
    peer[p] = (uint8_t*)ptr;
  }
  memcpy(m->tp_peer, peer, sizeof peer);
  m->tp_ex_on = true;
  return TCU_OK;
}

}  // extern "C"

// A memory-mapped GGUF StableLM checkpoint: the parsed file, the derived
// configuration and its tensors under their Hugging Face names (data
// pointing into the mapping).
struct tcu_gguf {
  GgufFile f;
  tcu_stablelm_config config{};
  std::vector<std::string> names;
  std::vector<tcu_tensor> tensors;
};

// loadStableGGUF's metadata rules (gguf.go:258-357), without the tokenizer
// check (the caller compares its tokenizer.json with the GGUF vocabulary).
static int gguf_stablelm(tcu_gguf* g) {
  const auto& meta = g->f.meta;
  auto get = [&](const char* k) -> const GgufValue* {
    auto it = meta.find(k);
    return it == meta.end() ? nullptr : &it->second;
  };
  const GgufValue* arch = get("general.architecture");
  const GgufValue* type = get("general.type");
  if (!arch || arch->kind != GgufValue::STR || arch->s != "stablelm" || (type && (type->kind != GgufValue::STR || type->s != "model")))
    return fail(TCU_EINVAL, "GGUF must contain a StableLM model");
  std::string bad;
  auto integer = [&](const char* k) -> int32_t {
    const GgufValue* v = get(k);
    if (!v || v->kind != GgufValue::UINT || v->u > (uint64_t)INT32_MAX) {
      if (bad.empty()) bad = k;
      return 0;
    }
    return (int32_t)v->u;
  };
  tcu_stablelm_config& c = g->config;
  c.hidden_size = integer("stablelm.embedding_length");
  c.intermediate_size = integer("stablelm.feed_forward_length");
  c.num_hidden_layers = integer("stablelm.block_count");
  c.num_attention_heads = integer("stablelm.attention.head_count");
  c.num_key_value_heads = integer("stablelm.attention.head_count_kv");
  c.max_position_embeddings = integer("stablelm.context_length");
  c.bos_token_id = integer("tokenizer.ggml.bos_token_id");
  c.eos_token_id = integer("tokenizer.ggml.eos_token_id");
  const GgufValue* par = get("stablelm.use_parallel_residual");
  const bool parallel = par && par->kind == GgufValue::BOOL && par->b;
  const GgufValue* eps = get("stablelm.attention.layer_norm_epsilon");
  c.layer_norm_eps = (eps && eps->kind == GgufValue::FLOAT) ? eps->f : 0.0;
  c.rope_theta = 10000.0;
  if (const GgufValue* th = get("stablelm.rope.freq_base")) {
    if (th->kind != GgufValue::FLOAT) return fail(TCU_EINVAL, "invalid GGUF RoPE frequency base");
    c.rope_theta = th->f;
  }
  if (c.hidden_size > 0 && c.num_attention_heads > 0)
    c.partial_rotary_factor = (double)integer("stablelm.rope.dimension_count") * (double)c.num_attention_heads / (double)c.hidden_size;
  const GgufValue* vocab = get("tokenizer.ggml.tokens");
  if (!vocab || vocab->kind != GgufValue::ARRAY) return fail(TCU_EINVAL, "GGUF missing vocabulary");
  c.vocab_size = (int32_t)vocab->count;
  if (!bad.empty()) return fail(TCU_EINVAL, "missing or invalid GGUF integer %s", bad.c_str());
  // validate() (stablelm.go:85-111).
  if (!parallel) return fail(TCU_EINVAL, "unsupported StableLM variant: require parallel residuals");
  if (c.hidden_size <= 0 || c.intermediate_size <= 0 || c.num_hidden_layers <= 0 || c.num_attention_heads <= 0 ||
      c.num_key_value_heads <= 0 || c.vocab_size <= 0 || c.max_position_embeddings <= 0 || c.hidden_size % c.num_attention_heads ||
      c.num_attention_heads % c.num_key_value_heads)
    return fail(TCU_EINVAL, "invalid StableLM dimensions");
  const double rotary = (double)(c.hidden_size / c.num_attention_heads) * c.partial_rotary_factor;
  if (!(c.layer_norm_eps > 0) || std::isinf(c.layer_norm_eps) || !(c.rope_theta > 0) || std::isinf(c.rope_theta) ||
      !(c.partial_rotary_factor > 0) || c.partial_rotary_factor > 1 || rotary != std::trunc(rotary) || (int)rotary % 2 != 0 || rotary < 2)
    return fail(TCU_EINVAL, "invalid LayerNorm or partial RoPE settings");
  if (c.bos_token_id < 0 || c.bos_token_id >= c.vocab_size || c.eos_token_id < 0 || c.eos_token_id >= c.vocab_size)
    return fail(TCU_EINVAL, "invalid BOS/EOS token IDs");
  const size_t nt = g->f.tensors.size();
  if (nt < 4 || (nt - 4) % 9 != 0 || (int)((nt - 4) / 9) != c.num_hidden_layers)
    return fail(TCU_EINVAL, "unexpected GGUF tensor count for %d StableLM layers", c.num_hidden_layers);
  if (const GgufValue* sc = get("stablelm.rope.scaling.type"))
    if (!(sc->kind == GgufValue::STR && sc->s == "none")) return fail(TCU_EINVAL, "GGUF RoPE scaling is not supported");
  for (const GgufTensor& t : g->f.tensors) {
    const std::string& n = t.name;
    const bool bias = n.size() >= 5 && n.compare(n.size() - 5, 5, ".bias") == 0;
    if (n.find("attn_q_norm") != std::string::npos || n.find("attn_k_norm") != std::string::npos ||
        n.find("ffn_norm") != std::string::npos || (bias && n.find("norm") == std::string::npos))
      return fail(TCU_EUNSUP, "unsupported StableLM tensor %s", n.c_str());
  }
  // The tensors loadStableWeights reads (stablelm.go:167-199), by their GGUF
  // names, with their row-major shapes checked.
  const int d = c.hidden_size, ff = c.intermediate_size, kv = d / c.num_attention_heads * c.num_key_value_heads;
  struct Want {
    std::string hf;
    std::vector<int64_t> shape;
  };
  std::vector<Want> want = {{"model.embed_tokens.weight", {c.vocab_size, d}}, {"lm_head.weight", {c.vocab_size, d}},
                            {"model.norm.weight", {d}}, {"model.norm.bias", {d}}};
  for (int l = 0; l < c.num_hidden_layers; l++) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    want.push_back({p + "input_layernorm.weight", {d}});
    want.push_back({p + "input_layernorm.bias", {d}});
    want.push_back({p + "self_attn.q_proj.weight", {d, d}});
    want.push_back({p + "self_attn.k_proj.weight", {kv, d}});
    want.push_back({p + "self_attn.v_proj.weight", {kv, d}});
    want.push_back({p + "self_attn.o_proj.weight", {d, d}});
    want.push_back({p + "mlp.gate_proj.weight", {ff, d}});
    want.push_back({p + "mlp.up_proj.weight", {ff, d}});
    want.push_back({p + "mlp.down_proj.weight", {d, ff}});
  }
  g->names.clear();
  g->tensors.clear();
  g->names.reserve(want.size());
  for (const Want& w : want) {
    const std::string gn = gguf_name(w.hf);
    auto it = g->f.by_name.find(gn);
    if (it == g->f.by_name.end()) return fail(TCU_EINVAL, "missing GGUF tensor %s", w.hf.c_str());
    const GgufTensor& t = g->f.tensors[it->second];
    if (t.shape != w.shape) return fail(TCU_EINVAL, "GGUF tensor %s: shape mismatch", w.hf.c_str());
    g->names.push_back(w.hf);
    tcu_tensor x{};
    x.dtype = t.dtype;
    x.ndim = (int32_t)t.shape.size();
    for (size_t j = 0; j < t.shape.size(); j++) x.shape[j] = t.shape[j];
    x.data = g->f.map + t.offset;
    x.nbytes = t.size;
    g->tensors.push_back(x);
  }
  for (size_t i = 0; i < g->tensors.size(); i++) g->tensors[i].name = g->names[i].c_str();
  return TCU_OK;
}

extern "C" {

int tcu_gguf_open(const char* path, tcu_gguf** out) {
  if (!path || !out) return fail(TCU_EINVAL, "null argument");
  *out = nullptr;
  tcu_gguf* g = new tcu_gguf();
  std::string err;
  if (!gguf_read(path, &g->f, &err)) {
    delete g;
    return fail(TCU_EINVAL, "%s", err.c_str());
  }
  const int rc = gguf_stablelm(g);
  if (rc != TCU_OK) {
    delete g;
    return rc;
  }
  *out = g;
  return TCU_OK;
}

int tcu_gguf_config(const tcu_gguf* g, tcu_stablelm_config* config) {
  if (!g || !config) return fail(TCU_EINVAL, "null argument");
  *config = g->config;
  return TCU_OK;
}

int tcu_gguf_tensor_count(const tcu_gguf* g, int32_t* n) {
  if (!g || !n) return fail(TCU_EINVAL, "null argument");
  *n = (int32_t)g->tensors.size();
  return TCU_OK;
}

int tcu_gguf_tensor(const tcu_gguf* g, int32_t i, tcu_tensor* out) {
  if (!g || !out) return fail(TCU_EINVAL, "null argument");
  if (i < 0 || i >= (int32_t)g->tensors.size()) return fail(TCU_EINVAL, "tensor index %d out of range", i);
  *out = g->tensors[i];
  return TCU_OK;
}

int tcu_gguf_load_stablelm(const tcu_gguf* g, const tcu_load_options* options, const tcu_tp_options* tp, tcu_model** out) {
  if (!g || !out) return fail(TCU_EINVAL, "null argument");
  if (tp) return tcu_stablelm_load_tp(&g->config, g->tensors.data(), (int32_t)g->tensors.size(), options, tp, out);
  return stablelm_load(&g->config, g->tensors.data(), (int32_t)g->tensors.size(), options, nullptr, out);
}

int tcu_gguf_close(tcu_gguf* g) {
  delete g;
  return TCU_OK;
}

int tcu_llama_load(const void* checkpoint, uint64_t nbytes, const tcu_load_options* options, tcu_model** out) {
  return llama_load(checkpoint, nbytes, options, out);
}

int tcu_model_info(const tcu_model* m, int32_t* vocab, int32_t* hidden, int32_t* layers, int32_t* heads, int32_t* kv_heads,
                   int32_t* max_positions) {
  if (!m) return fail(TCU_EINVAL, "null model");
  if (vocab) *vocab = m->V;
  if (hidden) *hidden = m->d;
  if (layers) *layers = m->L;
  if (heads) *heads = m->H;
  if (kv_heads) *kv_heads = m->KVH;
  if (max_positions) *max_positions = m->max_pos;
  return TCU_OK;
}

int tcu_model_memory(const tcu_model* m, uint64_t* weight_bytes, uint64_t* kv_pool_bytes, uint64_t* kv_used_bytes) {
  if (!m) return fail(TCU_EINVAL, "null model");
  uint64_t pool = 0, used = 0;
  for (KVPool* p : m->pools)
    if (p) {
      const uint64_t pb = (uint64_t)p->L * p->page_elems() * p->elem() * 2;
      pool += pb * p->num_pages;
      used += pb * p->used();
    }
  if (weight_bytes) *weight_bytes = m->weight_bytes;
  if (kv_pool_bytes) *kv_pool_bytes = pool;
  if (kv_used_bytes) *kv_used_bytes = used;
  return TCU_OK;
}

int tcu_model_free(tcu_model* m) {
  if (!m) return TCU_OK;
  if (m->sessions > 0) return fail(TCU_EINVAL, "%d sessions still open", m->sessions);
  model_release(m);
  return TCU_OK;
}

int tcu_session_new(tcu_model* m, int32_t kv_dtype, tcu_session** out) {
  if (!m || !out) return fail(TCU_EINVAL, "null argument");
  if (kv_dtype != TCU_F32 && kv_dtype != TCU_F16) return fail(TCU_EINVAL, "unsupported KV cache precision %d: use f32 or f16", kv_dtype);
  CK(cudaSetDevice(m->device));
  tcu_session* s = new tcu_session();
  s->m = m;
  s->half = kv_dtype == TCU_F16;
  int rc = pool_get(m, s->half, &s->pool);
  if (rc == TCU_OK) rc = work_take(m, &s->w, CHUNK, 1, 1, m->max_pos + 1);
  if (rc == TCU_OK && cudaStreamCreateWithFlags(&s->own_stream, cudaStreamNonBlocking) != cudaSuccess) rc = fail(TCU_ECUDA, "stream create");
  s->stream = s->own_stream;
  if (rc != TCU_OK) {
    if (s->own_stream) cudaStreamDestroy(s->own_stream);
    work_give(m, s->w);
    delete s;
    return rc;
  }
  {
    std::lock_guard<std::mutex> g(m->mu);
    m->sessions++;
  }
  *out = s;
  return TCU_OK;
}

int tcu_session_free(tcu_session* s) {
  if (!s) return TCU_OK;
  cudaSetDevice(s->m->device);
  if (s->branches_open) return fail(TCU_EINVAL, "close the open branches first");
  cudaStreamSynchronize(s->stream);
  release_pages(s->m, s->pool, s->pages, 0);
  if (s->graph) cudaGraphExecDestroy(s->graph);
  if (s->own_stream) cudaStreamDestroy(s->own_stream);
  work_give(s->m, s->w);
  {
    std::lock_guard<std::mutex> g(s->m->mu);
    s->m->sessions--;
  }
  delete s;
  return TCU_OK;
}

int tcu_session_length(const tcu_session* s, int32_t* length) {
  if (!s || !length) return fail(TCU_EINVAL, "null argument");
  *length = s->length;
  return TCU_OK;
}

int tcu_session_forward(tcu_session* s, int32_t prefix, const int32_t* tokens, int32_t n, int32_t want_logits, float* logits_out) {
  TRY(validate_forward(s, prefix, tokens, n));
  if (want_logits && !logits_out) return fail(TCU_EINVAL, "null logits buffer");
  CK(cudaSetDevice(s->m->device));
  ProfScope ps(s);
  int rc = session_run(s, prefix, tokens, n, nullptr);
  if (rc == TCU_OK && want_logits) {
    cudaError_t e = cudaMemcpyAsync(logits_out, s->w->logits, (size_t)s->m->V * 4, cudaMemcpyDeviceToHost, s->stream);
    if (e != cudaSuccess) rc = fail(TCU_ECUDA, "logits copy: %s", cudaGetErrorString(e));
  }
  return session_finish(s, rc, prefix + n);
}

int tcu_session_forward_all(tcu_session* s, int32_t prefix, const int32_t* tokens, int32_t n, float* logits_out) {
  TRY(validate_forward(s, prefix, tokens, n));
  if (!logits_out) return fail(TCU_EINVAL, "null logits buffer");
  CK(cudaSetDevice(s->m->device));
  ProfScope ps(s);
  int rc = session_run(s, prefix, tokens, n, logits_out);
  return session_finish(s, rc, prefix + n);
}

// Launches one persistent decode step (decode_mega.cuh) as a cooperative
// grid of one CTA per SM.
static int launch_mega(tcu_session* s) {
  tcu_model* m = s->m;
  MegaArgs a{};
  a.L = m->L;
  a.d = m->d;
  a.ff = m->ff;
  a.V = m->V;
  a.H = m->H;
  a.KVH = m->KVH;
  a.hd = m->hd;
  a.s1_stride = m->layers[0].w1.sstride;
  a.s2_stride = m->layers[0].w2.sstride;
  a.sh_stride = m->head.sstride;
  a.se_stride = m->embed.sstride;
  a.eps = m->eps;
  a.layers = m->mega_layers;
  a.head_w = (const int8_t*)m->head.w;
  a.head_s = m->head.s;
  a.emb_w = (const int8_t*)m->embed.w;
  a.emb_s = m->embed.s;
  a.fnw = m->fnw;
  a.fnb = m->fnb;
  a.rope = m->rope;
  a.kv = s->pool->view();
  a.page_table = s->w->pt;
  a.split = m->mega_split;
  a.max_splits = s->w->max_splits;
  a.scale = (float)sqrt((double)m->hd);
  a.pos = s->w->pos;
  a.keys = s->w->keys;
  a.step = s->w->step;
  a.out_tokens = s->w->out_tokens;
  a.out_count = s->w->out_count;
  a.logits = s->w->logits;
  a.xl = s->w->xl;
  a.qkv = s->w->qkv;
  a.part = s->w->part;
  a.counters = s->w->counters;
  a.adig = s->w->adig;
  a.asx = s->w->asx;
  a.asx_stride = s->w->asx_stride;
  a.att_warp = m->mega_att_warp;
  a.grab = s->w->grab;
  a.done = s->w->done;
  mega_dn_scales(m, &a.dn_sstride, &a.dn_soff);
  a.xdn = s->w->xdn;
  a.err = s->w->err;
  a.hold_layer = s->hold_layer;
  a.slot_bytes = m->mega_slot_bytes;
  a.nslots = m->mega_slots;
  a.off_x = m->mega_off[0];
  a.off_att = m->mega_off[1];
  a.off_dig = m->mega_off[2];
  a.off_sx = m->mega_off[3];
  a.off_slots = m->mega_off[4];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m->sm_count);
  cfg.blockDim = dim3(MG_THREADS);
  cfg.dynamicSmemBytes = m->mega_smem;
  cfg.stream = s->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PROF_BEGIN(ST_MEGA, s->stream);
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_decode_mega, a);
  PROF_END(s->stream);
  if (e != cudaSuccess) return fail(TCU_ECUDA, "persistent decode launch: %s", cudaGetErrorString(e));
  return TCU_OK;
}

int tcu_session_generate_greedy(tcu_session* s, int32_t prefix, const int32_t* tokens, int32_t n, int32_t steps, int32_t* out_tokens) {
  TRY(validate_forward(s, prefix, tokens, n));
  if (steps < 1 || !out_tokens) return fail(TCU_EINVAL, "invalid steps or output buffer");
  tcu_model* m = s->m;
  if (prefix + n + steps - 1 > m->max_pos) return fail(TCU_EINVAL, "generation exceeds the context length %d", m->max_pos);
  CK(cudaSetDevice(m->device));
  ProfScope ps(s);
  int rc = session_run(s, prefix, tokens, n, nullptr);
  if (rc == TCU_OK && s->prof.on) {
    rc = session_sync(s);
    prof_collect(s);
  }
  const int end = prefix + n + steps - 1;  // resident positions afterwards
  if (rc == TCU_OK) rc = prepare_pages(m, s->pool, s->pages, prefix + n, end, s->stream);
  if (rc == TCU_OK) rc = upload_pt(s);
  if (rc == TCU_OK && m->mega && steps > 1) {
    // Persistent decode: one cooperative launch per generated token.
    // TCU_TEST_HOLD_ARRIVAL=<layer> makes the first launch hold back one
    // arrival in that layer (a failure-detection test: its waits run out).
    const char* hold = getenv("TCU_TEST_HOLD_ARRIVAL");
    s->hold_layer = (hold && *hold) ? std::max(-1, std::min(m->L - 1, atoi(hold))) : -1;
    const int first = prefix + n;
    CK(cudaMemcpyAsync(s->w->pos, &first, sizeof(int), cudaMemcpyHostToDevice, s->stream));
    CK(cudaMemcpyAsync(s->w->keys, s->w->argmax, sizeof(unsigned long long), cudaMemcpyDeviceToDevice, s->stream));
    CK(cudaMemsetAsync(s->w->keys + 1, 0, sizeof(unsigned long long), s->stream));
    CK(cudaMemsetAsync(s->w->step, 0, sizeof(int), s->stream));
    CK(cudaMemsetAsync(s->w->out_count, 0, sizeof(int), s->stream));
    // Work and arrival counters start at zero (a run cut short by a timeout
    // may have left them set).
    const size_t nctl = (size_t)2 * (m->L + 1) * MG_CTL * sizeof(int);
    CK(cudaMemsetAsync(s->w->grab, 0, nctl, s->stream));
    CK(cudaMemsetAsync(s->w->done, 0, nctl, s->stream));
    CK(cudaMemsetAsync(s->w->counters, 0, (size_t)m->KVH * sizeof(int), s->stream));
    for (int i = 1; rc == TCU_OK && i < steps; i++) {
      rc = launch_mega(s);
      if (rc == TCU_OK && s->prof.on) {
        rc = session_sync(s);
        prof_collect(s);
      }
    }
    if (rc == TCU_OK) {
      k_finish_mega<<<1, 32, 0, s->stream>>>(s->w->keys, s->w->step, s->w->out_tokens, s->w->out_count);
      NOTE("k_finish_mega");
      cudaError_t e = cudaMemcpyAsync(out_tokens, s->w->out_tokens, (size_t)steps * sizeof(int), cudaMemcpyDeviceToHost, s->stream);
      if (e != cudaSuccess) rc = fail(TCU_ECUDA, "token copy: %s", cudaGetErrorString(e));
    }
    return session_finish(s, rc, end);
  }
  if (rc == TCU_OK) {
    const int last = prefix + n - 1;
    cudaMemcpyAsync(s->w->pos, &last, sizeof(int), cudaMemcpyHostToDevice, s->stream);
    NOTE("cudaMemcpyAsync(s->w->pos, &last, sizeof(");
    cudaMemsetAsync(s->w->out_count, 0, sizeof(int), s->stream);
    NOTE("cudaMemsetAsync(s->w->out_count, 0, sizeo");
    const int split = SPLIT_PAGES * m->P;
    int splits = (end + split - 1) / split;
    int bucket = 1;
    while (bucket < splits) bucket *= 2;
    bucket = std::min(bucket, s->w->max_splits);
    // Tensor-parallel models on NCCL enqueue each step (the all-reduce stays
    // out of captured graphs); others, the peer exchange included, replay one
    // captured step.
    const bool tp = m->tp_world > 1 && !m->tp_ex_on;
    if (steps > 1 && !tp) rc = session_graph(s, bucket);
    for (int i = 1; rc == TCU_OK && i < steps; i++) {
      if (tp) {
        enqueue_decode(m, s->pool, s->w, 1, true, bucket, true, s->stream);
        rc = comm_check();
        if (rc == TCU_OK && s->prof.on) {
          rc = session_sync(s);
          prof_collect(s);
        }
        continue;
      }
      cudaError_t e = cudaGraphLaunch(s->graph, s->stream);
      if (e != cudaSuccess) rc = fail(TCU_ECUDA, "graph launch: %s", cudaGetErrorString(e));
      if (rc == TCU_OK && s->prof.on) {
        // Events inside the graph are re-recorded by every replay.
        rc = session_sync(s);
        s->prof.collect(s->graph_events);
      }
    }
    if (rc == TCU_OK) {
      k_finish_greedy<<<1, 32, 0, s->stream>>>(s->w->argmax, s->w->out_tokens, s->w->out_cap, s->w->out_count, 1);
      NOTE("k_finish_greedy");
      cudaError_t e = cudaMemcpyAsync(out_tokens, s->w->out_tokens, (size_t)steps * sizeof(int), cudaMemcpyDeviceToHost, s->stream);
      if (e != cudaSuccess) rc = fail(TCU_ECUDA, "token copy: %s", cudaGetErrorString(e));
    }
  }
  return session_finish(s, rc, end);
}

int tcu_session_shortlist(tcu_session* s, int32_t k, int32_t* ids, float* logits, double* logsumexp, int32_t* n_out) {
  if (!s || !ids || !logits || !logsumexp || !n_out) return fail(TCU_EINVAL, "null argument");
  if (s->closed) return fail(TCU_ECLOSED, "session is closed");
  if (k < 1 || k > 256) return fail(TCU_EINVAL, "shortlist size must be in [1, 256]");
  if (s->length == 0) return fail(TCU_EINVAL, "no logits: forward first");
  CK(cudaSetDevice(s->m->device));
  const int kk = std::min<int>(k, s->m->V);
  const size_t smem = ((size_t)s->m->V + 31) / 32 * 4;  // attribute set at load (sampling_smem_attrs)
  k_shortlist<<<1, 1024, smem, s->stream>>>(s->w->logits, s->m->V, kk, s->w->sl_ids, s->w->sl_vals, s->w->sl_lse);
  NOTE("k_shortlist");
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(ids, s->w->sl_ids, kk * sizeof(int), cudaMemcpyDeviceToHost, s->stream));
  CK(cudaMemcpyAsync(logits, s->w->sl_vals, kk * sizeof(float), cudaMemcpyDeviceToHost, s->stream));
  CK(cudaMemcpyAsync(logsumexp, s->w->sl_lse, sizeof(double), cudaMemcpyDeviceToHost, s->stream));
  TRY(session_sync(s));
  *n_out = kk;
  return TCU_OK;
}

int tcu_session_forward_logprobs(tcu_session* s, int32_t prefix, const int32_t* tokens, const int32_t* targets, int32_t n,
                                 int32_t count, double* chosen, int32_t* top_ids, double* top_logprobs, float* logits_out) {
  TRY(validate_forward(s, prefix, tokens, n));
  if (!targets || !chosen || !top_ids || !top_logprobs) return fail(TCU_EINVAL, "null argument");
  // mlx_native.go:303-313
  if (count < 1 || count > s->m->V || count > 256) return fail(TCU_EINVAL, "invalid probability request (count %d)", count);
  for (int i = 0; i < n; i++)
    if (targets[i] < 0 || targets[i] >= s->m->V) return fail(TCU_EINVAL, "invalid probability target %d", targets[i]);
  CK(cudaSetDevice(s->m->device));
  ProfScope ps(s);
  const LogprobReq lp{targets, count, chosen, top_ids, top_logprobs};
  int rc = session_run(s, prefix, tokens, n, nullptr, &lp);
  if (rc == TCU_OK && logits_out) {
    cudaError_t e = cudaMemcpyAsync(logits_out, s->w->logits, (size_t)s->m->V * 4, cudaMemcpyDeviceToHost, s->stream);
    if (e != cudaSuccess) rc = fail(TCU_ECUDA, "logits copy: %s", cudaGetErrorString(e));
  }
  return session_finish(s, rc, prefix + n);
}

int tcu_session_sample_candidates(tcu_session* s, const int32_t* history, int32_t n_history, const tcu_penalties* p, int32_t k,
                                  int32_t* ids, double* scores, int32_t* n_out) {
  if (!s || !ids || !scores || !n_out || (n_history > 0 && !history) || n_history < 0) return fail(TCU_EINVAL, "null argument");
  if (s->closed) return fail(TCU_ECLOSED, "session is closed");
  if (k < 1 || k > 256) return fail(TCU_EINVAL, "candidate count must be in [1, 256]");
  if (s->length == 0) return fail(TCU_EINVAL, "no logits: forward first");
  const tcu_penalties neutral{1.0, 0.0, 0.0, 0.0, 0};
  const tcu_penalties& pp = p ? *p : neutral;
  TRY(penalties_check(pp));
  CK(cudaSetDevice(s->m->device));
  const int kk = std::min<int>(k, s->m->V);
  PenaltyHost h;
  penalties_add_row(h, history, n_history, pp, s->m->V);
  TRY(enqueue_candidates(s->m, s->w, s->w->logits, 1, h, kk, s->stream));
  CK(cudaMemcpyAsync(ids, s->w->cd_ids, kk * sizeof(int), cudaMemcpyDeviceToHost, s->stream));
  CK(cudaMemcpyAsync(scores, s->w->cd_vals, kk * sizeof(double), cudaMemcpyDeviceToHost, s->stream));
  TRY(session_sync(s));
  *n_out = kk;
  return TCU_OK;
}

// KV snapshots (cache_file.go:16-258) of a session's resident positions.

// Device staging for one layer of the payload, freed on every return path.
struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

int tcu_session_save_cache(tcu_session* s, const char* path, const uint8_t* model_sha256, const int32_t* tokens, int32_t n_tokens) {
  if (!s || !path || !model_sha256 || (n_tokens > 0 && !tokens)) return fail(TCU_EINVAL, "null argument");
  if (s->closed) return fail(TCU_ECLOSED, "session is closed");
  if (s->branches_open) return fail(TCU_EINVAL, "close the open branches first");
  if (n_tokens != s->length) return fail(TCU_EINVAL, "%d tokens given for %d resident positions", n_tokens, s->length);
  tcu_model* m = s->m;
  CK(cudaSetDevice(m->device));
  CK(cudaStreamSynchronize(s->stream));
  const std::string js = kv_header_json(model_sha256, s->half != 0, tokens, n_tokens);
  // A temporary file beside the target, renamed over it when complete
  // (SaveCache writes the same way, with mode 0600: prompt-derived data).
  std::string dir = path;
  const size_t slash = dir.find_last_of('/');
  dir = slash == std::string::npos ? std::string(".") : dir.substr(0, slash == 0 ? 1 : slash);
  std::string tmpl = dir + "/.tinyoai-kv-XXXXXX";
  std::vector<char> name(tmpl.begin(), tmpl.end());
  name.push_back('\0');
  const int fd = mkstemp(name.data());
  if (fd < 0) return fail(TCU_EINVAL, "cannot create a file beside %s: %s", path, strerror(errno));
  fchmod(fd, 0600);
  FILE* f = fdopen(fd, "wb");
  if (!f) {
    close(fd);
    unlink(name.data());
    return fail(TCU_EINVAL, "fdopen: %s", strerror(errno));
  }
  auto abandon = [&](int code) {
    fclose(f);
    unlink(name.data());
    return code;
  };
  Sha256 dg;
  auto put = [&](const void* p, size_t n) {
    dg.update(p, n);
    return fwrite(p, 1, n, f) == n;
  };
  uint8_t prefix[12];
  memcpy(prefix, "TNYKV001", 8);
  const uint32_t hl = (uint32_t)js.size();
  memcpy(prefix + 8, &hl, 4);
  if (!put(prefix, 12) || !put(js.data(), js.size())) return abandon(fail(TCU_EINVAL, "write %s: %s", path, strerror(errno)));
  if (n_tokens > 0) {
    const int es = s->half ? 2 : 4;
    const size_t layer_bytes = (size_t)m->KVH * 2 * n_tokens * m->hd * es;
    DevBuf dbuf;
    if (cudaMalloc(&dbuf.p, layer_bytes) != cudaSuccess) {
      cudaGetLastError();
      return abandon(fail(TCU_ENOMEM, "snapshot staging: cannot allocate %zu bytes", layer_bytes));
    }
    std::vector<uint8_t> hbuf(layer_bytes);
    int rc = upload_pt(s);
    if (rc != TCU_OK) return abandon(rc);
    for (int l = 0; l < m->L; l++) {
      k_kv_gather<<<m->sm_count * 4, 256, 0, s->stream>>>(s->pool->view(), l, s->w->pt, n_tokens, (uint8_t*)dbuf.p);
      if (cudaMemcpyAsync(hbuf.data(), dbuf.p, layer_bytes, cudaMemcpyDeviceToHost, s->stream) != cudaSuccess ||
          cudaStreamSynchronize(s->stream) != cudaSuccess)
        return abandon(fail(TCU_ECUDA, "snapshot copy: %s", cudaGetErrorString(cudaGetLastError())));
      if (!put(hbuf.data(), layer_bytes)) return abandon(fail(TCU_EINVAL, "write %s: %s", path, strerror(errno)));
    }
  }
  uint8_t sum[32];
  dg.final(sum);
  if (fwrite(sum, 1, 32, f) != 32 || fflush(f) != 0 || fsync(fileno(f)) != 0)
    return abandon(fail(TCU_EINVAL, "write %s: %s", path, strerror(errno)));
  if (fclose(f) != 0) {
    unlink(name.data());
    return fail(TCU_EINVAL, "close %s: %s", path, strerror(errno));
  }
  if (rename(name.data(), path) != 0) {
    unlink(name.data());
    return fail(TCU_EINVAL, "rename to %s: %s", path, strerror(errno));
  }
  return TCU_OK;
}

int tcu_session_load_cache(tcu_session* s, const char* path, const uint8_t* model_sha256, int32_t* tokens, int32_t capacity,
                           int32_t* n_tokens) {
  if (!s || !path || !model_sha256 || !n_tokens || (capacity > 0 && !tokens)) return fail(TCU_EINVAL, "null argument");
  if (s->closed) return fail(TCU_ECLOSED, "session is closed");
  if (s->branches_open) return fail(TCU_EINVAL, "close the open branches first");
  tcu_model* m = s->m;
  FILE* f = fopen(path, "rb");
  if (!f) return fail(TCU_EINVAL, "open %s: %s", path, strerror(errno));
  struct FileCloser {
    FILE* f;
    ~FileCloser() { fclose(f); }
  } closer{f};
  Sha256 dg;
  auto get = [&](void* p, size_t n) {
    if (fread(p, 1, n, f) != n) return false;
    dg.update(p, n);
    return true;
  };
  uint8_t prefix[12];
  if (!get(prefix, 12)) return fail(TCU_EINVAL, "KV cache: unexpected end of file");
  if (memcmp(prefix, "TNYKV001", 8) != 0) return fail(TCU_EINVAL, "unsupported KV cache format");
  uint32_t hl;
  memcpy(&hl, prefix + 8, 4);
  if (hl > (1u << 20)) return fail(TCU_EINVAL, "KV cache header too large");
  std::string js(hl, '\0');
  if (hl && !get(&js[0], hl)) return fail(TCU_EINVAL, "KV cache: unexpected end of file");
  uint8_t model[32];
  bool half = false;
  std::vector<int32_t> toks;
  if (!kv_header_parse(js, model, &half, &toks)) return fail(TCU_EINVAL, "KV cache header is not valid");
  // LoadCache's checks, in its order (cache_file.go:128-153).
  if ((int64_t)toks.size() > m->max_pos) return fail(TCU_EINVAL, "KV cache exceeds model context");
  for (int32_t id : toks)
    if (id < 0 || id >= m->V) return fail(TCU_EINVAL, "invalid KV cache token %d", id);
  if (memcmp(model, model_sha256, 32) != 0) return fail(TCU_EINVAL, "KV cache model does not match checkpoint");
  if (half != (s->half != 0)) return fail(TCU_EINVAL, "KV cache precision does not match model options");
  const int T = (int)toks.size();
  const int es = half ? 2 : 4;
  const uint64_t values = (uint64_t)m->L * 2 * m->KVH * m->hd * T;
  const uint64_t expected = 12 + (uint64_t)hl + values * es + 32;
  struct stat st;
  if (fstat(fileno(f), &st) != 0 || (uint64_t)st.st_size != expected)
    return fail(TCU_EINVAL, "KV cache size %lld, expected %llu", (long long)st.st_size, (unsigned long long)expected);
  if (T > capacity) return fail(TCU_EINVAL, "token buffer holds %d of %d snapshot tokens", capacity, T);
  CK(cudaSetDevice(m->device));
  CK(cudaStreamSynchronize(s->stream));
  // Fresh pages for the restored positions; the session keeps its own until
  // the whole file is verified.
  std::vector<int> pages;
  auto drop = [&](int code) {
    release_pages(m, s->pool, pages, 0);
    return code;
  };
  if (T > 0) {
    int rc = prepare_pages(m, s->pool, pages, 0, T, s->stream);
    if (rc != TCU_OK) return drop(rc);
    const size_t layer_bytes = (size_t)m->KVH * 2 * T * m->hd * es;
    DevBuf dbuf, dpt;
    if (cudaMalloc(&dbuf.p, layer_bytes) != cudaSuccess || cudaMalloc(&dpt.p, pages.size() * sizeof(int)) != cudaSuccess) {
      cudaGetLastError();
      return drop(fail(TCU_ENOMEM, "snapshot staging: cannot allocate %zu bytes", layer_bytes));
    }
    std::vector<uint8_t> hbuf(layer_bytes);
    if (cudaMemcpy(dpt.p, pages.data(), pages.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
      return drop(fail(TCU_ECUDA, "snapshot page table copy failed"));
    for (int l = 0; l < m->L; l++) {
      if (!get(hbuf.data(), layer_bytes)) return drop(fail(TCU_EINVAL, "KV cache: unexpected end of file"));
      if (cudaMemcpyAsync(dbuf.p, hbuf.data(), layer_bytes, cudaMemcpyHostToDevice, s->stream) != cudaSuccess)
        return drop(fail(TCU_ECUDA, "snapshot copy failed"));
      k_kv_scatter<<<m->sm_count * 4, 256, 0, s->stream>>>(s->pool->view(), l, (const int*)dpt.p, T, (const uint8_t*)dbuf.p);
      if (cudaStreamSynchronize(s->stream) != cudaSuccess)
        return drop(fail(TCU_ECUDA, "snapshot scatter: %s", cudaGetErrorString(cudaGetLastError())));
    }
  }
  uint8_t want[32], got[32];
  dg.final(want);
  if (fread(got, 1, 32, f) != 32 || memcmp(got, want, 32) != 0) return drop(fail(TCU_EINVAL, "KV cache checksum mismatch"));
  // Verified: the restored positions replace the session's context.
  release_pages(m, s->pool, s->pages, 0);
  s->pages.swap(pages);
  s->length = T;
  if (T > 0) memcpy(tokens, toks.data(), (size_t)T * sizeof(int32_t));
  *n_tokens = T;
  return TCU_OK;
}

int tcu_session_fork(tcu_session* s, tcu_session** child) {
  if (!s || !child) return fail(TCU_EINVAL, "null argument");
  if (s->closed) return fail(TCU_ECLOSED, "session is closed");
  tcu_session* c = nullptr;
  TRY(tcu_session_new(s->m, s->half ? TCU_F16 : TCU_F32, &c));
  CK(cudaStreamSynchronize(s->stream));
  for (int pg : s->pages) page_ref(s->m, s->pool, pg);
  c->pages = s->pages;
  c->length = s->length;
  // The child starts with the parent's last logits row (sessions.go:36-72
  // keeps probability rows; the next Forward recomputes them anyway).
  CK(cudaMemcpyAsync(c->w->logits, s->w->logits, (size_t)s->m->V * 4, cudaMemcpyDeviceToDevice, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  *child = c;
  return TCU_OK;
}

int tcu_session_limit(tcu_session* s, int32_t window, int32_t* cleared) {
  if (!s) return fail(TCU_EINVAL, "null session");
  if (window <= 0 || window > s->m->max_pos) return fail(TCU_EINVAL, "invalid window %d", window);
  int c = 0;
  if (s->length > window) {
    cudaStreamSynchronize(s->stream);
    session_invalidate(s);
    c = 1;
  }
  if (cleared) *cleared = c;
  return TCU_OK;
}

int tcu_session_set_kv_dtype(tcu_session* s, int32_t kv_dtype, int32_t* cleared) {
  if (!s) return fail(TCU_EINVAL, "null session");
  if (kv_dtype != TCU_F32 && kv_dtype != TCU_F16) return fail(TCU_EINVAL, "unsupported KV cache precision %d", kv_dtype);
  const int half = kv_dtype == TCU_F16;
  int c = 0;
  if (half != s->half) {
    if (s->branches_open) return fail(TCU_EINVAL, "close the open branches first");
    KVPool* p = nullptr;
    TRY(pool_get(s->m, half, &p));
    cudaStreamSynchronize(s->stream);
    c = s->length > 0;
    session_invalidate(s);
    if (s->graph) {
      cudaGraphExecDestroy(s->graph);
      s->graph = nullptr;
      s->graph_splits = 0;
    }
    s->pool = p;
    s->half = half;
  }
  if (cleared) *cleared = c;
  return TCU_OK;
}

int tcu_session_reset(tcu_session* s) {
  if (!s) return fail(TCU_EINVAL, "null session");
  cudaStreamSynchronize(s->stream);
  session_invalidate(s);
  return TCU_OK;
}

int tcu_session_set_stream(tcu_session* s, void* stream) {
  if (!s) return fail(TCU_EINVAL, "null session");
  if (s->closed) return fail(TCU_ECLOSED, "session is closed");
  CK(cudaSetDevice(s->m->device));
  CK(cudaStreamSynchronize(s->stream));
  cudaStream_t next = stream ? (cudaStream_t)stream : s->own_stream;
  if (next != s->stream && s->graph) {
    cudaGraphExecDestroy(s->graph);
    s->graph = nullptr;
    s->graph_splits = 0;
  }
  s->stream = next;
  return TCU_OK;
}

int tcu_session_profile(tcu_session* s, int32_t enable) {
  if (!s) return fail(TCU_EINVAL, "null session");
  s->prof.on = enable != 0;
  s->prof.used = 0;
  return TCU_OK;
}

int tcu_session_profile_read(tcu_session* s, int32_t n_stages, int64_t* launches, double* ms, int32_t reset) {
  if (!s || !launches || !ms) return fail(TCU_EINVAL, "null argument");
  for (int i = 0; i < n_stages && i < ST_COUNT; i++) {
    launches[i] = s->prof.launches[i];
    ms[i] = s->prof.ms[i];
  }
  if (reset)
    for (int i = 0; i < ST_COUNT; i++) {
      s->prof.launches[i] = 0;
      s->prof.ms[i] = 0;
    }
  return ST_COUNT;
}

int tcu_branches_open(tcu_session* s, int32_t prefix, int32_t count, tcu_branches** out) {
  if (!s || !out) return fail(TCU_EINVAL, "null argument");
  if (s->closed) return fail(TCU_ECLOSED, "session is closed");
  // mlx_branches.go:25-32 (GQA is supported here).
  if (prefix < 0 || prefix > s->length || count < 1 || count > s->m->V || prefix >= s->m->max_pos)
    return fail(TCU_EINVAL, "invalid branch prefix or batch size");
  CK(cudaSetDevice(s->m->device));
  tcu_branches* b = new tcu_branches();
  b->s = s;
  b->prefix = prefix;
  b->count = count;
  int rc = work_take(s->m, &b->w, count, count, count, 2);
  if (rc != TCU_OK) {
    delete b;
    return rc;
  }
  CK(cudaStreamSynchronize(s->stream));
  const size_t shared = (size_t)(prefix + s->m->P - 1) / s->m->P;
  b->pages.resize(count);
  for (int i = 0; i < count; i++) {
    b->pages[i].assign(s->pages.begin(), s->pages.begin() + shared);
    for (int pg : b->pages[i]) page_ref(s->m, s->pool, pg);
  }
  s->branches_open++;
  *out = b;
  return TCU_OK;
}

int tcu_branches_forward(tcu_branches* b, const int32_t* tokens, float* rows_out) {
  if (!b) return fail(TCU_EINVAL, "null branches");
  if (b->closed) return fail(TCU_ECLOSED, "token branches are closed");
  tcu_session* s = b->s;
  tcu_model* m = s->m;
  if (b->prefix + b->step >= m->max_pos) return fail(TCU_EINVAL, "invalid branch batch or context length");
  TRY(check_tokens(m, tokens, b->count));
  CK(cudaSetDevice(m->device));
  ProfScope ps(s, b->w->err);
  const int pos = b->prefix + b->step;
  int rc = TCU_OK;
  std::vector<int> pt((size_t)b->count * b->w->pt_stride, 0);
  for (int i = 0; rc == TCU_OK && i < b->count; i++) {
    rc = prepare_pages(m, s->pool, b->pages[i], pos, pos + 1, s->stream);
    std::copy(b->pages[i].begin(), b->pages[i].end(), pt.begin() + (size_t)i * b->w->pt_stride);
  }
  if (rc == TCU_OK) {
    std::vector<int> posv(b->count, pos);
    cudaMemcpyAsync(b->w->pt, pt.data(), pt.size() * sizeof(int), cudaMemcpyHostToDevice, s->stream);
    NOTE("cudaMemcpyAsync(b->w->pt, pt.data(), pt.s");
    cudaMemcpyAsync(b->w->pos, posv.data(), b->count * sizeof(int), cudaMemcpyHostToDevice, s->stream);
    NOTE("cudaMemcpyAsync(b->w->pos, posv.data(), b");
    cudaMemcpyAsync(b->w->tokens, tokens, b->count * sizeof(int), cudaMemcpyHostToDevice, s->stream);
    NOTE("cudaMemcpyAsync(b->w->tokens, tokens, b->");
    cudaMemsetAsync(b->w->argmax, 0, b->count * sizeof(unsigned long long), s->stream);
    NOTE("cudaMemsetAsync(b->w->argmax, 0, b->count");
    const int split = SPLIT_PAGES * m->P;
    // Whole splits inside the prefix's full pages are shared by every branch.
    b->w->shared_splits = (b->prefix / m->P) / SPLIT_PAGES;
    enqueue_decode(m, s->pool, b->w, b->count, false, (pos + 1 + split - 1) / split, true, s->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = fail(TCU_ECUDA, "launch: %s", cudaGetErrorString(e));
    if (rc == TCU_OK) rc = comm_check();
    if (rc == TCU_OK && rows_out) {
      e = cudaMemcpyAsync(rows_out, b->w->logits, (size_t)b->count * m->V * 4, cudaMemcpyDeviceToHost, s->stream);
      if (e != cudaSuccess) rc = fail(TCU_ECUDA, "rows copy: %s", cudaGetErrorString(e));
    }
  }
  if (rc == TCU_OK) rc = sync_stream(s->stream, b->w->err);
  if (rc == TCU_OK) prof_collect(s);
  s->prof.used = 0;
  if (rc != TCU_OK) {
    // mlx_branches.go:176-178: evaluation errors close the suffix caches; the
    // handle stays valid until tcu_branches_close.
    std::string msg = g_err;
    branches_release(b);
    g_err = msg;
    return rc;
  }
  b->step++;
  return TCU_OK;
}

int tcu_branches_argmax(tcu_branches* b, int32_t* ids) {
  if (!b || !ids) return fail(TCU_EINVAL, "null argument");
  if (b->closed) return fail(TCU_ECLOSED, "token branches are closed");
  if (b->step == 0) return fail(TCU_EINVAL, "no rows: forward first");
  std::vector<unsigned long long> keys(b->count);
  CK(cudaMemcpy(keys.data(), b->w->argmax, b->count * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
  for (int i = 0; i < b->count; i++) ids[i] = (int)(0xffffffffu - (uint32_t)(keys[i] & 0xffffffffu));
  return TCU_OK;
}

int tcu_branches_close(tcu_branches* b) {
  if (!b) return TCU_OK;
  branches_release(b);  // synchronises the session's stream
  work_give(b->s->m, b->w);
  delete b;
  return TCU_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Continuous batching: one decode step for several independent sessions of
// one model, each at its own position (a server's active requests). The
// per-row kernels take each row's position and page table, so the step is
// the branch step with unrelated rows.
struct tcu_batch {
  tcu_model* m = nullptr;
  int max_rows = 0;
  int last_rows = 0;  // rows of the last successful step (their logits stay in w->logits)
  Work* w = nullptr;  // from the model's workspace pool (work_take)
  cudaStream_t stream = nullptr;
};

extern "C" {

int tcu_batch_open(tcu_model* m, int32_t max_rows, tcu_batch** out) {
  if (!m || !out) return fail(TCU_EINVAL, "null argument");
  if (max_rows < 1 || max_rows > 1024) return fail(TCU_EINVAL, "batch size %d outside 1..1024", max_rows);
  CK(cudaSetDevice(m->device));
  tcu_batch* b = new tcu_batch();
  b->m = m;
  b->max_rows = max_rows;
  int rc = work_take(m, &b->w, max_rows, max_rows, max_rows, 2);
  if (rc == TCU_OK && cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking) != cudaSuccess)
    rc = fail(TCU_ECUDA, "stream creation failed");
  if (rc != TCU_OK) {
    if (b->stream) cudaStreamDestroy(b->stream);
    work_give(m, b->w);
    delete b;
    return rc;
  }
  *out = b;
  return TCU_OK;
}

int tcu_batch_forward(tcu_batch* b, tcu_session* const* sessions, const int32_t* tokens, int32_t n, float* rows_out,
                      int32_t* ids_out) {
  if (!b || !sessions || !tokens) return fail(TCU_EINVAL, "null argument");
  if (n < 1 || n > b->max_rows) return fail(TCU_EINVAL, "batch of %d rows outside 1..%d", n, b->max_rows);
  tcu_model* m = b->m;
  KVPool* pool = nullptr;
  for (int i = 0; i < n; i++) {
    tcu_session* s = sessions[i];
    if (!s || s->m != m) return fail(TCU_EINVAL, "row %d: not a session of this model", i);
    if (s->closed) return fail(TCU_ECLOSED, "row %d: session is closed", i);
    if (s->branches_open) return fail(TCU_EINVAL, "row %d: session has open branches", i);
    if (s->length < 1 || s->length >= m->max_pos) return fail(TCU_EINVAL, "row %d: invalid position %d", i, s->length);
    if (pool && s->pool != pool) return fail(TCU_EINVAL, "rows mix KV precisions");
    pool = s->pool;
    for (int j = 0; j < i; j++)
      if (sessions[j] == s) return fail(TCU_EINVAL, "session appears twice in the batch");
  }
  TRY(check_tokens(m, tokens, n));
  CK(cudaSetDevice(m->device));
  ProfScope ps(nullptr, b->w->err);
  // Each session's earlier work precedes this step.
  for (int i = 0; i < n; i++) CK(cudaStreamSynchronize(sessions[i]->stream));
  int rc = TCU_OK, max_len = 0;
  std::vector<int> pt((size_t)n * b->w->pt_stride, 0), posv(n);
  for (int i = 0; rc == TCU_OK && i < n; i++) {
    tcu_session* s = sessions[i];
    rc = prepare_pages(m, pool, s->pages, s->length, s->length + 1, b->stream);
    std::copy(s->pages.begin(), s->pages.end(), pt.begin() + (size_t)i * b->w->pt_stride);
    posv[i] = s->length;
    max_len = std::max(max_len, s->length + 1);
  }
  if (rc == TCU_OK) {
    cudaMemcpyAsync(b->w->pt, pt.data(), pt.size() * sizeof(int), cudaMemcpyHostToDevice, b->stream);
    cudaMemcpyAsync(b->w->pos, posv.data(), n * sizeof(int), cudaMemcpyHostToDevice, b->stream);
    cudaMemcpyAsync(b->w->tokens, tokens, n * sizeof(int), cudaMemcpyHostToDevice, b->stream);
    cudaMemsetAsync(b->w->argmax, 0, n * sizeof(unsigned long long), b->stream);
    const int split = SPLIT_PAGES * m->P;
    b->w->shared_splits = 0;
    enqueue_decode(m, pool, b->w, n, false, (max_len + split - 1) / split, true, b->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = fail(TCU_ECUDA, "launch: %s", cudaGetErrorString(e));
    if (rc == TCU_OK) rc = comm_check();
    if (rc == TCU_OK && rows_out) {
      e = cudaMemcpyAsync(rows_out, b->w->logits, (size_t)n * m->V * 4, cudaMemcpyDeviceToHost, b->stream);
      if (e != cudaSuccess) rc = fail(TCU_ECUDA, "rows copy: %s", cudaGetErrorString(e));
    }
  }
  std::vector<unsigned long long> keys(n);
  if (rc == TCU_OK && ids_out) {
    cudaError_t e = cudaMemcpyAsync(keys.data(), b->w->argmax, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost, b->stream);
    if (e != cudaSuccess) rc = fail(TCU_ECUDA, "argmax copy: %s", cudaGetErrorString(e));
  }
  if (rc == TCU_OK) rc = sync_stream(b->stream, b->w->err);
  if (rc != TCU_OK) return rc;  // lengths unchanged: the new positions are rewritten next time
  if (ids_out)
    for (int i = 0; i < n; i++) ids_out[i] = (int)(0xffffffffu - (uint32_t)(keys[i] & 0xffffffffu));
  for (int i = 0; i < n; i++) sessions[i]->length++;
  b->last_rows = n;
  return TCU_OK;
}

int tcu_batch_sample_candidates(tcu_batch* b, int32_t n, const int32_t* history, const int32_t* history_len, const tcu_penalties* p,
                                int32_t k, int32_t* ids, double* scores) {
  if (!b || !history_len || !p || !ids || !scores) return fail(TCU_EINVAL, "null argument");
  if (n < 1 || n > b->last_rows) return fail(TCU_EINVAL, "%d rows requested, the last step had %d", n, b->last_rows);
  if (k < 1 || k > 256 || k > b->m->V) return fail(TCU_EINVAL, "candidate count must be in [1, min(256, vocab)]");
  PenaltyHost h;
  size_t off = 0;
  for (int i = 0; i < n; i++) {
    if (history_len[i] < 0 || (history_len[i] > 0 && !history)) return fail(TCU_EINVAL, "row %d: invalid history", i);
    TRY(penalties_check(p[i]));
    penalties_add_row(h, history + off, history_len[i], p[i], b->m->V);
    off += (size_t)history_len[i];
  }
  CK(cudaSetDevice(b->m->device));
  TRY(enqueue_candidates(b->m, b->w, b->w->logits, n, h, k, b->stream));
  CK(cudaMemcpyAsync(ids, b->w->cd_ids, (size_t)n * k * sizeof(int), cudaMemcpyDeviceToHost, b->stream));
  CK(cudaMemcpyAsync(scores, b->w->cd_vals, (size_t)n * k * sizeof(double), cudaMemcpyDeviceToHost, b->stream));
  return sync_stream(b->stream, b->w->err);
}

int tcu_batch_close(tcu_batch* b) {
  if (!b) return TCU_OK;
  cudaSetDevice(b->m->device);
  if (b->stream) {
    cudaStreamSynchronize(b->stream);
    cudaStreamDestroy(b->stream);
  }
  work_give(b->m, b->w);
  delete b;
  return TCU_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// weightTensor.readValues (matmul.go:12-50) through the device decoders.

namespace {
// Device buffers of one tcu_read_values call, freed on every return path.
struct ReadBufs {
  std::vector<void*> p;
  ~ReadBufs() {
    for (void* q : p) cudaFree(q);
  }
  int get(void** out, size_t bytes) {
    *out = nullptr;
    cudaError_t e = cudaMalloc(out, std::max<size_t>(bytes, 16));
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(e == cudaErrorMemoryAllocation ? TCU_ENOMEM : TCU_ECUDA, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    p.push_back(*out);
    return TCU_OK;
  }
};
}  // namespace

extern "C" int tcu_read_values(int32_t device, int32_t dtype, const void* data, uint64_t nbytes, int32_t rows, int32_t cols,
                               int64_t offset, int64_t n, int32_t decoder, float* out) {
  if (!data || (n > 0 && !out)) return fail(TCU_EINVAL, "null argument");
  if (!fmt_known(dtype)) return fail(TCU_EUNSUP, "unsupported dtype %d", dtype);
  if (rows <= 0 || cols <= 0) return fail(TCU_EINVAL, "invalid shape %d x %d", rows, cols);
  if ((dtype == FMT_Q8_0 || dtype == FMT_Q5_1) && cols % 32) return fail(TCU_EINVAL, "rows of this format must be divisible by 32");
  if ((dtype == FMT_Q5_K || dtype == FMT_Q6_K) && cols % 256) return fail(TCU_EINVAL, "K-quant rows must be divisible by 256");
  if (nbytes != file_bytes(dtype, rows, cols))
    return fail(TCU_EINVAL, "%llu bytes, want %zu", (unsigned long long)nbytes, file_bytes(dtype, rows, cols));
  const int64_t total = (int64_t)rows * cols;
  if (offset < 0 || n < 0 || offset > total || n > total - offset)
    return fail(TCU_EINVAL, "read of %lld values at %lld exceeds %lld", (long long)n, (long long)offset, (long long)total);
  const bool kq = dtype == FMT_Q5_K || dtype == FMT_Q6_K;
  if (decoder == RD_GROUP8 && !kq) return fail(TCU_EUNSUP, "the 8-value group decoder serves Q6_K and Q5_K");
  if (decoder == RD_TC && !kq && dtype != FMT_Q8_0) return fail(TCU_EUNSUP, "the tensor-core operand serves Q8_0, Q6_K and Q5_K");
  if (decoder != RD_ELEMENT && decoder != RD_GROUP8 && decoder != RD_TC) return fail(TCU_EINVAL, "unknown decoder %d", decoder);
  TRY(check_device(device));
  if (n == 0) return TCU_OK;
  ReadBufs bufs;
  void *raw = nullptr, *dout = nullptr, *scratch = nullptr;
  TRY(bufs.get(&raw, nbytes));
  TRY(bufs.get(&dout, (size_t)n * 4));
  TRY(bufs.get(&scratch, sizeof(unsigned)));
  CK(cudaMemcpy(raw, data, nbytes, cudaMemcpyHostToDevice));
  DMat W{};
  W.fmt = dtype;
  W.rows = rows;
  W.cols = cols;
  if (dtype == FMT_Q8_0) {
    // The device layout of a loaded Q8_0 matrix, made by the load-time repack.
    W.sstride = (cols / 32 + 7) / 8 * 8;
    void *q = nullptr, *sc = nullptr;
    TRY(bufs.get(&q, (size_t)rows * cols));
    TRY(bufs.get(&sc, (size_t)rows * W.sstride * 2));
    W.w = (const uint8_t*)q;
    W.s = (const __half*)sc;
    RepackArgs ra{(const uint8_t*)raw, dtype, rows, cols, W, 0, 1, 0};
    k_repack<<<1184, 256>>>(ra);
    CK(cudaGetLastError());
  } else {
    // K-quants: the device super-block size of a loaded matrix.
    void* q = nullptr;
    TRY(bufs.get(&q, (size_t)rows * fmt_row_bytes(dtype, cols)));
    W.w = (const uint8_t*)q;
    RepackArgs ra{(const uint8_t*)raw, dtype, rows, cols, W, 0, 1, 0};
    k_repack<<<1184, 256>>>(ra);
    CK(cudaGetLastError());
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (decoder == RD_TC) TRY(tc_shift_of(&W, (unsigned*)scratch, sms));
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8);
  k_read_values<<<blocks, 256>>>(W, offset, n, decoder, (float*)dout);
  CK(cudaGetLastError());
  CK(cudaMemcpy(out, dout, (size_t)n * 4, cudaMemcpyDeviceToHost));
  return TCU_OK;
}

// ---------------------------------------------------------------------------
// Shortlist with no device allocation (tcu_shortlist_static). No counterpart
// in the reference.
//
// Some callers must not allocate device memory when they call: a host whose
// own caching allocator already reserved the free HBM (a cudaMalloc then fails
// or fragments that pool), or a caller on a latency budget, for which
// cudaMalloc's cost and cudaFree's device-wide synchronisation are too much.
// This path runs the unchanged k_shortlist kernel over a logits row the
// caller already holds on the device. Session workspace is not used: the
// kernel's results go to one fixed file-scope device array.
//
// Scratch layout (TCU_SHORTLIST_STATIC_SCRATCH_BYTES):
//   [0, 1024)     int32  ids[TCU_SHORTLIST_STATIC_MAX_K]
//   [1024, 2048)  float  values[TCU_SHORTLIST_STATIC_MAX_K]
//   [2048, 2056)  double logsumexp
// The kernel writes every word the host then reads back (ids and values
// 0..n-1, the log-sum-exp), so nothing has to start at zero and nothing is
// cleared. The array keeps the last call's results. Calls on one device share
// it, so two calls in flight at the same time on one device overwrite each
// other's results.

static_assert(TCU_SHORTLIST_STATIC_MAX_K * 8 + 8 <= TCU_SHORTLIST_STATIC_SCRATCH_BYTES, "shortlist scratch too small");
static_assert(((size_t)TCU_SHORTLIST_STATIC_MAX_VOCAB + 31) / 32 * 4 <= 200 * 1024, "taken bitmap exceeds shared memory");

static __device__ __align__(256) unsigned char g_shortlist_scratch[TCU_SHORTLIST_STATIC_SCRATCH_BYTES];

static const int SL_STATIC_MAX_DEVICES = 64;
static std::mutex g_sl_static_mu;
static unsigned char* g_sl_static_ptr[SL_STATIC_MAX_DEVICES] = {};

// Once per device, with that device current: checks the architecture and
// looks up the device address of g_shortlist_scratch.
static int shortlist_static_setup(int device, unsigned char** out) {
  std::lock_guard<std::mutex> g(g_sl_static_mu);
  if (!g_sl_static_ptr[device]) {
    int major = 0;
    cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    if (e != cudaSuccess) return fail(TCU_ECUDA, "shortlist set-up on device %d: %s", device, cudaGetErrorString(e));
    if (major != 10) return fail(TCU_ENODEV, "device %d is not sm_100; this library is built for sm_100a", device);
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_shortlist_scratch);
    if (e != cudaSuccess || !p)
      return fail(TCU_ECUDA, "shortlist set-up on device %d: cudaGetSymbolAddress: %s", device, cudaGetErrorString(e));
    // The kernel's largest bitmap, once per device (not per call, where
    // another thread could lower it between this call's set and launch).
    TRY(sampling_smem_attrs(device));
    g_sl_static_ptr[device] = (unsigned char*)p;
  }
  *out = g_sl_static_ptr[device];
  return TCU_OK;
}

extern "C" int tcu_shortlist_static(int32_t device, const float* logits, int32_t vocab, int32_t k, void* stream, int32_t* ids,
                                    float* values, double* logsumexp, int32_t* n_out) {
  if (!logits || !ids || !values || !logsumexp || !n_out) return fail(TCU_EINVAL, "null argument");
  if (k < 1 || k > TCU_SHORTLIST_STATIC_MAX_K)
    return fail(TCU_EINVAL, "shortlist size %d is outside [1, %d], the capacity of the static scratch", k, TCU_SHORTLIST_STATIC_MAX_K);
  if (vocab < 1 || vocab > TCU_SHORTLIST_STATIC_MAX_VOCAB)
    return fail(TCU_EINVAL, "vocabulary of %d is outside [1, %d], the largest the static shortlist handles", vocab,
                TCU_SHORTLIST_STATIC_MAX_VOCAB);
  if ((reinterpret_cast<uintptr_t>(logits) & 3) != 0) return fail(TCU_EINVAL, "logits pointer is not 4-byte aligned");
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return fail(TCU_ENODEV, "no CUDA device available");
  }
  if (device < 0 || device >= n || device >= SL_STATIC_MAX_DEVICES)
    return fail(TCU_ENODEV, "device %d out of range (%d devices)", device, n);
  CK(cudaSetDevice(device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The call synchronises the stream and copies into host memory, neither of
  // which a graph can hold.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  CK(cudaStreamIsCapturing(st, &cap));
  if (cap != cudaStreamCaptureStatusNone) return fail(TCU_EINVAL, "the stream is being captured; this call cannot be");
  cudaPointerAttributes pa;
  CK(cudaPointerGetAttributes(&pa, logits));
  if ((pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged) || pa.device != device)
    return fail(TCU_EINVAL, "logits must be device memory on device %d", device);
  unsigned char* scratch = nullptr;
  TRY(shortlist_static_setup(device, &scratch));
  int32_t* d_ids = reinterpret_cast<int32_t*>(scratch);
  float* d_vals = reinterpret_cast<float*>(scratch + TCU_SHORTLIST_STATIC_MAX_K * 4);
  double* d_lse = reinterpret_cast<double*>(scratch + TCU_SHORTLIST_STATIC_MAX_K * 8);
  const int kk = std::min<int>(k, vocab);
  const size_t smem = ((size_t)vocab + 31) / 32 * 4;  // within the attribute set up once per device
  k_shortlist<<<1, 1024, smem, st>>>(logits, vocab, kk, d_ids, d_vals, d_lse);
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(ids, d_ids, kk * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(values, d_vals, kk * sizeof(float), cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(logsumexp, d_lse, sizeof(double), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  *n_out = kk;
  return TCU_OK;
}
