/*
 * CPU oracle: a plain-C restatement of the reference's Go scalar path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h). Every function cites the Go
 * source (path:line inside the wbrown/tinyoai project) whose arithmetic it
 * restates. Build with -ffp-contract=off so that no multiply-add is fused,
 * matching the reference's amd64 code generation. OpenMP splits rows and
 * heads across threads exactly as parallelRows (dot.go:76-89) does: the split
 * never changes the reduction order inside a row or head.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;

void oc_set_threads(int n) {
  g_threads = n;
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#endif
}

int oc_get_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static inline float bits_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint32_t f32_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

/* safetensors.go:250-264 halfFloat */
float oc_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t ex = (h >> 10) & 31, frac = h & 1023;
  if (ex == 0) {
    float v = (float)ldexp((double)frac, -24);
    return sign ? -v : v;
  }
  if (ex == 31) return bits_f32(sign | 0x7f800000u | frac << 13);
  return bits_f32(sign | (ex + 112) << 23 | frac << 13);
}

/* kv_cache.go:27-51 floatHalf: round to nearest even, subnormals, overflow. */
uint16_t oc_float_to_half(float value) {
  uint32_t bits = f32_bits(value);
  uint16_t sign = (uint16_t)(bits >> 16) & 0x8000;
  uint32_t magnitude = bits & 0x7fffffff;
  if (magnitude >= 0x7f800000u) {
    if (magnitude > 0x7f800000u) return sign | 0x7e00;
    return sign | 0x7c00;
  }
  int exponent = (int)(magnitude >> 23) - 127 + 15;
  if (exponent >= 31) return sign | 0x7c00;
  if (exponent <= 0) {
    if (exponent < -10) return sign;
    uint32_t mantissa = (magnitude & 0x7fffff) | 0x800000;
    unsigned shift = (unsigned)(14 - exponent);
    uint32_t rounded = (mantissa + ((1u << (shift - 1)) - 1) + ((mantissa >> shift) & 1)) >> shift;
    return sign | (uint16_t)rounded;
  }
  magnitude += 0xfff + ((magnitude >> 13) & 1);
  return sign | (uint16_t)((magnitude >> 13) - 0x1c000);
}

/* quant_k.go:8-25 */
static int kblock_bytes(int dtype) { return dtype == OC_Q5_1 ? 24 : dtype == OC_Q6_K ? 210 : 176; }
static int kblock_width(int dtype) { return dtype == OC_Q5_1 ? 32 : 256; }

/* quant_k.go:31-86 decodeKBlock; every product and difference is a separate
 * float32 operation. */
void oc_decode_kblock(float* out, const uint8_t* block, int dtype) {
  if (dtype == OC_Q5_1) {
    float d = oc_half_to_float(rd16(block)), minimum = oc_half_to_float(rd16(block + 2));
    uint32_t high = rd32(block + 4);
    for (int i = 0; i < 32; i++) {
      uint8_t low = (block[8 + i % 16] >> (unsigned)(i / 16 * 4)) & 15;
      uint8_t q = low | (uint8_t)(((high >> (unsigned)i) & 1) << 4);
      float prod = d * (float)q;
      out[i] = prod + minimum;
    }
    return;
  }
  if (dtype == OC_Q6_K) {
    float d = oc_half_to_float(rd16(block + 208));
    for (int group = 0; group < 16; group++) {
      float scale = d * (float)(int8_t)block[192 + group];
      for (int j = 0; j < 16; j++) {
        int i = group * 16 + j;
        int low = (block[(i / 128) * 64 + i % 64] >> (unsigned)((i % 128) / 64 * 4)) & 15;
        int high = (block[128 + (i / 128) * 32 + i % 32] >> (unsigned)((i % 128) / 32 * 2)) & 3;
        out[i] = scale * (float)((low | high << 4) - 32);
      }
    }
    return;
  }
  float d = oc_half_to_float(rd16(block));
  float dmin = oc_half_to_float(rd16(block + 2));
  const uint8_t* scales = block + 4;
  for (int group = 0; group < 8; group++) {
    uint8_t scale, minimum;
    if (group < 4) {
      scale = scales[group] & 63;
      minimum = scales[group + 4] & 63;
    } else {
      scale = (scales[group + 4] & 15) | (uint8_t)((scales[group - 4] >> 6) << 4);
      minimum = (scales[group + 4] >> 4) | (uint8_t)((scales[group] >> 6) << 4);
    }
    float ds = d * (float)scale, dm = dmin * (float)minimum;
    for (int j = 0; j < 32; j++) {
      int low = (block[48 + (group / 2) * 32 + j] >> (unsigned)(group % 2 * 4)) & 15;
      int high = (block[16 + j] >> (unsigned)group) & 1;
      float prod = ds * (float)(low | high << 4);
      out[group * 32 + j] = prod - dm;
    }
  }
}

/* safetensors.go:230-246 at() for one element. */
static float tensor_at(const oc_tensor* w, int64_t i) {
  switch (w->dtype) {
    case OC_BF16:
      return bits_f32((uint32_t)rd16(w->data + i * 2) << 16);
    case OC_F16:
      return oc_half_to_float(rd16(w->data + i * 2));
    case OC_Q8_0: {
      const uint8_t* block = w->data + i / 32 * 34;
      return oc_half_to_float(rd16(block)) * (float)(int8_t)block[2 + i % 32];
    }
    case OC_Q5_K:
    case OC_Q6_K:
    case OC_Q5_1: {
      float v;
      oc_read_values(&v, w, i, 1);
      return v;
    }
    default:
      return bits_f32(rd32(w->data + i * 4));
  }
}

/* matmul.go:12-50 readValues */
void oc_read_values(float* out, const oc_tensor* w, int64_t offset, int64_t n) {
  switch (w->dtype) {
    case OC_BF16:
      for (int64_t i = 0; i < n; i++) out[i] = bits_f32((uint32_t)rd16(w->data + (offset + i) * 2) << 16);
      return;
    case OC_F32:
      for (int64_t i = 0; i < n; i++) out[i] = bits_f32(rd32(w->data + (offset + i) * 4));
      return;
    case OC_Q8_0:
      for (int64_t i = 0; i < n;) {
        int64_t index = offset + i;
        const uint8_t* block = w->data + index / 32 * 34;
        float scale = oc_half_to_float(rd16(block));
        int64_t m = 32 - index % 32;
        if (m > n - i) m = n - i;
        for (int64_t j = 0; j < m; j++) out[i + j] = scale * (float)(int8_t)block[2 + index % 32 + j];
        i += m;
      }
      return;
    case OC_Q5_K:
    case OC_Q6_K:
    case OC_Q5_1: {
      int size = kblock_bytes(w->dtype), width = kblock_width(w->dtype);
      float decoded[256];
      for (int64_t i = 0; i < n;) {
        int64_t index = offset + i;
        oc_decode_kblock(decoded, w->data + index / width * size, w->dtype);
        int64_t m = width - index % width;
        if (m > n - i) m = n - i;
        memcpy(out + i, decoded + index % width, (size_t)m * sizeof(float));
        i += m;
      }
      return;
    }
    default:
      for (int64_t i = 0; i < n; i++) out[i] = tensor_at(w, offset + i);
  }
}

/* dot.go:14-70 mulRowsScalar for one row. */
static float mul_row(const oc_tensor* w, const float* x, int64_t i) {
  int64_t cols = w->cols;
  double sum = 0;
  switch (w->dtype) {
    case OC_Q5_K:
    case OC_Q6_K:
    case OC_Q5_1: {
      float decoded[256];
      for (int64_t j = 0; j < cols; j += 256) {
        int64_t n = cols - j < 256 ? cols - j : 256;
        oc_read_values(decoded, w, i * cols + j, n);
        for (int64_t k = 0; k < n; k++) sum += (double)x[j + k] * (double)decoded[k];
      }
      break;
    }
    case OC_Q8_0: {
      const uint8_t* row = w->data + i * cols / 32 * 34;
      for (int64_t j = 0; j < cols; j += 32) {
        const uint8_t* block = row + j / 32 * 34;
        double dot = 0;
        for (int k = 0; k < 32; k++) dot += (double)x[j + k] * (double)(int8_t)block[2 + k];
        sum += dot * (double)oc_half_to_float(rd16(block));
      }
      break;
    }
    case OC_BF16: {
      const uint8_t* row = w->data + i * cols * 2;
      double a = 0, b = 0, c = 0, d = 0;
      int64_t j = 0;
      for (; j + 3 < cols; j += 4) {
        a += (double)x[j] * (double)bits_f32((uint32_t)rd16(row + j * 2) << 16);
        b += (double)x[j + 1] * (double)bits_f32((uint32_t)rd16(row + j * 2 + 2) << 16);
        c += (double)x[j + 2] * (double)bits_f32((uint32_t)rd16(row + j * 2 + 4) << 16);
        d += (double)x[j + 3] * (double)bits_f32((uint32_t)rd16(row + j * 2 + 6) << 16);
      }
      sum = (a + b) + (c + d);
      for (; j < cols; j++) sum += (double)x[j] * (double)bits_f32((uint32_t)rd16(row + j * 2) << 16);
      break;
    }
    case OC_F32: {
      const uint8_t* row = w->data + i * cols * 4;
      for (int64_t j = 0; j < cols; j++) sum += (double)x[j] * (double)bits_f32(rd32(row + j * 4));
      break;
    }
    default:
      for (int64_t j = 0; j < cols; j++) sum += (double)x[j] * (double)tensor_at(w, i * cols + j);
  }
  return (float)sum;
}

/* safetensors.go:275-280 mulScratch -> mulRows -> mulRowsScalar */
void oc_mul_rows(float* out, const float* x, const oc_tensor* w) {
  int64_t rows = w->rows;
#pragma omp parallel for schedule(static) if (rows * w->cols >= (1 << 20))
  for (int64_t i = 0; i < rows; i++) out[i] = mul_row(w, x, i);
}

/* matmul.go:55-95 mulBatch with the scalar batchDot4 (matmul_scalar.go:7-27):
 * 4-row groups, 512-wide reduction tiles, float32 partials -> float64 totals. */
void oc_mul_batch(float* out, const float* x, int n, const oc_tensor* w) {
  if (n == 1) {
    oc_mul_rows(out, x, w);
    return;
  }
  const int64_t rows = w->rows, cols = w->cols;
  const int stride = (n + 3) / 4 * 4;
  const int block = 512;
  float* packed = (float*)calloc((size_t)cols * stride, sizeof(float));
  for (int token = 0; token < n; token++)
    for (int64_t col = 0; col < cols; col++) packed[col * stride + token] = x[token * cols + col];
  int64_t groups = (rows + 3) / 4;
#pragma omp parallel
  {
    float* tile = (float*)malloc(4 * block * sizeof(float));
    double* totals = (double*)malloc((size_t)4 * stride * sizeof(double));
#pragma omp for schedule(static)
    for (int64_t group = 0; group < groups; group++) {
      int64_t row = group * 4;
      int nr = rows - row < 4 ? (int)(rows - row) : 4;
      memset(totals, 0, (size_t)4 * stride * sizeof(double));
      for (int64_t col = 0; col < cols; col += block) {
        int nk = cols - col < block ? (int)(cols - col) : block;
        if (nr != 4) memset(tile, 0, 4 * block * sizeof(float));
        for (int r = 0; r < nr; r++) oc_read_values(tile + r * nk, w, (row + r) * cols + col, nk);
        const float* xp = packed + col * stride;
        for (int token = 0; token < stride; token++) {
          float a = 0, b = 0, c = 0, d = 0;
          for (int j = 0; j < nk; j++) {
            float v = xp[(int64_t)j * stride + token];
            a += v * tile[j];
            b += v * tile[nk + j];
            c += v * tile[2 * nk + j];
            d += v * tile[3 * nk + j];
          }
          totals[token] += (double)a;
          totals[stride + token] += (double)b;
          totals[2 * stride + token] += (double)c;
          totals[3 * stride + token] += (double)d;
        }
      }
      for (int r = 0; r < nr; r++)
        for (int token = 0; token < n; token++) out[(int64_t)token * rows + row + r] = (float)totals[r * stride + token];
    }
    free(tile);
    free(totals);
  }
  free(packed);
}

/* stablelm.go:288-305 layerNorm: float64 moments, float32 affine. */
void oc_layer_norm(float* out, const float* x, int n, const oc_tensor* weight, const oc_tensor* bias, double eps) {
  double mean = 0, variance = 0;
  for (int i = 0; i < n; i++) mean += (double)x[i];
  mean /= (double)n;
  for (int i = 0; i < n; i++) {
    double d = (double)x[i] - mean;
    variance += d * d;
  }
  float inv = (float)(1 / sqrt(variance / (double)n + eps));
  float fmean = (float)mean;
  for (int i = 0; i < n; i++) {
    float t = x[i] - fmean;
    t = t * inv;
    t = t * tensor_at(weight, i);
    out[i] = t + tensor_at(bias, i);
  }
}

/* stablelm.go:309-326 stableRotate: split-half rotation of the rotary prefix. */
void oc_stable_rotate(float* x, int len, int head_size, int rotary, int pos, double theta) {
  for (int i = 0; i < rotary / 2; i++) {
    float power = (float)pow((double)(float)theta, (double)((float)(2 * i) / (float)rotary));
    float inv_freq = 1.0f / power;
    float angle = (float)pos * inv_freq;
    float sn = (float)sin((double)angle), cs = (float)cos((double)angle);
    for (int h = 0; h < len; h += head_size) {
      float a = x[h + i], b = x[h + i + rotary / 2];
      float p1 = a * cs, p2 = b * sn;
      float p3 = b * cs, p4 = a * sn;
      x[h + i] = p1 - p2;
      x[h + i + rotary / 2] = p3 + p4;
    }
  }
}

/* model.go:552-570 softmax */
void oc_softmax(float* x, int n) {
  if (n == 0) return;
  float max_val = x[0];
  for (int i = 1; i < n; i++)
    if (x[i] > max_val) max_val = x[i];
  float sum = 0;
  for (int i = 0; i < n; i++) {
    x[i] = (float)exp((double)(x[i] - max_val));
    sum += x[i];
  }
  for (int i = 0; i < n; i++) x[i] /= sum;
}

/* model.go:622-630 argmax: strict comparison keeps the earliest index. */
int oc_argmax(const float* v, int n) {
  int best = 0;
  float bv = v[0];
  for (int i = 1; i < n; i++)
    if (v[i] > bv) {
      best = i;
      bv = v[i];
    }
  return best;
}

/* ------------------------------------------------------------------------ */
/* StableLM (stablelm.go, prefill.go, kv_cache.go)                           */

struct oc_stablelm {
  oc_stablelm_config c;
  oc_tensor* t; /* 9 per layer + embed, head, norm, bias */
  int n_tensors;
  int half_kv, capacity;
  float** keys;       /* [layer] -> [kvh][capacity][head] */
  float** values;
  uint16_t** keys16;
  uint16_t** values16;
  float *key_ws, *value_ws;
  /* scratch */
  float *x, *norm, *att_out, *proj, *gate, *up, *q, *k, *v, *att, *logits;
};

enum { T_NORM, T_BIAS, T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN };
#define LT(m, l, which) (&(m)->t[(l) * 9 + (which)])
#define T_EMBED(m) (&(m)->t[(m)->c.num_hidden_layers * 9 + 0])
#define T_HEAD(m) (&(m)->t[(m)->c.num_hidden_layers * 9 + 1])
#define T_FNORM(m) (&(m)->t[(m)->c.num_hidden_layers * 9 + 2])
#define T_FBIAS(m) (&(m)->t[(m)->c.num_hidden_layers * 9 + 3])

/* stablelm.go:256-282 newState */
oc_stablelm* oc_stablelm_new(const oc_stablelm_config* c, const oc_tensor* tensors, int n_tensors, int half_kv, int capacity) {
  if (n_tensors != c->num_hidden_layers * 9 + 4) return NULL;
  oc_stablelm* m = (oc_stablelm*)calloc(1, sizeof(*m));
  m->c = *c;
  m->n_tensors = n_tensors;
  m->t = (oc_tensor*)malloc(sizeof(oc_tensor) * n_tensors);
  memcpy(m->t, tensors, sizeof(oc_tensor) * n_tensors);
  m->half_kv = half_kv;
  m->capacity = capacity;
  int d = c->hidden_size, L = c->num_hidden_layers;
  int kv = d / c->num_attention_heads * c->num_key_value_heads;
  size_t per = (size_t)capacity * kv;
  if (half_kv) {
    m->keys16 = (uint16_t**)calloc(L, sizeof(uint16_t*));
    m->values16 = (uint16_t**)calloc(L, sizeof(uint16_t*));
    for (int l = 0; l < L; l++) {
      m->keys16[l] = (uint16_t*)calloc(per, 2);
      m->values16[l] = (uint16_t*)calloc(per, 2);
    }
    m->key_ws = (float*)calloc(per, 4);
    m->value_ws = (float*)calloc(per, 4);
  } else {
    m->keys = (float**)calloc(L, sizeof(float*));
    m->values = (float**)calloc(L, sizeof(float*));
    for (int l = 0; l < L; l++) {
      m->keys[l] = (float*)calloc(per, 4);
      m->values[l] = (float*)calloc(per, 4);
    }
  }
  int h = c->intermediate_size;
  m->x = (float*)calloc(d, 4);
  m->norm = (float*)calloc(d, 4);
  m->att_out = (float*)calloc(d, 4);
  m->proj = (float*)calloc(d, 4);
  m->gate = (float*)calloc(h, 4);
  m->up = (float*)calloc(h, 4);
  m->q = (float*)calloc(d, 4);
  m->k = (float*)calloc(kv, 4);
  m->v = (float*)calloc(kv, 4);
  m->att = (float*)calloc((size_t)capacity * c->num_attention_heads, 4);
  m->logits = (float*)calloc(c->vocab_size, 4);
  return m;
}

void oc_stablelm_free(oc_stablelm* m) {
  if (!m) return;
  for (int l = 0; l < m->c.num_hidden_layers; l++) {
    if (m->keys) {
      free(m->keys[l]);
      free(m->values[l]);
    }
    if (m->keys16) {
      free(m->keys16[l]);
      free(m->values16[l]);
    }
  }
  free(m->keys);
  free(m->values);
  free(m->keys16);
  free(m->values16);
  free(m->key_ws);
  free(m->value_ws);
  free(m->x);
  free(m->norm);
  free(m->att_out);
  free(m->proj);
  free(m->gate);
  free(m->up);
  free(m->q);
  free(m->k);
  free(m->v);
  free(m->att);
  free(m->logits);
  free(m->t);
  free(m);
}

/* kv_cache.go:55-65 storeKV */
static void store_kv(oc_stablelm* m, int l, int64_t offset, const float* key, const float* value, int n) {
  if (!m->half_kv) {
    memcpy(m->keys[l] + offset, key, n * 4);
    memcpy(m->values[l] + offset, value, n * 4);
    return;
  }
  for (int i = 0; i < n; i++) {
    m->keys16[l][offset + i] = oc_float_to_half(key[i]);
    m->values16[l][offset + i] = oc_float_to_half(value[i]);
  }
}

/* kv_cache.go:71-96 prepareKV + kvLayer */
static void kv_layer(oc_stablelm* m, int l, int positions, float** keys, float** values) {
  if (!m->half_kv) {
    *keys = m->keys[l];
    *values = m->values[l];
    return;
  }
  int head = m->c.hidden_size / m->c.num_attention_heads;
  int cap = m->capacity;
  for (int h = 0; h < m->c.num_key_value_heads; h++) {
    int64_t start = (int64_t)h * cap * head, end = ((int64_t)h * cap + positions) * head;
    for (int64_t i = start; i < end; i++) {
      m->key_ws[i] = oc_half_to_float(m->keys16[l][i]);
      m->value_ws[i] = oc_half_to_float(m->values16[l][i]);
    }
  }
  *keys = m->key_ws;
  *values = m->value_ws;
}

/* stablelm.go:401-427 attendHeads for one query vector q at position pos. */
static void attend_heads(const oc_stablelm* m, const float* keys, const float* values, int pos, const float* q, float* att_scratch,
                         float* att_out) {
  const oc_stablelm_config* c = &m->c;
  int head = c->hidden_size / c->num_attention_heads;
  int group = c->num_attention_heads / c->num_key_value_heads;
  int cap = m->capacity;
  float scale = (float)sqrt((double)head);
#pragma omp parallel for schedule(static) if ((int64_t)c->hidden_size * (pos + 1) >= (1 << 20))
  for (int h = 0; h < c->num_attention_heads; h++) {
    float* att = att_scratch + (int64_t)h * cap;
    const float* qh = q + h * head;
    int64_t offset = (int64_t)(h / group) * cap * head;
    for (int t = 0; t <= pos; t++) {
      const float* k = keys + offset + (int64_t)t * head;
      float score = 0; /* dot_scalar.go:23-29 */
      for (int i = 0; i < head; i++) score += qh[i] * k[i];
      att[t] = score / scale;
    }
    oc_softmax(att, pos + 1);
    float* out = att_out + h * head;
    memset(out, 0, head * 4);
    for (int t = 0; t <= pos; t++) {
      const float* v = values + offset + (int64_t)t * head;
      float s = att[t];
      for (int i = 0; i < head; i++) out[i] += s * v[i]; /* dot_scalar.go:31-37 */
    }
  }
}

static inline float silu_mul(float v, float up) { /* stablelm.go:371-373 */
  float e = (float)exp(-(double)v);
  float den = 1 + e;
  float s = v / den;
  return s * up;
}

/* stablelm.go:332-387 forward */
int oc_stablelm_forward(oc_stablelm* m, int token, int pos, int want_logits, float* logits) {
  const oc_stablelm_config* c = &m->c;
  int d = c->hidden_size, head = d / c->num_attention_heads;
  int rotary = (int)((double)head * c->partial_rotary_factor);
  int kvw = head * c->num_key_value_heads;
  if (pos < 0 || pos >= m->capacity || token < 0 || token >= c->vocab_size) return -1;
  oc_read_values(m->x, T_EMBED(m), (int64_t)token * d, d);
  for (int l = 0; l < c->num_hidden_layers; l++) {
    oc_layer_norm(m->norm, m->x, d, LT(m, l, T_NORM), LT(m, l, T_BIAS), c->layer_norm_eps);
    oc_mul_rows(m->q, m->norm, LT(m, l, T_Q));
    oc_mul_rows(m->k, m->norm, LT(m, l, T_K));
    oc_mul_rows(m->v, m->norm, LT(m, l, T_V));
    oc_stable_rotate(m->q, d, head, rotary, pos, c->rope_theta);
    oc_stable_rotate(m->k, kvw, head, rotary, pos, c->rope_theta);
    for (int h = 0; h < c->num_key_value_heads; h++) {
      int64_t offset = ((int64_t)h * m->capacity + pos) * head;
      store_kv(m, l, offset, m->k + h * head, m->v + h * head, head);
    }
    float *keys, *values;
    kv_layer(m, l, pos + 1, &keys, &values);
    attend_heads(m, keys, values, pos, m->q, m->att, m->att_out);
    oc_mul_rows(m->proj, m->att_out, LT(m, l, T_O));
    oc_mul_rows(m->gate, m->norm, LT(m, l, T_GATE));
    oc_mul_rows(m->up, m->norm, LT(m, l, T_UP));
    for (int i = 0; i < c->intermediate_size; i++) m->gate[i] = silu_mul(m->gate[i], m->up[i]);
    oc_mul_rows(m->att_out, m->gate, LT(m, l, T_DOWN));
    for (int i = 0; i < d; i++) {
      float t = m->x[i] + m->proj[i];
      m->x[i] = t + m->att_out[i];
    }
  }
  if (want_logits) {
    oc_layer_norm(m->norm, m->x, d, T_FNORM(m), T_FBIAS(m), c->layer_norm_eps);
    oc_mul_rows(m->logits, m->norm, T_HEAD(m));
    if (logits) memcpy(logits, m->logits, (size_t)c->vocab_size * 4);
  }
  return 0;
}

/* prefill.go:33-115 prefill (scalar build: attendBatch reduces to attendHeads
 * per query, attention.go:6-45 with attentionBatchWidth()==1). */
int oc_stablelm_prefill(oc_stablelm* m, const int* ids, int n_ids, int start, int chunk, float* logits) {
  const oc_stablelm_config* c = &m->c;
  int d = c->hidden_size, h = c->intermediate_size, head = d / c->num_attention_heads;
  int kvw = head * c->num_key_value_heads;
  int rotary = (int)((double)head * c->partial_rotary_factor);
  if (n_ids <= 0) return 0;
  if (start < 0 || start + n_ids > m->capacity) return -1;
  for (int i = 0; i < n_ids; i++)
    if (ids[i] < 0 || ids[i] >= c->vocab_size) return -1;
  if (chunk <= 0) chunk = 128; /* matmul.go:8 prefillBatch */
  float *bx = (float*)malloc((size_t)chunk * d * 4), *bn = (float*)malloc((size_t)chunk * d * 4);
  float *bq = (float*)malloc((size_t)chunk * d * 4), *bk = (float*)malloc((size_t)chunk * kvw * 4);
  float *bv = (float*)malloc((size_t)chunk * kvw * 4), *bo = (float*)malloc((size_t)chunk * d * 4);
  float *bp = (float*)malloc((size_t)chunk * d * 4), *bg = (float*)malloc((size_t)chunk * h * 4);
  float* bu = (float*)malloc((size_t)chunk * h * 4);
  for (int offset = 0; offset < n_ids; offset += chunk) {
    int n = n_ids - offset < chunk ? n_ids - offset : chunk;
    int last = offset + n == n_ids;
    if (n == 1) {
      oc_stablelm_forward(m, ids[offset], start + offset, last, last ? logits : NULL);
      continue;
    }
    for (int j = 0; j < n; j++) oc_read_values(bx + (int64_t)j * d, T_EMBED(m), (int64_t)ids[offset + j] * d, d);
    for (int l = 0; l < c->num_hidden_layers; l++) {
      for (int j = 0; j < n; j++)
        oc_layer_norm(bn + (int64_t)j * d, bx + (int64_t)j * d, d, LT(m, l, T_NORM), LT(m, l, T_BIAS), c->layer_norm_eps);
      oc_mul_batch(bq, bn, n, LT(m, l, T_Q));
      oc_mul_batch(bk, bn, n, LT(m, l, T_K));
      oc_mul_batch(bv, bn, n, LT(m, l, T_V));
      for (int j = 0; j < n; j++) {
        oc_stable_rotate(bq + (int64_t)j * d, d, head, rotary, start + offset + j, c->rope_theta);
        oc_stable_rotate(bk + (int64_t)j * kvw, kvw, head, rotary, start + offset + j, c->rope_theta);
      }
      for (int j = 0; j < n; j++)
        for (int kh = 0; kh < c->num_key_value_heads; kh++) {
          int64_t at = ((int64_t)kh * m->capacity + start + offset + j) * head;
          store_kv(m, l, at, bk + (int64_t)j * kvw + kh * head, bv + (int64_t)j * kvw + kh * head, head);
        }
      float *keys, *values;
      kv_layer(m, l, start + offset + n, &keys, &values);
      for (int j = 0; j < n; j++) attend_heads(m, keys, values, start + offset + j, bq + (int64_t)j * d, m->att, bo + (int64_t)j * d);
      oc_mul_batch(bp, bo, n, LT(m, l, T_O));
      oc_mul_batch(bg, bn, n, LT(m, l, T_GATE));
      oc_mul_batch(bu, bn, n, LT(m, l, T_UP));
      for (int64_t i = 0; i < (int64_t)n * h; i++) bg[i] = silu_mul(bg[i], bu[i]);
      oc_mul_batch(bo, bg, n, LT(m, l, T_DOWN));
      for (int64_t i = 0; i < (int64_t)n * d; i++) {
        float t = bx[i] + bp[i];
        bx[i] = t + bo[i];
      }
    }
    if (last) {
      memcpy(m->x, bx + (int64_t)(n - 1) * d, d * 4);
      oc_layer_norm(m->norm, m->x, d, T_FNORM(m), T_FBIAS(m), c->layer_norm_eps);
      oc_mul_rows(m->logits, m->norm, T_HEAD(m));
      if (logits) memcpy(logits, m->logits, (size_t)c->vocab_size * 4);
    }
  }
  free(bx);
  free(bn);
  free(bq);
  free(bk);
  free(bv);
  free(bo);
  free(bp);
  free(bg);
  free(bu);
  return 0;
}

static float top_margin(const float* v, int n) {
  int best = oc_argmax(v, n);
  float second = -INFINITY;
  for (int i = 0; i < n; i++)
    if (i != best && v[i] > second) second = v[i];
  return v[best] - second;
}

/* stablelm.go:503-540: prefill, then sample (greedy) / forward in turn. */
int oc_stablelm_greedy(oc_stablelm* m, const int* prompt, int n_prompt, int steps, int chunk, int* out, float* margins) {
  int V = m->c.vocab_size;
  if (oc_stablelm_prefill(m, prompt, n_prompt, 0, chunk, NULL) != 0) return -1;
  int pos = n_prompt - 1;
  for (int i = 0; i < steps; i++) {
    int token = oc_argmax(m->logits, V);
    if (margins) margins[i] = top_margin(m->logits, V);
    out[i] = token;
    if (i + 1 < steps) {
      if (oc_stablelm_forward(m, token, pos + 1, 1, NULL) != 0) return -1;
      pos++;
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Legacy llama2.c engine (model.go)                                          */

struct oc_llama {
  int dim, hidden, layers, heads, kv_heads, vocab, seq;
  float *emb, *rms_att, *wq, *wk, *wv, *wo, *rms_ffn, *w1, *w2, *w3, *rms_final, *fcr, *fci;
  float *data;
  float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *key_cache, *value_cache;
};

/* model.go:90-166 LoadModel/readWeights (checkpoint only). */
oc_llama* oc_llama_new(const uint8_t* ck, size_t nbytes) {
  if (nbytes < 28) return NULL;
  int32_t h[7];
  memcpy(h, ck, 28);
  if (h[0] <= 0 || h[1] <= 0 || h[2] <= 0 || h[3] <= 0 || h[4] <= 0 || h[3] % h[4] != 0 || h[5] < 2 || h[6] <= 0 || h[0] % h[3] != 0 ||
      (h[0] / h[3]) % 2 != 0)
    return NULL;
  oc_llama* m = (oc_llama*)calloc(1, sizeof(*m));
  m->dim = h[0];
  m->hidden = h[1];
  m->layers = h[2];
  m->heads = h[3];
  m->kv_heads = h[4];
  m->vocab = h[5];
  m->seq = h[6];
  int64_t hs = m->dim / m->heads, kvd = hs * m->kv_heads, dim = m->dim, hid = m->hidden, L = m->layers;
  int64_t sizes[13] = {m->vocab * dim, L * dim, L * dim * dim, L * dim * kvd, L * dim * kvd, L * dim * dim, L * dim,
                       L * hid * dim,  L * dim * hid, L * hid * dim, dim, m->seq * hs / 2, m->seq * hs / 2};
  int64_t total = 0;
  for (int i = 0; i < 13; i++) total += sizes[i];
  if ((size_t)(28 + total * 4) != nbytes) {
    free(m);
    return NULL;
  }
  m->data = (float*)malloc((size_t)total * 4);
  memcpy(m->data, ck + 28, (size_t)total * 4);
  float** dst[13] = {&m->emb, &m->rms_att, &m->wq, &m->wk, &m->wv, &m->wo, &m->rms_ffn, &m->w1, &m->w2, &m->w3, &m->rms_final, &m->fcr, &m->fci};
  float* p = m->data;
  for (int i = 0; i < 13; i++) {
    *dst[i] = p;
    p += sizes[i];
  }
  m->x = (float*)calloc(dim, 4);
  m->xb = (float*)calloc(dim, 4);
  m->xb2 = (float*)calloc(dim, 4);
  m->hb = (float*)calloc(hid, 4);
  m->hb2 = (float*)calloc(hid, 4);
  m->q = (float*)calloc(dim, 4);
  m->k = (float*)calloc(kvd, 4);
  m->v = (float*)calloc(kvd, 4);
  m->att = (float*)calloc(m->seq, 4);
  m->key_cache = (float*)calloc((size_t)L * m->seq * kvd, 4);
  m->value_cache = (float*)calloc((size_t)L * m->seq * kvd, 4);
  return m;
}

void oc_llama_free(oc_llama* m) {
  if (!m) return;
  free(m->data);
  free(m->x);
  free(m->xb);
  free(m->xb2);
  free(m->hb);
  free(m->hb2);
  free(m->q);
  free(m->k);
  free(m->v);
  free(m->att);
  free(m->key_cache);
  free(m->value_cache);
  free(m);
}

int oc_llama_config(const oc_llama* m, int* o) {
  o[0] = m->dim;
  o[1] = m->hidden;
  o[2] = m->layers;
  o[3] = m->heads;
  o[4] = m->kv_heads;
  o[5] = m->vocab;
  o[6] = m->seq;
  return 0;
}

/* model.go:575-586 matmul: sequential float32 accumulation. */
static void llama_matmul(float* xout, const float* x, const float* w, int n, int d) {
  for (int i = 0; i < d; i++) {
    float val = 0;
    const float* row = w + (int64_t)i * n;
    for (int j = 0; j < n; j++) val += row[j] * x[j];
    xout[i] = val;
  }
}

/* model.go:591-600 rmsNorm */
static void llama_rmsnorm(float* dest, const float* src, const float* weight, int n) {
  float ss = 0;
  for (int i = 0; i < n; i++) ss += src[i] * src[i];
  float mean = ss / (float)n;
  mean = mean + 1e-5f;
  float r = (float)sqrt((double)mean);
  float inv = 1.0f / r;
  for (int i = 0; i < n; i++) {
    float t = inv * src[i];
    dest[i] = weight[i] * t;
  }
}

/* model.go:611-618 rotateHead */
static void llama_rotate(float* vec, const float* fr, const float* fi, int hs) {
  for (int i = 0; i < hs; i += 2) {
    float v0 = vec[i], v1 = vec[i + 1], c = fr[i / 2], s = fi[i / 2];
    float a = v0 * c, b = v1 * s, e = v0 * s, f = v1 * c;
    vec[i] = a - b;
    vec[i + 1] = e + f;
  }
}

/* model.go:407-481 transformer */
int oc_llama_transformer(oc_llama* m, int token, int pos, float* logits) {
  if (token < 0 || token >= m->vocab || pos < 0 || pos >= m->seq) return -1;
  int dim = m->dim, hid = m->hidden, hs = dim / m->heads, kvd = hs * m->kv_heads, kvmul = m->heads / m->kv_heads;
  float* x = m->x;
  memcpy(x, m->emb + (int64_t)token * dim, dim * 4);
  const float* fr = m->fcr + (int64_t)pos * hs / 2;
  const float* fi = m->fci + (int64_t)pos * hs / 2;
  float scale = (float)sqrt((double)hs);
  for (int l = 0; l < m->layers; l++) {
    llama_rmsnorm(m->xb, x, m->rms_att + (int64_t)l * dim, dim);
    llama_matmul(m->q, m->xb, m->wq + (int64_t)l * dim * dim, dim, dim);
    llama_matmul(m->k, m->xb, m->wk + (int64_t)l * dim * kvd, dim, kvd);
    llama_matmul(m->v, m->xb, m->wv + (int64_t)l * dim * kvd, dim, kvd);
    for (int h = 0; h < m->heads; h++) llama_rotate(m->q + h * hs, fr, fi, hs);
    for (int h = 0; h < m->kv_heads; h++) llama_rotate(m->k + h * hs, fr, fi, hs);
    int64_t loff = (int64_t)l * m->seq * kvd;
    memcpy(m->key_cache + loff + (int64_t)pos * kvd, m->k, kvd * 4);
    memcpy(m->value_cache + loff + (int64_t)pos * kvd, m->v, kvd * 4);
    for (int h = 0; h < m->heads; h++) {
      const float* q = m->q + h * hs;
      int kvoff = (h / kvmul) * hs;
      for (int t = 0; t <= pos; t++) {
        const float* k = m->key_cache + loff + (int64_t)t * kvd + kvoff;
        float score = 0;
        for (int i = 0; i < hs; i++) score += q[i] * k[i];
        m->att[t] = score / scale;
      }
      oc_softmax(m->att, pos + 1);
      for (int i = 0; i < hs; i++) {
        float val = 0;
        for (int t = 0; t <= pos; t++) val += m->att[t] * m->value_cache[loff + (int64_t)t * kvd + kvoff + i];
        m->xb[h * hs + i] = val;
      }
    }
    llama_matmul(m->xb2, m->xb, m->wo + (int64_t)l * dim * dim, dim, dim);
    for (int i = 0; i < dim; i++) x[i] += m->xb2[i];
    llama_rmsnorm(m->xb, x, m->rms_ffn + (int64_t)l * dim, dim);
    llama_matmul(m->hb, m->xb, m->w1 + (int64_t)l * dim * hid, dim, hid);
    llama_matmul(m->hb2, m->xb, m->w3 + (int64_t)l * dim * hid, dim, hid);
    for (int i = 0; i < hid; i++) {
      float e = (float)exp(-(double)m->hb[i]);
      float den = 1.0f + e;
      float r = 1.0f / den;
      float t = m->hb[i] * r;
      m->hb[i] = t * m->hb2[i];
    }
    llama_matmul(m->xb, m->hb, m->w2 + (int64_t)l * dim * hid, hid, dim);
    for (int i = 0; i < dim; i++) x[i] += m->xb[i];
  }
  llama_rmsnorm(x, x, m->rms_final, dim);
  llama_matmul(logits, x, m->emb, dim, m->vocab);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Sampling helpers                                                           */

/* logprobs.go:64-95 summarizeLogits */
double oc_summarize_logits(const float* logits, int n, int chosen, int count, int* ids, double* values, int* n_out) {
  if (count > n) count = n;
  double best = (double)logits[0];
  for (int i = 0; i < n; i++) best = fmax(best, (double)logits[i]);
  double total = 0;
  int len = 0;
  for (int i = 0; i < n; i++) {
    float v = logits[i];
    total += exp((double)v - best);
    if (count > 0 && len == count && v <= logits[ids[count - 1]]) continue;
    int at = 0;
    while (at < len && !(v > logits[ids[at]])) at++;
    if (at < count) {
      int end = len < count ? len : count - 1;
      for (int j = end; j > at; j--) ids[j] = ids[j - 1];
      ids[at] = i;
      if (len < count) len++;
    }
  }
  double z = best + log(total);
  for (int i = 0; i < len; i++) values[i] = (double)logits[ids[i]] - z;
  *n_out = len;
  return (double)logits[chosen] - z;
}

/* sampling.go:64-70 repetitionWeight */
double oc_repetition_weight(int age, int window, double slope) {
  if (slope == 0 || window <= 1) return 1;
  double x = 1 - 2 * (double)age / (double)(window - 1);
  return 1 + slope * x / (1 + fabs(x) * (slope - 1));
}

/* sampling.go:76-101 penalizedLogits: float64 copy of the logits, then for
 * each of the last `window` history ids (most recent first) the frequency
 * penalty times its recency weight, and on an id's most recent occurrence
 * also (log(repetition) + presence) times that weight. */
void oc_penalized_logits(const float* logits, int n, const int* history, int n_history, double repetition_penalty,
                         int repetition_range, double repetition_slope, double presence_penalty, double frequency_penalty,
                         double* out) {
  for (int i = 0; i < n; i++) out[i] = (double)logits[i];
  int window = repetition_range == 0 ? n_history : repetition_range;
  int m = window < n_history ? window : n_history;
  unsigned char* seen = (unsigned char*)calloc((size_t)n, 1);
  for (int age = 0; age < m; age++) {
    int id = history[n_history - 1 - age];
    if (id < 0 || id >= n) continue;
    double weight = oc_repetition_weight(age, window, repetition_slope);
    out[id] -= frequency_penalty * weight;
    if (!seen[id]) {
      out[id] -= (log(repetition_penalty) + presence_penalty) * weight;
      seen[id] = 1;
    }
  }
  free(seen);
}

/* sampling.go:112-143 samplingCandidates over float64 scores (k > 0). */
int oc_sampling_candidates_f64(const double* scores, int n, int k, int* ids, double* values) {
  if (k <= 0 || k > n) k = n;
  int len = 0;
  for (int id = 0; id < n; id++) {
    double p = scores[id];
    if (len == k && p <= values[k - 1]) continue;
    int at = 0;
    while (at < len && !(p > values[at])) at++;
    int end = len < k ? len : k - 1;
    for (int j = end; j > at; j--) {
      ids[j] = ids[j - 1];
      values[j] = values[j - 1];
    }
    ids[at] = id;
    values[at] = p;
    if (len < k) len++;
  }
  return len;
}

/* sampling.go:112-143 samplingCandidates (k > 0): descending score, ties by
 * ascending id, at most k entries. */
int oc_sampling_candidates(const float* logits, int n, int k, int* ids, double* values) {
  if (k <= 0 || k > n) k = n;
  int len = 0;
  for (int id = 0; id < n; id++) {
    double p = (double)logits[id];
    if (len == k && p <= values[k - 1]) continue;
    int at = 0;
    while (at < len && !(p > values[at])) at++;
    int end = len < k ? len : k - 1;
    for (int j = end; j > at; j--) {
      ids[j] = ids[j - 1];
      values[j] = values[j - 1];
    }
    ids[at] = id;
    values[at] = p;
    if (len < k) len++;
  }
  return len;
}
