/*
 * CPU oracle for the tinyoai StableLM / llama2.c forward path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference's
 * Go scalar CPU path (wbrown/tinyoai), used by tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg as the checker. The product library
 * (tinyoai_b200/) never links, loads or calls it.
 *
 * Parity is pinned against the reference's own golden vectors:
 *   testdata/gguf/{q5_k,q6_k,q5_1}.bin + -f32.bin  (bitwise decode)
 *   testdata/stablelm/expected.json                (HF fp32 logits, 3e-5)
 *   testdata/stablelm/rope.json                    (split-half RoPE, 5e-7)
 *   exhaustive binary16 round trip                 (kv_cache_test.go:12-41)
 * converted into tests/golden/ by tests/golden/make_golden.py.
 *
 * Numeric semantics follow the Go source as written for amd64 (no fused
 * multiply-add: build with -ffp-contract=off): float64 accumulation in the
 * matrix-vector product (dot.go:14-70), float32 partials promoted to float64
 * in the batched product (matmul.go:55-95, matmul_scalar.go:12-27), float64
 * LayerNorm moments (stablelm.go:288-305) and float32 attention
 * (stablelm.go:401-427).
 */
#ifndef TINYOAI_ORACLE_H
#define TINYOAI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF type codes (gguf.go:177-205). */
enum { OC_F32 = 0, OC_F16 = 1, OC_Q5_1 = 7, OC_Q8_0 = 8, OC_Q5_K = 13, OC_Q6_K = 14, OC_BF16 = 30 };

typedef struct {
  int dtype;
  int64_t rows, cols; /* 1-D tensors use rows = 1 */
  const uint8_t* data;
} oc_tensor;

float oc_half_to_float(uint16_t h);
uint16_t oc_float_to_half(float v);
void oc_decode_kblock(float* out, const uint8_t* block, int dtype);
void oc_read_values(float* out, const oc_tensor* w, int64_t offset, int64_t n);
void oc_mul_rows(float* out, const float* x, const oc_tensor* w);
void oc_mul_batch(float* out, const float* x, int n, const oc_tensor* w);
void oc_layer_norm(float* out, const float* x, int n, const oc_tensor* weight, const oc_tensor* bias, double eps);
void oc_stable_rotate(float* x, int len, int head_size, int rotary, int pos, double theta);
void oc_softmax(float* x, int n);
int oc_argmax(const float* v, int n);

typedef struct {
  int vocab_size, hidden_size, intermediate_size, num_hidden_layers;
  int num_attention_heads, num_key_value_heads, max_position_embeddings;
  double layer_norm_eps, rope_theta, partial_rotary_factor;
} oc_stablelm_config;

/* Tensor order per layer: norm, bias, q, k, v, o, gate, up, down (9 per layer),
 * then embed, head, final norm, final bias. */
typedef struct oc_stablelm oc_stablelm;
oc_stablelm* oc_stablelm_new(const oc_stablelm_config* c, const oc_tensor* tensors, int n_tensors, int half_kv, int capacity);
void oc_stablelm_free(oc_stablelm* m);
/* One-token forward at absolute position pos (stablelm.go:332-387). */
int oc_stablelm_forward(oc_stablelm* m, int token, int pos, int want_logits, float* logits);
/* Chunked prefill of ids[0..n) starting at position start (prefill.go:33-115). */
int oc_stablelm_prefill(oc_stablelm* m, const int* ids, int n, int start, int chunk, float* logits);
/* Greedy continuation: prefill prompt then `steps` argmax tokens (stablelm.go:519-540). */
int oc_stablelm_greedy(oc_stablelm* m, const int* prompt, int n_prompt, int steps, int chunk, int* out, float* margins);

typedef struct oc_llama oc_llama;
oc_llama* oc_llama_new(const uint8_t* checkpoint, size_t nbytes);
void oc_llama_free(oc_llama* m);
int oc_llama_config(const oc_llama* m, int* out7);
/* model.go:407-481 */
int oc_llama_transformer(oc_llama* m, int token, int pos, float* logits);

/* logprobs.go:64-95 summarizeLogits: returns chosen log probability; writes
 * up to count (id, logprob) pairs, descending, ties by lower id. */
double oc_summarize_logits(const float* logits, int n, int chosen, int count, int* ids, double* values, int* n_out);
/* sampling.go:112-143 samplingCandidates over float32 logits promoted to float64. */
int oc_sampling_candidates(const float* logits, int n, int k, int* ids, double* values);

/* sampling.go:64-70 repetitionWeight and sampling.go:76-101 penalizedLogits
 * (float64 scores with recency-weighted frequency, presence and logarithmic
 * repetition penalties). */
double oc_repetition_weight(int age, int window, double slope);
void oc_penalized_logits(const float* logits, int n, const int* history, int n_history, double repetition_penalty,
                         int repetition_range, double repetition_slope, double presence_penalty, double frequency_penalty,
                         double* out);
/* sampling.go:112-143 samplingCandidates over float64 scores. */
int oc_sampling_candidates_f64(const double* scores, int n, int k, int* ids, double* values);

void oc_set_threads(int n);
int oc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
