/*
 * tinyoai_cuda.h - C ABI of the B200 (sm_100a) inference backend for tinyoai.
 *
 * The Go package binds these entry points through cgo (build tag `cuda`) in
 * place of its native MLX forwarders. Each entry point names the reference
 * interface it replaces (path:line inside the wbrown/tinyoai project).
 *
 * Conventions
 *  - Every function returns an int status: TCU_OK (0) or a negative TCU_E*
 *    code. The message of the last failure on the calling thread is returned
 *    by tcu_last_error() (pattern of internal/mlx/bridge.c:13-33).
 *  - Buffers are plain host pointers owned by the caller. Nothing is retained
 *    after a call returns except where stated (weights are copied to the GPU
 *    during load, so the caller may free its tensor bytes afterwards).
 *  - Handles are opaque. A session (and its branches) must be used from one
 *    thread at a time, as the Go wrapper guarantees with its request gate
 *    (mlx.go:32, 291-296). Distinct sessions may run concurrently.
 *  - No call allocates host memory for the caller, and no call falls back to
 *    the CPU: without a usable sm_100a GPU, loading fails with TCU_ENODEV.
 */
#ifndef TINYOAI_CUDA_H
#define TINYOAI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TCU_ABI_VERSION 1

/* Status codes. */
#define TCU_OK 0
#define TCU_EINVAL (-1)    /* bad argument: token, prefix, length, shape, dtype */
#define TCU_ENODEV (-2)    /* no usable sm_100 device */
#define TCU_ENOMEM (-3)    /* device memory or KV pool exhausted */
#define TCU_ECUDA (-4)     /* CUDA runtime error (message has the detail) */
#define TCU_ECLOSED (-5)   /* handle already closed */
#define TCU_EUNSUP (-6)    /* valid request this backend does not implement */
#define TCU_ETIMEOUT (-7)  /* a bounded device wait expired */

/* Tensor dtypes: GGUF type codes (gguf.go:177-205). */
#define TCU_F32 0
#define TCU_F16 1
#define TCU_Q5_1 7
#define TCU_Q8_0 8
#define TCU_Q5_K 13
#define TCU_Q6_K 14
#define TCU_BF16 30

/* One checkpoint tensor as the Go loaders hold it: weightTensor{data, dtype,
 * shape} (safetensors.go:193-197), row-major with the file's block encoding.
 * Names use the Hugging Face convention (stablelm.go:180-191). */
typedef struct {
  const char* name;
  int32_t dtype;
  int32_t ndim;       /* 1 or 2 */
  int64_t shape[2];   /* shape[0] = rows (or length), shape[1] = cols */
  const void* data;
  uint64_t nbytes;
} tcu_tensor;

/* StableLMConfig after validate() (stablelm.go:18-111). */
typedef struct {
  int32_t vocab_size, hidden_size, intermediate_size, num_hidden_layers;
  int32_t num_attention_heads, num_key_value_heads, max_position_embeddings;
  int32_t bos_token_id, eos_token_id;
  double layer_norm_eps, rope_theta, partial_rotary_factor;
} tcu_stablelm_config;

/* Load-time options. Zero-initialise for defaults. */
typedef struct {
  int32_t device;         /* CUDA ordinal */
  int32_t kv_page_tokens; /* positions per KV page; 0 -> 32 */
  int64_t kv_pool_bytes;  /* KV pool budget per KV dtype; 0 -> 1/4 of free HBM after weights */
} tcu_load_options;

typedef struct tcu_model tcu_model;
typedef struct tcu_session tcu_session;
typedef struct tcu_branches tcu_branches;

/* Library and device queries. */
int tcu_abi_version(void);
const char* tcu_last_error(void);
int tcu_device_count(int32_t* count);

/* Replaces LoadStableLM/loadStableWeights (stablelm.go:136-199) and
 * LoadMLXNative (mlx_native.go:56-160): validates the config, checks every
 * tensor's shape, uploads and repacks weights into the device layout. */
int tcu_stablelm_load(const tcu_stablelm_config* config, const tcu_tensor* tensors, int32_t n_tensors,
                      const tcu_load_options* options, tcu_model** out);

/* Head-parallel tensor parallelism for one long sequence (an 8K-token
 * prefill, say): `world` processes, one GPU each, load the same checkpoint
 * and each keeps a contiguous block of query heads (and their KV heads),
 * the matching rows of q/k/v, a block of MLP rows (gate/up rows, down
 * columns) and the matching columns of o_proj; embedding, norms and lm_head
 * are replicated. Every layer sums the ranks' out + down partials with one
 * NCCL all-reduce (the parallel residual, stablelm.go:365-377, lets both
 * products share it) and adds the sum to the residual. Rank 0 makes the
 * communicator id with tcu_tp_unique_id and shares its 128 bytes with the
 * others (any host channel); every rank then calls tcu_stablelm_load_tp with
 * the same id. world must divide the heads, KV heads and MLP width, and the
 * o/down column slices must be whole quantisation blocks. A tensor-parallel
 * model serves one session at a time (every rank runs the same calls, in the
 * same order, with the same tokens). NCCL is loaded at run time
 * (libnccl.so.2); without it these return TCU_EUNSUP. */
typedef struct {
  int32_t world;
  int32_t rank;
  uint8_t nccl_id[128];
} tcu_tp_options;
int tcu_tp_unique_id(uint8_t* id);
int tcu_stablelm_load_tp(const tcu_stablelm_config* config, const tcu_tensor* tensors, int32_t n_tensors,
                         const tcu_load_options* options, const tcu_tp_options* tp, tcu_model** out);
/* The share of rank `rank`: out[0..6) = first query head, query heads, first
 * KV head, KV heads, first MLP row, MLP rows. Needs no GPU. */
int tcu_tp_plan(const tcu_stablelm_config* config, int32_t world, int32_t rank, int32_t* out);

/* The per-layer exchange over NVLink peer memory instead of NCCL (no
 * counterpart in the reference): every rank calls tcu_tp_exchange_handle
 * (allocates its exchange buffer, returns its CUDA IPC handle), the ranks
 * share the handles (any host channel), and every rank calls
 * tcu_tp_exchange_open with all of them in rank order. From then on the
 * exchange of up to 64 rows (decode steps) is one kernel per layer that stores
 * this rank's partial into every rank's buffer, waits (bounded) for the
 * others' and adds the rank-ordered sum to the residual, and tensor-parallel
 * decode steps replay a captured CUDA graph; prefill chunks keep NCCL. Ranks
 * on one node, at most 8. A wait that runs out returns TCU_ETIMEOUT. */
#define TCU_TP_HANDLE_BYTES 64
int tcu_tp_exchange_handle(tcu_model* model, uint8_t* handle);
int tcu_tp_exchange_open(tcu_model* model, const uint8_t* handles);

/* GGUF StableLM checkpoints (readGGUF and loadStableGGUF, gguf.go:139-357):
 * tcu_gguf_open memory-maps a GGUF v3 file, validates its header as the
 * reference does (magic and version, counts, metadata types, tensor ranks,
 * dimensions and types, alignment, bounds, overlap, the StableLM metadata and
 * tensor set) and derives the configuration. The vocabulary size is the
 * length of tokenizer.ggml.tokens; comparing that vocabulary with the
 * tokenizer.json beside the file stays with the caller's tokenizer.
 * tcu_gguf_tensor returns tensor i under its Hugging Face name (the inverse of
 * ggufNames, gguf.go:250-255) with data pointing into the mapping, valid until
 * tcu_gguf_close. tcu_gguf_load_stablelm uploads the model straight from the
 * mapping (no host copy of the weights); tp may be NULL (the whole model) or a
 * rank's share as for tcu_stablelm_load_tp. Needs no GPU except the load. */
typedef struct tcu_gguf tcu_gguf;
int tcu_gguf_open(const char* path, tcu_gguf** out);
int tcu_gguf_config(const tcu_gguf* gguf, tcu_stablelm_config* config);
int tcu_gguf_tensor_count(const tcu_gguf* gguf, int32_t* n);
int tcu_gguf_tensor(const tcu_gguf* gguf, int32_t index, tcu_tensor* out);
int tcu_gguf_load_stablelm(const tcu_gguf* gguf, const tcu_load_options* options, const tcu_tp_options* tp, tcu_model** out);
int tcu_gguf_close(tcu_gguf* gguf);

/* Replaces LoadModel/readWeights (model.go:90-166) for the legacy llama2.c
 * checkpoint (7 x int32 header then float32 tensors), and DefaultMLX /
 * LoadLlamaMLX (mlx_llama.go:37-53). */
int tcu_llama_load(const void* checkpoint, uint64_t nbytes, const tcu_load_options* options, tcu_model** out);

/* Model dimensions: vocab, hidden, layers, heads, kv heads, max positions. */
int tcu_model_info(const tcu_model* model, int32_t* vocab, int32_t* hidden, int32_t* layers, int32_t* heads,
                   int32_t* kv_heads, int32_t* max_positions);
/* Device bytes held by weights, and by the KV pool (allocated / in use). */
int tcu_model_memory(const tcu_model* model, uint64_t* weight_bytes, uint64_t* kv_pool_bytes, uint64_t* kv_used_bytes);
/* Releases weights and the KV pool. Every session must be closed first. */
int tcu_model_free(tcu_model* model);

/* weightTensor.readValues (matmul.go:12-50, decodeKBlock quant_k.go:31-86) on
 * the device: decodes n values, starting at row-major element `offset`, of a
 * rows x cols tensor given in its file encoding (host bytes, checked against
 * the format's size), into out (n host floats). `decoder` names which of the
 * device decoders produces them:
 *   TCU_DECODE_ELEMENT  the per-element decoder of the matrix-vector kernels
 *                       (every format);
 *   TCU_DECODE_GROUP8   the 8-value decoder of the batched products (Q6_K,
 *                       Q5_K);
 *   TCU_DECODE_TC       the tensor-core operand: the binary16 pieces the
 *                       tcgen05 GEMM multiplies, summed back and unscaled
 *                       (Q8_0, Q6_K, Q5_K).
 * Each returns the reference's float32 values bit for bit, which is what this
 * entry point lets a host check (quant_k_test.go:14-48 checks the Go decoder
 * the same way). It allocates and frees its own device buffers. */
#define TCU_DECODE_ELEMENT 0
#define TCU_DECODE_GROUP8 1
#define TCU_DECODE_TC 2
int tcu_read_values(int32_t device, int32_t dtype, const void* data, uint64_t nbytes, int32_t rows, int32_t cols,
                    int64_t offset, int64_t n, int32_t decoder, float* out);

/* A generation session: the resident token prefix of one request stream and
 * its paged KV (the state nativeMLX keeps per model, mlx_native.go:24-45).
 * kv_dtype is TCU_F32 or TCU_F16 (StableLMOptions.KVCache, kv_cache.go:8-24). */
int tcu_session_new(tcu_model* model, int32_t kv_dtype, tcu_session** out);
int tcu_session_free(tcu_session* session);
/* Number of resident positions (nativeMLX.offset). */
int tcu_session_length(const tcu_session* session, int32_t* length);

/* mlxForwarder.Forward (mlx.go:45-51, mlx_native.go:294-297): evaluates tokens
 * at positions prefix.. after keeping the first `prefix` resident positions.
 * When want_logits != 0 the final vocabulary row is written to logits_out
 * (vocab floats). Requires 0 <= prefix <= length and prefix + n <= max
 * positions. On failure the resident prefix is discarded (mlx_native.go:487-489). */
int tcu_session_forward(tcu_session* session, int32_t prefix, const int32_t* tokens, int32_t n, int32_t want_logits,
                        float* logits_out);

/* llamaMLXForwarder.Forward with allLogits (mlx_llama.go:27-35): one logits
 * row per input token (n x vocab floats). */
int tcu_session_forward_all(tcu_session* session, int32_t prefix, const int32_t* tokens, int32_t n, float* logits_out);

/* Greedy decoding on the device (sampleWithOptions with Temperature == 0,
 * sampling.go:150-163 / model.go:622-630, inside the loops of
 * stablelm.go:519-540 and mlx.go:414-468): evaluates tokens after `prefix`,
 * then emits `steps` argmax tokens, feeding each back without a host round
 * trip. The resident prefix afterwards holds prompt + steps-1 tokens, as in
 * the reference loop (the final sampled token is not evaluated). */
int tcu_session_generate_greedy(tcu_session* session, int32_t prefix, const int32_t* tokens, int32_t n, int32_t steps,
                                int32_t* out_tokens);

/* Device-side sampling shortlist over the logits of the last forward:
 * samplingCandidates (sampling.go:112-143) over float32 logits, returning up to
 * k (id, logit) pairs in descending order with ties broken by lower id, plus
 * the full-vocabulary log-sum-exp (logprobs.go:64-95). */
int tcu_session_shortlist(tcu_session* session, int32_t k, int32_t* ids, float* logits, double* logsumexp,
                          int32_t* n_out);

/* mlxProbabilityForwarder.ForwardWithLogprobs (mlx.go:53-57,
 * mlx_native.go:303-313 and 436-478) with summarizeLogits semantics
 * (logprobs.go:64-95): evaluates tokens[0..n) after `prefix` as
 * tcu_session_forward does, and for every input position i writes
 *   chosen[i]                          log P(targets[i]) after position i,
 *   top_ids[i * count .. + count)      the count most likely next ids,
 *   top_logprobs[i * count .. + count) their log probabilities,
 * descending, ties by lower id, all normalised over the full vocabulary in
 * float64. logits_out (vocab floats, may be NULL) receives the final row.
 * targets pair one-for-one with tokens; 1 <= count <= min(256, vocab).
 * On failure the resident prefix is discarded, as for tcu_session_forward. */
int tcu_session_forward_logprobs(tcu_session* session, int32_t prefix, const int32_t* tokens, const int32_t* targets, int32_t n,
                                 int32_t count, double* chosen, int32_t* top_ids, double* top_logprobs, float* logits_out);

/* SamplingOptions' penalties (sampling.go:12-58), validated as Validate does:
 * finite, repetition_penalty >= 1, repetition_range >= 0 (0: the whole
 * history), repetition_slope >= 0. Neutral: {1, 0, 0, 0, 0}. */
typedef struct {
  double repetition_penalty;
  double presence_penalty;
  double frequency_penalty;
  double repetition_slope;
  int32_t repetition_range;
} tcu_penalties;

/* samplingCandidates(penalizedLogits(logits, history, opts), k)
 * (sampling.go:76-143) over the logits of the session's last forward, on
 * the device: float64 scores with recency-weighted frequency, presence and
 * logarithmic repetition penalties from `history` (the story's token ids,
 * oldest first), then the k best (id, score) pairs, descending, ties by
 * lower id (1 <= k <= 256). ids[0] is the greedy choice of sampleWithOptions
 * (sampling.go:155-163). The caller draws from the pairs with its own RNG
 * (temperature, top-p and tail-free filtering run on these k scores). At most
 * 16384 distinct ids may carry a penalty. */
int tcu_session_sample_candidates(tcu_session* session, const int32_t* history, int32_t n_history, const tcu_penalties* penalties,
                                  int32_t k, int32_t* ids, double* scores, int32_t* n_out);

/* SaveCache / LoadCache (cache_file.go:55-176) for a session, in the
 * reference's TNYKV001 format: "TNYKV001", the header length, the JSON header
 * {"model_sha256", "float16", "tokens"} as encoding/json writes it, the
 * resident positions' KV in layer -> KV head -> keys, values order (float32
 * little-endian or binary16 bits, cachePayload cache_file.go:203-258), then
 * the SHA-256 of all of that. model_sha256 is the caller's model identity
 * (modelIdentity, cache_file.go:26-48: the config and tensor bytes), tokens
 * the session's resident token ids (n_tokens == its length).
 * Save writes a 0600 temporary file beside `path`, syncs it and renames it
 * over `path`. Load checks, in LoadCache's order, the format, header size,
 * context length, token ids, model identity, KV precision, file size and
 * checksum; only then do the restored positions replace the session's
 * context (on any error the session is unchanged) and the tokens go to
 * tokens[0 .. *n_tokens) (capacity entries available). */
int tcu_session_save_cache(tcu_session* session, const char* path, const uint8_t* model_sha256, const int32_t* tokens,
                           int32_t n_tokens);
int tcu_session_load_cache(tcu_session* session, const char* path, const uint8_t* model_sha256, int32_t* tokens, int32_t capacity,
                           int32_t* n_tokens);

/* mlxForker.Fork (sessions.go:26-30, mlx_sessions.go:10-71): the child shares
 * every full KV page copy-free (reference counted) and copies only the
 * partially filled tail page. Parent and child then diverge independently. */
int tcu_session_fork(tcu_session* session, tcu_session** child);

/* LimitCache / SetKVBits (mlx_native.go:231-244, mlx_kv.go:78-91). cleared
 * reports whether resident KV was discarded. */
int tcu_session_limit(tcu_session* session, int32_t window, int32_t* cleared);
int tcu_session_set_kv_dtype(tcu_session* session, int32_t kv_dtype, int32_t* cleared);
/* llamaMLXForwarder.Reset: drop all resident positions. */
int tcu_session_reset(tcu_session* session);

/* Runs the session's work on a caller-owned CUDA stream (a cudaStream_t;
 * NULL restores the session's own stream). Lets a host that already owns a
 * stream order its copies and events with the session's kernels. */
int tcu_session_set_stream(tcu_session* session, void* stream);

/* Opt-in stage timing, the device counterpart of stableProfile
 * (stablelm.go:229-250): when enabled, CUDA events bracket every kernel and
 * the per-stage launch counts and milliseconds accumulate. Stages, in order:
 * embedding, norm+q/k/v/gate/up projection, decode attention, out/down
 * projection + residual, final norm+head, prefill projection, prefill
 * attention, other, whole persistent decode step, tensor-parallel
 * all-reduce. tcu_session_profile_read returns the number of stages (10) and
 * fills up to n_stages entries;
 * reset != 0 clears the totals.
 * Profiling synchronises after every decode step, so it is for diagnosis,
 * not for throughput runs. */
int tcu_session_profile(tcu_session* session, int32_t enable);
int tcu_session_profile_read(tcu_session* session, int32_t n_stages, int64_t* launches, double* ms, int32_t reset);

/* mlxBrancher.NewBranches (branches.go:55-59, mlx_branches.go:25-32): count
 * suffixes that share the first `prefix` resident positions read-only.
 * Unlike the MLX backend, grouped-query attention is supported. */
int tcu_branches_open(tcu_session* session, int32_t prefix, int32_t count, tcu_branches** out);
/* mlxBranches.Forward (mlx_branches.go:120-184): one token per branch at the
 * same absolute position; writes count x vocab logits (rows_out may be NULL
 * to skip the copy). */
int tcu_branches_forward(tcu_branches* branches, const int32_t* tokens, float* rows_out);
/* Greedy argmax of each branch's last row (count ints). */
int tcu_branches_argmax(tcu_branches* branches, int32_t* ids);
/* mlxBranches.Close: releases suffix pages (the shared prefix stays resident)
 * and frees the handle, which must not be used afterwards. A failed
 * tcu_branches_forward already released the pages; close it all the same. */
int tcu_branches_close(tcu_branches* branches);

/* Continuous batching (a serving load of many sessions). The reference's
 * Go server runs one request at a time per model (the request gate,
 * mlx.go:291-296); a batching scheduler instead advances all active
 * sessions together. tcu_batch_open reserves a workspace and stream for up
 * to max_rows rows (1..1024) so that steps allocate no device memory. */
typedef struct tcu_batch tcu_batch;
int tcu_batch_open(tcu_model* model, int32_t max_rows, tcu_batch** out);
/* One decode step for n sessions of the batch's model that share one KV
 * precision: tokens[i] is appended to sessions[i] at its current length
 * (which must be >= 1) and its logits row computed, exactly as
 * tcu_session_forward(sessions[i], length, &tokens[i], 1, 1, row) would.
 * Writes n x vocab logits (rows_out may be NULL) and each row's greedy
 * argmax (ids_out may be NULL); each session's length then grows by one.
 * Sessions with open branches, repeated or closed sessions are rejected.
 * Work already queued on a session's own stream completes first. */
int tcu_batch_forward(tcu_batch* batch, tcu_session* const* sessions, const int32_t* tokens, int32_t n, float* rows_out,
                      int32_t* ids_out);
/* tcu_session_sample_candidates for every row of the batch's last step
 * (n = that step's row count): row i's history is history[off_i ..
 * off_i + history_len[i]) with off_i the sum of the earlier lengths, its
 * penalties penalties[i]; writes n x k ids and scores. */
int tcu_batch_sample_candidates(tcu_batch* batch, int32_t n, const int32_t* history, const int32_t* history_len,
                                const tcu_penalties* penalties, int32_t k, int32_t* ids, double* scores);
int tcu_batch_close(tcu_batch* batch);

/* Sampling shortlist over a logits row the caller already holds in device
 * memory, allocating no device memory. This entry point has no counterpart in
 * the reference (its Go path keeps logits on the host); it serves callers that
 * must not allocate on the device when they call, for example a host whose
 * own caching allocator already holds the free HBM.
 *
 * Same kernel and results as tcu_session_shortlist: up to k (id, logit)
 * pairs, descending, ties by lower id (sampling.go:112-143), plus the float64
 * log-sum-exp of the whole row (logprobs.go:64-95). logits: `vocab` floats on
 * `device`; stream: a CUDA stream of that device, or NULL for the legacy
 * default stream. The call makes `device` current, returns after the stream
 * has synchronised, and writes *n_out = min(k, vocab) entries to the host
 * arrays ids and values.
 *
 * The kernel's results pass through one fixed device array of
 * TCU_SHORTLIST_STATIC_SCRATCH_BYTES per device, so k is limited to
 * TCU_SHORTLIST_STATIC_MAX_K. vocab is limited to
 * TCU_SHORTLIST_STATIC_MAX_VOCAB (the kernel marks taken ids in shared memory).
 * Larger values fail with TCU_EINVAL. The first call on a device does the set-up
 * (it looks up that array's device address). The call synchronises the stream
 * and copies into host memory, so it cannot be captured into a CUDA graph: a
 * stream under capture fails with TCU_EINVAL before any work is queued.
 * Calls on one device share the array: two calls in flight at the same time on
 * one device, from different host threads, overwrite each other's results. */
#define TCU_SHORTLIST_STATIC_MAX_K 256
#define TCU_SHORTLIST_STATIC_MAX_VOCAB 1048576
#define TCU_SHORTLIST_STATIC_SCRATCH_BYTES 4096
int tcu_shortlist_static(int32_t device, const float* logits, int32_t vocab, int32_t k, void* stream, int32_t* ids,
                         float* values, double* logsumexp, int32_t* n_out);

#ifdef __cplusplus
}
#endif
#endif
