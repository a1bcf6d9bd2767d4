/*
 * smallmind_cuda.h — C-ABI of the SmallMind.Cuda native library (sm_100a).
 *
 * Drop-in boundary for SmallMind's quantized decode/prefill hot path.  The
 * reference engine (C#) binds these entry points through P/Invoke; every
 * declaration names the reference interface it replaces (paths relative to the
 * reference project root).  Plain C types only: pointers, sizes, ints.
 *
 * Conventions
 *   - Every call returns an int status: SM_OK (0) or a negative SM_ERR_* code.
 *     sm_last_error() returns the calling thread's last error text.
 *   - Shape/length mismatches return SM_ERR_SHAPE, the counterpart of the
 *     ArgumentException thrown by the reference (e.g. Q4KWeightTensor.cs:43-48).
 *   - Outputs are OVERWRITTEN, never accumulated (the reference clears C first,
 *     e.g. FusedQ4KMatMul.cs:54).
 *   - Pointer-location flags: SM_PTR_HOST means the call copies host buffers
 *     in/out and synchronises; SM_PTR_DEVICE means device pointers and the
 *     call is asynchronous on the context's stream.
 *   - Threading: one sm_ctx per device and stream.  Calls on different
 *     contexts may run on different threads; calls on one context are not
 *     re-entrant (sessions are single-owner, InferenceSession.cs:28-29,127-144).
 */
#ifndef SMALLMIND_CUDA_H
#define SMALLMIND_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SM_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------- status */
#define SM_OK 0
#define SM_ERR_INVALID_ARG (-1)
#define SM_ERR_SHAPE (-2)
#define SM_ERR_CUDA (-3)
#define SM_ERR_OOM (-4)
#define SM_ERR_UNSUPPORTED (-5)
#define SM_ERR_STATE (-6)
#define SM_ERR_TIMEOUT (-7)
#define SM_ERR_NCCL (-8)

/* QuantScheme values of src/SmallMind.Quantization/Abstractions/IWeightTensor.cs:47-72 */
#define SM_F32 0
#define SM_F16 1
#define SM_Q8_0 2
#define SM_Q4_0 3
#define SM_Q4_1 4
#define SM_Q5_0 5
#define SM_Q4_K 6
#define SM_Q6_K 7

/* Weight orientation.
 * SM_LAYOUT_INTENDED: rows = N (out features), cols = K (in features); the
 *   packed bytes quantize W[N][K] along the linear index (blocks run along K;
 *   K-quant block n*(K/256)+kb, the GGUF order).  matmul computes y = x . W^T,
 *   the contract IWeightTensor documents (IWeightTensor.cs:25-26) and the
 *   orientation Linear.SetQuantizedWeight requires (NeuralNet.cs:89).
 * SM_LAYOUT_REFERENCE: the kernels as written: rows = K, cols = N; Q8_0/Q4_0
 *   linear row-major KxN (MatMulF32Q8.cs:61-79); K-quant block (k/256)*N + n
 *   (FusedQ4KMatMul.cs:122,127).  matmul computes C = A . B.                  */
#define SM_LAYOUT_INTENDED 0
#define SM_LAYOUT_REFERENCE 1

#define SM_PTR_HOST 0
#define SM_PTR_DEVICE 1

typedef struct sm_ctx sm_ctx;
typedef struct sm_weight sm_weight;
typedef struct sm_model sm_model;
typedef struct sm_kv sm_kv;

/* ---------------------------------------------------------------- library */
SM_API int sm_version(void);
/* copies the calling thread's last error message (NUL-terminated) */
SM_API int sm_last_error(char* buf, size_t n);
SM_API int sm_device_count(int* out);

/* ---------------------------------------------------------------- context */
/* One device + one CUDA stream.  Replaces nothing in the reference (managed
 * arrays need no context); the C# shim owns it as an IDisposable. */
SM_API int sm_ctx_create(int device, sm_ctx** out);
/* Destroying the context does not free the weights, models and KV caches made on it;
 * their destroy calls stay valid afterwards (they wait on the whole device). */
SM_API int sm_ctx_destroy(sm_ctx* ctx);
/* Use an external cudaStream_t (e.g. one owned by a host framework); NULL = own stream. */
SM_API int sm_ctx_set_stream(sm_ctx* ctx, void* cuda_stream);
SM_API int sm_stream_sync(sm_ctx* ctx);
/* Last kernel-side status (bounded device waits report SM_ERR_TIMEOUT here). */
SM_API int sm_ctx_device_status(sm_ctx* ctx);

/* ---------------------------------------------------------------- weights */
/* Upload a packed weight.  Replaces the managed Q8Tensor/Q4Tensor/Q4KTensor/
 * Q6KTensor byte arrays wrapped by Q*WeightTensor (Q4KWeightTensor.cs:10-36) and
 * the factory SmqModelLoader.CreateWeightTensor (SmqModelLoader.cs:299-338).
 *   data/nbytes: Q8_0 int8[rows*cols]; Q4_0 bytes[(rows*cols+1)/2];
 *                Q4_K 144 B per 256 elements; Q6_K 210 B per 256; F32 float[rows*cols].
 *   scales/nscales: fp32 block scales for Q8_0/Q4_0 (Q8Tensor.cs:36), else NULL/0.
 *   block_size: Q8_0/Q4_0 block size (reference default 64, Q8Tensor.cs:72); ignored otherwise.
 *   data and scales are host pointers. */
SM_API int sm_weight_upload(sm_ctx* ctx, int scheme, int rows, int cols, int block_size, const void* data,
                            size_t nbytes, const float* scales, size_t nscales, int layout, sm_weight** out);
/* Same, from device pointers (no host round trip). */
SM_API int sm_weight_upload_device(sm_ctx* ctx, int scheme, int rows, int cols, int block_size,
                                   const void* data_dev, size_t nbytes, const float* scales_dev, size_t nscales,
                                   int layout, sm_weight** out);
SM_API int sm_weight_destroy(sm_weight* w);
/* IWeightTensor.Rows / Cols / Scheme (IWeightTensor.cs:12-22) */
SM_API int sm_weight_info(const sm_weight* w, int* scheme, int* rows, int* cols, int* layout);
/* Device bytes held by the weight (packed data + scales). */
SM_API int sm_weight_nbytes(const sm_weight* w, size_t* out);

/* IWeightTensor.MatMul(activations, output, m, k, n) (IWeightTensor.cs:33):
 *   INTENDED layout: requires k == Cols, n == Rows; c[m][n] = sum_k a[m][k] w[n][k].
 *   REFERENCE layout: requires k == Rows, n == Cols (Q4KWeightTensor.cs:43-44); c = a . B.
 * a: fp32 [m][k] row-major; c: fp32 [m][n]; flags: SM_PTR_HOST / SM_PTR_DEVICE.   */
SM_API int sm_matmul(sm_weight* w, const float* a, float* c, int m, int k, int n, int flags);

/* IWeightTensor.ToFloat32() (IWeightTensor.cs:41): bit-exact dequantization of
 * the uploaded tensor, rows*cols fp32 in the uploaded linear order
 * (Q8Tensor.cs:131-158, Q4Tensor.cs:150-179, Q4KTensor.cs:71-148, Q6KTensor.cs:72-127). */
SM_API int sm_dequant(sm_weight* w, float* out, int flags);

/* Quantize fp32 -> packed on the device.  Q8_0 / Q4_0 are bit-exact with
 * Q8Tensor.Quantize (Q8Tensor.cs:72-125) / Q4Tensor.Quantize (Q4Tensor.cs:75-134);
 * Q4_K / Q6_K use this library's own quantizer (the reference has none).
 * src/data/scales are device pointers; data holds the packed bytes, scales the
 * fp32 block scales (Q8_0/Q4_0 only). */
SM_API int sm_quantize(sm_ctx* ctx, int scheme, const float* src, int64_t n, int block_size, void* data,
                       float* scales);

/* ---------------------------------------------------------------- ops */
/* RMSNormOps.RMSNorm (RMSNormOps.cs:28-220): y = gamma * (x / sqrt(mean(x^2) + eps)) per row. */
SM_API int sm_op_rmsnorm(sm_ctx* ctx, const float* x, const float* gamma, float* y, int rows, int features,
                         float eps, int flags);
/* RotaryEmbedding.ApplyInPlace on one token row [n_heads][head_dim] at position
 * pos (RotaryEmbedding.cs:69-121), interleaved pairs, theta tables as
 * RotaryEmbedding.cs:45-60.  x is rotated in place. */
SM_API int sm_op_rope(sm_ctx* ctx, float* x, int rows, int n_heads, int head_dim, const int* positions,
                      float theta, int max_seq, int flags);
/* ActivationOps.FusedSiLUMul (ActivationOps.cs:565-580) */
SM_API int sm_op_silu_mul(sm_ctx* ctx, const float* gate, const float* up, float* out, int n, int flags);
/* Causal GQA attention of one sequence (MultiHeadAttention.cs:676-744, 810-844
 * with OptimizedOps.FusedScaleMaskSoftmax, OptimizedOps.cs:39-95, and the Pade
 * MathUtils.FastExp, MathUtils.cs:20-32).  q: [T][n_heads*hd]; k, v:
 * [S][n_kv*hd]; query row i is at absolute position S-T+i.  out: [T][n_heads*hd]. */
SM_API int sm_attention(sm_ctx* ctx, const float* q, const float* k, const float* v, float* out, int T, int S,
                        int n_heads, int n_kv, int head_dim, int flags);
/* Decode attention for a batch of sequences of ragged lengths (one query row
 * each) over a head-major cache: k_cache/v_cache [B][n_kv][max_ctx][hd],
 * q/out [B][n_heads*hd], lens[B] >= 1.  Device pointers only. */
SM_API int sm_attention_decode(sm_ctx* ctx, const float* q, const float* k_cache, const float* v_cache,
                               float* out, const int* lens_dev, int B, int max_ctx, int n_heads, int n_kv,
                               int head_dim);

/* Same computation as sm_attention_decode, for callers that cannot let the
 * library allocate device memory (hosts that reserve their whole device budget
 * up front, or run where another allocator owns the device).  No counterpart in
 * the reference: it has no device memory at all.  Shapes the scratch-free
 * cluster kernel takes (head_dim 64, at most 8 q heads per kv head) use it;
 * other shapes take working memory from a fixed 16 MiB static device array held
 * by every GPU that loads the library, and those needing more
 * (B * n_heads * (max_ctx + 66 * ceil(max_ctx/64)) floats) return SM_ERR_SHAPE.
 * The first call on a device that uses the array looks up its address (make it
 * before any stream capture; a later reset of the device's primary context is
 * not supported).  Calls share the array: calls that overlap on the GPU race and
 * must be serialised.  Device pointers only. */
SM_API int sm_attention_decode_noalloc(sm_ctx* ctx, const float* q, const float* k_cache, const float* v_cache,
                                       float* out, const int* lens_dev, int B, int max_ctx, int n_heads, int n_kv,
                                       int head_dim);

/* ---------------------------------------------------------------- model */
/* ModelConfig fields used by the LLaMA path (ModelConfig.cs:14-136). */
typedef struct sm_model_config {
  int vocab_size;
  int hidden;       /* EmbeddingLength */
  int n_layers;     /* BlockCount */
  int n_heads;      /* HeadCount */
  int n_kv_heads;   /* HeadCountKv */
  int head_dim;
  int ffn_hidden;   /* FeedForwardLength */
  int max_context;  /* ContextLength (blockSize) */
  float norm_eps;   /* NormEps */
  float rope_theta; /* RopeFreqBase */
} sm_model_config;

/* Tensor roles of one transformer block (TransformerBlock.cs, MultiHeadAttention.cs:92-93,
 * GatedMLP.cs) and the model (TransformerModel.cs:163-259). */
#define SM_ROLE_ATTN_NORM 0
#define SM_ROLE_WQ 1
#define SM_ROLE_WK 2
#define SM_ROLE_WV 3
#define SM_ROLE_WO 4
#define SM_ROLE_FFN_NORM 5
#define SM_ROLE_W_GATE 6
#define SM_ROLE_W_UP 7
#define SM_ROLE_W_DOWN 8
#define SM_ROLE_TOKEN_EMBD 9 /* fp32 [vocab][hidden], layer ignored */
#define SM_ROLE_OUT_NORM 10  /* layer ignored */
#define SM_ROLE_OUTPUT 11    /* LM head weight, layer ignored */

/* new TransformerModel(ModelConfig) (TransformerModel.cs:163-259): an empty
 * device-resident model; fill it with sm_model_set_weight / _vector. */
SM_API int sm_model_create(sm_ctx* ctx, const sm_model_config* cfg, sm_model** out);
/* Linear.SetQuantizedWeight (NeuralNet.cs:84-107).  The model borrows w (INTENDED
 * layout, rows = out features, cols = in features); w must outlive the model. */
SM_API int sm_model_set_weight(sm_model* m, int layer, int role, sm_weight* w);
/* RMSNorm gamma (fp32[hidden]) or the fp32 token embedding (vocab*hidden); host pointer. */
SM_API int sm_model_set_vector(sm_model* m, int layer, int role, const float* data, size_t n);
/* Validates that every tensor is present with matching shapes. */
SM_API int sm_model_finalize(sm_model* m);
SM_API int sm_model_destroy(sm_model* m);
/* Device bytes held by the model's own buffers (embedding, norms, tables, workspace). */
SM_API int sm_model_nbytes(const sm_model* m, size_t* out);

/* ---- tensor-parallel decode (one process per GPU, NCCL loaded at run time) ----
 * The reference runs one CPU process; these entry points split one model over a
 * group of GPUs.  Each rank builds an ordinary model from its weight shards: the
 * column-split projections keep its q / kv heads and its FFN units (the rows of
 * Wq / Wk / Wv, MultiHeadAttention.cs:92-93 _qkv, and of gate / up,
 * GatedMLP.cs:38-40), the row-split ones keep the matching input columns (Wo,
 * MultiHeadAttention.cs:92-93 _proj; down, GatedMLP.cs:38-40) in whole 256-weight
 * blocks; embedding, norms and LM head are replicated.  After the O and down
 * projections every rank sums the partial outputs with one all-reduce before the
 * residual add (TransformerBlock.cs:170, :184), so all ranks hold the same
 * residual stream and produce the same logits. */
/* Writes the group's 128-byte id (rank 0 makes it; every rank passes the same bytes). */
SM_API int sm_tp_unique_id(void* id, size_t n);
/* Joins ctx to the group as rank tp_rank of tp_size (blocking until all ranks join). */
SM_API int sm_tp_init(sm_ctx* ctx, int tp_size, int tp_rank, const void* id, size_t n);
/* In-place sum of n floats (device pointer) over the group, on the context stream. */
SM_API int sm_tp_allreduce(sm_ctx* ctx, float* buf, size_t n);
/* Marks m as this rank's shard of a tensor-parallel model (enable = 1) or not (0).
 * SM_ERR_STATE if ctx has no group. */
SM_API int sm_model_set_tp(sm_model* m, int enable);

/* HBM KV cache for up to max_seqs sequences of max_tokens positions each
 * (replaces the per-layer caches of MultiHeadAttention.cs:252-274 and the session
 * store semantics of KvCacheEntry.cs:42-43).  fp32, [layer][seq][kv_head][pos][hd]. */
SM_API int sm_kv_create(sm_model* m, int max_seqs, int max_tokens, sm_kv** out);
SM_API int sm_kv_destroy(sm_kv* kv);
/* InferenceSession.ResetKVCache (InferenceSession.cs:485-526): length of seq -> 0. */
SM_API int sm_kv_reset(sm_kv* kv, int seq_id);
SM_API int sm_kv_length(sm_kv* kv, int seq_id, int* len);
/* Keep the first len tokens of seq_id (0 <= len <= current length): the cached
 * prefix that a new prompt shares (ChatSession.cs:282-300 reuses the cache when
 * the longest common prefix covers it; this also keeps a partial prefix). */
SM_API int sm_kv_truncate(sm_kv* kv, int seq_id, int len);
/* KvCacheEntry.Slide (KvCacheEntry.cs:203-229): keep the last `window` tokens,
 * moved to positions 0 .. window-1 of every layer; no-op when window >= length;
 * window < 0 is an error.  Cached keys keep the rotation of their old positions,
 * as in the reference. */
SM_API int sm_kv_slide(sm_kv* kv, int seq_id, int window);
/* KvCacheEntry.GetKeys / GetValues (KvCacheEntry.cs:155-189): tokens [start,
 * start + count) of one layer, into host arrays laid out [token][kv_head][head_dim]
 * (either may be NULL); the range must lie inside the cached tokens. */
SM_API int sm_kv_read(sm_kv* kv, int layer, int seq_id, int start, int count, float* keys, float* values);

/* Prefill: TransformerModel.Forward(idx[1,T], positionOffset = current length)
 * (TransformerModel.cs:272-344) appending T tokens to seq_id's cache; writes the
 * logits of the last position ([vocab]) and/or its greedy argmax.  tokens is
 * a host array; last_logits / next_token are host pointers (either may be NULL). */
SM_API int sm_prefill(sm_model* m, sm_kv* kv, int seq_id, const int* tokens, int n_tokens, float* last_logits,
                      int* next_token);
/* Several prompts in one pass (batched prefill, the multi-sequence form of
 * sm_prefill; BatchedInferenceEngine.cs:226-233 leaves batching unimplemented):
 * prompt i appends n_tokens[i] tokens to seq_ids[i]'s cache at its current
 * length.  tokens holds the prompts back to back.  The linear layers run once
 * over all the rows; attention runs per prompt over its own slot.  last_logits
 * [n][vocab] and/or next_tokens[n] (greedy) are host pointers (either may be
 * NULL).  Each sequence id appears at most once. */
SM_API int sm_prefill_batch(sm_model* m, sm_kv* kv, const int* seq_ids, const int* tokens, const int* n_tokens,
                            int n, float* last_logits, int* next_tokens);

/* One decode step for n sequences (InferenceSession.GenerateNextTokenAsync decode
 * branch, InferenceSession.cs:527-563, batched): token[i] is appended to
 * seq_ids[i]; logits [n][vocab] and/or greedy argmax next_tokens[n] (TopK = 1,
 * InferenceSession.cs:635-670; ties pick the lowest id) are written.
 * flags: SM_PTR_HOST (all arrays host) or SM_PTR_DEVICE (all arrays device; no sync). */
SM_API int sm_decode(sm_model* m, sm_kv* kv, const int* seq_ids, const int* tokens, int n, float* logits,
                     int* next_tokens, int flags);

/* Sampling options of InferenceSession's pipeline (InferenceSession.cs:565-606).
 * Disabled values: temperature 1, top_k <= 0, top_p >= 1, min_p <= 0,
 * repetition_penalty 1, presence / frequency penalty 0.  repetition_window 0
 * means min(context length, 256) (:780-783). */
typedef struct sm_sampling_params {
  double temperature;
  int top_k;
  double top_p;
  double min_p;
  float repetition_penalty;
  float presence_penalty;
  float frequency_penalty;
  int repetition_window;
} sm_sampling_params;

#define SM_SAMPLE_MAX_VOCAB 53248

/* One token per logits row through the reference sampling pipeline, on the
 * device (replaces InferenceSession.SampleNextToken's host stages: penalties
 * :769-850, temperature :741-763, top-k :635-670, softmax :672-712, top-p
 * :862-907, min-p :913-935, SampleFromProbs :714-734).
 * logits [n_rows][vocab] (vocab <= SM_SAMPLE_MAX_VOCAB); targets[n_rows] are the
 * uniform draws in [0, 1) that SampleFromProbs compares the cumulative sum with
 * (the reference takes them from DeterministicRng.NextDouble); context
 * [n_rows][context_stride] with context_lens[n_rows] (each <= context_stride) are
 * each row's token history for the penalties (NULL when no penalty is set; ids
 * outside [0, vocab) are skipped).  tokens[n_rows] receives the samples; probs (may be NULL)
 * [n_rows][vocab] the final distribution.  flags: SM_PTR_HOST (all arrays host,
 * synchronous) or SM_PTR_DEVICE (all arrays device; stream-ordered, no
 * allocation). */
SM_API int sm_sample(sm_ctx* ctx, const float* logits, int n_rows, int vocab, const sm_sampling_params* params,
                     const int* context, const int* context_lens, int context_stride, const double* targets,
                     int* tokens, float* probs, int flags);

/* Number of kernels the library launched on this context so far (evidence
 * counter for benchmarks). */
SM_API int sm_ctx_launch_count(sm_ctx* ctx, int64_t* out);

#ifdef __cplusplus
}
#endif
#endif /* SMALLMIND_CUDA_H */
