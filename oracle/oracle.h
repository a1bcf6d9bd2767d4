/*
 * SmallMind quantized-path ORACLE — test infrastructure only.
 *
 * A plain C++17 CPU restatement of the reference (justinamiller/SmallMind,
 * C# / .NET 10) arithmetic for the quantized decode/prefill hot path.  It is
 * the checker for the CUDA library and the timed CPU baseline of bench.py; no
 * product code path may call it.  Every function cites the reference
 * file:line it restates (paths relative to the reference project root).
 *
 * Parity pinning: the reference cannot be built here (no .NET toolchain), so
 * this restatement is pinned against every exact known-answer the reference's
 * own tests hold for the path (nibble decode, block sizes/bytes, RoPE identity
 * at position 0, RMSNorm formula values) and replays the reference's seeded
 * matmul tests (System.Random(42) restated below) at the reference's own
 * tolerances.  Q4_K/Q6_K dequant values, attention and end-to-end logits are
 * not pinned by any reference test (theirs are skipped or placeholders); for
 * those rows parity means agreement with this restatement.
 *
 * All arithmetic is compiled with -ffp-contract=off: the reference's .NET JIT
 * does not contract a*b+c into FMA, so every product and sum rounds separately.
 */
#ifndef SMALLMIND_ORACLE_H
#define SMALLMIND_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* QuantScheme values of src/SmallMind.Quantization/Abstractions/IWeightTensor.cs:47-72 */
enum { OR_F32 = 0, OR_F16 = 1, OR_Q8_0 = 2, OR_Q4_0 = 3, OR_Q4_1 = 4, OR_Q5_0 = 5, OR_Q4_K = 6, OR_Q6_K = 7 };

/* ---- System.Random(seed) (legacy seeded algorithm, Knuth subtractive) ---- */
typedef struct { int32_t seed_array[56]; int inext, inextp; } or_dotnet_random;
void   or_dotnet_random_init(or_dotnet_random* r, int32_t seed);
double or_dotnet_random_next_double(or_dotnet_random* r);
/* GenerateRandomFloats of tests/SmallMind.Quantization.Tests/QuantKernelsTests.cs:260-269 */
void   or_dotnet_random_floats(or_dotnet_random* r, float* out, int count, float min, float max);

/* ---- fp16 ---- */
float    or_half_to_float(uint16_t h);        /* Q4KTensor.cs:155-191 */
uint16_t or_float_to_half_rne(float f);       /* used by the K-quant quantizers of this build */

/* ---- Q8_0 (Q8Tensor.cs) ---- */
int  or_q8_quantize(const float* src, int64_t n, int block_size, int8_t* data, float* scales);
void or_q8_dequantize(const int8_t* data, const float* scales, int64_t n, int block_size, float* out);
/* ---- Q4_0 (Q4Tensor.cs) ---- */
int  or_q4_decode_nibble(int nibble);
int  or_q4_quantize(const float* src, int64_t n, int block_size, uint8_t* data, float* scales);
void or_q4_dequantize(const uint8_t* data, const float* scales, int64_t n, int block_size, float* out);
/* ---- Q4_1 (Q4_1Tensor.cs) and Q5_0 (Q5_0Tensor.cs), block size 32 ----
 * In or_matmul: Q4_1 `scales` = the block scales followed by the block mins;
 * Q5_0 `data` = the low nibbles ((n+1)/2 bytes) followed by the 4-byte high-bit words. */
int  or_q41_quantize(const float* src, int64_t n, uint8_t* data, float* scales, float* mins);
void or_q41_dequantize(const uint8_t* data, const float* scales, const float* mins, int64_t n, float* out);
int  or_q50_quantize(const float* src, int64_t n, uint8_t* low, uint8_t* high, float* scales);
void or_q50_dequantize(const uint8_t* low, const uint8_t* high, const float* scales, int64_t n, float* out);
/* ---- Q4_K / Q6_K (Q4KTensor.cs, Q6KTensor.cs); quantizers are this build's own ---- */
void or_q4k_quantize(const float* src, int64_t n, uint8_t* out);
void or_q4k_dequantize(const uint8_t* src, int64_t n, float* out);
void or_q6k_quantize(const float* src, int64_t n, uint8_t* out);
void or_q6k_dequantize(const uint8_t* src, int64_t n, float* out);

/* ---- Quantized matmul ----
 * mode 0 = reference-literal: C[MxN] = A[MxK] * B with B the tensor (rows=K, cols=N);
 *          Q8/Q4: linear row-major KxN; K-quants: block (k/256)*N + n.
 *          Follows MatMulF32Q8.cs:53-80, MatMulF32Q4.cs:61-92,
 *          FusedQ4KMatMul.cs:76-197, FusedQ6KMatMul.cs:66-164 accumulation order.
 * mode 1 = intended (x . W^T, IWeightTensor.cs:25-26): W is [N][K] row-major,
 *          quantized linearly (blocks along K; K-quant block n*(K/256)+kb),
 *          y[m][n] = sum_k a[m][k] * w[n][k] with w the reference element formula.
 * data: packed bytes; scales: fp32 block scales (Q8/Q4 only, else NULL).
 * out64 (optional): same sum in double precision (error budget twin).        */
int or_matmul(int scheme, int mode, const void* data, const float* scales, int block_size,
              const float* A, float* C, double* C64, int M, int K, int N);

/* ---- Model-level ops ---- */
/* RMSNormOps.cs:28-220 */
void  or_rmsnorm(const float* x, const float* gamma, float* y, int rows, int features, float eps);
/* RotaryEmbedding.cs:45-60: tables [max_seq][head_dim/2] */
void  or_rope_tables(int max_seq, int head_dim, float theta, float* sin_t, float* cos_t);
/* RotaryEmbedding.cs:69-121 on one [n_heads][head_dim] token row */
void  or_rope_apply(float* x, int n_heads, int head_dim, int pos, const float* sin_t, const float* cos_t);
/* MathUtils.cs:20-32 */
float or_fast_exp(float x);
/* ActivationOps.cs:304-309,565-580 */
void  or_silu_mul(const float* gate, const float* up, float* out, int n);
/* Causal GQA attention over a full sequence (cache-off semantics,
 * MultiHeadAttention.cs:676-744,810-844; OptimizedOps.cs:39-95).
 * q: [T][n_heads*hd]; k,v: [S][n_kv*hd]; query row i sits at absolute
 * position (S - T + i) and sees keys 0..S-T+i. out: [T][n_heads*hd]. */
void  or_attention(const float* q, const float* k, const float* v, float* out,
                   int T, int S, int n_heads, int n_kv, int head_dim, int n_threads);

/* ---- LLaMA-shaped model (TransformerModel.cs:272-344, TransformerBlock.cs:153-187) ---- */
typedef struct {
  int vocab_size, hidden, n_layers, n_heads, n_kv_heads, head_dim, ffn_hidden, max_context;
  float norm_eps, rope_theta;
} or_model_config;

/* one quantized linear: intended orientation, W [rows=N][cols=K] */
typedef struct {
  int scheme;          /* OR_Q8_0 / OR_Q4_0 / OR_Q4_K / OR_Q6_K / OR_F32 */
  int block_size;      /* Q8/Q4 block size */
  const void* data;    /* packed bytes (or float* for F32) */
  const float* scales; /* Q8/Q4 scales */
} or_linear;

typedef struct {
  const float* attn_norm; const float* ffn_norm;
  or_linear wq, wk, wv, wo, w_gate, w_up, w_down;
} or_layer;

typedef struct {
  or_model_config cfg;
  const float* token_embd;  /* [vocab][hidden] fp32 */
  const float* out_norm;
  or_linear output;
  const or_layer* layers;
} or_model;

/* Full forward over tokens[0..T) from position 0 (cache-off recompute),
 * writing logits of the last n_last positions into logits [n_last][vocab].
 * The reference computes the head for all T rows (TransformerModel.cs:343);
 * rows other than the last n_last are skipped here since nothing reads them. */
int or_model_forward(const or_model* m, const int* tokens, int T, int n_last, float* logits, int n_threads);

/* KV-cached decode twin used by the CPU baseline: same math, but keeps K/V
 * for past positions so each new token costs one row.  kv: [layers][2][max_ctx][n_kv*hd]. */
/* 0: linears use the caller's n_threads; 1: single-threaded, as the reference runs them. */
void or_set_linear_threads(int n);
int or_model_step(const or_model* m, float* kv, int pos, const int* tokens, int T, float* last_logits, int n_threads);

/* One token from one logits row through the reference sampling pipeline
 * (InferenceSession.cs:565-606): repetition / presence / frequency penalties
 * over the context window (:769-850), temperature (:741-763), top-k (:635-670),
 * softmax (:672-712), top-p (:862-907), min-p (:913-935), then the first index
 * whose double cumulative probability reaches `target` (:714-734), `target`
 * being the caller's uniform draw.  logits is modified in place; probs_out
 * (may be NULL) receives the final distribution.  Disabled values:
 * temperature 1, top_k <= 0, top_p >= 1, min_p <= 0, penalties 1 / 0 / 0. */
int or_sample(float* logits, int V, double temperature, int top_k, double top_p, double min_p, float rep_penalty,
              float presence_penalty, float frequency_penalty, int rep_window, const int* context, int ctx_len,
              double target, float* probs_out);

/* DeterministicRng (src/SmallMind.Core/Rng/DeterministicRng.cs): SplitMix64-seeded
 * xoroshiro128+; writes n NextDouble() draws. */
void or_deterministic_rng_doubles(int32_t seed, int n, double* out);

/* synthetic weights: N(0, std) from a counter-based generator (SplitMix64 + Box-Muller) */
void or_fill_normal(float* out, int64_t n, uint64_t seed, float std_dev, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
