// Element-wise / row kernels of the LLaMA block: RMSNorm, RoPE + KV append,
// SiLU-gate, embedding gather, greedy argmax.
#include <cfloat>

#include "common.cuh"

namespace sm {
namespace {

// RMSNormOps.cs:28-220: invRms = 1/sqrt(sumSq/F + eps); y = gamma * (x * invRms).
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ gamma, float* __restrict__ y,
                               int F, float eps) {
  const int row = blockIdx.x;
  const float* xr = x + (int64_t)row * F;
  float s = 0.f;
  for (int f = threadIdx.x; f < F; f += blockDim.x) s = fmaf(xr[f], xr[f], s);
  __shared__ float red[32];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(red[0], (float)F), eps)));
  float* yr = y + (int64_t)row * F;
  for (int f = threadIdx.x; f < F; f += blockDim.x) yr[f] = __fmul_rn(gamma[f], __fmul_rn(xr[f], inv));
}

// RotaryEmbedding.cs:103-116 on interleaved pairs with host-built tables.
__global__ void rope_rows_kernel(float* __restrict__ x, int row_stride, int n_heads, int hd,
                                 const int* __restrict__ positions, const float* __restrict__ sin_t,
                                 const float* __restrict__ cos_t) {
  const int row = blockIdx.x;
  const int half = hd / 2;
  const int pos = positions[row];
  float* xr = x + (int64_t)row * row_stride;
  for (int t = threadIdx.x; t < n_heads * half; t += blockDim.x) {
    const int h = t / half, i = t - h * half;
    float* p = xr + h * hd + 2 * i;
    const float x0 = p[0], x1 = p[1];
    const float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
    p[0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    p[1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  }
}

// Fused: RoPE on the Q and K parts of a merged [Q | K | V] row
// (MultiHeadAttention.cs:229-243) and append of rotated K and raw V to the
// head-major cache [seq][kv_head][pos][hd] (MultiHeadAttention.cs:262-274).
__global__ void rope_qk_append_kernel(float* __restrict__ qkv, int qkv_stride, int nH, int nKv, int hd,
                                      const int* __restrict__ positions, const int* __restrict__ seq_ids,
                                      const float* __restrict__ sin_t, const float* __restrict__ cos_t,
                                      float* __restrict__ kcache, float* __restrict__ vcache, int max_ctx) {
  const int row = blockIdx.x;
  const int half = hd / 2;
  const int pos = positions[row];
  const int64_t seq = seq_ids[row];
  float* r = qkv + (int64_t)row * qkv_stride;
  const int qd = nH * hd, kd = nKv * hd;
  // Q heads
  for (int t = threadIdx.x; t < nH * half; t += blockDim.x) {
    const int h = t / half, i = t - h * half;
    float* p = r + h * hd + 2 * i;
    const float x0 = p[0], x1 = p[1];
    const float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
    p[0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    p[1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  }
  // K heads -> rotated into cache; V -> cache
  for (int t = threadIdx.x; t < nKv * half; t += blockDim.x) {
    const int h = t / half, i = t - h * half;
    const float* p = r + qd + h * hd + 2 * i;
    const float x0 = p[0], x1 = p[1];
    const float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
    float* kd_ = kcache + ((seq * nKv + h) * max_ctx + pos) * hd + 2 * i;
    kd_[0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    kd_[1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    const float* pv = r + qd + kd + h * hd + 2 * i;
    float* vd = vcache + ((seq * nKv + h) * max_ctx + pos) * hd + 2 * i;
    vd[0] = pv[0];
    vd[1] = pv[1];
  }
}

// ActivationOps.cs:304-309,565-580: silu(g) * u with sigmoid = 1/(1+exp(-clamp(g,+-20))).
__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ out,
                                int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = g[i];
    const float c = fmaxf(-20.f, fminf(x, 20.f));
    const float sig = __fdiv_rn(1.f, __fadd_rn(1.f, expf(-c)));
    out[i] = __fmul_rn(__fmul_rn(x, sig), u[i]);
  }
}

// Embedding.Forward (NeuralNet.cs:376-): row gather.
__global__ void embed_kernel(const float* __restrict__ table, const int* __restrict__ tokens, float* __restrict__ x,
                             int H) {
  const int row = blockIdx.x;
  const float4* src = (const float4*)(table + (int64_t)tokens[row] * H);
  float4* dst = (float4*)(x + (int64_t)row * H);
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
  for (int i = (H / 4) * 4 + threadIdx.x; i < H; i += blockDim.x)
    x[(int64_t)row * H + i] = table[(int64_t)tokens[row] * H + i];
}

// Greedy TopK = 1 (InferenceSession.cs:635-670): max logit, lowest id on ties.
__global__ void argmax_kernel(const float* __restrict__ logits, int V, int* __restrict__ out) {
  const int row = blockIdx.x;
  const float* l = logits + (int64_t)row * V;
  float best = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = l[i];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  if ((threadIdx.x & 31) == 0) {
    sb[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sb[w] > best || (sb[w] == best && si[w] < bi)) {
        best = sb[w];
        bi = si[w];
      }
    out[row] = bi;
  }
}

}  // namespace

int launch_rmsnorm(const float* x, const float* gamma, float* y, int rows, int F, float eps, cudaStream_t st) {
  if (rows <= 0) return SM_OK;
  rmsnorm_kernel<<<rows, 256, 0, st>>>(x, gamma, y, F, eps);
  SM_CUDA_TRY(cudaGetLastError());
  return SM_OK;
}

int launch_rope_rows(float* x, int rows, int row_stride, int n_heads, int hd, const int* positions, const float* sin_t,
                     const float* cos_t, cudaStream_t st) {
  if (rows <= 0) return SM_OK;
  rope_rows_kernel<<<rows, 128, 0, st>>>(x, row_stride, n_heads, hd, positions, sin_t, cos_t);
  SM_CUDA_TRY(cudaGetLastError());
  return SM_OK;
}

int launch_rope_qk_append(float* qkv, int rows, int qkv_stride, int nH, int nKv, int hd, const int* positions,
                          const int* seq_ids, const float* sin_t, const float* cos_t, float* kc, float* vc,
                          int max_ctx, cudaStream_t st) {
  if (rows <= 0) return SM_OK;
  rope_qk_append_kernel<<<rows, 128, 0, st>>>(qkv, qkv_stride, nH, nKv, hd, positions, seq_ids, sin_t, cos_t, kc,
                                               vc, max_ctx);
  SM_CUDA_TRY(cudaGetLastError());
  return SM_OK;
}

int launch_silu_mul(const float* g, const float* u, float* out, int64_t n, cudaStream_t st) {
  if (n <= 0) return SM_OK;
  int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  silu_mul_kernel<<<grid, 256, 0, st>>>(g, u, out, n);
  SM_CUDA_TRY(cudaGetLastError());
  return SM_OK;
}

int launch_embed(const float* table, const int* tokens, float* x, int n, int H, cudaStream_t st) {
  if (n <= 0) return SM_OK;
  embed_kernel<<<n, 128, 0, st>>>(table, tokens, x, H);
  SM_CUDA_TRY(cudaGetLastError());
  return SM_OK;
}

int launch_argmax(const float* logits, int rows, int V, int* out, cudaStream_t st) {
  if (rows <= 0) return SM_OK;
  argmax_kernel<<<rows, 1024, 0, st>>>(logits, V, out);
  SM_CUDA_TRY(cudaGetLastError());
  return SM_OK;
}

}  // namespace sm
