// Token sampling on the device: the reference's per-token sampling pipeline
// (InferenceSession.cs:565-606) over logits rows that already sit in HBM,
// replacing the host full-vocab sort of the reference (ApplyTopK, :635-670;
// ApplyTopP, :862-907).
//
// One 1024-thread CTA per row; the row is staged once in shared memory
// (vocab <= SM_SAMPLE_MAX_VOCAB) and every stage works there:
//   penalties   one thread per distinct token of the window (first occurrence)
//   temperature x * (1 / T)
//   top-k       exact k-th largest value: the row turned into order-preserving
//               keys, the largest key x with count(key >= x) >= k found bit by
//               bit (key_search: one barrier per block step; the last bits on a
//               compacted bucket in one warp)
//   softmax     block max, expf, block sum, division
//   top-p       the cut value by the same search over the probability's bits
//               (fp32 per thread, float64 across threads); ties at the cut kept
//               in index order
//   min-p       block max, threshold, renormalise (multiply by 1 / sum)
//   sample      per-thread contiguous chunks, block scan of the chunk sums in
//               double, first index whose cumulative sum reaches the target.
// The caller supplies the uniform target per row (the reference draws it from
// DeterministicRng / System.Random, DeterministicRng.cs).
#include <cfloat>

#include "common.cuh"

namespace sm {
int ctx_view(sm_ctx* ctx, int* device, cudaStream_t* stream, int64_t** launches);

namespace {

// current device switched for the call's duration
struct SampleDeviceGuard {
  int prev = -1;
  explicit SampleDeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~SampleDeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

constexpr int ST = 1024;
constexpr int SW = ST / 32;

struct SampleArgs {
  const float* logits;
  int vocab;
  sm_sampling_params p;
  const int* context;
  const int* context_lens;
  int context_stride;
  const double* targets;
  int* tokens;
  float* probs;
};

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide reductions through a 32-entry shared scratch; every thread gets the result.
template <typename T>
__device__ __forceinline__ T block_sum(T v, T* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = lane < SW ? red[lane] : T(0);
  return warp_sum(v);
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = lane < SW ? red[lane] : -INFINITY;
  return warp_max(v);
}
// Exclusive scan of one value per thread (thread order); returns this thread's prefix.
__device__ __forceinline__ double block_exclusive_scan(double v, double* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  double x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) red[w] = x;
  __syncthreads();
  if (w == 0) {
    double s = lane < SW ? red[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < SW) red[lane] = s;  // inclusive warp prefix
  }
  __syncthreads();
  return (w ? red[w - 1] : 0.0) + x - v;
}

// order-preserving key of a float (ascending)
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// 1 / s in float, s > 0 (NormalizeProbabilities, InferenceSession.cs:1011-1030)
__device__ __forceinline__ void normalize(float* P, int V, float* redf) {
  float s = 0.f;
  for (int i = threadIdx.x; i < V; i += ST) s += P[i];
  s = block_sum(s, redf);
  if (s > 0.f) {
    const float inv = __fdiv_rn(1.0f, s);
    for (int i = threadIdx.x; i < V; i += ST) P[i] = __fmul_rn(P[i], inv);
  }
  __syncthreads();
}

// Bitwise search for the largest key x with  W(key >= x) >= need,  W = element
// count (top-k) or the sum of the probabilities (top-p; keys are then the bits of
// p >= 0).  Block-wide steps (one barrier each, double-buffered partials) narrow
// the bucket of keys sharing x's decided bits; once it holds <= LIST_MAX
// elements they are compacted into `list` and warp 0 decides the remaining bits
// alone.  Returns x, the weight strictly above x and the number of keys equal to x.
constexpr int LIST_MAX = 1024;
struct Found {
  uint32_t x;
  double above;
  int eq;
};

template <bool SUM>
__device__ Found key_search(const uint32_t* K, int V, double need, int top_bit, uint32_t* list, double* redw,
                            int* redc, int* list_n, Found* out) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t x = 0, mask = 0;
  double above = 0.0;
  int pop = V, bit = top_bit, ph = 0;
  for (; bit >= 0 && pop > LIST_MAX; --bit) {
    const uint32_t b = 1u << bit;
    float sw = 0.f;
    int sc = 0;
    for (int i = threadIdx.x; i < V; i += ST) {
      const uint32_t k = K[i];
      if ((k & mask) == x && (k & b)) {
        if (SUM) sw += __uint_as_float(k);
        ++sc;
      }
    }
    const double dw = warp_sum(SUM ? (double)sw : 0.0);
    sc = warp_sum(sc);
    if (lane == 0) {
      redw[ph * 32 + w] = dw;
      redc[ph * 32 + w] = sc;
    }
    __syncthreads();
    const double tw = SUM ? warp_sum(lane < SW ? redw[ph * 32 + lane] : 0.0) : 0.0;
    const int tc = warp_sum(lane < SW ? redc[ph * 32 + lane] : 0);
    ph ^= 1;
    const double t = SUM ? tw : (double)tc;
    if (above + t >= need) {
      x |= b;
      pop = tc;
    } else {
      above += t;
      pop -= tc;
    }
    mask |= b;
  }
  if (bit >= 0) {
    // compact the bucket (pop <= LIST_MAX keys) and finish in warp 0
    if (threadIdx.x == 0) *list_n = 0;
    __syncthreads();
    for (int i0 = 0; i0 < V; i0 += ST) {
      const int i = i0 + threadIdx.x;
      const uint32_t k = i < V ? K[i] : 0u;
      const bool in = i < V && (k & mask) == x;
      const unsigned bal = __ballot_sync(0xffffffffu, in);
      int base = 0;
      if (lane == 0 && bal) base = atomicAdd(list_n, __popc(bal));
      base = __shfl_sync(0xffffffffu, base, 0);
      if (in) list[base + __popc(bal & ((1u << lane) - 1u))] = k;
    }
    __syncthreads();
    if (w == 0) {
      const int n = *list_n;
      for (; bit >= 0; --bit) {
        const uint32_t b = 1u << bit;
        float sw = 0.f;
        int sc = 0;
        for (int j = lane; j < n; j += 32) {
          const uint32_t k = list[j];
          if ((k & mask) == x && (k & b)) {
            if (SUM) sw += __uint_as_float(k);
            ++sc;
          }
        }
        const double t = SUM ? warp_sum((double)sw) : (double)warp_sum(sc);
        const int tc = warp_sum(sc);
        if (above + t >= need) {
          x |= b;
          pop = tc;
        } else {
          above += t;
          pop -= tc;
        }
        mask |= b;
      }
      if (lane == 0) *out = Found{x, above, pop};
    }
    __syncthreads();
    return *out;
  }
  return Found{x, above, pop};
}

__global__ void __launch_bounds__(ST, 1) sample_kernel(const __grid_constant__ SampleArgs a) {
  extern __shared__ float P[];  // the row: logits, then probabilities
  __shared__ float redf[32];
  __shared__ double redd[32];
  __shared__ int redi[32];
  __shared__ double sredw[64];
  __shared__ int sredc[64];
  __shared__ uint32_t slist[LIST_MAX];
  __shared__ int slist_n;
  __shared__ Found sfound;
  const int V = a.vocab, row = blockIdx.x, tid = threadIdx.x;
  const sm_sampling_params& p = a.p;
  const float* src = a.logits + (size_t)row * V;
  for (int i = tid; i < V; i += ST) P[i] = src[i];
  __syncthreads();

  // 1. penalties (InferenceSession.cs:769-850): one thread per distinct window token
  if (!(p.repetition_penalty == 1.0f && p.presence_penalty == 0.0f && p.frequency_penalty == 0.0f) && a.context) {
    const int* ctx = a.context + (size_t)row * a.context_stride;
    const int n = a.context_lens ? a.context_lens[row] : 0;
    const int win = p.repetition_window > 0 ? p.repetition_window : min(n, 256);
    const int start = max(0, n - win);
    for (int i = start + tid; i < n; i += ST) {
      const int t = ctx[i];
      bool first = t >= 0 && t < V;
      for (int j = start; j < i && first; ++j) first = ctx[j] != t;
      if (!first) continue;
      int cnt = 0;
      for (int j = start; j < n; ++j) cnt += ctx[j] == t;
      float x = P[t];
      if (p.repetition_penalty != 1.0f) x = x > 0.f ? __fdiv_rn(x, p.repetition_penalty) : __fmul_rn(x, p.repetition_penalty);
      if (p.presence_penalty != 0.0f) x = __fsub_rn(x, p.presence_penalty);
      if (p.frequency_penalty != 0.0f) x = __fsub_rn(x, __fmul_rn((float)cnt, p.frequency_penalty));
      P[t] = x;
    }
    __syncthreads();
  }
  // 2. temperature (:741-763)
  if (p.temperature != 1.0) {
    const float inv = __fdiv_rn(1.0f, (float)p.temperature);
    for (int i = tid; i < V; i += ST) P[i] = __fmul_rn(P[i], inv);
    __syncthreads();
  }
  // 3. top-k (:635-670): exact k-th largest (descending-sort position k-1), values below -> -inf.
  // The row becomes order-preserving keys; the k-th largest key is the largest x with
  // count(key >= x) >= k.
  if (p.top_k > 0 && p.top_k < V) {
    uint32_t* K = reinterpret_cast<uint32_t*>(P);
    for (int i = tid; i < V; i += ST) K[i] = fkey(P[i]);
    __syncthreads();
    const uint32_t x = key_search<false>(K, V, (double)p.top_k, 31, slist, sredw, sredc, &slist_n, &sfound).x;
    for (int i = tid; i < V; i += ST) {
      const uint32_t k = K[i];
      const float v = __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
      P[i] = k >= x ? v : -INFINITY;
    }
    __syncthreads();
  }
  // 4. softmax (:672-712)
  {
    float m = -INFINITY;
    for (int i = tid; i < V; i += ST)
      if (P[i] != -INFINITY) m = fmaxf(m, P[i]);
    m = block_max(m, redf);
    float s = 0.f;
    for (int i = tid; i < V; i += ST) {
      const float x = P[i];
      const float e = x != -INFINITY ? expf(__fsub_rn(x, m)) : 0.f;
      P[i] = e;
      s += e;
    }
    s = block_sum(s, redf);
    if (s > 0.f)
      for (int i = tid; i < V; i += ST) P[i] = __fdiv_rn(P[i], s);
    __syncthreads();
  }
  // contiguous per-thread chunks of odd length (no shared-memory bank conflicts)
  int chunk = (V + ST - 1) / ST;
  chunk |= 1;
  const int c0 = min(V, tid * chunk), c1 = min(V, c0 + chunk);
  // 5. top-p (:862-907): the cut value tau = the largest p with sum(p >= tau) >= top_p
  if (p.top_p < 1.0) {
    // top_p <= 0: the reference's first sorted token already reaches it (:891-896), so only the top
    // probability is kept; a tiny positive target gives that cut
    const double need = p.top_p > 0.0 ? p.top_p : 1e-300;
    const Found f = key_search<true>(reinterpret_cast<const uint32_t*>(P), V, need, 30, slist, sredw, sredc,
                                     &slist_n, &sfound);
    const float tau = __uint_as_float(f.x);
    const double above = f.above;
    const int neq = f.eq;
    // keep the first m ties at the cut (index order)
    int m = neq;
    if (tau > 0.f && above < need) m = min(neq, max(1, (int)ceil((need - above) / (double)tau)));
    int mine = 0;
    for (int i = c0; i < c1; ++i) mine += P[i] == tau;
    int before = (int)block_exclusive_scan((double)mine, redd);
    for (int i = c0; i < c1; ++i) {
      const float v = P[i];
      if (v < tau) P[i] = 0.f;
      else if (v == tau) {
        if (before >= m) P[i] = 0.f;
        ++before;
      }
    }
    __syncthreads();
    normalize(P, V, redf);
  }
  // 6. min-p (:913-935)
  if (p.min_p > 0.0) {
    float m = -INFINITY;
    for (int i = tid; i < V; i += ST) m = fmaxf(m, P[i]);
    m = block_max(m, redf);
    const float thr = __fmul_rn(m, (float)p.min_p);
    for (int i = tid; i < V; i += ST)
      if (P[i] < thr) P[i] = 0.f;
    __syncthreads();
    normalize(P, V, redf);
  }
  if (a.probs) {
    float* dst = a.probs + (size_t)row * V;
    for (int i = tid; i < V; i += ST) dst[i] = P[i];
  }
  // 7. SampleFromProbs (:714-734): first index whose double cumulative sum reaches the target
  {
    double mine = 0.0;
    for (int i = c0; i < c1; ++i) mine += (double)P[i];
    double cum = block_exclusive_scan(mine, redd);
    const double target = a.targets[row];
    int found = V;
    for (int i = c0; i < c1; ++i) {
      cum += (double)P[i];
      if (cum >= target) {
        found = i;
        break;
      }
    }
    int f = found;
#pragma unroll
    for (int o = 16; o; o >>= 1) f = min(f, __shfl_xor_sync(0xffffffffu, f, o));
    __syncthreads();
    if ((tid & 31) == 0) redi[tid >> 5] = f;
    __syncthreads();
    if (tid < 32) {
      f = tid < SW ? redi[tid] : V;
#pragma unroll
      for (int o = 16; o; o >>= 1) f = min(f, __shfl_xor_sync(0xffffffffu, f, o));
      if (tid == 0) a.tokens[row] = f < V ? f : V - 1;
    }
  }
}

}  // namespace

int launch_sample(const float* logits, int n_rows, int vocab, const sm_sampling_params& p, const int* context,
                  const int* context_lens, int context_stride, const double* targets, int* tokens, float* probs,
                  cudaStream_t st, int64_t* launches) {
  const size_t smem = sizeof(float) * (size_t)vocab;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    SM_CUDA_TRY(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)(sizeof(float) * SM_SAMPLE_MAX_VOCAB)));
    attr[dev] = true;
  }
  SampleArgs a{logits, vocab, p, context, context_lens, context_stride, targets, tokens, probs};
  sample_kernel<<<n_rows, ST, smem, st>>>(a);
  SM_CUDA_TRY(cudaGetLastError());
  if (launches) ++*launches;
  return SM_OK;
}

}  // namespace sm

using namespace sm;

SM_API int sm_sample(sm_ctx* ctx, const float* logits, int n_rows, int vocab, const sm_sampling_params* params,
                     const int* context, const int* context_lens, int context_stride, const double* targets,
                     int* tokens, float* probs, int flags) {
  int dev = 0;
  cudaStream_t st = nullptr;
  int64_t* launches = nullptr;
  SM_TRY(ctx_view(ctx, &dev, &st, &launches));
  if (!logits || !params || !targets || !tokens) return fail(SM_ERR_INVALID_ARG, "sample: null argument");
  if (n_rows <= 0 || vocab <= 0) return fail(SM_ERR_SHAPE, "sample: rows and vocab must be positive");
  if (vocab > SM_SAMPLE_MAX_VOCAB) return fail(SM_ERR_UNSUPPORTED, "sample: vocab above SM_SAMPLE_MAX_VOCAB");
  const sm_sampling_params p = *params;
  if (!(p.temperature > 0.0)) return fail(SM_ERR_INVALID_ARG, "sample: temperature must be positive");
  const bool pen = !(p.repetition_penalty == 1.0f && p.presence_penalty == 0.0f && p.frequency_penalty == 0.0f);
  if (pen && context && (!context_lens || context_stride <= 0))
    return fail(SM_ERR_INVALID_ARG, "sample: context needs context_lens and a positive stride");
  if (flags != SM_PTR_HOST && flags != SM_PTR_DEVICE) return fail(SM_ERR_INVALID_ARG, "sample: bad pointer flags");
  SampleDeviceGuard g(dev);
  if (flags == SM_PTR_DEVICE)
    return launch_sample(logits, n_rows, vocab, p, pen ? context : nullptr, context_lens, context_stride, targets,
                         tokens, probs, st, launches);
  // host buffers: one device staging block, copies in, kernel, copies out, synchronise
  if (pen && context)
    for (int r = 0; r < n_rows; ++r)
      if (context_lens[r] < 0 || context_lens[r] > context_stride)
        return fail(SM_ERR_SHAPE, "sample: context length outside [0, stride]");
  const size_t nl = (size_t)n_rows * vocab, nc = pen && context ? (size_t)n_rows * context_stride : 0;
  const size_t off_probs = nl * 4, off_tgt = off_probs + (probs ? nl * 4 : 0), off_ctx = off_tgt + 8 * (size_t)n_rows,
               off_len = off_ctx + 4 * nc, off_tok = off_len + 4 * (size_t)n_rows, total = off_tok + 4 * (size_t)n_rows;
  uint8_t* buf = nullptr;
  if (cudaMallocAsync((void**)&buf, total, st) != cudaSuccess) return fail(SM_ERR_OOM, "sample: device allocation failed");
  int rc = SM_OK;
  auto cp = [&](void* d, const void* h, size_t n) {
    if (rc == SM_OK && n && cudaMemcpyAsync(d, h, n, cudaMemcpyHostToDevice, st) != cudaSuccess)
      rc = fail(SM_ERR_CUDA, "sample: copy to device failed");
  };
  cp(buf, logits, nl * 4);
  cp(buf + off_tgt, targets, 8 * (size_t)n_rows);
  if (nc) {
    cp(buf + off_ctx, context, 4 * nc);
    cp(buf + off_len, context_lens, 4 * (size_t)n_rows);
  }
  if (rc == SM_OK)
    rc = launch_sample((const float*)buf, n_rows, vocab, p, nc ? (const int*)(buf + off_ctx) : nullptr,
                       nc ? (const int*)(buf + off_len) : nullptr, context_stride, (const double*)(buf + off_tgt),
                       (int*)(buf + off_tok), probs ? (float*)(buf + off_probs) : nullptr, st, launches);
  if (rc == SM_OK && cudaMemcpyAsync(tokens, buf + off_tok, 4 * (size_t)n_rows, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    rc = fail(SM_ERR_CUDA, "sample: copy to host failed");
  if (rc == SM_OK && probs &&
      cudaMemcpyAsync(probs, buf + off_probs, nl * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    rc = fail(SM_ERR_CUDA, "sample: copy to host failed");
  cudaFreeAsync(buf, st);
  if (cudaStreamSynchronize(st) != cudaSuccess && rc == SM_OK) rc = fail(SM_ERR_CUDA, "sample: stream error");
  return rc;
}
