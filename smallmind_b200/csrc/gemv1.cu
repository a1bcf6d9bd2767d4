// Decode GEMV for one activation row (M = 1), the bs1 hot path.
//
// y[n] = sum_k x[k] * w[n][k] for INTENDED-layout weights (W[N][K], blocks
// along K), for Q4_K, Q6_K (device layout), Q8_0 and Q4_0.
//
// Per weight the inner loop costs one PRMT and one FFMA: the packed integer q
// is turned into the exact float f = 1 + q/16 (Q4_K, Q4_0) or 1 + q/64 (Q6_K)
// by placing its bits in the mantissa of 1.0f with a byte permute, and the
// sub-block partial is recovered from sum(f*x) and the precomputed sum(x):
//   Q4_K: sum((sc*q - m) x) = 16 sc sum(f x) - (16 sc + m) sum(x)       (Q4KTensor.cs:129-147)
//   Q6_K: sum(d s (q - 32) x) = d s (64 sum(f x) - 96 sum(x))          (Q6KTensor.cs:99-125)
//   Q4_0: sum(scale q x), q = nibble - 8 after XOR 8 (Q4Tensor.cs:140-144) = scale (16 sum(f x) - 24 sum(x))
//   Q8_0: f = 2^23 + q + 128 exactly, q = f - (2^23 + 128)              (Q8Tensor.cs:151)
// The reference rounds each dequantized weight before the product; this
// kernel reassociates, which stays within the 1e-4 GEMV tolerance (the
// sums of x are exact-order fp32 over 16/32 elements).
//
// One launch covers up to four weights ("segments": Q|K|V, or one linear) with
// a fused RMSNorm prologue (RMSNormOps.cs:114,215-216) and a store, residual-add
// (TransformerBlock.cs:170,184) or SiLU-gate (GatedMLP.cs:84, ActivationOps.cs:565-580)
// epilogue.  Launched with programmatic dependent launch: each CTA prefetches
// its weight rows into L2, lets the next kernel start, and only then waits
// for the previous kernel's output.
#include <algorithm>

#include "common.cuh"
#include "gemv1.cuh"
#include "gemv_units.cuh"

namespace sm {
namespace {

constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;

__device__ __forceinline__ int swz(int k) { return k ^ (((k >> 5) & 7) << 2); }

// Partial dot products of R rows over this warp's share of K (units sub, sub+S, ...).
template <int FMT, int R>
__device__ __forceinline__ void group_partial(const GemvArgs& a, const GemvSeg& s, int lg, const float* xs,
                                              const float* x16, int lane, int sub, float* acc) {
  const int K = a.K, units = K >> 5;
  const int j = lane & 7;
  const bool glu = s.mode == GEMV_GLU;
  GemvSeg up = s;  // GLU rows R/2.. read the up-projection weight
  if (glu) {
    up.data = s.data2;
    up.aux = s.aux2;
  }
  int rows[R];
#pragma unroll
  for (int r = 0; r < R; ++r) rows[r] = group_row<R>(s, lg, r);
  for (int u = sub * 32 + lane; u < units; u += 32 * a.S) {
    typename Unit<FMT>::Raw raw[R];
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (rows[r] < s.rows) Unit<FMT>::load((glu && r >= R / 2) ? up : s, rows[r], u, K, raw[r]);
    float xr[32];
    const float* xp = xs + 32 * u;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 v = *(const float4*)(xp + 4 * (c ^ j));
      xr[4 * c] = v.x; xr[4 * c + 1] = v.y; xr[4 * c + 2] = v.z; xr[4 * c + 3] = v.w;
    }
    const float xa = x16[2 * u], xb = x16[2 * u + 1];
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (rows[r] < s.rows) acc[r] += Unit<FMT>::dot(raw[r], j, xr, xa, xb);
  }
}

__device__ __forceinline__ void prefetch_rows(const GemvArgs& a, const GemvSeg& s, int lg, int R, int sub,
                                              int lane) {
  const int K = a.K;
  int64_t row_bytes;
  switch (s.fmt) {
    case SM_Q4_K: row_bytes = (int64_t)(K >> 8) * Q4K_BLOCK_BYTES; break;
    case SM_Q6_K: row_bytes = (int64_t)(K >> 8) * Q6K_BODY_BYTES; break;
    case SM_Q8_0: row_bytes = K; break;
    default: row_bytes = K >> 1; break;
  }
  const bool glu = s.mode == GEMV_GLU;
  const int rg = glu ? R / 2 : R;
  const int r0 = lg * rg;
  const int nr = min(rg, s.rows - r0);
  for (int w = 0; w < (glu ? 2 : 1); ++w) {
    const uint8_t* base = (w == 0 ? s.data : s.data2) + r0 * row_bytes;
    const int64_t bytes = nr * row_bytes;
    for (int64_t off = (int64_t)(sub * 32 + lane) * 128; off < bytes; off += 32 * 128 * a.S)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(base + off));
  }
}

__device__ __forceinline__ int seg_of(const GemvArgs& a, int g) {
  int si = 0;
  while (si + 1 < a.nseg && g >= a.seg[si + 1].group_begin) ++si;
  return si;
}

// A CTA of 8 warps works on 8/S row groups at a time; the S warps of a group
// split K and combine their partials through shared memory.
template <int FA, int FB, int R>
__global__ void __launch_bounds__(THREADS, 2) gemv1_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ float smem[];
  float* xs = smem;             // [K] swizzled
  float* x16 = xs + a.K;        // [K/16] sums of 16 consecutive x
  float* red = x16 + a.K / 16;  // [WARPS][R]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int S = a.S, gpc = WARPS / S;
  const int sub = warp % S;
  // 1. weights do not depend on the previous kernel: start pulling them into L2
  for (int base = blockIdx.x * gpc; base < a.ngroups; base += gridDim.x * gpc) {
    const int g = base + warp / S;
    if (g < a.ngroups) {
      const int si = seg_of(a, g);
      prefetch_rows(a, a.seg[si], g - a.seg[si].group_begin, R, sub, lane);
    }
  }
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // 2. stage x (optionally RMS-normalised) and its 16-element sums
  const int K = a.K;
  float ss = 0.f;
  for (int k = threadIdx.x; k < K; k += THREADS) {
    const float v = a.x[k];
    xs[swz(k)] = v;
    ss = fmaf(v, v, ss);
  }
  if (a.gamma) {
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) tot += red[w];
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), a.eps)));
    for (int k = threadIdx.x; k < K; k += THREADS) {
      const int p = swz(k);
      xs[p] = __fmul_rn(a.gamma[k], __fmul_rn(xs[p], inv));
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < K / 16; t += THREADS) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) s += xs[swz(16 * t + i)];
    x16[t] = s;
  }
  __syncthreads();
  // 3. row groups
  for (int base = blockIdx.x * gpc; base < a.ngroups; base += gridDim.x * gpc) {
    const int g = base + warp / S;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    int si = 0;
    if (g < a.ngroups) {
      si = seg_of(a, g);
      const GemvSeg& s = a.seg[si];
      if (FA == FB || s.fmt == FA)
        group_partial<FA, R>(a, s, g - s.group_begin, xs, x16, lane, sub, acc);
      else
        group_partial<FB, R>(a, s, g - s.group_begin, xs, x16, lane, sub, acc);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = warp_sum(acc[r]);
    if (S > 1) {
      if (lane == 0)
#pragma unroll
        for (int r = 0; r < R; ++r) red[warp * R + r] = acc[r];
      __syncthreads();
      if (sub == 0 && lane == 0)
        for (int w = 1; w < S; ++w)
#pragma unroll
          for (int r = 0; r < R; ++r) acc[r] += red[(warp + w) * R + r];
    }
    if (g < a.ngroups && sub == 0 && lane == 0) group_store<R>(a, a.seg[si], g - a.seg[si].group_begin, acc);
    if (S > 1) __syncthreads();
  }
}

}  // namespace

bool gemv1_supports(const DevWeight& w, int K) {
  if (w.layout != SM_LAYOUT_INTENDED || w.K() != K || (K & 31)) return false;
  switch (w.scheme) {
    case SM_Q4_K: case SM_Q6_K: return (K & 255) == 0;
    case SM_Q8_0: case SM_Q4_0: return w.block_size % 32 == 0;
    case SM_Q4_1: case SM_Q5_0: return w.aux_stride > 0;  // row-padded [scales | second] aux
    default: return false;
  }
}

int gemv1_segment(GemvArgs& a, const DevWeight& w, const DevWeight* w2, float* y, int mode) {
  if (a.nseg >= GEMV_MAX_SEG) return fail(SM_ERR_INVALID_ARG, "gemv1: too many segments");
  if (!gemv1_supports(w, a.K) || (w2 && (!gemv1_supports(*w2, a.K) || w2->scheme != w.scheme || w2->rows != w.rows)))
    return fail(SM_ERR_UNSUPPORTED, "gemv1: unsupported weight for the M=1 path");
  if ((mode == GEMV_ROPE_Q || mode == GEMV_ROPE_K_CACHE) && (a.head_dim <= 0 || w.rows % a.head_dim))
    return fail(SM_ERR_INVALID_ARG, "gemv1: RoPE epilogue needs whole heads");
  GemvSeg& s = a.seg[a.nseg];
  s.fmt = w.scheme;
  s.rows = w.rows;
  s.bs = w.block_size;
  s.aux_bpr = w.aux_bpr;
  s.aux_stride = w.aux_stride;
  s.mode = mode;
  s.data = (const uint8_t*)w.data;
  s.aux = w.aux;
  s.data2 = w2 ? (const uint8_t*)w2->data : nullptr;
  s.aux2 = w2 ? w2->aux : nullptr;
  s.y = y;
  a.nseg++;
  return SM_OK;
}

namespace {
int set_groups(GemvArgs& a, int R) {
  a.ngroups = 0;
  for (int i = 0; i < a.nseg; ++i) {
    GemvSeg& s = a.seg[i];
    s.group_begin = a.ngroups;
    a.ngroups += s.mode == GEMV_GLU ? ceil_div(s.rows, R / 2) : ceil_div(s.rows, R);
  }
  return a.ngroups;
}

template <int R>
void* pick_kernel(int fa, int fb) {
  if (fa == fb) {
    switch (fa) {
      case SM_Q4_K: return (void*)gemv1_kernel<SM_Q4_K, SM_Q4_K, R>;
      case SM_Q6_K: return (void*)gemv1_kernel<SM_Q6_K, SM_Q6_K, R>;
      case SM_Q8_0: return (void*)gemv1_kernel<SM_Q8_0, SM_Q8_0, R>;
      case SM_Q4_0: return (void*)gemv1_kernel<SM_Q4_0, SM_Q4_0, R>;
      case SM_Q4_1: return (void*)gemv1_kernel<SM_Q4_1, SM_Q4_1, R>;
      case SM_Q5_0: return (void*)gemv1_kernel<SM_Q5_0, SM_Q5_0, R>;
    }
  } else if (fa == SM_Q4_K && fb == SM_Q6_K) {
    return (void*)gemv1_kernel<SM_Q4_K, SM_Q6_K, R>;
  }
  return nullptr;
}
}  // namespace

bool gemv1_mix_ok(int fa, int fb) {
  if (fb == SM_Q4_K && fa == SM_Q6_K) std::swap(fa, fb);
  return pick_kernel<4>(fa, fb) != nullptr;
}

int launch_gemv1(const GemvArgs& args, cudaStream_t st, int* n_launch) {
  GemvArgs a = args;
  const size_t smem = sizeof(float) * ((size_t)a.K + a.K / 16 + WARPS * 4);
  if (smem > 200 * 1024) return fail(SM_ERR_UNSUPPORTED, "gemv1: K too large");
  // one or two distinct formats per launch (each pair is its own instantiation)
  int fa = a.seg[0].fmt, fb = fa;
  for (int i = 1; i < a.nseg; ++i) {
    if (a.seg[i].fmt == fa || a.seg[i].fmt == fb) continue;
    if (fb != fa) return fail(SM_ERR_UNSUPPORTED, "gemv1: more than two formats in one launch");
    fb = a.seg[i].fmt;
  }
  if (fb == SM_Q4_K && fa == SM_Q6_K) std::swap(fa, fb);
  // rows per group R and warps per group S: fill the SMs (2 CTAs x 8 warps each) while keeping
  // every lane of a warp busy over K (units of 32 weights strided by 32*S)
  const int units = a.K / 32;
  const int target_warps = 148 * 2 * WARPS;
  int bestR = 4, bestS = 1;
  double best = -1;
  for (int R : {4, 2})
    for (int S : {1, 2, 4, 8}) {
      const int ng = set_groups(a, R);
      const int per = 32 * S;
      const double lane_eff = (double)units / (per * ((units + per - 1) / per));
      const double par_eff = std::min(1.0, (double)ng * S / target_warps);
      const double score = lane_eff * par_eff * (R == 4 ? 1.0 : 0.85);
      if (score > best + 1e-9) {
        best = score;
        bestR = R;
        bestS = S;
      }
    }
  a.S = bestS;
  set_groups(a, bestR);
  void* kern = bestR == 4 ? pick_kernel<4>(fa, fb) : pick_kernel<2>(fa, fb);
  if (!kern) return fail(SM_ERR_UNSUPPORTED, "gemv1: unsupported format mix in one launch");
  static bool attr_set[64][8][8][2] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int ri = bestR == 4 ? 0 : 1;
  if (dev < 64 && !attr_set[dev][fa][fb][ri]) {
    SM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_set[dev][fa][fb][ri] = true;
  }
  const int gpc = WARPS / bestS;
  const int grid = std::max(1, std::min(ceil_div(a.ngroups, gpc), 148 * 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* params[] = {&a};
  SM_CUDA_TRY(cudaLaunchKernelExC(&cfg, kern, params));
  if (n_launch) ++*n_launch;
  return SM_OK;
}

}  // namespace sm
