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

namespace sm {
namespace {

constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;

__device__ __forceinline__ int swz(int k) { return k ^ (((k >> 5) & 7) << 2); }

__device__ __forceinline__ float fbyte(uint32_t t, int b) {
  // bytes (0, 0, t.byte_b, 0x3F): the float 1.0 with t.byte_b's low 7 bits in the top mantissa bits
  return __uint_as_float(__byte_perm(t, 0x3F000000u, 0x7044u | (b << 8)));
}

template <int FMT>
struct Unit;

// Q4_K block (144 B): d, dmin fp16 | 12 B of 6-bit scales/mins | 128 B nibbles.
template <>
struct Unit<SM_Q4_K> {
  struct Raw {
    int4 hdr, qs;
  };
  __device__ __forceinline__ static void load(const GemvSeg& s, int row, int u, int K, Raw& r) {
    const uint8_t* blk = s.data + ((int64_t)row * (K >> 8) + (u >> 3)) * Q4K_BLOCK_BYTES;
    r.hdr = __ldg((const int4*)blk);
    r.qs = __ldg((const int4*)(blk + 16 + 16 * (u & 7)));
  }
  __device__ __forceinline__ static float dot(const Raw& r, int j, const float* x, float x16a, float x16b) {
    const float d = __half2float(__ushort_as_half((unsigned short)(r.hdr.x & 0xFFFF)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)((uint32_t)r.hdr.x >> 16)));
    // 8 six-bit scales are bits 6j..6j+5 of bytes 4..9, mins of bytes 10..15 (Q4KTensor.cs:109-126)
    const uint64_t sb = (uint32_t)r.hdr.y | ((uint64_t)((uint32_t)r.hdr.z & 0xFFFFu) << 32);
    const uint64_t mb = ((uint32_t)r.hdr.z >> 16) | ((uint64_t)(uint32_t)r.hdr.w << 16);
    const float sc = d * (float)((sb >> (6 * j)) & 63);
    const float mn = dmin * (float)((mb >> (6 * j)) & 63);
    const uint32_t w[4] = {(uint32_t)r.qs.x, (uint32_t)r.qs.y, (uint32_t)r.qs.z, (uint32_t)r.qs.w};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t tl = ((w[i] << 3) & 0x78787878u) | 0x80808080u;
      const uint32_t th = ((w[i] >> 1) & 0x78787878u) | 0x80808080u;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        a0 = fmaf(fbyte(tl, b), x[8 * i + 2 * b], a0);
        a1 = fmaf(fbyte(th, b), x[8 * i + 2 * b + 1], a1);
      }
    }
    const float s16 = 16.f * sc;
    return s16 * (a0 + a1) - (s16 + mn) * (x16a + x16b);
  }
};

// Q6_K device body (208 B): ql 128 | qh' 64 (re-packed) | int8 scales 16; d in aux.
template <>
struct Unit<SM_Q6_K> {
  struct Raw {
    int4 ql;
    int2 qh;
    unsigned short sc;
    unsigned short d;
  };
  __device__ __forceinline__ static void load(const GemvSeg& s, int row, int u, int K, Raw& r) {
    const int64_t b = (int64_t)row * (K >> 8) + (u >> 3);
    const uint8_t* blk = s.data + b * Q6K_BODY_BYTES;
    const int j = u & 7;
    r.ql = __ldg((const int4*)(blk + 16 * j));
    r.qh = __ldg((const int2*)(blk + 128 + 8 * j));
    r.sc = __ldg((const unsigned short*)(blk + 192 + 2 * j));
    r.d = __ldg((const unsigned short*)s.aux + b);
  }
  __device__ __forceinline__ static float half16(uint32_t w0, uint32_t w1, uint32_t W, const float* x) {
    // elements 0..7 from w0, 8..15 from w1; byte b of W holds highs of 2b, 2b+1, 8+2b, 9+2b
    const uint32_t t0 = ((w0 << 1) & 0x1E1E1E1Eu) | ((W << 5) & 0x60606060u) | 0x80808080u;
    const uint32_t t1 = ((w0 >> 3) & 0x1E1E1E1Eu) | ((W << 3) & 0x60606060u) | 0x80808080u;
    const uint32_t t2 = ((w1 << 1) & 0x1E1E1E1Eu) | ((W << 1) & 0x60606060u) | 0x80808080u;
    const uint32_t t3 = ((w1 >> 3) & 0x1E1E1E1Eu) | ((W >> 1) & 0x60606060u) | 0x80808080u;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      a0 = fmaf(fbyte(t0, b), x[2 * b], a0);
      a1 = fmaf(fbyte(t1, b), x[2 * b + 1], a1);
      a0 = fmaf(fbyte(t2, b), x[8 + 2 * b], a0);
      a1 = fmaf(fbyte(t3, b), x[9 + 2 * b], a1);
    }
    return a0 + a1;
  }
  __device__ __forceinline__ static float dot(const Raw& r, int, const float* x, float x16a, float x16b) {
    const float d = __half2float(__ushort_as_half(r.d));
    const float sa = d * (float)(int8_t)(r.sc & 0xFF), sb = d * (float)(int8_t)(r.sc >> 8);
    const float fa = half16((uint32_t)r.ql.x, (uint32_t)r.ql.y, (uint32_t)r.qh.x, x);
    const float fb = half16((uint32_t)r.ql.z, (uint32_t)r.ql.w, (uint32_t)r.qh.y, x + 16);
    return sa * (64.f * fa - 96.f * x16a) + sb * (64.f * fb - 96.f * x16b);
  }
};

// Q8_0: 32 int8 + fp32 block scale (block size a multiple of 32).
template <>
struct Unit<SM_Q8_0> {
  struct Raw {
    int4 a, b;
    float sc;
  };
  __device__ __forceinline__ static void load(const GemvSeg& s, int row, int u, int K, Raw& r) {
    const int64_t e0 = (int64_t)row * K + 32 * u;
    r.a = __ldg((const int4*)(s.data + e0));
    r.b = __ldg((const int4*)(s.data + e0) + 1);
    r.sc = __ldg((const float*)s.aux + e0 / s.bs);
  }
  __device__ __forceinline__ static float dot(const Raw& r, int, const float* x, float, float) {
    const uint32_t w[8] = {(uint32_t)r.a.x, (uint32_t)r.a.y, (uint32_t)r.a.z, (uint32_t)r.a.w,
                           (uint32_t)r.b.x, (uint32_t)r.b.y, (uint32_t)r.b.z, (uint32_t)r.b.w};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t v = w[i] ^ 0x80808080u;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const float q = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | b)) - 8388736.f;
        if (b & 1)
          a1 = fmaf(q, x[4 * i + b], a1);
        else
          a0 = fmaf(q, x[4 * i + b], a0);
      }
    }
    return r.sc * (a0 + a1);
  }
};

// Q4_0: 32 signed nibbles (global-index order: even low) + fp32 block scale.
template <>
struct Unit<SM_Q4_0> {
  struct Raw {
    int4 q;
    float sc;
  };
  __device__ __forceinline__ static void load(const GemvSeg& s, int row, int u, int K, Raw& r) {
    const int64_t e0 = (int64_t)row * K + 32 * u;
    r.q = __ldg((const int4*)(s.data + (e0 >> 1)));
    r.sc = __ldg((const float*)s.aux + e0 / s.bs);
  }
  __device__ __forceinline__ static float dot(const Raw& r, int, const float* x, float x16a, float x16b) {
    const uint32_t w[4] = {(uint32_t)r.q.x, (uint32_t)r.q.y, (uint32_t)r.q.z, (uint32_t)r.q.w};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t v = w[i] ^ 0x88888888u;  // two's-complement nibble -> nibble + 8
      const uint32_t tl = ((v << 3) & 0x78787878u) | 0x80808080u;
      const uint32_t th = ((v >> 1) & 0x78787878u) | 0x80808080u;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        a0 = fmaf(fbyte(tl, b), x[8 * i + 2 * b], a0);
        a1 = fmaf(fbyte(th, b), x[8 * i + 2 * b + 1], a1);
      }
    }
    return r.sc * (16.f * (a0 + a1) - 24.f * (x16a + x16b));
  }
};

// One warp, four weight rows (GLU: two output rows = two gate rows + two up rows).
template <int FMT>
__device__ __forceinline__ void group_rows(const GemvArgs& a, const GemvSeg& s, int lg, const float* xs,
                                           const float* x16, int lane) {
  const int K = a.K, units = K >> 5;
  const int j = lane & 7;
  const bool glu = s.mode == GEMV_GLU;
  int rows[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) rows[r] = glu ? lg * 2 + (r & 1) : lg * 4 + r;
  GemvSeg up = s;  // GLU rows 2, 3 read the up-projection weight
  if (glu) {
    up.data = s.data2;
    up.aux = s.aux2;
  }
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int u = lane; u < units; u += 32) {
    typename Unit<FMT>::Raw raw[4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
      if (rows[r] < s.rows) Unit<FMT>::load(r >= 2 ? up : s, rows[r], u, K, raw[r]);
    float xr[32];
    const float* xp = xs + 32 * u;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 v = *(const float4*)(xp + 4 * (c ^ j));
      xr[4 * c] = v.x; xr[4 * c + 1] = v.y; xr[4 * c + 2] = v.z; xr[4 * c + 3] = v.w;
    }
    const float xa = x16[2 * u], xb = x16[2 * u + 1];
#pragma unroll
    for (int r = 0; r < 4; ++r)
      if (rows[r] < s.rows) acc[r] += Unit<FMT>::dot(raw[r], j, xr, xa, xb);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) acc[r] = warp_sum(acc[r]);
  if (lane < 4) {
    if (glu) {
      if (lane < 2 && rows[lane] < s.rows) {
        const float g = lane == 0 ? acc[0] : acc[1];
        const float uu = lane == 0 ? acc[2] : acc[3];
        const float c = fmaxf(-20.f, fminf(g, 20.f));
        const float sig = __fdiv_rn(1.f, __fadd_rn(1.f, expf(-c)));
        s.y[rows[lane]] = __fmul_rn(__fmul_rn(g, sig), uu);
      }
    } else if (rows[lane] < s.rows) {
      const float v = acc[lane];
      float* dst = s.y + rows[lane];
      *dst = s.mode == GEMV_ADD ? *dst + v : v;
    }
  }
}

__device__ __forceinline__ void prefetch_rows(const GemvArgs& a, const GemvSeg& s, int lg, int lane) {
  const int K = a.K;
  int64_t row_bytes;
  switch (s.fmt) {
    case SM_Q4_K: row_bytes = (int64_t)(K >> 8) * Q4K_BLOCK_BYTES; break;
    case SM_Q6_K: row_bytes = (int64_t)(K >> 8) * Q6K_BODY_BYTES; break;
    case SM_Q8_0: row_bytes = K; break;
    default: row_bytes = K >> 1; break;
  }
  const bool glu = s.mode == GEMV_GLU;
  const int r0 = glu ? lg * 2 : lg * 4;
  const int nr = min(glu ? 2 : 4, s.rows - r0);
  for (int w = 0; w < (glu ? 2 : 1); ++w) {
    const uint8_t* base = (w == 0 ? s.data : s.data2) + r0 * row_bytes;
    const int64_t bytes = nr * row_bytes;
    for (int64_t off = (int64_t)lane * 128; off < bytes; off += 32 * 128)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(base + off));
  }
}

template <int FA, int FB>
__global__ void __launch_bounds__(THREADS, 2) gemv1_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ float smem[];
  float* xs = smem;             // [K] swizzled
  float* x16 = xs + a.K;        // [K/16] sums of 16 consecutive x
  float* red = x16 + a.K / 16;  // [WARPS]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gw = blockIdx.x * WARPS + warp, nw = gridDim.x * WARPS;
  // 1. weights do not depend on the previous kernel: start pulling them into L2
  for (int g = gw; g < a.ngroups; g += nw) {
    int si = 0;
    while (si + 1 < a.nseg && g >= a.seg[si + 1].group_begin) ++si;
    prefetch_rows(a, a.seg[si], g - a.seg[si].group_begin, lane);
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
  for (int g = gw; g < a.ngroups; g += nw) {
    int si = 0;
    while (si + 1 < a.nseg && g >= a.seg[si + 1].group_begin) ++si;
    const GemvSeg& s = a.seg[si];
    const int lg = g - s.group_begin;
    if (FA == FB || s.fmt == FA)
      group_rows<FA>(a, s, lg, xs, x16, lane);
    else
      group_rows<FB>(a, s, lg, xs, x16, lane);
  }
}

}  // namespace

bool gemv1_supports(const DevWeight& w, int K) {
  if (w.layout != SM_LAYOUT_INTENDED || w.K() != K || (K & 31)) return false;
  switch (w.scheme) {
    case SM_Q4_K: case SM_Q6_K: return (K & 255) == 0;
    case SM_Q8_0: case SM_Q4_0: return w.block_size % 32 == 0;
    default: return false;
  }
}

int gemv1_segment(GemvArgs& a, const DevWeight& w, const DevWeight* w2, float* y, int mode) {
  if (a.nseg >= GEMV_MAX_SEG) return fail(SM_ERR_INVALID_ARG, "gemv1: too many segments");
  if (!gemv1_supports(w, a.K) || (w2 && (!gemv1_supports(*w2, a.K) || w2->scheme != w.scheme || w2->rows != w.rows)))
    return fail(SM_ERR_UNSUPPORTED, "gemv1: unsupported weight for the M=1 path");
  GemvSeg& s = a.seg[a.nseg];
  s.fmt = w.scheme;
  s.rows = w.rows;
  s.bs = w.block_size;
  s.mode = mode;
  s.data = (const uint8_t*)w.data;
  s.aux = w.aux;
  s.data2 = w2 ? (const uint8_t*)w2->data : nullptr;
  s.aux2 = w2 ? w2->aux : nullptr;
  s.y = y;
  s.group_begin = a.ngroups;
  a.ngroups += mode == GEMV_GLU ? (w.rows + 1) / 2 : (w.rows + 3) / 4;
  a.nseg++;
  return SM_OK;
}

int launch_gemv1(const GemvArgs& a, cudaStream_t st, int* n_launch) {
  const size_t smem = sizeof(float) * ((size_t)a.K + a.K / 16 + WARPS);
  // one or two distinct formats per launch (each pair is its own instantiation)
  int fa = a.seg[0].fmt, fb = fa;
  for (int i = 1; i < a.nseg; ++i) {
    if (a.seg[i].fmt == fa || a.seg[i].fmt == fb) continue;
    if (fb != fa) return fail(SM_ERR_UNSUPPORTED, "gemv1: more than two formats in one launch");
    fb = a.seg[i].fmt;
  }
  if (fb == SM_Q4_K && fa == SM_Q6_K) std::swap(fa, fb);
  void (*kern)(GemvArgs) = nullptr;
  if (fa == fb) {
    switch (fa) {
      case SM_Q4_K: kern = gemv1_kernel<SM_Q4_K, SM_Q4_K>; break;
      case SM_Q6_K: kern = gemv1_kernel<SM_Q6_K, SM_Q6_K>; break;
      case SM_Q8_0: kern = gemv1_kernel<SM_Q8_0, SM_Q8_0>; break;
      case SM_Q4_0: kern = gemv1_kernel<SM_Q4_0, SM_Q4_0>; break;
    }
  } else if (fa == SM_Q4_K && fb == SM_Q6_K) {
    kern = gemv1_kernel<SM_Q4_K, SM_Q6_K>;
  }
  if (!kern) return fail(SM_ERR_UNSUPPORTED, "gemv1: unsupported format mix in one launch");
  if (smem > 200 * 1024) return fail(SM_ERR_UNSUPPORTED, "gemv1: K too large");
  static bool attr_set[64][8][8] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev][fa][fb]) {
    SM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_set[dev][fa][fb] = true;
  }
  const int grid = std::max(1, std::min(ceil_div(a.ngroups, WARPS), 148 * 2));
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
  SM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  if (n_launch) ++*n_launch;
  return SM_OK;
}

}  // namespace sm
