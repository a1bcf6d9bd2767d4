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

// Rows of group lg handled by this segment (GLU: R/2 gate rows then the same R/2 up rows).
template <int R>
__device__ __forceinline__ int group_row(const GemvSeg& s, int lg, int r) {
  return s.mode == GEMV_GLU ? lg * (R / 2) + (r % (R / 2)) : lg * R + r;
}

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

__device__ __forceinline__ void rope_pair(float& x0, float& x1, const GemvArgs& a, int pos, int d) {
  // RotaryEmbedding.cs:103-116 on the pair (d, d+1), d even
  const int half = a.head_dim / 2, i = d / 2;
  const float c = a.cos_t[pos * half + i], sn = a.sin_t[pos * half + i];
  const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
  const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
  x0 = y0;
  x1 = y1;
}

// Epilogue of one group, final row values v[0..R-1].
template <int R>
__device__ __forceinline__ void group_store(const GemvArgs& a, const GemvSeg& s, int lg, float* v) {
  if (s.mode == GEMV_GLU) {
#pragma unroll
    for (int r = 0; r < R / 2; ++r) {
      const int row = group_row<R>(s, lg, r);
      if (row >= s.rows) continue;
      const float g = v[r], u = v[r + R / 2];
      const float c = fmaxf(-20.f, fminf(g, 20.f));
      const float sig = __fdiv_rn(1.f, __fadd_rn(1.f, expf(-c)));  // ActivationOps.cs:304-309
      s.y[row] = __fmul_rn(__fmul_rn(g, sig), u);
    }
    return;
  }
  const int row0 = group_row<R>(s, lg, 0);
  if (s.mode == GEMV_ROPE_Q || s.mode == GEMV_ROPE_K_CACHE) {
    const int pos = *a.pos;
#pragma unroll
    for (int r = 0; r < R; r += 2) rope_pair(v[r], v[r + 1], a, pos, (row0 + r) % a.head_dim);
  }
  if (s.mode == GEMV_ROPE_K_CACHE || s.mode == GEMV_V_CACHE) {
    // head-major cache [seq][kv_head][pos][hd] (MultiHeadAttention.cs:262-274)
    const int64_t seq = *a.seq, pos = *a.pos;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = row0 + r;
      if (row >= s.rows) continue;
      const int h = row / a.head_dim, d = row - h * a.head_dim;
      s.y[((seq * a.n_kv + h) * a.max_ctx + pos) * a.head_dim + d] = v[r];
    }
    return;
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r;
    if (row >= s.rows) continue;
    s.y[row] = s.mode == GEMV_ADD ? s.y[row] + v[r] : v[r];
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
    }
  } else if (fa == SM_Q4_K && fb == SM_Q6_K) {
    return (void*)gemv1_kernel<SM_Q4_K, SM_Q6_K, R>;
  }
  return nullptr;
}
}  // namespace

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
