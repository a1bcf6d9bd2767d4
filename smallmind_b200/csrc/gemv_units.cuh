// Per-format 32-weight "units" and the row epilogues shared by the M = 1 GEMVs
// (gemv1.cu, decode_mega.cu).  Exact byte-permute dequant: see gemv1.cu.
#pragma once
#include "common.cuh"
#include "gemv1.cuh"

namespace sm {

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
  // from a copy of the row (shared memory)
  __device__ __forceinline__ static void load_row(const GemvSeg&, const uint8_t* rowp, int, int u, int, bool,
                                                  Raw& r) {
    const uint8_t* blk = rowp + (u >> 3) * Q4K_BLOCK_BYTES;
    r.hdr = *(const int4*)blk;
    r.qs = *(const int4*)(blk + 16 + 16 * (u & 7));
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
    r.d = __ldg((const unsigned short*)s.aux + aux_idx(b, s.aux_bpr, s.aux_stride));
  }
  __device__ __forceinline__ static void load_row(const GemvSeg& s, const uint8_t* rowp, int row, int u, int K,
                                                  bool up, Raw& r) {
    const uint8_t* blk = rowp + (u >> 3) * Q6K_BODY_BYTES;
    const int j = u & 7;
    r.ql = *(const int4*)(blk + 16 * j);
    r.qh = *(const int2*)(blk + 128 + 8 * j);
    r.sc = *(const unsigned short*)(blk + 192 + 2 * j);
    r.d = __ldg((const unsigned short*)(up ? s.aux2 : s.aux) +
                aux_idx((int64_t)row * (K >> 8) + (u >> 3), s.aux_bpr, s.aux_stride));
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
    r.sc = __ldg((const float*)s.aux + aux_idx(e0 / s.bs, s.aux_bpr, s.aux_stride));
  }
  __device__ __forceinline__ static void load_row(const GemvSeg& s, const uint8_t* rowp, int row, int u, int K,
                                                  bool up, Raw& r) {
    r.a = *(const int4*)(rowp + 32 * u);
    r.b = *((const int4*)(rowp + 32 * u) + 1);
    r.sc = __ldg((const float*)(up ? s.aux2 : s.aux) + aux_idx(((int64_t)row * K + 32 * u) / s.bs, s.aux_bpr, s.aux_stride));
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
    r.sc = __ldg((const float*)s.aux + aux_idx(e0 / s.bs, s.aux_bpr, s.aux_stride));
  }
  __device__ __forceinline__ static void load_row(const GemvSeg& s, const uint8_t* rowp, int row, int u, int K,
                                                  bool up, Raw& r) {
    r.q = *(const int4*)(rowp + 16 * u);
    r.sc = __ldg((const float*)(up ? s.aux2 : s.aux) + aux_idx(((int64_t)row * K + 32 * u) / s.bs, s.aux_bpr, s.aux_stride));
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

// Q4_1 / Q5_0: 32 nibbles (global-index order: even low) + fp32 scale and a
// second per-block word in the row-padded aux (Q4_1: the min; Q5_0: the 32
// fifth bits).  Q4_1: sum((sc u + mn) x) = 16 sc sum(f x) + (mn - 16 sc) sum(x),
// f = 1 + u/16 (Q4_1Tensor.cs:153-156).  Q5_0: the fifth bit joins the nibble
// in the byte, f = 1 + u5/32, sum(sc (u5 - 16) x) = sc (32 sum(f x) - 48 sum(x))
// (Q5_0Tensor.cs:157-172).
template <int FMT>
struct Unit4150 {
  struct Raw {
    int4 q;
    float sc;
    uint32_t second;
  };
  __device__ __forceinline__ static void load(const GemvSeg& s, int row, int u, int K, Raw& r) {
    const int64_t e0 = (int64_t)row * K + 32 * u, b = e0 >> 5;
    r.q = __ldg((const int4*)(s.data + (e0 >> 1)));
    r.sc = __ldg((const float*)s.aux + aux_idx(b, s.aux_bpr, s.aux_stride));
    r.second = __ldg((const uint32_t*)s.aux + aux_second_idx(b, s.aux_bpr, s.aux_stride, 0));
  }
  __device__ __forceinline__ static void load_row(const GemvSeg& s, const uint8_t* rowp, int row, int u, int K,
                                                  bool up, Raw& r) {
    const int64_t b = ((int64_t)row * K >> 5) + u;
    const void* aux = up ? s.aux2 : s.aux;
    r.q = *(const int4*)(rowp + 16 * u);
    r.sc = __ldg((const float*)aux + aux_idx(b, s.aux_bpr, s.aux_stride));
    r.second = __ldg((const uint32_t*)aux + aux_second_idx(b, s.aux_bpr, s.aux_stride, 0));
  }
  // bits 0, 2, 4, 6 of h -> bit 6 of bytes 0..3
  __device__ __forceinline__ static uint32_t spread_even(uint32_t h) {
    uint32_t t = h & 0x55u;
    t = (t | (t << 12)) & 0x00050005u;
    t = (t | (t << 6)) & 0x01010101u;
    return t << 6;
  }
  __device__ __forceinline__ static float dot(const Raw& r, int, const float* x, float x16a, float x16b) {
    const uint32_t w[4] = {(uint32_t)r.q.x, (uint32_t)r.q.y, (uint32_t)r.q.z, (uint32_t)r.q.w};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t tl, th;
      if (FMT == SM_Q4_1) {
        tl = ((w[i] << 3) & 0x78787878u) | 0x80808080u;
        th = ((w[i] >> 1) & 0x78787878u) | 0x80808080u;
      } else {
        const uint32_t h = r.second >> (8 * i);
        tl = ((w[i] << 2) & 0x3C3C3C3Cu) | spread_even(h) | 0x80808080u;
        th = ((w[i] >> 2) & 0x3C3C3C3Cu) | spread_even(h >> 1) | 0x80808080u;
      }
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        a0 = fmaf(fbyte(tl, b), x[8 * i + 2 * b], a0);
        a1 = fmaf(fbyte(th, b), x[8 * i + 2 * b + 1], a1);
      }
    }
    const float sx = x16a + x16b;
    if (FMT == SM_Q4_1) {
      const float s16 = 16.f * r.sc;
      return s16 * (a0 + a1) + (__uint_as_float(r.second) - s16) * sx;
    }
    return r.sc * (32.f * (a0 + a1) - 48.f * sx);
  }
};
template <>
struct Unit<SM_Q4_1> : Unit4150<SM_Q4_1> {};
template <>
struct Unit<SM_Q5_0> : Unit4150<SM_Q5_0> {};

// Rows of group lg handled by this segment (GLU: R/2 gate rows then the same R/2 up rows).
template <int R>
__device__ __forceinline__ int group_row(const GemvSeg& s, int lg, int r) {
  if constexpr (R >= 2) {
    if (s.mode == GEMV_GLU) return lg * (R / 2) + (r % (R / 2));
  }
  return lg * R + r;
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
    s.y[row] = s.mode == GEMV_ADD ? __ldcg(&s.y[row]) + v[r] : v[r];
  }
}


}  // namespace sm

namespace sm {

// ---------------------------------------------------------------------------
// Integer dot path.  The 32 activations of a unit become 24-bit fixed point
// with one power-of-two exponent per unit, X_i = round(x_i * 2^(23-e)), split
// into three byte planes X = a*2^16 + b*2^8 + c (a signed, b and c unsigned).
// The packed weights' integer codes then meet the planes in dp4a (exact int32
// sums), and sum(q x) = 2^(e-23) * (A*65536 + B*256 + C).  Rounding x to 24
// bits relative to the unit's largest |x| keeps the result well inside the
// 1e-4 GEMV tolerance.
//
// PAIR packing (Q4_K, Q4_0, Q6_K code words): plane words 0..3 hold elements
// 8i, 8i+2, 8i+4, 8i+6 (low nibbles of code word i), words 4..7 elements
// 8i+1, ... (high nibbles).  NATURAL packing (Q8_0): word i = elements 4i..4i+3.
struct XPlanes {
  uint32_t a[8], b[8], c[8];
  float inv;        // 2^(e-23)
  float x16a, x16b; // sums of x over elements 0..15 and 16..31 (exact-order fp32)
};

__device__ __forceinline__ void make_planes(const float* x, bool pair, XPlanes& p) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
  int ex = 0;
  frexpf(amax, &ex);  // amax < 2^ex
  const float up = ldexpf(1.f, 23 - ex);
  p.inv = ldexpf(1.f, ex - 23);
  int X[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) X[i] = amax > 0.f ? __float2int_rn(x[i] * up) : 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    int e[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) e[j] = pair ? (8 * (w & 3) + 2 * j + (w >> 2)) : (4 * w + j);
    // byte 2 / 1 / 0 of four 32-bit values -> one word per plane
    const uint32_t x0 = X[e[0]], x1 = X[e[1]], x2 = X[e[2]], x3 = X[e[3]];
    p.a[w] = __byte_perm(__byte_perm(x0, x1, 0x0062), __byte_perm(x2, x3, 0x0062), 0x5410);
    p.b[w] = __byte_perm(__byte_perm(x0, x1, 0x0051), __byte_perm(x2, x3, 0x0051), 0x5410);
    p.c[w] = __byte_perm(__byte_perm(x0, x1, 0x0040), __byte_perm(x2, x3, 0x0040), 0x5410);
  }
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    s0 += x[i];
    s1 += x[16 + i];
  }
  p.x16a = s0;
  p.x16b = s1;
}

// dp4a with a signed first operand (weight codes) and a signed / unsigned plane
__device__ __forceinline__ int dp_ss(uint32_t q, uint32_t a, int acc) {
  int r;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(q), "r"(a), "r"(acc));
  return r;
}
__device__ __forceinline__ int dp_su(uint32_t q, uint32_t b, int acc) {
  int r;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(q), "r"(b), "r"(acc));
  return r;
}

struct IAcc {
  int A = 0, B = 0, C = 0;
  __device__ __forceinline__ void add(uint32_t q, const XPlanes& p, int w) {
    A = dp_ss(q, p.a[w], A);
    B = dp_su(q, p.b[w], B);
    C = dp_su(q, p.c[w], C);
  }
  __device__ __forceinline__ float value(float inv) const {
    return inv * fmaf((float)A, 65536.f, fmaf((float)B, 256.f, (float)C));
  }
};

// sum over the unit of (code * x) for each format; codes as in the reference:
// Q4_K q in [0,15]; Q6_K q in [0,63] per 16-element half; Q8_0 q in [-127,127];
// Q4_0 nibble + 8 in [0,15].
__device__ __forceinline__ float dot_i8_q4k(const Unit<SM_Q4_K>::Raw& r, int j, const XPlanes& p) {
  const float d = __half2float(__ushort_as_half((unsigned short)(r.hdr.x & 0xFFFF)));
  const float dmin = __half2float(__ushort_as_half((unsigned short)((uint32_t)r.hdr.x >> 16)));
  const uint64_t sb = (uint32_t)r.hdr.y | ((uint64_t)((uint32_t)r.hdr.z & 0xFFFFu) << 32);
  const uint64_t mb = ((uint32_t)r.hdr.z >> 16) | ((uint64_t)(uint32_t)r.hdr.w << 16);
  const float sc = d * (float)((sb >> (6 * j)) & 63);
  const float mn = dmin * (float)((mb >> (6 * j)) & 63);
  const uint32_t w[4] = {(uint32_t)r.qs.x, (uint32_t)r.qs.y, (uint32_t)r.qs.z, (uint32_t)r.qs.w};
  IAcc acc;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc.add(w[i] & 0x0F0F0F0Fu, p, i);
    acc.add((w[i] >> 4) & 0x0F0F0F0Fu, p, 4 + i);
  }
  return sc * acc.value(p.inv) - mn * (p.x16a + p.x16b);
}

__device__ __forceinline__ float dot_i8_q6k(const Unit<SM_Q6_K>::Raw& r, const XPlanes& p) {
  const float d = __half2float(__ushort_as_half(r.d));
  const float sa = d * (float)(int8_t)(r.sc & 0xFF), sb = d * (float)(int8_t)(r.sc >> 8);
  const uint32_t w0 = r.ql.x, w1 = r.ql.y, w2 = r.ql.z, w3 = r.ql.w;
  const uint32_t W0 = r.qh.x, W1 = r.qh.y;
  // byte b of W holds the highs of elements 2b, 2b+1, 8+2b, 9+2b of its 16-element half
  IAcc h0, h1;
  h0.add((w0 & 0x0F0F0F0Fu) | ((W0 << 4) & 0x30303030u), p, 0);
  h0.add(((w0 >> 4) & 0x0F0F0F0Fu) | ((W0 << 2) & 0x30303030u), p, 4);
  h0.add((w1 & 0x0F0F0F0Fu) | (W0 & 0x30303030u), p, 1);
  h0.add(((w1 >> 4) & 0x0F0F0F0Fu) | ((W0 >> 2) & 0x30303030u), p, 5);
  h1.add((w2 & 0x0F0F0F0Fu) | ((W1 << 4) & 0x30303030u), p, 2);
  h1.add(((w2 >> 4) & 0x0F0F0F0Fu) | ((W1 << 2) & 0x30303030u), p, 6);
  h1.add((w3 & 0x0F0F0F0Fu) | (W1 & 0x30303030u), p, 3);
  h1.add(((w3 >> 4) & 0x0F0F0F0Fu) | ((W1 >> 2) & 0x30303030u), p, 7);
  return sa * (h0.value(p.inv) - 32.f * p.x16a) + sb * (h1.value(p.inv) - 32.f * p.x16b);
}

__device__ __forceinline__ float dot_i8_q8(const Unit<SM_Q8_0>::Raw& r, const XPlanes& p) {
  const uint32_t w[8] = {(uint32_t)r.a.x, (uint32_t)r.a.y, (uint32_t)r.a.z, (uint32_t)r.a.w,
                         (uint32_t)r.b.x, (uint32_t)r.b.y, (uint32_t)r.b.z, (uint32_t)r.b.w};
  IAcc acc;
#pragma unroll
  for (int i = 0; i < 8; ++i) acc.add(w[i], p, i);
  return r.sc * acc.value(p.inv);
}

__device__ __forceinline__ float dot_i8_q4_0(const Unit<SM_Q4_0>::Raw& r, const XPlanes& p) {
  const uint32_t w[4] = {(uint32_t)r.q.x, (uint32_t)r.q.y, (uint32_t)r.q.z, (uint32_t)r.q.w};
  IAcc acc;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t v = w[i] ^ 0x88888888u;  // nibble + 8
    acc.add(v & 0x0F0F0F0Fu, p, i);
    acc.add((v >> 4) & 0x0F0F0F0Fu, p, 4 + i);
  }
  return r.sc * (acc.value(p.inv) - 8.f * (p.x16a + p.x16b));
}

}  // namespace sm
