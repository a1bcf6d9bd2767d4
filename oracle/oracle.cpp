// SmallMind quantized-path ORACLE — test infrastructure only (see oracle.h).
// C++17 restatement of the reference C# arithmetic; compiled -ffp-contract=off.
// Every function cites the reference file:line it restates.
#include "oracle.h"

#include <algorithm>
#include <limits>
#include <cmath>
#include <cstring>
#include <atomic>
#include <thread>
#include <vector>

namespace {

template <class F>
void parallel_for(int n, int n_threads, F&& f) {
  if (n_threads <= 1 || n <= 1) {
    for (int i = 0; i < n; ++i) f(i);
    return;
  }
  int nt = std::min(n_threads, n);
  std::vector<std::thread> th;
  th.reserve(nt);
  for (int t = 0; t < nt; ++t) {
    th.emplace_back([&, t] {
      for (int i = t; i < n; i += nt) f(i);
    });
  }
  for (auto& x : th) x.join();
}

// MathF.Round: round half to even (default MidpointRounding.ToEven).
inline float round_half_even(float x) { return std::nearbyint(x); }

inline float clampf(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }

// Unpack of the 12-byte K-quant scale field, sequential 6-bit packing:
// Q4KTensor.cs:109-126 (== FusedQ4KMatMul.cs:203-224).
inline void unpack_q4k_scales(const uint8_t* s, uint8_t* sc, uint8_t* mn) {
  sc[0] = (uint8_t)(s[0] & 0x3F);
  sc[1] = (uint8_t)((s[0] >> 6) | ((s[1] & 0x0F) << 2));
  sc[2] = (uint8_t)((s[1] >> 4) | ((s[2] & 0x03) << 4));
  sc[3] = (uint8_t)((s[2] >> 2) & 0x3F);
  sc[4] = (uint8_t)(s[3] & 0x3F);
  sc[5] = (uint8_t)((s[3] >> 6) | ((s[4] & 0x0F) << 2));
  sc[6] = (uint8_t)((s[4] >> 4) | ((s[5] & 0x03) << 4));
  sc[7] = (uint8_t)((s[5] >> 2) & 0x3F);
  mn[0] = (uint8_t)(s[6] & 0x3F);
  mn[1] = (uint8_t)((s[6] >> 6) | ((s[7] & 0x0F) << 2));
  mn[2] = (uint8_t)((s[7] >> 4) | ((s[8] & 0x03) << 4));
  mn[3] = (uint8_t)((s[8] >> 2) & 0x3F);
  mn[4] = (uint8_t)(s[9] & 0x3F);
  mn[5] = (uint8_t)((s[9] >> 6) | ((s[10] & 0x0F) << 2));
  mn[6] = (uint8_t)((s[10] >> 4) | ((s[11] & 0x03) << 4));
  mn[7] = (uint8_t)((s[11] >> 2) & 0x3F);
}

// One Q4_K block -> 256 floats.  Q4KTensor.cs:84-147: sc = d*scale, m = dmin*min,
// byte qs[16j+i] holds element 2i (low nibble) and 2i+1 (high), w = sc*q - m.
inline void dequant_q4k_block(const uint8_t* b, float* out) {
  uint16_t db, dmb;
  std::memcpy(&db, b, 2);
  std::memcpy(&dmb, b + 2, 2);
  float d = or_half_to_float(db), dmin = or_half_to_float(dmb);
  uint8_t sc[8], mn[8];
  unpack_q4k_scales(b + 4, sc, mn);
  const uint8_t* qs = b + 16;
  for (int j = 0; j < 8; ++j) {
    float s = d * (float)sc[j];
    float m = dmin * (float)mn[j];
    for (int i = 0; i < 16; ++i) {
      uint8_t p = qs[16 * j + i];
      int q0 = p & 0xF, q1 = (p >> 4) & 0xF;
      float t0 = s * (float)q0;
      float t1 = s * (float)q1;
      out[32 * j + 2 * i] = t0 - m;
      out[32 * j + 2 * i + 1] = t1 - m;
    }
  }
}

// One Q6_K block -> 256 floats.  Q6KTensor.cs:85-125: ql @0 (128 B), qh @128 (64 B),
// int8 scales @192 (16), d fp16 @208; element v: low4 = nibble(ql[v/2], v&1),
// high2 = (qh[v/4] >> 2(v%4)) & 3, w = (d*scale[v/16]) * (q - 32).
inline void dequant_q6k_block(const uint8_t* b, float* out) {
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const int8_t* scales = (const int8_t*)(b + 192);
  uint16_t db;
  std::memcpy(&db, b + 208, 2);
  float d = or_half_to_float(db);
  for (int sb = 0; sb < 16; ++sb) {
    float s = d * (float)scales[sb];
    for (int i = 0; i < 16; ++i) {
      int v = sb * 16 + i;
      uint8_t qlb = ql[v / 2];
      int low4 = (v % 2 == 0) ? (qlb & 0xF) : ((qlb >> 4) & 0xF);
      int high2 = (qh[v / 4] >> ((v % 4) * 2)) & 3;
      int q = low4 | (high2 << 4);
      out[v] = s * (float)(q - 32);
    }
  }
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// System.Random(int seed): the legacy seeded generator (Knuth's subtractive
// method, Numerical Recipes "ran3"), which .NET keeps for seeded instances.
// Restated from the published algorithm; reproduces the inputs of the
// reference's seeded tests (tests/SmallMind.Quantization.Tests/*.cs, new Random(42)).
void or_dotnet_random_init(or_dotnet_random* r, int32_t seed) {
  const int32_t MBIG = 2147483647, MSEED = 161803398;
  int32_t* sa = r->seed_array;
  std::memset(sa, 0, sizeof(r->seed_array));
  int32_t subtraction = (seed == INT32_MIN) ? INT32_MAX : (seed < 0 ? -seed : seed);
  int32_t mj = MSEED - subtraction;
  sa[55] = mj;
  int32_t mk = 1;
  int ii = 0;
  for (int i = 1; i < 55; i++) {
    if ((ii += 21) >= 55) ii -= 55;
    sa[ii] = mk;
    mk = mj - mk;
    if (mk < 0) mk += MBIG;
    mj = sa[ii];
  }
  for (int k = 1; k < 5; k++) {
    for (int i = 1; i < 56; i++) {
      int n = i + 30;
      if (n >= 55) n -= 55;
      sa[i] = (int32_t)((uint32_t)sa[i] - (uint32_t)sa[1 + n]);
      if (sa[i] < 0) sa[i] += MBIG;
    }
  }
  r->inext = 0;
  r->inextp = 21;
}

double or_dotnet_random_next_double(or_dotnet_random* r) {
  const int32_t MBIG = 2147483647;
  int a = r->inext, b = r->inextp;
  if (++a >= 56) a = 1;
  if (++b >= 56) b = 1;
  int32_t ret = (int32_t)((uint32_t)r->seed_array[a] - (uint32_t)r->seed_array[b]);
  if (ret == MBIG) ret--;
  if (ret < 0) ret += MBIG;
  r->seed_array[a] = ret;
  r->inext = a;
  r->inextp = b;
  return ret * (1.0 / MBIG);
}

void or_dotnet_random_floats(or_dotnet_random* r, float* out, int count, float min, float max) {
  float range = max - min;
  for (int i = 0; i < count; i++) out[i] = (float)or_dotnet_random_next_double(r) * range + min;
}

// ---------------------------------------------------------------------------
// Q4KTensor.cs:155-191 HalfToFloat (exact fp16 -> fp32, subnormals normalised).
float or_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t exponent = (uint32_t)(h & 0x7C00) >> 10;
  uint32_t mantissa = (uint32_t)(h & 0x03FF);
  uint32_t bits;
  if (exponent == 0) {
    if (mantissa == 0) {
      bits = sign;
      float f;
      std::memcpy(&f, &bits, 4);
      return f;
    }
    while ((mantissa & 0x0400) == 0) {
      mantissa <<= 1;
      exponent--;
    }
    exponent++;
    mantissa &= 0x03FF;
  } else if (exponent == 31) {
    bits = sign | 0x7F800000u | (mantissa << 13);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
  }
  exponent = exponent + (127 - 15);
  mantissa = mantissa << 13;
  bits = sign | (exponent << 23) | mantissa;
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// IEEE round-to-nearest-even fp32 -> fp16 (integer restatement; no reference
// counterpart — the reference has no K-quant quantizer).
uint16_t or_float_to_half_rne(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t absx = x & 0x7FFFFFFFu;
  if (absx >= 0x7F800000u) return (uint16_t)(sign | (absx > 0x7F800000u ? 0x7E00u : 0x7C00u));
  if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to >= 65520 -> inf
  if (absx < 0x38800000u) {                                     // subnormal half (< 2^-14)
    if (absx < 0x33000000u) return (uint16_t)sign;              // < 2^-25 -> 0 (ties at 2^-25 round to even 0)
    uint32_t e = absx >> 23;
    uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
    int shift = 126 - (int)e;  // result = m >> (shift) with 14 + ... alignment
    // half subnormal unit is 2^-24; value = m * 2^(e-150); units = m * 2^(e-126)
    uint32_t units = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (units & 1))) units++;
    return (uint16_t)(sign | units);
  }
  uint32_t e = (absx >> 23) - 127 + 15;
  uint32_t m = absx & 0x7FFFFFu;
  uint32_t h = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
  return (uint16_t)(sign | h);
}

// ---------------------------------------------------------------------------
// Q8Tensor.cs:72-125 Quantize: per block over the linear index,
// scale = maxAbs>0 ? maxAbs/127f : 1f; q = (sbyte)round_half_even(clamp(x*(1/scale), -127, 127)).
int or_q8_quantize(const float* src, int64_t n, int bs, int8_t* data, float* scales) {
  if (bs <= 0 || n <= 0) return -1;
  int64_t nb = (n + bs - 1) / bs;
  for (int64_t b = 0; b < nb; ++b) {
    int64_t s = b * bs, e = std::min<int64_t>(s + bs, n);
    float maxAbs = 0.f;
    for (int64_t i = s; i < e; ++i) {
      float a = std::fabs(src[i]);
      if (a > maxAbs) maxAbs = a;
    }
    float scale = maxAbs > 0.f ? maxAbs / 127.f : 1.f;
    scales[b] = scale;
    float inv = 1.f / scale;
    for (int64_t i = s; i < e; ++i) {
      float q = src[i] * inv;
      data[i] = (int8_t)(int)round_half_even(clampf(q, -127.f, 127.f));
    }
  }
  return 0;
}

// Q8Tensor.cs:131-158: w = q * scale.
void or_q8_dequantize(const int8_t* data, const float* scales, int64_t n, int bs, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = (float)data[i] * scales[i / bs];
}

// Q4Tensor.cs:140-144: 4-bit two's complement.
int or_q4_decode_nibble(int nibble) { return nibble < 8 ? nibble : nibble - 16; }

// Q4Tensor.cs:75-134: scale = maxAbs/7f; q = round_half_even(clamp(x*(1/scale), -8, 7));
// global linear index i: even -> low nibble, odd -> high nibble.
int or_q4_quantize(const float* src, int64_t n, int bs, uint8_t* data, float* scales) {
  if (bs <= 0 || n <= 0) return -1;
  int64_t nb = (n + bs - 1) / bs;
  for (int64_t b = 0; b < nb; ++b) {
    int64_t s = b * bs, e = std::min<int64_t>(s + bs, n);
    float maxAbs = 0.f;
    for (int64_t i = s; i < e; ++i) {
      float a = std::fabs(src[i]);
      if (a > maxAbs) maxAbs = a;
    }
    float scale = maxAbs > 0.f ? maxAbs / 7.f : 1.f;
    scales[b] = scale;
    float inv = 1.f / scale;
    for (int64_t i = s; i < e; ++i) {
      int c = (int)round_half_even(clampf(src[i] * inv, -8.f, 7.f));
      int64_t bi = i / 2;
      if (i % 2 == 0)
        data[bi] = (uint8_t)(c & 0xF);
      else
        data[bi] = (uint8_t)((data[bi] & 0x0F) | ((c & 0xF) << 4));
    }
  }
  return 0;
}

// Q4Tensor.cs:150-179.
void or_q4_dequantize(const uint8_t* data, const float* scales, int64_t n, int bs, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    uint8_t p = data[i / 2];
    int nib = (i % 2 == 0) ? (p & 0xF) : ((p >> 4) & 0xF);
    out[i] = (float)or_q4_decode_nibble(nib) * scales[i / bs];
  }
}

// Q4_1Tensor.cs:47-112 (block 32 fixed): per block min and max, scale =
// range > 0 ? range/15f : 1f, q = (int)round_half_even(clamp((x - min) * (1/scale), 0, 15)),
// nibbles packed by global index (even -> low).  Scales and mins are two arrays.
int or_q41_quantize(const float* src, int64_t n, uint8_t* data, float* scales, float* mins) {
  if (n <= 0) return -1;
  const int bs = 32;
  const int64_t nb = (n + bs - 1) / bs;
  for (int64_t b = 0; b < nb; ++b) {
    const int64_t s = b * bs, e = std::min<int64_t>(s + bs, n);
    float lo = std::numeric_limits<float>::max(), hi = std::numeric_limits<float>::lowest();
    for (int64_t i = s; i < e; ++i) {
      if (src[i] < lo) lo = src[i];
      if (src[i] > hi) hi = src[i];
    }
    const float range = hi - lo;
    const float scale = range > 0.f ? range / 15.f : 1.f;
    scales[b] = scale;
    mins[b] = lo;
    const float inv = 1.f / scale;
    for (int64_t i = s; i < e; ++i) {
      const float nv = (src[i] - lo) * inv;
      const int c = (int)round_half_even(clampf(nv, 0.f, 15.f));
      const int64_t bi = i / 2;
      if (i % 2 == 0)
        data[bi] = (uint8_t)(c & 0xF);
      else
        data[bi] = (uint8_t)((data[bi] & 0x0F) | ((c & 0xF) << 4));
    }
  }
  return 0;
}

// Q4_1Tensor.cs:129-160: w = q * scale + min (q the unsigned nibble).
void or_q41_dequantize(const uint8_t* data, const float* scales, const float* mins, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    const uint8_t p = data[i / 2];
    const int q = (i % 2 == 0) ? (p & 0xF) : ((p >> 4) & 0xF);
    out[i] = (float)q * scales[i / 32] + mins[i / 32];
  }
}

// Q5_0Tensor.cs:47-130 (block 32 fixed): scale = maxAbs > 0 ? maxAbs/15f : 1f,
// q = (int)round_half_even(clamp(x * (1/scale), -16, 15)) + 16; the low nibble packed
// by global index, bit (i - blockStart) of the block's little-endian 32-bit word the high bit.
int or_q50_quantize(const float* src, int64_t n, uint8_t* low, uint8_t* high, float* scales) {
  if (n <= 0) return -1;
  const int bs = 32;
  const int64_t nb = (n + bs - 1) / bs;
  for (int64_t b = 0; b < nb; ++b) {
    const int64_t s = b * bs, e = std::min<int64_t>(s + bs, n);
    float maxAbs = 0.f;
    for (int64_t i = s; i < e; ++i) maxAbs = std::max(maxAbs, std::fabs(src[i]));
    const float scale = maxAbs > 0.f ? maxAbs / 15.f : 1.f;
    scales[b] = scale;
    const float inv = 1.f / scale;
    uint32_t hb = 0;
    for (int64_t i = s; i < e; ++i) {
      const int c = (int)round_half_even(clampf(src[i] * inv, -16.f, 15.f)) + 16;
      const int64_t bi = i / 2;
      if (i % 2 == 0)
        low[bi] = (uint8_t)(c & 0xF);
      else
        low[bi] = (uint8_t)((low[bi] & 0x0F) | ((c & 0xF) << 4));
      hb |= (uint32_t)((c >> 4) & 1) << (i - s);
    }
    for (int k = 0; k < 4; ++k) high[4 * b + k] = (uint8_t)(hb >> (8 * k));
  }
  return 0;
}

// Q5_0Tensor.cs:136-182: w = (((low | high << 4)) - 16) * scale.
void or_q50_dequantize(const uint8_t* low, const uint8_t* high, const float* scales, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    const int64_t b = i / 32;
    const uint32_t hb = (uint32_t)high[4 * b] | ((uint32_t)high[4 * b + 1] << 8) | ((uint32_t)high[4 * b + 2] << 16) |
                        ((uint32_t)high[4 * b + 3] << 24);
    const uint8_t p = low[i / 2];
    const int lo4 = (i % 2 == 0) ? (p & 0xF) : ((p >> 4) & 0xF);
    const int q = (lo4 | (int)(((hb >> (i - 32 * b)) & 1) << 4)) - 16;
    out[i] = (float)q * scales[b];
  }
}

// Q4_K quantizer (this build's own; the reference has none).  Emits the
// reference's byte layout (Q4KTensor.cs:84-147): per 32-element sub-block a
// 6-bit scale and 6-bit min under fp16 super-scales d/dmin, w ~= d*s*q - dmin*m.
void or_q4k_quantize(const float* src, int64_t n, uint8_t* out) {
  int64_t nb = n / 256;
  for (int64_t b = 0; b < nb; ++b) {
    const float* x = src + b * 256;
    uint8_t* o = out + b * 144;
    float sub_scale[8], sub_min[8];
    for (int j = 0; j < 8; ++j) {
      float mn = x[32 * j], mx = x[32 * j];
      for (int i = 1; i < 32; ++i) {
        mn = std::min(mn, x[32 * j + i]);
        mx = std::max(mx, x[32 * j + i]);
      }
      if (mn > 0.f) mn = 0.f;
      sub_scale[j] = (mx - mn) / 15.f;
      sub_min[j] = -mn;
    }
    float max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; ++j) {
      max_scale = std::max(max_scale, sub_scale[j]);
      max_min = std::max(max_min, sub_min[j]);
    }
    uint16_t dh = or_float_to_half_rne(max_scale / 63.f);
    uint16_t dmh = or_float_to_half_rne(max_min / 63.f);
    float d = or_half_to_float(dh), dmin = or_half_to_float(dmh);
    uint8_t sc[8], mnq[8];
    for (int j = 0; j < 8; ++j) {
      int s = d > 0.f ? (int)round_half_even(sub_scale[j] / d) : 0;
      int m = dmin > 0.f ? (int)round_half_even(sub_min[j] / dmin) : 0;
      sc[j] = (uint8_t)std::min(63, std::max(0, s));
      mnq[j] = (uint8_t)std::min(63, std::max(0, m));
    }
    std::memcpy(o, &dh, 2);
    std::memcpy(o + 2, &dmh, 2);
    uint8_t* s = o + 4;
    for (int g = 0; g < 2; ++g) {  // inverse of the unpack in Q4KTensor.cs:109-126
      const uint8_t* v = (g == 0) ? sc : mnq;
      for (int h = 0; h < 2; ++h) {
        const uint8_t* w = v + 4 * h;
        uint8_t* t = s + 6 * g + 3 * h;
        t[0] = (uint8_t)((w[0] & 0x3F) | ((w[1] & 0x03) << 6));
        t[1] = (uint8_t)(((w[1] >> 2) & 0x0F) | ((w[2] & 0x0F) << 4));
        t[2] = (uint8_t)(((w[2] >> 4) & 0x03) | ((w[3] & 0x3F) << 2));
      }
    }
    uint8_t* qs = o + 16;
    for (int j = 0; j < 8; ++j) {
      float ss = d * (float)sc[j];
      float mm = dmin * (float)mnq[j];
      int q[32];
      for (int i = 0; i < 32; ++i) {
        int v = ss > 0.f ? (int)round_half_even((x[32 * j + i] + mm) / ss) : 0;
        q[i] = std::min(15, std::max(0, v));
      }
      for (int i = 0; i < 16; ++i) qs[16 * j + i] = (uint8_t)(q[2 * i] | (q[2 * i + 1] << 4));
    }
  }
}

void or_q4k_dequantize(const uint8_t* src, int64_t n, float* out) {
  for (int64_t b = 0; b < n / 256; ++b) dequant_q4k_block(src + b * 144, out + b * 256);
}

// Q6_K quantizer (this build's own).  Emits the reference layout
// (Q6KTensor.cs:85-125): symmetric 6-bit, int8 sub-block scales under an fp16 d.
void or_q6k_quantize(const float* src, int64_t n, uint8_t* out) {
  int64_t nb = n / 256;
  for (int64_t b = 0; b < nb; ++b) {
    const float* x = src + b * 256;
    uint8_t* o = out + b * 210;
    std::memset(o, 0, 210);
    float sub_scale[16];
    float max_scale = 0.f;
    for (int j = 0; j < 16; ++j) {
      float amax = 0.f;
      for (int i = 0; i < 16; ++i) amax = std::max(amax, std::fabs(x[16 * j + i]));
      sub_scale[j] = amax / 31.f;
      max_scale = std::max(max_scale, sub_scale[j]);
    }
    uint16_t dh = or_float_to_half_rne(max_scale / 127.f);
    float d = or_half_to_float(dh);
    int8_t* scales = (int8_t*)(o + 192);
    for (int j = 0; j < 16; ++j) {
      int s = d > 0.f ? (int)round_half_even(sub_scale[j] / d) : 0;
      scales[j] = (int8_t)std::min(127, std::max(-128, s));
    }
    std::memcpy(o + 208, &dh, 2);
    for (int v = 0; v < 256; ++v) {
      float ss = d * (float)scales[v / 16];
      int q = ss > 0.f ? (int)round_half_even(x[v] / ss) + 32 : 32;
      q = std::min(63, std::max(0, q));
      o[v / 2] |= (uint8_t)((q & 0xF) << ((v % 2) * 4));
      o[128 + v / 4] |= (uint8_t)(((q >> 4) & 3) << ((v % 4) * 2));
    }
  }
}

void or_q6k_dequantize(const uint8_t* src, int64_t n, float* out) {
  for (int64_t b = 0; b < n / 256; ++b) dequant_q6k_block(src + b * 210, out + b * 256);
}

// ---------------------------------------------------------------------------
// Quantized matmul.
// Element li of a Q4_1 / Q5_0 tensor of n_total elements.  Q4_1: `scales` holds
// the block scales then the block mins; Q5_0: `data` holds the low nibbles then
// the 4-byte high-bit words of the blocks.
static float q41_q50_elem(int scheme, const void* data, const float* scales, int64_t n_total, int64_t li) {
  const uint8_t* q = (const uint8_t*)data;
  const int64_t b = li / 32, nb = (n_total + 31) / 32;
  const uint8_t p = q[li / 2];
  const int lo4 = (li % 2 == 0) ? (p & 0xF) : ((p >> 4) & 0xF);
  if (scheme == OR_Q4_1) return (float)lo4 * scales[b] + scales[nb + b];
  const uint8_t* high = q + (n_total + 1) / 2 + 4 * b;
  const uint32_t hb = (uint32_t)high[0] | ((uint32_t)high[1] << 8) | ((uint32_t)high[2] << 16) | ((uint32_t)high[3] << 24);
  const int v = (lo4 | (int)(((hb >> (li - 32 * b)) & 1) << 4)) - 16;
  return (float)v * scales[b];
}

static void decode_row_intended(int scheme, const void* data, const float* scales, int bs, int64_t n, int K,
                                float* w, int64_t n_total) {
  // Row n of W[N][K] in linear-index order (Q*Tensor.Dequantize element formulas).
  int64_t base = n * (int64_t)K;
  switch (scheme) {
    case OR_F32:
      std::memcpy(w, (const float*)data + base, sizeof(float) * K);
      break;
    case OR_Q8_0: {
      const int8_t* q = (const int8_t*)data;
      for (int k = 0; k < K; ++k) w[k] = (float)q[base + k] * scales[(base + k) / bs];
      break;
    }
    case OR_Q4_0: {
      const uint8_t* q = (const uint8_t*)data;
      for (int k = 0; k < K; ++k) {
        int64_t i = base + k;
        uint8_t p = q[i / 2];
        int nib = (i % 2 == 0) ? (p & 0xF) : ((p >> 4) & 0xF);
        w[k] = (float)or_q4_decode_nibble(nib) * scales[i / bs];
      }
      break;
    }
    case OR_Q4_1:
    case OR_Q5_0: {
      for (int k = 0; k < K; ++k) w[k] = q41_q50_elem(scheme, data, scales, n_total, base + k);
      break;
    }
    case OR_Q4_K: {
      const uint8_t* q = (const uint8_t*)data;
      for (int kb = 0; kb < K / 256; ++kb) dequant_q4k_block(q + (base / 256 + kb) * 144, w + 256 * kb);
      break;
    }
    case OR_Q6_K: {
      const uint8_t* q = (const uint8_t*)data;
      for (int kb = 0; kb < K / 256; ++kb) dequant_q6k_block(q + (base / 256 + kb) * 210, w + 256 * kb);
      break;
    }
  }
}

int or_matmul(int scheme, int mode, const void* data, const float* scales, int bs, const float* A, float* C,
              double* C64, int M, int K, int N) {
  if (M <= 0 || K <= 0 || N <= 0) return -1;
  if ((scheme == OR_Q4_K || scheme == OR_Q6_K) && K % 256 != 0) return -2;
  if (mode == 1) {
    std::vector<float> w(K);
    for (int n = 0; n < N; ++n) {
      decode_row_intended(scheme, data, scales, bs, n, K, w.data(), (int64_t)N * K);
      for (int m = 0; m < M; ++m) {
        const float* a = A + (int64_t)m * K;
        float s = 0.f;
        double s64 = 0.0;
        for (int k = 0; k < K; ++k) {
          float p = a[k] * w[k];
          s += p;
          if (C64) s64 += (double)a[k] * (double)w[k];
        }
        C[(int64_t)m * N + n] = s;
        if (C64) C64[(int64_t)m * N + n] = s64;
      }
    }
    return 0;
  }
  // mode 0: reference-literal orientation (B is KxN).
  std::fill(C, C + (int64_t)M * N, 0.f);
  if (C64) std::fill(C64, C64 + (int64_t)M * N, 0.0);
  if (scheme == OR_Q8_0 || scheme == OR_Q4_0 || scheme == OR_F32) {
    // MatMulF32Q8.cs:53-80 / MatMulF32Q4.cs:61-92: c[col] += aVal * quantVal * scale,
    // K ascending in the outer loop, exact-zero activations skipped.
    for (int m = 0; m < M; ++m) {
      const float* a = A + (int64_t)m * K;
      float* c = C + (int64_t)m * N;
      for (int k = 0; k < K; ++k) {
        float av = a[k];
        if (av == 0.f) continue;
        int64_t ro = (int64_t)k * N;
        for (int n = 0; n < N; ++n) {
          int64_t li = ro + n;
          float q, sc;
          if (scheme == OR_F32) {
            q = ((const float*)data)[li];
            sc = 1.f;
          } else if (scheme == OR_Q8_0) {
            q = (float)((const int8_t*)data)[li];
            sc = scales[li / bs];
          } else {
            uint8_t p = ((const uint8_t*)data)[li >> 1];
            q = (float)or_q4_decode_nibble((p >> ((li & 1) << 2)) & 0xF);
            sc = scales[li / bs];
          }
          float t = av * q;
          c[n] += t * sc;
          if (C64) C64[(int64_t)m * N + n] += (double)av * (double)q * (double)sc;
        }
      }
    }
    return 0;
  }
  if (scheme == OR_Q4_1 || scheme == OR_Q5_0) {
    // FusedQ4_1MatMul.cs:356-385 / FusedQ5_0MatMul.cs:388-426 (scalar paths): bkj =
    // the dequantized element at linear index k*N + j, C[i][j] += a[i][k] * bkj, k ascending
    const int64_t nt = (int64_t)K * N;
    for (int m = 0; m < M; ++m) {
      const float* a = A + (int64_t)m * K;
      float* c = C + (int64_t)m * N;
      for (int k = 0; k < K; ++k)
        for (int n = 0; n < N; ++n) {
          const float bkj = q41_q50_elem(scheme, data, scales, nt, (int64_t)k * N + n);
          c[n] += a[k] * bkj;
          if (C64) C64[(int64_t)m * N + n] += (double)a[k] * (double)bkj;
        }
    }
    return 0;
  }
  // FusedQ4KMatMul.cs:76-197 / FusedQ6KMatMul.cs:66-164: block (k/256)*N + n,
  // accum += a * (dequantized element), K ascending per (m, n).
  const int bpb = scheme == OR_Q4_K ? 144 : 210;
  std::vector<float> w(256);
  for (int m = 0; m < M; ++m) {
    for (int n = 0; n < N; ++n) {
      float acc = 0.f;
      double acc64 = 0.0;
      for (int kb = 0; kb < K / 256; ++kb) {
        const uint8_t* blk = (const uint8_t*)data + ((int64_t)kb * N + n) * bpb;
        if (scheme == OR_Q4_K)
          dequant_q4k_block(blk, w.data());
        else
          dequant_q6k_block(blk, w.data());
        const float* a = A + (int64_t)m * K + kb * 256;
        for (int i = 0; i < 256; ++i) {
          float p = a[i] * w[i];
          acc += p;
          if (C64) acc64 += (double)a[i] * (double)w[i];
        }
      }
      C[(int64_t)m * N + n] = acc;
      if (C64) C64[(int64_t)m * N + n] = acc64;
    }
  }
  return 0;
}

// ---------------------------------------------------------------------------
// RMSNormOps.cs:28-220: sumSq via 8-lane Vector<float> partials when F >= 128
// (lanes summed in order, then the scalar tail), invRms = 1/sqrt(sumSq/F + eps),
// y = gamma * (x * invRms).
void or_rmsnorm(const float* x, const float* gamma, float* y, int rows, int F, float eps) {
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (int64_t)r * F;
    float sumSq = 0.f;
    if (F >= 128) {
      float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      int f = 0;
      for (; f <= F - 8; f += 8)
        for (int l = 0; l < 8; ++l) lanes[l] += xr[f + l] * xr[f + l];
      for (int l = 0; l < 8; ++l) sumSq += lanes[l];
      for (; f < F; ++f) sumSq += xr[f] * xr[f];
    } else {
      for (int f = 0; f < F; ++f) sumSq += xr[f] * xr[f];
    }
    float invRms = 1.f / std::sqrt(sumSq / (float)F + eps);
    for (int f = 0; f < F; ++f) {
      float nrm = xr[f] * invRms;
      y[(int64_t)r * F + f] = gamma[f] * nrm;
    }
  }
}

// RotaryEmbedding.cs:45-60: freq = 1/powf(theta, 2i/hd); angle = pos*freq.
void or_rope_tables(int max_seq, int hd, float theta, float* sin_t, float* cos_t) {
  int half = hd / 2;
  for (int pos = 0; pos < max_seq; ++pos)
    for (int i = 0; i < half; ++i) {
      float freq = 1.0f / std::pow(theta, (2.0f * (float)i) / (float)hd);
      float angle = (float)pos * freq;
      sin_t[pos * half + i] = std::sin(angle);
      cos_t[pos * half + i] = std::cos(angle);
    }
}

// RotaryEmbedding.cs:103-116: interleaved pairs (2i, 2i+1).
void or_rope_apply(float* x, int n_heads, int hd, int pos, const float* sin_t, const float* cos_t) {
  int half = hd / 2;
  for (int h = 0; h < n_heads; ++h) {
    float* r = x + h * hd;
    for (int i = 0; i < half; ++i) {
      float x0 = r[2 * i], x1 = r[2 * i + 1];
      float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
      float a0 = x0 * c, b0 = x1 * s, a1 = x0 * s, b1 = x1 * c;
      r[2 * i] = a0 - b0;
      r[2 * i + 1] = a1 + b1;
    }
  }
}

// MathUtils.cs:20-32: Pade(2,2) exp with clamp to [-87.3, 88.7].
float or_fast_exp(float x) {
  x = std::max(-87.3f, std::min(x, 88.7f));
  float x2 = x * x;
  float num = 1.0f + x * 0.5f + x2 * 0.08333333f;
  float den = 1.0f - x * 0.5f + x2 * 0.08333333f;
  return num / den;
}

// ActivationOps.cs:304-309 FastSigmoid, :565-580 FusedSiLUMul.
void or_silu_mul(const float* g, const float* u, float* out, int n) {
  for (int i = 0; i < n; ++i) {
    float x = g[i];
    float c = std::max(-20.f, std::min(x, 20.f));
    float sig = 1.f / (1.f + std::exp(-c));
    float silu = x * sig;
    out[i] = silu * u[i];
  }
}

// Attention: MultiHeadAttention.cs:676-744 (S = Q K^T unscaled, GQA map
// kvHead = h / (nH/nKv)), OptimizedOps.cs:39-95 (max of s*scale, e =
// FastExp(s*scale - max), p = e * (1/sum)), MultiHeadAttention.cs:810-844 (O = P V).
void or_attention(const float* q, const float* k, const float* v, float* out, int T, int S, int nH, int nKv, int hd,
                  int n_threads) {
  const float scale = 1.0f / std::sqrt((float)hd);
  const int group = nH / nKv;
  const int qd = nH * hd, kd = nKv * hd;
  const int cache_offset = S - T;
  parallel_for(nH, n_threads, [&](int h) {
    int kvh = h / group;
    std::vector<float> sc(S);
    for (int i = 0; i < T; ++i) {
      const float* qi = q + (int64_t)i * qd + h * hd;
      int valid = cache_offset + i + 1;
      for (int j = 0; j < valid; ++j) {
        const float* kj = k + (int64_t)j * kd + kvh * hd;
        float s = 0.f;
        for (int d = 0; d < hd; ++d) s += qi[d] * kj[d];
        sc[j] = s;
      }
      float mx = -INFINITY;
      for (int j = 0; j < valid; ++j) {
        float s = sc[j] * scale;
        if (s > mx) mx = s;
      }
      float sum = 0.f;
      for (int j = 0; j < valid; ++j) {
        float e = or_fast_exp(sc[j] * scale - mx);
        sc[j] = e;
        sum += e;
      }
      float inv = 1.f / sum;
      for (int j = 0; j < valid; ++j) sc[j] *= inv;
      float* o = out + (int64_t)i * qd + h * hd;
      for (int d = 0; d < hd; ++d) o[d] = 0.f;
      for (int j = 0; j < valid; ++j) {
        const float* vj = v + (int64_t)j * kd + kvh * hd;
        float p = sc[j];
        for (int d = 0; d < hd; ++d) o[d] += p * vj[d];
      }
    }
  });
}

// ---------------------------------------------------------------------------
// Threads of the quantized linears: 0 = the caller's n_threads (rows split across
// threads); 1 = single-threaded, the reference's own threading (its MatMulF32Q8 /
// FusedQ4KMatMul / FusedQ6KMatMul run on the calling thread).  Attention keeps
// n_threads either way (Parallel.For over B*nH, MultiHeadAttention.cs:686-712).
static std::atomic<int> g_linear_threads{0};
void or_set_linear_threads(int n) { g_linear_threads.store(n < 0 ? 0 : n); }

static void linear_fwd(const or_linear& L, const float* x, float* y, int M, int K, int N, int n_threads) {
  // x . W^T for W [N][K]; rows split across threads (each row is independent).
  const int lt = g_linear_threads.load();
  if (lt > 0) n_threads = lt;
  int chunks = std::max(1, std::min(n_threads, N / 64));
  parallel_for(chunks, chunks, [&](int c) {
    int n0 = (int)((int64_t)N * c / chunks), n1 = (int)((int64_t)N * (c + 1) / chunks);
    std::vector<float> w(K);
    for (int n = n0; n < n1; ++n) {
      decode_row_intended(L.scheme, L.data, L.scales, L.block_size, n, K, w.data(), (int64_t)N * K);
      for (int m = 0; m < M; ++m) {
        const float* a = x + (int64_t)m * K;
        float s = 0.f;
        for (int k = 0; k < K; ++k) {
          float p = a[k] * w[k];
          s += p;
        }
        y[(int64_t)m * N + n] = s;
      }
    }
  });
}

// One pass of T tokens at positions pos..pos+T-1 over the cached K/V
// (TransformerBlock.cs:153-187 per layer; TransformerModel.cs:272-344 overall).
int or_model_step(const or_model* mdl, float* kv, int pos, const int* tokens, int T, float* last_logits,
                  int n_threads) {
  const or_model_config& c = mdl->cfg;
  const int H = c.hidden, hd = c.head_dim, nH = c.n_heads, nKv = c.n_kv_heads, F = c.ffn_hidden;
  const int qd = nH * hd, kd = nKv * hd, S = pos + T;
  if (S > c.max_context || T <= 0) return -1;
  std::vector<float> x((size_t)T * H), h((size_t)T * H), q((size_t)T * qd), att((size_t)T * qd),
      o((size_t)T * H), g((size_t)T * F), u((size_t)T * F), a((size_t)T * F);
  std::vector<float> sin_t((size_t)c.max_context * hd / 2), cos_t((size_t)c.max_context * hd / 2);
  or_rope_tables(c.max_context, hd, c.rope_theta, sin_t.data(), cos_t.data());
  for (int t = 0; t < T; ++t) {  // Embedding.Forward (NeuralNet.cs:376-): row gather
    int id = tokens[t];
    if (id < 0 || id >= c.vocab_size) return -2;
    std::memcpy(&x[(size_t)t * H], mdl->token_embd + (int64_t)id * H, sizeof(float) * H);
  }
  const size_t layer_stride = (size_t)2 * c.max_context * kd;
  for (int l = 0; l < c.n_layers; ++l) {
    const or_layer& L = mdl->layers[l];
    float* kc = kv + layer_stride * l;
    float* vc = kc + (size_t)c.max_context * kd;
    or_rmsnorm(x.data(), L.attn_norm, h.data(), T, H, c.norm_eps);
    linear_fwd(L.wq, h.data(), q.data(), T, H, qd, n_threads);
    linear_fwd(L.wk, h.data(), kc + (size_t)pos * kd, T, H, kd, n_threads);
    linear_fwd(L.wv, h.data(), vc + (size_t)pos * kd, T, H, kd, n_threads);
    for (int t = 0; t < T; ++t) {
      or_rope_apply(&q[(size_t)t * qd], nH, hd, pos + t, sin_t.data(), cos_t.data());
      or_rope_apply(kc + (size_t)(pos + t) * kd, nKv, hd, pos + t, sin_t.data(), cos_t.data());
    }
    or_attention(q.data(), kc, vc, att.data(), T, S, nH, nKv, hd, n_threads);
    linear_fwd(L.wo, att.data(), o.data(), T, qd, H, n_threads);
    for (size_t i = 0; i < x.size(); ++i) x[i] = x[i] + o[i];  // TransformerBlock.cs:170
    or_rmsnorm(x.data(), L.ffn_norm, h.data(), T, H, c.norm_eps);
    linear_fwd(L.w_gate, h.data(), g.data(), T, H, F, n_threads);  // GatedMLP.cs:51-93
    linear_fwd(L.w_up, h.data(), u.data(), T, H, F, n_threads);
    or_silu_mul(g.data(), u.data(), a.data(), T * F);
    linear_fwd(L.w_down, a.data(), o.data(), T, F, H, n_threads);
    for (size_t i = 0; i < x.size(); ++i) x[i] = x[i] + o[i];  // TransformerBlock.cs:184
  }
  // final RMSNorm + LM head on the last position only (what the generation loop reads,
  // InferenceSession.cs:548-563)
  std::vector<float> hl(H);
  or_rmsnorm(&x[(size_t)(T - 1) * H], mdl->out_norm, hl.data(), 1, H, c.norm_eps);
  linear_fwd(mdl->output, hl.data(), last_logits, 1, H, c.vocab_size, n_threads);
  return 0;
}

int or_model_forward(const or_model* mdl, const int* tokens, int T, int n_last, float* logits, int n_threads) {
  const or_model_config& c = mdl->cfg;
  if (n_last < 1 || n_last > T) return -1;
  const int kd = c.n_kv_heads * c.head_dim;
  std::vector<float> kv((size_t)c.n_layers * 2 * c.max_context * kd);
  // Cache-off semantics: position p's logits come from a full recompute of
  // tokens[0..p] (TransformerModel.Forward with positionOffset 0).  Causality
  // makes that equal to one pass over tokens[0..T) read at row p.
  for (int r = 0; r < n_last; ++r) {
    int p = T - n_last + r;
    int rc = or_model_step(mdl, kv.data(), 0, tokens, p + 1, logits + (int64_t)r * c.vocab_size, n_threads);
    if (rc) return rc;
  }
  return 0;
}

// Counter-based N(0, std): SplitMix64 of (seed, index) -> two uniforms -> Box-Muller.
static inline uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// ---------------------------------------------------------------- sampling
// NormalizeProbabilities (InferenceSession.cs:982-1031): Vector<float> lane sums
// (8 lanes), horizontal sum, remainder, then multiply by 1 / sum.
static void or_normalize(float* p, int V) {
  float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int i = 0;
  for (; i + 8 <= V; i += 8)
    for (int j = 0; j < 8; ++j) lanes[j] += p[i + j];
  float sum = 0.f;
  for (int j = 0; j < 8; ++j) sum += lanes[j];
  for (; i < V; ++i) sum += p[i];
  if (sum > 0.f) {
    const float inv = 1.0f / sum;
    for (int k = 0; k < V; ++k) p[k] *= inv;
  }
}

int or_sample(float* L, int V, double temperature, int top_k, double top_p, double min_p, float rep_penalty,
              float presence_penalty, float frequency_penalty, int rep_window, const int* context, int ctx_len,
              double target, float* probs_out) {
  // 1. penalties (InferenceSession.cs:769-850): distinct tokens of the window, first-seen order, with counts
  if (!(rep_penalty == 1.0f && presence_penalty == 0.0f && frequency_penalty == 0.0f)) {
    const int win = rep_window > 0 ? rep_window : std::min(ctx_len, 256);
    const int start = std::max(0, ctx_len - win);
    std::vector<int> ids, counts;
    for (int i = start; i < ctx_len; ++i) {
      const int t = context[i];
      int f = -1;
      for (size_t j = 0; j < ids.size(); ++j)
        if (ids[j] == t) { f = (int)j; break; }
      if (f >= 0) ++counts[f];
      else { ids.push_back(t); counts.push_back(1); }
    }
    for (size_t j = 0; j < ids.size(); ++j) {
      float& x = L[ids[j]];
      if (rep_penalty != 1.0f) x = x > 0 ? x / rep_penalty : x * rep_penalty;
      if (presence_penalty != 0.0f) x -= presence_penalty;
      if (frequency_penalty != 0.0f) x -= (float)counts[j] * frequency_penalty;
    }
  }
  // 2. temperature (:741-763)
  if (temperature != 1.0) {
    const float inv = 1.0f / (float)temperature;
    for (int i = 0; i < V; ++i) L[i] *= inv;
  }
  // 3. top-k (:635-670): the k-th largest value of a descending sort; values below it -> -inf
  if (top_k > 0 && top_k < V) {
    std::vector<float> s(L, L + V);
    std::sort(s.begin(), s.end(), [](float a, float b) { return a > b; });
    const float kth = s[std::min(top_k - 1, V - 1)];
    for (int i = 0; i < V; ++i)
      if (!(L[i] >= kth)) L[i] = -INFINITY;
  }
  // 4. softmax (:672-712)
  std::vector<float> p(V);
  float mx = -INFINITY;
  for (int i = 0; i < V; ++i)
    if (L[i] != -INFINITY) mx = std::max(mx, L[i]);
  float sum = 0.f;
  for (int i = 0; i < V; ++i) {
    if (L[i] != -INFINITY) {
      p[i] = std::exp(L[i] - mx);
      sum += p[i];
    } else {
      p[i] = 0.f;
    }
  }
  if (sum > 0)
    for (int i = 0; i < V; ++i) p[i] /= sum;
  // 5. top-p (:862-907): descending order (ties by index here; the reference's sort leaves them unspecified)
  if (top_p < 1.0) {
    std::vector<int> idx(V);
    for (int i = 0; i < V; ++i) idx[i] = i;
    std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return p[a] > p[b]; });
    float cum = 0.f;
    int cut = V;
    for (int i = 0; i < V; ++i) {
      cum += p[idx[i]];
      if ((double)cum >= top_p) { cut = i + 1; break; }
    }
    for (int i = cut; i < V; ++i) p[idx[i]] = 0.f;
    or_normalize(p.data(), V);
  }
  // 6. min-p (:913-935)
  if (min_p > 0.0) {
    float mp = -INFINITY;
    for (int i = 0; i < V; ++i) mp = std::max(mp, p[i]);
    const float thr = mp * (float)min_p;
    for (int i = 0; i < V; ++i)
      if (p[i] < thr) p[i] = 0.f;
    or_normalize(p.data(), V);
  }
  if (probs_out) std::memcpy(probs_out, p.data(), sizeof(float) * V);
  // 7. SampleFromProbs (:714-734)
  double cum = 0.0;
  for (int i = 0; i < V; ++i) {
    cum += p[i];
    if (cum >= target) return i;
  }
  return V - 1;
}

// DeterministicRng.cs: SplitMix64 seeding, xoroshiro128+ (rotations 24 / 16 / 37), 53-bit doubles
void or_deterministic_rng_doubles(int32_t seed, int n, double* out) {
  uint64_t s = (uint64_t)(int64_t)seed;
  auto splitmix = [&]() {
    s += 0x9e3779b97f4a7c15ULL;
    uint64_t z = s;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
  };
  uint64_t s0 = splitmix(), s1 = splitmix();
  if (s0 == 0 && s1 == 0) s0 = s1 = 1;
  auto rotl = [](uint64_t x, int k) { return (x << k) | (x >> (64 - k)); };
  for (int i = 0; i < n; ++i) {
    const uint64_t r = s0 + s1;
    s1 ^= s0;
    s0 = rotl(s0, 24) ^ s1 ^ (s1 << 16);
    s1 = rotl(s1, 37);
    out[i] = (double)(r & ((1ULL << 53) - 1)) * (1.0 / (double)(1ULL << 53));
  }
}

void or_fill_normal(float* out, int64_t n, uint64_t seed, float std_dev, int n_threads) {
  int chunks = std::max(1, n_threads);
  parallel_for(chunks, chunks, [&](int c) {
    int64_t i0 = n * c / chunks, i1 = n * (c + 1) / chunks;
    for (int64_t i = i0; i < i1; ++i) {
      uint64_t r = splitmix64(seed * 0x100000001B3ull ^ (uint64_t)i);
      double u1 = ((r >> 11) + 1) * (1.0 / 9007199254740993.0);
      double u2 = ((splitmix64(r) >> 11)) * (1.0 / 9007199254740992.0);
      double z = std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
      out[i] = (float)(z * std_dev);
    }
  });
}

}  // extern "C"
