// Quantize / dequantize kernels (bit-exact with the reference element formulas).
#include "common.cuh"

namespace sm {
namespace {

// ---------------------------------------------------------------- dequant
// Q8Tensor.cs:131-158: w = (float)q * scale.
__global__ void dequant_q8_kernel(const int8_t* __restrict__ q, const float* __restrict__ scales, int64_t n, int bs,
                                  int bpr, int stride, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __fmul_rn((float)q[i], scales[aux_idx(i / bs, bpr, stride)]);
}

// Q4Tensor.cs:150-179: nibble by global index (even low), two's complement, * scale.
__global__ void dequant_q4_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scales, int64_t n, int bs,
                                  int bpr, int stride, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    uint8_t p = q[i >> 1];
    int nib = (i & 1) ? (p >> 4) : (p & 0xF);
    int v = nib < 8 ? nib : nib - 16;
    out[i] = __fmul_rn((float)v, scales[aux_idx(i / bs, bpr, stride)]);
  }
}

// Q4KTensor.cs:79-147.  One 64-thread group per block; thread t owns qs byte
// pair... simple mapping: thread t in [0,128) decodes qs byte t (2 elements).
__global__ void dequant_q4k_kernel(const uint8_t* __restrict__ src, int64_t nblocks, float* __restrict__ out) {
  const int t = threadIdx.x;  // 128 threads, one per qs byte
  for (int64_t b = blockIdx.x; b < nblocks; b += gridDim.x) {
    const uint8_t* blk = src + b * Q4K_BLOCK_BYTES;
    const uint16_t db = (uint16_t)blk[0] | ((uint16_t)blk[1] << 8);
    const uint16_t dmb = (uint16_t)blk[2] | ((uint16_t)blk[3] << 8);
    const float d = half_bits_to_float(db), dmin = half_bits_to_float(dmb);
    const int j = t >> 4, i = t & 15;
    int sc, mn;
    unpack_q4k_scales(blk + 4, j, sc, mn);
    const float s = __fmul_rn(d, (float)sc);
    const float m = __fmul_rn(dmin, (float)mn);
    const uint8_t p = blk[16 + t];
    float* o = out + b * 256 + 32 * j + 2 * i;
    o[0] = __fsub_rn(__fmul_rn(s, (float)(p & 0xF)), m);
    o[1] = __fsub_rn(__fmul_rn(s, (float)(p >> 4)), m);
  }
}

// Q6KTensor.cs:80-125 on the device layout (208 B body + separate d; the high
// 2-bit plane is re-packed, see q6k_relayout_kernel).
__device__ __forceinline__ int q6k_high2(const uint8_t* qhp, int v) {
  const int t = v >> 4, e = v & 15;
  const int b = (e & 7) >> 1;
  const int shift = ((e >> 3) << 2) + ((e & 1) << 1);
  return (qhp[4 * t + b] >> shift) & 3;
}

__global__ void dequant_q6k_kernel(const uint8_t* __restrict__ body, const uint16_t* __restrict__ dv, int64_t nblocks,
                                   int bpr, int stride, float* __restrict__ out) {
  const int v = threadIdx.x;  // 256 threads, one per element
  for (int64_t b = blockIdx.x; b < nblocks; b += gridDim.x) {
    const uint8_t* blk = body + b * Q6K_BODY_BYTES;
    const float d = half_bits_to_float(dv[aux_idx(b, bpr, stride)]);
    const int8_t scale = (int8_t)blk[192 + v / 16];
    const float s = __fmul_rn(d, (float)scale);
    const uint8_t qlb = blk[v >> 1];
    const int low4 = (v & 1) ? (qlb >> 4) : (qlb & 0xF);
    const int q = low4 | (q6k_high2(blk + 128, v) << 4);
    out[b * 256 + v] = __fmul_rn(s, (float)(q - 32));
  }
}

__global__ void dequant_f32_kernel(const float* __restrict__ w, int64_t n, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = w[i];
}

// Q6_K reference block (210 B) -> device body (208 B) + d.  The body keeps ql
// (128 B) and the int8 scales (16 B, at 192) as they are; the high-bit plane is
// re-packed so that one 32-bit word covers 16 consecutive elements 16t..16t+15
// and byte b of it holds the 2-bit highs of elements 16t+2b, 16t+2b+1,
// 16t+8+2b, 16t+9+2b (bits 0-1, 2-3, 4-5, 6-7).  Byte b then lines up with
// byte b of the matching ql words, so the GEMV builds four 6-bit values with a
// few shifts and masks per 32-bit word.
__global__ void q6k_relayout_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ body,
                                    uint16_t* __restrict__ dv, int64_t nblocks, int bpr, int stride) {
  for (int64_t b = blockIdx.x; b < nblocks; b += gridDim.x) {
    const uint8_t* s = src + b * Q6K_BLOCK_BYTES;
    uint8_t* o = body + b * Q6K_BODY_BYTES;
    for (int i = threadIdx.x; i < Q6K_BODY_BYTES; i += blockDim.x) {
      if (i < 128 || i >= 192) {
        o[i] = s[i];
      } else {
        const int idx = i - 128, t = idx >> 2, bb = idx & 3;
        auto h = [&](int v) { return (s[128 + (v >> 2)] >> (2 * (v & 3))) & 3; };
        const int v0 = 16 * t + 2 * bb;
        o[i] = (uint8_t)(h(v0) | (h(v0 + 1) << 2) | (h(v0 + 8) << 4) | (h(v0 + 9) << 6));
      }
    }
    if (threadIdx.x == 0) dv[aux_idx(b, bpr, stride)] = (uint16_t)s[208] | ((uint16_t)s[209] << 8);
  }
}

// ---------------------------------------------------------------- quantize
// Q8Tensor.cs:94-120 / Q4Tensor.cs:91-131: one warp per scale block.
// scale = maxAbs > 0 ? maxAbs / qmax : 1; inv = 1 / scale (IEEE divisions).
__global__ void block_scales_kernel(const float* __restrict__ src, int64_t n, int bs, float qmax,
                                    float* __restrict__ scales, float* __restrict__ inv_scales, int64_t nb) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t b = warp; b < nb; b += nwarps) {
    const int64_t s = b * bs;
    const int64_t e = min(s + bs, n);
    float mx = 0.f;
    for (int64_t i = s + lane; i < e; i += 32) mx = fmaxf(mx, fabsf(src[i]));
    mx = warp_max(mx);
    if (lane == 0) {
      float scale = mx > 0.f ? __fdiv_rn(mx, qmax) : 1.f;
      scales[b] = scale;
      inv_scales[b] = __fdiv_rn(1.f, scale);
    }
  }
}

__device__ __forceinline__ int quant_elem(float x, float inv, float lo, float hi) {
  float q = __fmul_rn(x, inv);
  q = fminf(fmaxf(q, lo), hi);  // Math.Clamp
  return (int)rintf(q);         // MathF.Round: half to even
}

__global__ void q8_pack_kernel(const float* __restrict__ src, int64_t n, int bs, const float* __restrict__ inv,
                               int8_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (int8_t)quant_elem(src[i], inv[i / bs], -127.f, 127.f);
}

__global__ void q4_pack_kernel(const float* __restrict__ src, int64_t n, int bs, const float* __restrict__ inv,
                               uint8_t* __restrict__ out) {
  const int64_t nbytes = (n + 1) / 2;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nbytes; b += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i0 = 2 * b, i1 = 2 * b + 1;
    int c0 = quant_elem(src[i0], inv[i0 / bs], -8.f, 7.f);
    int c1 = i1 < n ? quant_elem(src[i1], inv[i1 / bs], -8.f, 7.f) : 0;
    out[b] = (uint8_t)((c0 & 0xF) | ((c1 & 0xF) << 4));
  }
}

// Q4_K quantizer (this library's own; identical arithmetic to the oracle's
// or_q4k_quantize): one warp per 256-element block.
__global__ void q4k_quantize_kernel(const float* __restrict__ src, int64_t nblocks, uint8_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t b = warp; b < nblocks; b += nwarps) {
    const float* x = src + b * 256;
    uint8_t* o = out + b * Q4K_BLOCK_BYTES;
    // lane j<8 computes sub-block j statistics
    float xs[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) xs[r] = x[32 * r + lane];  // element lane of sub-block r
    float sub_scale = 0.f, sub_min = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      float mn = xs[r], mx = xs[r];
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
      }
      if (mn > 0.f) mn = 0.f;
      if (lane == r) {
        sub_scale = __fdiv_rn(__fsub_rn(mx, mn), 15.f);
        sub_min = -mn;
      }
    }
    float ms = lane < 8 ? sub_scale : 0.f, mm = lane < 8 ? sub_min : 0.f;
    ms = warp_max(ms);
    mm = warp_max(mm);
    const __half dh = __float2half_rn(__fdiv_rn(ms, 63.f));
    const __half dmh = __float2half_rn(__fdiv_rn(mm, 63.f));
    const float d = __half2float(dh), dmin = __half2float(dmh);
    int scq = d > 0.f ? (int)rintf(__fdiv_rn(sub_scale, d)) : 0;
    int mnq = dmin > 0.f ? (int)rintf(__fdiv_rn(sub_min, dmin)) : 0;
    scq = min(63, max(0, scq));
    mnq = min(63, max(0, mnq));
    // gather the 8 scales/mins to every lane
    int sc[8], mnv[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      sc[r] = __shfl_sync(0xffffffffu, scq, r);
      mnv[r] = __shfl_sync(0xffffffffu, mnq, r);
    }
    if (lane == 0) {
      uint16_t dbits = __half_as_ushort(dh), dmbits = __half_as_ushort(dmh);
      o[0] = dbits & 0xFF; o[1] = dbits >> 8; o[2] = dmbits & 0xFF; o[3] = dmbits >> 8;
      for (int g = 0; g < 2; ++g) {
        const int* v = g == 0 ? sc : mnv;
        for (int h = 0; h < 2; ++h) {
          const int* w = v + 4 * h;
          uint8_t* t = o + 4 + 6 * g + 3 * h;
          t[0] = (uint8_t)((w[0] & 0x3F) | ((w[1] & 0x03) << 6));
          t[1] = (uint8_t)(((w[1] >> 2) & 0x0F) | ((w[2] & 0x0F) << 4));
          t[2] = (uint8_t)(((w[2] >> 4) & 0x03) | ((w[3] & 0x3F) << 2));
        }
      }
    }
    // quantize: lane handles element pairs (2i, 2i+1) of sub-block r for i = lane&15, r in {lane>>4, +2, ...}
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int r = 2 * it + (lane >> 4);
      const int i = lane & 15;
      const float ss = __fmul_rn(d, (float)sc[r]);
      const float m = __fmul_rn(dmin, (float)mnv[r]);
      int q0 = 0, q1 = 0;
      if (ss > 0.f) {
        q0 = (int)rintf(__fdiv_rn(__fadd_rn(x[32 * r + 2 * i], m), ss));
        q1 = (int)rintf(__fdiv_rn(__fadd_rn(x[32 * r + 2 * i + 1], m), ss));
      }
      q0 = min(15, max(0, q0));
      q1 = min(15, max(0, q1));
      o[16 + 16 * r + i] = (uint8_t)(q0 | (q1 << 4));
    }
  }
}

// Q6_K quantizer (own; identical arithmetic to or_q6k_quantize), writes the
// reference 210-byte layout.  One warp per block.
__global__ void q6k_quantize_kernel(const float* __restrict__ src, int64_t nblocks, uint8_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t b = warp; b < nblocks; b += nwarps) {
    const float* x = src + b * 256;
    uint8_t* o = out + b * Q6K_BLOCK_BYTES;
    // lane handles elements 8*lane .. 8*lane+7 (sub-block lane/2)
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = x[8 * lane + i];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));  // sub-block = lane pair
    const float sub_scale = __fdiv_rn(amax, 31.f);
    const float ms = warp_max(sub_scale);
    const __half dh = __float2half_rn(__fdiv_rn(ms, 127.f));
    const float d = __half2float(dh);
    int s = d > 0.f ? (int)rintf(__fdiv_rn(sub_scale, d)) : 0;
    s = min(127, max(-128, s));
    const float ss = __fmul_rn(d, (float)s);
    int q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int qq = ss > 0.f ? (int)rintf(__fdiv_rn(v[i], ss)) + 32 : 32;
      q[i] = min(63, max(0, qq));
    }
    // ql bytes 4*lane .. 4*lane+3 ; qh bytes 2*lane, 2*lane+1
#pragma unroll
    for (int i = 0; i < 4; ++i) o[4 * lane + i] = (uint8_t)((q[2 * i] & 0xF) | ((q[2 * i + 1] & 0xF) << 4));
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint8_t h = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) h |= (uint8_t)(((q[4 * i + e] >> 4) & 3) << (2 * e));
      o[128 + 2 * lane + i] = h;
    }
    if ((lane & 1) == 0) o[192 + lane / 2] = (uint8_t)(int8_t)s;
    if (lane == 0) {
      uint16_t db = __half_as_ushort(dh);
      o[208] = db & 0xFF;
      o[209] = db >> 8;
    }
  }
}

inline int grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  return (int)std::min<int64_t>(std::max<int64_t>(g, 1), 148 * 32);
}

}  // namespace

__global__ void dequant_q41_q50_kernel(DevWeight w, float* __restrict__ out) {
  const int64_t nb = (w.n + 31) / 32;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < w.n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = q41_q50_weight(w.scheme, w.data, w.aux, w.aux_bpr, w.aux_stride, nb, i);
}

int launch_dequant(const DevWeight& w, float* out, cudaStream_t st) {
  switch (w.scheme) {
    case SM_Q4_1:
    case SM_Q5_0:
      dequant_q41_q50_kernel<<<grid_for(w.n, 256), 256, 0, st>>>(w, out);
      break;
    case SM_Q8_0:
      dequant_q8_kernel<<<grid_for(w.n, 256), 256, 0, st>>>((const int8_t*)w.data, (const float*)w.aux, w.n,
                                                             w.block_size, w.aux_bpr, w.aux_stride, out);
      break;
    case SM_Q4_0:
      dequant_q4_kernel<<<grid_for(w.n, 256), 256, 0, st>>>((const uint8_t*)w.data, (const float*)w.aux, w.n,
                                                             w.block_size, w.aux_bpr, w.aux_stride, out);
      break;
    case SM_Q4_K:
      dequant_q4k_kernel<<<grid_for(w.n / 256, 1), 128, 0, st>>>((const uint8_t*)w.data, w.n / 256, out);
      break;
    case SM_Q6_K:
      dequant_q6k_kernel<<<grid_for(w.n / 256, 1), 256, 0, st>>>((const uint8_t*)w.data, (const uint16_t*)w.aux,
                                                                  w.n / 256, w.aux_bpr, w.aux_stride, out);
      break;
    case SM_F32:
      dequant_f32_kernel<<<grid_for(w.n, 256), 256, 0, st>>>((const float*)w.data, w.n, out);
      break;
    default:
      return fail(SM_ERR_UNSUPPORTED, "dequant: unsupported scheme");
  }
  SM_CUDA_TRY(cudaGetLastError());
  return SM_OK;
}

int launch_q6k_relayout(const uint8_t* src, uint8_t* body, uint16_t* d, int64_t nblocks, int bpr, int stride,
                        cudaStream_t st) {
  q6k_relayout_kernel<<<grid_for(nblocks, 1), 64, 0, st>>>(src, body, d, nblocks, bpr, stride);
  SM_CUDA_TRY(cudaGetLastError());
  return SM_OK;
}

int launch_quantize(int scheme, const float* src, int64_t n, int bs, void* data, float* scales, cudaStream_t st) {
  if (n <= 0) return fail(SM_ERR_SHAPE, "quantize: n must be positive");
  if (scheme == SM_Q8_0 || scheme == SM_Q4_0) {
    if (bs <= 0) return fail(SM_ERR_INVALID_ARG, "quantize: block size must be positive");
    const int64_t nb = (n + bs - 1) / bs;
    float* inv = nullptr;
    SM_CUDA_TRY(cudaMallocAsync((void**)&inv, sizeof(float) * nb, st));
    block_scales_kernel<<<grid_for(nb * 32, 256), 256, 0, st>>>(src, n, bs, scheme == SM_Q8_0 ? 127.f : 7.f, scales,
                                                                 inv, nb);
    if (scheme == SM_Q8_0)
      q8_pack_kernel<<<grid_for(n, 256), 256, 0, st>>>(src, n, bs, inv, (int8_t*)data);
    else
      q4_pack_kernel<<<grid_for((n + 1) / 2, 256), 256, 0, st>>>(src, n, bs, inv, (uint8_t*)data);
    SM_CUDA_TRY(cudaGetLastError());
    SM_CUDA_TRY(cudaFreeAsync(inv, st));
    return SM_OK;
  }
  if (scheme == SM_Q4_K || scheme == SM_Q6_K) {
    if (n % 256) return fail(SM_ERR_SHAPE, "quantize: K-quant element count must be a multiple of 256");
    const int64_t nb = n / 256;
    if (scheme == SM_Q4_K)
      q4k_quantize_kernel<<<grid_for(nb * 32, 256), 256, 0, st>>>(src, nb, (uint8_t*)data);
    else
      q6k_quantize_kernel<<<grid_for(nb * 32, 256), 256, 0, st>>>(src, nb, (uint8_t*)data);
    SM_CUDA_TRY(cudaGetLastError());
    return SM_OK;
  }
  return fail(SM_ERR_UNSUPPORTED, "quantize: unsupported scheme");
}

}  // namespace sm
