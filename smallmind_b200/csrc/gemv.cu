// Fused dequant-GEMV (decode, M <= 8 per pass) on CUDA cores.
//
// INTENDED layout (y = x . W^T, W[N][K], blocks along K): one warp computes
// ROWS output rows at a time; each lane owns 32-element "units" of K (a Q4_K
// sub-block, two Q6_K sub-blocks, one 32-weight Q8_0/Q4_0 run), loads the
// unit's packed bytes with 128-bit loads, decodes them in registers with the
// reference element formula (sc*q - m, separately rounded) and FMAs against
// the activations staged once per CTA in shared memory.  Partial sums are
// combined with warp shuffles.
//
// REFERENCE layout (C = A . B, B[K][N]): the orientation the reference kernels
// are written in (MatMulF32Q8.cs:61-79, FusedQ4KMatMul.cs:122,127).  Kept for
// op-level parity; one thread per output column.
#include <cstdlib>

#include "common.cuh"
#include "gemv1.cuh"

namespace sm {
namespace {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int ROWS = 2;

// x staged as xs[m][k'] with k' = k ^ (((k >> 5) & 7) << 2): the 16-byte
// chunk index inside a 32-float unit is XORed with the unit index, so the 8
// lanes of a quarter-warp reading chunk j of 8 consecutive units hit 8
// different bank groups.
__device__ __forceinline__ int swz(int k) { return k ^ (((k >> 5) & 7) << 2); }

struct UnitW {
  float w[32];
};

template <int FMT>
struct Decoder;

// Q8_0: w = q * scale (Q8Tensor.cs:151); unit scale = scales[(row*K + 32u) / bs].
template <>
struct Decoder<SM_Q8_0> {
  __device__ __forceinline__ static void decode(const DevWeight& W, int row, int u, int K, bool literal_kq, int N,
                                                UnitW& o) {
    const int8_t* q = (const int8_t*)W.data + (int64_t)row * K + 32 * u;
    const float sc = ((const float*)W.aux)[aux_idx(((int64_t)row * K + 32 * u) / W.block_size, W.aux_bpr, W.aux_stride)];
    int4 a = __ldg((const int4*)q), b = __ldg((const int4*)q + 1);
    const int v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) o.w[4 * i + e] = __fmul_rn((float)(int8_t)(v[i] >> (8 * e)), sc);
  }
};

// Q4_0: nibble by global index, even -> low (Q4Tensor.cs:119-129), w = q * scale.
template <>
struct Decoder<SM_Q4_0> {
  __device__ __forceinline__ static void decode(const DevWeight& W, int row, int u, int K, bool, int, UnitW& o) {
    const int64_t e0 = (int64_t)row * K + 32 * u;
    const uint8_t* q = (const uint8_t*)W.data + e0 / 2;
    const float sc = ((const float*)W.aux)[aux_idx(e0 / W.block_size, W.aux_bpr, W.aux_stride)];
    int4 a = __ldg((const int4*)q);
    const int v[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        int nib = (v[i] >> (4 * e)) & 0xF;
        o.w[8 * i + e] = __fmul_rn((float)(nib < 8 ? nib : nib - 16), sc);
      }
  }
};

// Q4_1 / Q5_0 (block 32 = one unit): Q4_1Tensor.cs:153-156 (q * scale + min),
// Q5_0Tensor.cs:157-172 ((low | high << 4) - 16, times scale); nibbles by global index.
template <int FMT>
struct Decoder41_50 {
  __device__ __forceinline__ static void decode(const DevWeight& W, int row, int u, int K, bool, int, UnitW& o) {
    const int64_t e0 = (int64_t)row * K + 32 * u;
    const int64_t b = e0 >> 5, nb = (W.n + 31) / 32;
    const int4 a = __ldg((const int4*)((const uint8_t*)W.data + e0 / 2));
    const float* af = (const float*)W.aux;
    const float sc = af[aux_idx(b, W.aux_bpr, W.aux_stride)];
    const int64_t i2 = aux_second_idx(b, W.aux_bpr, W.aux_stride, nb);
    const int v[4] = {a.x, a.y, a.z, a.w};
    if (FMT == SM_Q4_1) {
      const float mn = af[i2];
#pragma unroll
      for (int e = 0; e < 32; ++e) o.w[e] = __fadd_rn(__fmul_rn((float)((v[e >> 3] >> (4 * (e & 7))) & 0xF), sc), mn);
    } else {
      const uint32_t hb = ((const uint32_t*)W.aux)[i2];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int q = (((v[e >> 3] >> (4 * (e & 7))) & 0xF) | (int)(((hb >> e) & 1u) << 4)) - 16;
        o.w[e] = __fmul_rn((float)q, sc);
      }
    }
  }
};
template <>
struct Decoder<SM_Q4_1> : Decoder41_50<SM_Q4_1> {};
template <>
struct Decoder<SM_Q5_0> : Decoder41_50<SM_Q5_0> {};

__device__ __forceinline__ int64_t kq_block(int row, int kb, int K, int N, bool literal) {
  return literal ? (int64_t)kb * N + row : (int64_t)row * (K / 256) + kb;
}

// Q4_K: Q4KTensor.cs:129-147, unit u = sub-block (u & 7) of K-block (u >> 3).
template <>
struct Decoder<SM_Q4_K> {
  __device__ __forceinline__ static void decode(const DevWeight& W, int row, int u, int K, bool literal, int N,
                                                UnitW& o) {
    const uint8_t* blk = (const uint8_t*)W.data + kq_block(row, u >> 3, K, N, literal) * Q4K_BLOCK_BYTES;
    const int j = u & 7;
    int4 hdr = __ldg((const int4*)blk);
    int4 qs = __ldg((const int4*)(blk + 16 + 16 * j));
    const uint8_t* hb = (const uint8_t*)&hdr;
    const float d = half_bits_to_float((uint16_t)(hb[0] | (hb[1] << 8)));
    const float dmin = half_bits_to_float((uint16_t)(hb[2] | (hb[3] << 8)));
    int sc, mn;
    unpack_q4k_scales(hb + 4, j, sc, mn);
    const float s = __fmul_rn(d, (float)sc), m = __fmul_rn(dmin, (float)mn);
    const int v[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int bt = 0; bt < 4; ++bt) {
        const int p = (v[i] >> (8 * bt)) & 0xFF;
        o.w[8 * i + 2 * bt] = __fsub_rn(__fmul_rn(s, (float)(p & 0xF)), m);
        o.w[8 * i + 2 * bt + 1] = __fsub_rn(__fmul_rn(s, (float)(p >> 4)), m);
      }
  }
};

// Q6_K (device body layout): Q6KTensor.cs:99-125, unit u covers sub-blocks
// 2j, 2j+1 of K-block (u >> 3), j = u & 7.
template <>
struct Decoder<SM_Q6_K> {
  __device__ __forceinline__ static void decode(const DevWeight& W, int row, int u, int K, bool literal, int N,
                                                UnitW& o) {
    const int64_t b = kq_block(row, u >> 3, K, N, literal);
    const uint8_t* blk = (const uint8_t*)W.data + b * Q6K_BODY_BYTES;
    const int j = u & 7;
    const float d = half_bits_to_float(((const uint16_t*)W.aux)[aux_idx(b, W.aux_bpr, W.aux_stride)]);
    int4 ql = __ldg((const int4*)(blk + 16 * j));
    int2 qh = __ldg((const int2*)(blk + 128 + 8 * j));
    const unsigned short sc2 = __ldg((const unsigned short*)(blk + 192 + 2 * j));
    const float s0 = __fmul_rn(d, (float)(int8_t)(sc2 & 0xFF));
    const float s1 = __fmul_rn(d, (float)(int8_t)(sc2 >> 8));
    const int lq[4] = {ql.x, ql.y, ql.z, ql.w};
    const int hq[2] = {qh.x, qh.y};
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const int low4 = (lq[e >> 3] >> (4 * (e & 7))) & 0xF;
      const int ee = e & 15;  // re-packed high plane (q6k_relayout_kernel)
      const int high2 = (hq[e >> 4] >> (8 * ((ee & 7) >> 1) + ((ee >> 3) << 2) + ((ee & 1) << 1))) & 3;
      const int q = low4 | (high2 << 4);
      o.w[e] = __fmul_rn(e < 16 ? s0 : s1, (float)(q - 32));
    }
  }
};

template <>
struct Decoder<SM_F32> {
  __device__ __forceinline__ static void decode(const DevWeight& W, int row, int u, int K, bool, int, UnitW& o) {
    const float4* p = (const float4*)((const float*)W.data + (int64_t)row * K + 32 * u);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 t = __ldg(p + i);
      o.w[4 * i] = t.x; o.w[4 * i + 1] = t.y; o.w[4 * i + 2] = t.z; o.w[4 * i + 3] = t.w;
    }
  }
};

template <int FMT, int MB>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_rows_kernel(DevWeight W, const float* __restrict__ x, int ldx,
                                                                 float* __restrict__ y, int ldy, int K, int N,
                                                                 int accumulate, int literal) {
  extern __shared__ float xs[];  // [MB][K] swizzled
  for (int i = threadIdx.x; i < MB * K; i += GEMV_THREADS) {
    const int m = i / K, k = i - m * K;
    xs[m * K + swz(k)] = x[(int64_t)m * ldx + k];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int units = K / 32;
  const int ngroups = (N + ROWS - 1) / ROWS;
  for (int g = blockIdx.x * GEMV_WARPS + warp; g < ngroups; g += gridDim.x * GEMV_WARPS) {
    float acc[ROWS][MB];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int m = 0; m < MB; ++m) acc[r][m] = 0.f;
    for (int u = lane; u < units; u += 32) {
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int row = g * ROWS + r;
        if (row >= N) break;
        UnitW w;
        Decoder<FMT>::decode(W, row, u, K, literal != 0, N, w);
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          const float* xr = xs + m * K + 32 * u;
          float a = acc[r][m];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 xv = *(const float4*)(xr + 4 * (c ^ (u & 7)));
            a = fmaf(w.w[4 * c], xv.x, a);
            a = fmaf(w.w[4 * c + 1], xv.y, a);
            a = fmaf(w.w[4 * c + 2], xv.z, a);
            a = fmaf(w.w[4 * c + 3], xv.w, a);
          }
          acc[r][m] = a;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int row = g * ROWS + r;
#pragma unroll
      for (int m = 0; m < MB; ++m) {
        float v = warp_sum(acc[r][m]);
        if (lane == 0 && row < N) {
          float* dst = y + (int64_t)m * ldy + row;
          *dst = accumulate ? *dst + v : v;
        }
      }
    }
  }
}

// Generic element-wise path: any block size / shape (tiny shapes of the
// reference tests).  One thread per output; w(n, k) from the linear index.
__device__ __forceinline__ float elem_weight(const DevWeight& W, int64_t li) {
  switch (W.scheme) {
    case SM_Q8_0:
      return __fmul_rn((float)((const int8_t*)W.data)[li], ((const float*)W.aux)[aux_idx(li / W.block_size, W.aux_bpr, W.aux_stride)]);
    case SM_Q4_0: {
      const uint8_t p = ((const uint8_t*)W.data)[li >> 1];
      const int nib = (li & 1) ? (p >> 4) : (p & 0xF);
      return __fmul_rn((float)(nib < 8 ? nib : nib - 16), ((const float*)W.aux)[aux_idx(li / W.block_size, W.aux_bpr, W.aux_stride)]);
    }
    case SM_Q4_1:
    case SM_Q5_0:
      return q41_q50_weight(W.scheme, W.data, W.aux, W.aux_bpr, W.aux_stride, (W.n + 31) / 32, li);
    default:
      return ((const float*)W.data)[li];
  }
}

// REFERENCE-layout Q8_0/Q4_0/F32: C[m][n] = sum_k (a[m][k] * q[k][n]) * scale
// (MatMulF32Q8.cs:77: c[col] += aVal * quantVal * scale), k ascending.
__global__ void matmul_literal_linear_kernel(DevWeight W, const float* __restrict__ x, int ldx, float* __restrict__ y,
                                             int ldy, int M, int K, int N, int accumulate) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= N || m >= M) return;
  float acc = 0.f;
  for (int k = 0; k < K; ++k) {
    const float a = x[(int64_t)m * ldx + k];
    if (a == 0.f) continue;
    const int64_t li = (int64_t)k * N + n;
    float q, sc;
    if (W.scheme == SM_Q8_0) {
      q = (float)((const int8_t*)W.data)[li];
      sc = ((const float*)W.aux)[aux_idx(li / W.block_size, W.aux_bpr, W.aux_stride)];
    } else if (W.scheme == SM_Q4_0) {
      const uint8_t p = ((const uint8_t*)W.data)[li >> 1];
      const int nib = (li & 1) ? (p >> 4) : (p & 0xF);
      q = (float)(nib < 8 ? nib : nib - 16);
      sc = ((const float*)W.aux)[aux_idx(li / W.block_size, W.aux_bpr, W.aux_stride)];
    } else if (W.scheme == SM_Q4_1 || W.scheme == SM_Q5_0) {
      // FusedQ4_1MatMul.cs:380-383 / FusedQ5_0MatMul.cs:421-424: C += aik * bkj, bkj dequantized
      acc = __fadd_rn(acc, __fmul_rn(a, elem_weight(W, li)));
      continue;
    } else {
      q = ((const float*)W.data)[li];
      sc = 1.f;
    }
    acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(a, q), sc));
  }
  float* dst = y + (int64_t)m * ldy + n;
  *dst = accumulate ? *dst + acc : acc;
}

// INTENDED layout, block size not a multiple of 32 (or K % 32 != 0).
__global__ void matmul_intended_generic_kernel(DevWeight W, const float* __restrict__ x, int ldx,
                                               float* __restrict__ y, int ldy, int M, int K, int N, int accumulate) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= N || m >= M) return;
  float acc = 0.f;
  for (int k = 0; k < K; ++k) acc = fmaf(x[(int64_t)m * ldx + k], elem_weight(W, (int64_t)n * K + k), acc);
  float* dst = y + (int64_t)m * ldy + n;
  *dst = accumulate ? *dst + acc : acc;
}

template <int FMT>
int launch_rows(const DevWeight& W, const float* x, float* y, int M, int ldy, int accumulate, cudaStream_t st,
                int* n_launch) {
  const int K = W.K(), N = W.N();
  const bool literal = W.layout == SM_LAYOUT_REFERENCE;
  int done = 0;
  while (done < M) {
    int mb = M - done >= 8 ? 8 : (M - done >= 4 ? 4 : (M - done >= 2 ? 2 : 1));
    while (mb > 1 && (size_t)mb * K * 4 > 200 * 1024) mb >>= 1;
    const size_t smem = (size_t)mb * K * sizeof(float);
    if (smem > 220 * 1024) return fail(SM_ERR_UNSUPPORTED, "matmul: K too large for the staged GEMV");
    const int ngroups = (N + ROWS - 1) / ROWS;
    const int grid = std::max(1, std::min(ceil_div(ngroups, GEMV_WARPS), 148 * 8));
    const float* xp = x + (int64_t)done * K;
    float* yp = y + (int64_t)done * ldy;
#define SM_LAUNCH_MB(MBV)                                                                                  \
  case MBV: {                                                                                              \
    auto kern = gemv_rows_kernel<FMT, MBV>;                                                                \
    SM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));       \
    kern<<<grid, GEMV_THREADS, smem, st>>>(W, xp, K, yp, ldy, K, N, accumulate, literal ? 1 : 0);           \
    break;                                                                                                 \
  }
    switch (mb) {
      SM_LAUNCH_MB(1)
      SM_LAUNCH_MB(2)
      SM_LAUNCH_MB(4)
      SM_LAUNCH_MB(8)
    }
#undef SM_LAUNCH_MB
    SM_CUDA_TRY(cudaGetLastError());
    if (n_launch) ++*n_launch;
    done += mb;
  }
  return SM_OK;
}

}  // namespace

int launch_matmul(const DevWeight& W, const float* x, float* y, int M, int ldy, int accumulate, cudaStream_t st,
                  int* n_launch) {
  const int K = W.K(), N = W.N();
  const bool kq = W.scheme == SM_Q4_K || W.scheme == SM_Q6_K;
  const bool literal = W.layout == SM_LAYOUT_REFERENCE;
  if (!kq && literal) {
    dim3 grid(ceil_div(N, 128), M);
    matmul_literal_linear_kernel<<<grid, 128, 0, st>>>(W, x, K, y, ldy, M, K, N, accumulate);
    SM_CUDA_TRY(cudaGetLastError());
    if (n_launch) ++*n_launch;
    return SM_OK;
  }
  if (M == 1 && gemv1_supports(W, K)) {
    GemvArgs a;
    a.K = K;
    a.x = x;
    SM_TRY(gemv1_segment(a, W, nullptr, y, accumulate ? GEMV_ADD : GEMV_STORE));
    // Q4_K / Q6_K: integer tensor-core GEMV (SMALLMIND_GEMV_MMA=0 selects the CUDA-core kernel)
    const char* em = std::getenv("SMALLMIND_GEMV_MMA");
    if (!(em && em[0] == '0') && W.scheme == SM_Q4_K) {
      const int rc = launch_gemv_mma_q4k(W, x, y, accumulate, nullptr, st, n_launch);
      if (rc != SM_ERR_UNSUPPORTED) return rc;
    }
    if (!(em && em[0] == '0') && W.scheme == SM_Q6_K) {
      const int rc = launch_gemv_mma_q6k(W, x, y, accumulate, nullptr, st, n_launch);
      if (rc != SM_ERR_UNSUPPORTED) return rc;
    }
    if (!(em && em[0] == '0') && (W.scheme == SM_Q8_0 || W.scheme == SM_Q4_0)) {
      const int rc = launch_gemv_mma_q80(W, x, y, accumulate, nullptr, st, n_launch);
      if (rc != SM_ERR_UNSUPPORTED) return rc;
    }
    return launch_gemv1(a, st, n_launch);
  }
  {
    // 2 <= M <= 4, Q4_K / Q6_K: the integer tensor-core GEMV, all x rows in one pass over the
    // packed weights (more rows would take several passes: the tcgen05 GEMM is faster there)
    const char* em = std::getenv("SMALLMIND_GEMV_MMA");
    if (!(em && em[0] == '0') && W.scheme == SM_Q4_K && M > 1 && M <= 4) {
      const int rc = launch_gemv_mma_q4k_rows(W, x, M, y, ldy, accumulate, nullptr, st, n_launch);
      if (rc != SM_ERR_UNSUPPORTED) return rc;
    }
    if (!(em && em[0] == '0') && W.scheme == SM_Q6_K && M > 1 && M <= 4) {
      const int rc = launch_gemv_mma_q6k_rows(W, x, M, y, ldy, accumulate, nullptr, st, n_launch);
      if (rc != SM_ERR_UNSUPPORTED) return rc;
    }
  }
  {
    // M >= 5: tcgen05 GEMM (SMALLMIND_GEMM_TC=0 selects the CUDA-core row kernel)
    const char* et = std::getenv("SMALLMIND_GEMM_TC");
    if (!(et && et[0] == '0') && gemm_tc_supports(W, M)) {
      const int rc = launch_gemm_tc(W, x, y, M, ldy, accumulate, nullptr, st, n_launch);
      if (rc != SM_ERR_UNSUPPORTED) return rc;
    }
  }
  const bool fast = kq || (K % 32 == 0 && (W.scheme == SM_F32 || W.block_size % 32 == 0));
  if (!fast) {
    dim3 grid(ceil_div(N, 128), M);
    matmul_intended_generic_kernel<<<grid, 128, 0, st>>>(W, x, K, y, ldy, M, K, N, accumulate);
    SM_CUDA_TRY(cudaGetLastError());
    if (n_launch) ++*n_launch;
    return SM_OK;
  }
  switch (W.scheme) {
    case SM_Q8_0: return launch_rows<SM_Q8_0>(W, x, y, M, ldy, accumulate, st, n_launch);
    case SM_Q4_0: return launch_rows<SM_Q4_0>(W, x, y, M, ldy, accumulate, st, n_launch);
    case SM_Q4_1: return launch_rows<SM_Q4_1>(W, x, y, M, ldy, accumulate, st, n_launch);
    case SM_Q5_0: return launch_rows<SM_Q5_0>(W, x, y, M, ldy, accumulate, st, n_launch);
    case SM_Q4_K: return launch_rows<SM_Q4_K>(W, x, y, M, ldy, accumulate, st, n_launch);
    case SM_Q6_K: return launch_rows<SM_Q6_K>(W, x, y, M, ldy, accumulate, st, n_launch);
    case SM_F32: return launch_rows<SM_F32>(W, x, y, M, ldy, accumulate, st, n_launch);
  }
  return fail(SM_ERR_UNSUPPORTED, "matmul: unsupported scheme");
}

}  // namespace sm
