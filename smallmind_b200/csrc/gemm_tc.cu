// Prefill / batched GEMM y[M][N] (+)= x[M][K] W[N][K]^T on the tcgen05 tensor
// cores, for every quantized weight format (INTENDED layout).
//
// Precision.  The weight of element (n, k) is the exact fp32 value of the
// reference element formula (Q8Tensor.cs:151, Q4Tensor.cs:150-179,
// Q4KTensor.cs:129-147, Q6KTensor.cs:105-124).  Both operands are split into
// fp16 pairs, v = hi + lo with hi = fp16(v), lo = fp16(v - hi) (22 significant
// bits), and each 16-wide k step issues three kind::f16 MMAs into one fp32 TMEM
// accumulator: x_hi w_hi + x_hi w_lo + x_lo w_hi.  The dropped x_lo w_lo term
// and the residuals are ~2^-22 relative, far inside the 1e-4 tolerance.
// (|x| must stay below the fp16 range, 65504.)
//
// Structure (one 128 x 128 output tile per CTA, 320 threads):
//   * x is split once into fp16 hi / lo planes (gemm_split_kernel) and each
//     128 x 64 tile of both planes is brought in by TMA with the 128-byte
//     swizzle (warp 8, one elected lane; no multicast);
//   * warps 0..7 dequantize the 128 x 64 weight tile (thread = row, 32 k) to
//     the same swizzled K-major layout, hi and lo planes;
//   * warp 9, one lane, issues 4 k-steps x 3 tcgen05.mma per stage and
//     commits each stage back to its producers through an mbarrier;
//   * warps 0..3 read the accumulator from TMEM (tcgen05.ld 32x32b) and store y.
// Every mbarrier wait is bounded (SM_ERR_TIMEOUT in *status), and the TMEM
// columns are always released before the CTA exits.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "gemv1.cuh"
#include "mbar.cuh"

namespace sm {
namespace {

constexpr int BM = 128;  // x rows per tile (MMA M)
constexpr int BN = 128;  // weight rows per tile (MMA N)
constexpr int BK = 64;   // k per stage: one 128-byte swizzle atom of fp16
// warp roles: WT = false (weights dequantized in the kernel): warps 0..7 load
// weight tiles, 8 = TMA, 9 = MMA; WT = true (weights pre-split into fp16
// planes and loaded by TMA): 4 = TMA, 5 = MMA.  Warps 0..3 run the epilogue.
template <bool WT>
struct Roles {
  static constexpr int LOADER_WARPS = WT ? 0 : 8;
  static constexpr int TMA_WARP = WT ? 4 : 8;
  static constexpr int THREADS = (TMA_WARP + 2) * 32;
};
constexpr int TILE_A = BM * BK * 2;  // bytes of one fp16 plane of the x tile
// Tile geometry per weight-tile width NB (the MMA N): 128, or 256 for GEMMs with
// several x-row tiles whose weights come as resident planes.  A 256-wide tile reads
// A and B from shared memory once per twice the MACs of a 128-wide one; it leaves
// room for 2 stages instead of 3.
template <int NB>
struct Geo {
  static constexpr int TILE_W = NB * BK * 2;
  static constexpr int STAGE_BYTES = 2 * TILE_A + 2 * TILE_W;
  static constexpr int STAGES = NB == 256 ? 2 : 3;
  static constexpr int TMEM_COLS = NB;  // fp32 accumulator: 128 lanes x NB columns
  static constexpr size_t SMEM_BYTES = (size_t)STAGES * STAGE_BYTES + 1024 + 256;
};
constexpr size_t SMEM_BYTES = Geo<BN>::SMEM_BYTES;

constexpr int MAX_SEG = 3;

// Up to three weights with the same K, stacked along N (Q|K|V, gate|up); each
// segment but the last spans whole 128-row tiles and has its own output.
struct TcArgs {
  DevWeight W[MAX_SEG];
  int nseg;
  int seg_n0[MAX_SEG + 1];  // prefix sums of the segments' N
  float* seg_y[MAX_SEG];
  int seg_ldy[MAX_SEG];
  int M, N, K;              // N = total over the segments
  int accumulate;
  int* status;
  int kslices;      // split-K: blockIdx.z takes stages [z nk / kslices, (z+1) nk / kslices)
  float* partial;   // kslices > 1: [kslices][M][N] partial sums (reduced by gemm_reduce_kernel)
};

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand in the canonical 128-byte-swizzle layout: rows of 128 B,
// 8-row atoms of 1024 B (stride byte offset), version 1, layout type 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, both
// K-major, N = BN, M = BM.
template <int NB>
constexpr uint32_t idesc() { return (1u << 4) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(BM >> 4) << 24); }

template <int NB = BN>
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc<NB>()), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 columns of this warp's 32 TMEM lanes, without waiting (tmem_wait_ld completes them)
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Packed bytes of one unit, loaded ahead of their decode (register prefetch).
// Q4_K: a = block header, b = the unit's 16 code bytes.  Q6_K: a = ql, b.xy =
// high plane words, b.z = the two int8 scales, b.w = d bits.  Q8_0: a, b = 32
// codes, s = scale.  Q4_0: a = 16 code bytes, s = scale.  Q4_1 / Q5_0: a = 16
// code bytes, s = scale, b.x = the block's min (Q4_1) or high-bit word (Q5_0).
struct RawUnit {
  uint4 a, b;
  float s;
};

__device__ __forceinline__ void load_raw41_50(const DevWeight& W, int n, int k0, int K, RawUnit& r) {
  const int64_t i0 = (int64_t)n * K + k0, b = i0 >> 5;
  r.a = __ldg((const uint4*)((const uint8_t*)W.data + (i0 >> 1)));
  r.s = __ldg((const float*)W.aux + aux_idx(b, W.aux_bpr, W.aux_stride));
  r.b.x = __ldg((const uint32_t*)W.aux + aux_second_idx(b, W.aux_bpr, W.aux_stride, (W.n + 31) / 32));
}

// Q4_1Tensor.cs:153-156 (q * scale + min) and Q5_0Tensor.cs:157-172 ((low | high << 4) - 16, times scale)
__device__ __forceinline__ void decode_raw41_50(int scheme, const RawUnit& r, float (&w)[32]) {
  const uint32_t qw[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const uint32_t b = (qw[e >> 3] >> (8 * ((e >> 1) & 3))) & 0xFF;
    const int nib = (e & 1) ? (int)(b >> 4) : (int)(b & 0xF);
    if (scheme == SM_Q4_1)
      w[e] = __fadd_rn(__fmul_rn((float)nib, r.s), __uint_as_float(r.b.x));
    else
      w[e] = __fmul_rn((float)((nib | (int)(((r.b.x >> e) & 1u) << 4)) - 16), r.s);
  }
}

// ---------------------------------------------------------------- weight unit -> 32 fp32 values
// Elements k0 .. k0 + 31 (k0 % 32 == 0) of weight row n, exactly as the
// reference element formulas produce them.
__device__ __forceinline__ void weight_unit(const DevWeight& W, int n, int k0, int K, float (&w)[32]) {
  switch (W.scheme) {
    case SM_Q4_K: {
      const int kb = k0 >> 8, j = (k0 >> 5) & 7;
      const uint8_t* blk = (const uint8_t*)W.data + ((int64_t)n * (K >> 8) + kb) * Q4K_BLOCK_BYTES;
      const uint32_t h0 = *(const uint32_t*)blk;
      const float d = half_bits_to_float((uint16_t)(h0 & 0xFFFF)), dmin = half_bits_to_float((uint16_t)(h0 >> 16));
      int sc, mn;
      unpack_q4k_scales(blk + 4, j, sc, mn);
      const float s = __fmul_rn(d, (float)sc), m = __fmul_rn(dmin, (float)mn);
      const uint4 q = *(const uint4*)(blk + 16 + 16 * j);
      const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t b = (qw[i >> 2] >> (8 * (i & 3))) & 0xFF;
        w[2 * i] = __fsub_rn(__fmul_rn(s, (float)(b & 0xF)), m);
        w[2 * i + 1] = __fsub_rn(__fmul_rn(s, (float)(b >> 4)), m);
      }
      break;
    }
    case SM_Q6_K: {
      const int kb = k0 >> 8, j = (k0 >> 5) & 7;
      const int64_t b = (int64_t)n * (K >> 8) + kb;
      const uint8_t* blk = (const uint8_t*)W.data + b * Q6K_BODY_BYTES;
      const float d = half_bits_to_float(((const uint16_t*)W.aux)[aux_idx(b, W.aux_bpr, W.aux_stride)]);
      const float s0 = __fmul_rn(d, (float)(int8_t)blk[192 + 2 * j]);
      const float s1 = __fmul_rn(d, (float)(int8_t)blk[192 + 2 * j + 1]);
      const uint4 ql = *(const uint4*)(blk + 16 * j);
      const uint32_t qlw[4] = {ql.x, ql.y, ql.z, ql.w};
      // re-packed high plane: word t covers elements 16t .. 16t+15; byte bb holds
      // the highs of 16t+2bb, 16t+2bb+1 (bits 0-3) and 16t+8+2bb, 16t+9+2bb (bits 4-7)
      const uint2 qh = *(const uint2*)(blk + 128 + 8 * j);
      const uint32_t qhw[2] = {qh.x, qh.y};
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const uint32_t lb = (qlw[e >> 3] >> (8 * ((e >> 1) & 3))) & 0xFF;
        const int low4 = (e & 1) ? (int)(lb >> 4) : (int)(lb & 0xF);
        const int t = e >> 4, ee = e & 15;
        const int bb = (ee & 7) >> 1, sh = ((ee >> 3) << 2) + ((ee & 1) << 1);
        const int high2 = (int)((qhw[t] >> (8 * bb + sh)) & 3);
        w[e] = __fmul_rn(e < 16 ? s0 : s1, (float)((low4 | (high2 << 4)) - 32));
      }
      break;
    }
    case SM_Q8_0: {
      const int64_t i0 = (int64_t)n * K + k0;
      const int4* src = (const int4*)((const int8_t*)W.data + i0);
      const int4 v0 = src[0], v1 = src[1];
      const int vw[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      const float* sc = (const float*)W.aux;
      const bool one = W.block_size % 32 == 0;  // one scale block covers the unit
      const float s1 = sc[aux_idx(i0 / W.block_size, W.aux_bpr, W.aux_stride)];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float s = one ? s1 : sc[aux_idx((i0 + e) / W.block_size, W.aux_bpr, W.aux_stride)];
        w[e] = __fmul_rn((float)(int8_t)((vw[e >> 2] >> (8 * (e & 3))) & 0xFF), s);
      }
      break;
    }
    case SM_Q4_0: {
      const int64_t i0 = (int64_t)n * K + k0;  // even
      const uint4 q = *(const uint4*)((const uint8_t*)W.data + (i0 >> 1));
      const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
      const float* sc = (const float*)W.aux;
      const bool one = W.block_size % 32 == 0;
      const float s1 = sc[aux_idx(i0 / W.block_size, W.aux_bpr, W.aux_stride)];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const uint32_t b = (qw[e >> 3] >> (8 * ((e >> 1) & 3))) & 0xFF;
        const int nib = (e & 1) ? (int)(b >> 4) : (int)(b & 0xF);
        const float s = one ? s1 : sc[aux_idx((i0 + e) / W.block_size, W.aux_bpr, W.aux_stride)];
        w[e] = __fmul_rn((float)(nib < 8 ? nib : nib - 16), s);
      }
      break;
    }
    case SM_Q4_1:
    case SM_Q5_0: {
      RawUnit r;
      load_raw41_50(W, n, k0, K, r);
      decode_raw41_50(W.scheme, r, w);
      break;
    }
    default: {  // F32
      const float4* src = (const float4*)((const float*)W.data + (int64_t)n * K + k0);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 v = src[c];
        w[4 * c] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
      }
    }
  }
}

__device__ __forceinline__ bool raw_prefetchable(const DevWeight& W) {
  return W.scheme == SM_Q4_K || W.scheme == SM_Q6_K || W.scheme == SM_Q4_1 || W.scheme == SM_Q5_0 ||
         ((W.scheme == SM_Q8_0 || W.scheme == SM_Q4_0) && W.block_size % 32 == 0);
}

__device__ __forceinline__ void load_raw(const DevWeight& W, int n, int k0, int K, RawUnit& r) {
  switch (W.scheme) {
    case SM_Q4_K: {
      const uint8_t* blk = (const uint8_t*)W.data + ((int64_t)n * (K >> 8) + (k0 >> 8)) * Q4K_BLOCK_BYTES;
      r.a = __ldg((const uint4*)blk);
      r.b = __ldg((const uint4*)(blk + 16 + 16 * ((k0 >> 5) & 7)));
      break;
    }
    case SM_Q6_K: {
      const int j = (k0 >> 5) & 7;
      const int64_t b = (int64_t)n * (K >> 8) + (k0 >> 8);
      const uint8_t* blk = (const uint8_t*)W.data + b * Q6K_BODY_BYTES;
      r.a = __ldg((const uint4*)(blk + 16 * j));
      const uint2 qh = __ldg((const uint2*)(blk + 128 + 8 * j));
      r.b.x = qh.x;
      r.b.y = qh.y;
      r.b.z = __ldg((const unsigned short*)(blk + 192 + 2 * j));
      r.b.w = __ldg(((const unsigned short*)W.aux) + aux_idx(b, W.aux_bpr, W.aux_stride));
      break;
    }
    case SM_Q8_0: {
      const int64_t i0 = (int64_t)n * K + k0;
      const uint4* src = (const uint4*)((const int8_t*)W.data + i0);
      r.a = __ldg(src);
      r.b = __ldg(src + 1);
      r.s = __ldg((const float*)W.aux + aux_idx(i0 / W.block_size, W.aux_bpr, W.aux_stride));
      break;
    }
    case SM_Q4_1:
    case SM_Q5_0:
      load_raw41_50(W, n, k0, K, r);
      break;
    default: {  // Q4_0
      const int64_t i0 = (int64_t)n * K + k0;
      r.a = __ldg((const uint4*)((const uint8_t*)W.data + (i0 >> 1)));
      r.s = __ldg((const float*)W.aux + aux_idx(i0 / W.block_size, W.aux_bpr, W.aux_stride));
    }
  }
}

// The same element formulas as weight_unit, from prefetched bytes.
__device__ __forceinline__ void decode_raw(int scheme, int k0, const RawUnit& r, float (&w)[32]) {
  switch (scheme) {
    case SM_Q4_K: {
      const float d = half_bits_to_float((uint16_t)(r.a.x & 0xFFFF));
      const float dmin = half_bits_to_float((uint16_t)(r.a.x >> 16));
      // six-bit scale / min j at bits 6j of header bytes 4..9 / 10..15 (Q4KTensor.cs:109-126)
      const int j = (k0 >> 5) & 7;
      const uint64_t sb = (uint64_t)r.a.y | ((uint64_t)(r.a.z & 0xFFFFu) << 32);
      const uint64_t mb = (uint64_t)(r.a.z >> 16) | ((uint64_t)r.a.w << 16);
      const float s = __fmul_rn(d, (float)(int)((sb >> (6 * j)) & 63));
      const float m = __fmul_rn(dmin, (float)(int)((mb >> (6 * j)) & 63));
      const uint32_t qw[4] = {r.b.x, r.b.y, r.b.z, r.b.w};
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t b = (qw[i >> 2] >> (8 * (i & 3))) & 0xFF;
        w[2 * i] = __fsub_rn(__fmul_rn(s, (float)(b & 0xF)), m);
        w[2 * i + 1] = __fsub_rn(__fmul_rn(s, (float)(b >> 4)), m);
      }
      break;
    }
    case SM_Q6_K: {
      const float d = half_bits_to_float((uint16_t)r.b.w);
      const float s0 = __fmul_rn(d, (float)(int8_t)(r.b.z & 0xFF));
      const float s1 = __fmul_rn(d, (float)(int8_t)((r.b.z >> 8) & 0xFF));
      const uint32_t qlw[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
      const uint32_t qhw[2] = {r.b.x, r.b.y};
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const uint32_t lb = (qlw[e >> 3] >> (8 * ((e >> 1) & 3))) & 0xFF;
        const int low4 = (e & 1) ? (int)(lb >> 4) : (int)(lb & 0xF);
        const int t = e >> 4, ee = e & 15;
        const int bb = (ee & 7) >> 1, sh = ((ee >> 3) << 2) + ((ee & 1) << 1);
        const int high2 = (int)((qhw[t] >> (8 * bb + sh)) & 3);
        w[e] = __fmul_rn(e < 16 ? s0 : s1, (float)((low4 | (high2 << 4)) - 32));
      }
      break;
    }
    case SM_Q8_0: {
      const uint32_t vw[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
#pragma unroll
      for (int e = 0; e < 32; ++e) w[e] = __fmul_rn((float)(int8_t)((vw[e >> 2] >> (8 * (e & 3))) & 0xFF), r.s);
      break;
    }
    case SM_Q4_1:
    case SM_Q5_0:
      decode_raw41_50(scheme, r, w);
      break;
    default: {  // Q4_0
      const uint32_t qw[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const uint32_t b = (qw[e >> 3] >> (8 * ((e >> 1) & 3))) & 0xFF;
        const int nib = (e & 1) ? (int)(b >> 4) : (int)(b & 0xF);
        w[e] = __fmul_rn((float)(nib < 8 ? nib : nib - 16), r.s);
      }
    }
  }
}

// byte offset of 16-byte chunk c (8 fp16 along k) of row r in a 128B-swizzled tile
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

template <bool WT, int NB = BN>
__global__ void __launch_bounds__(Roles<WT>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_hi, const __grid_constant__ CUtensorMap tm_lo,
                   const __grid_constant__ CUtensorMap tm_whi, const __grid_constant__ CUtensorMap tm_wlo,
                   const __grid_constant__ TcArgs a) {
  constexpr int LOADER_WARPS = Roles<WT>::LOADER_WARPS;
  constexpr int TMA_WARP = Roles<WT>::TMA_WARP;
  static_assert(WT || NB == BN, "the loader warps fill 128-row weight tiles");
  constexpr int STAGES = Geo<NB>::STAGES;
  constexpr int STAGE_BYTES = Geo<NB>::STAGE_BYTES;
  constexpr int TILE_W = Geo<NB>::TILE_W;
  constexpr int TMEM_COLS = Geo<NB>::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full_a = (uint64_t*)(smem + STAGES * STAGE_BYTES);
  uint64_t* full_w = full_a + STAGES;
  uint64_t* empty = full_w + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = (uint32_t*)(done + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // x-row tiles vary fastest: consecutive CTAs share one weight tile, which then
  // comes from L2 for all the row tiles instead of from DRAM once per row tile
  const int n0 = blockIdx.y * NB, m0 = blockIdx.x * BM;
  const int K = a.K;
  const int nk_all = K / BK;
  const int kt0 = (int)((int64_t)nk_all * blockIdx.z / a.kslices);
  const int nk = (int)((int64_t)nk_all * (blockIdx.z + 1) / a.kslices) - kt0;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&full_w[s], WT ? 1 : LOADER_WARPS * 32);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (!WT && warp < LOADER_WARPS) {
    // ---- weight tiles: thread = (row r, k half h); the packed bytes of the
    // next two stages are in flight while this one is decoded
    const int r = tid & (BN - 1), h = tid >> 7;
    int sg = 0;
    while (sg + 1 < a.nseg && n0 >= a.seg_n0[sg + 1]) ++sg;
    const DevWeight& W = a.W[sg];
    const int n = n0 + r - a.seg_n0[sg];  // row inside the segment's weight
    const bool live = n0 + r < a.seg_n0[sg + 1];
    const bool pf = raw_prefetchable(W);
    RawUnit r0, r1;
    if (pf && live) {
      if (nk > 0) load_raw(W, n, (kt0 + 0) * BK + 32 * h, K, r0);
      if (nk > 1) load_raw(W, n, (kt0 + 1) * BK + 32 * h, K, r1);
    }
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % STAGES;
      const int k0 = (kt0 + kt) * BK + 32 * h;
      float w[32];
      if (!live) {
#pragma unroll
        for (int e = 0; e < 32; ++e) w[e] = 0.f;
      } else if (pf) {
        const RawUnit cur = r0;
        r0 = r1;
        if (kt + 2 < nk) load_raw(W, n, k0 + 2 * BK, K, r1);
        decode_raw(W.scheme, k0, cur, w);
      } else {
        weight_unit(W, n, k0, K, w);
      }
      if (kt >= STAGES && !mbar_wait_bounded(&empty[s], ((kt / STAGES) - 1) & 1, a.status)) break;
      uint8_t* whi = smem + s * STAGE_BYTES + 2 * TILE_A;
      uint8_t* wlo = whi + TILE_W;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t hp[4], lp[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float v0 = w[8 * c + 2 * e], v1 = w[8 * c + 2 * e + 1];
          const __half2 hh = __floats2half2_rn(v0, v1);
          const float2 hf = __half22float2(hh);
          const __half2 ll = __floats2half2_rn(__fsub_rn(v0, hf.x), __fsub_rn(v1, hf.y));
          hp[e] = *(const uint32_t*)&hh;
          lp[e] = *(const uint32_t*)&ll;
        }
        const uint32_t off = sw_off(r, 4 * h + c);
        *(uint4*)(whi + off) = make_uint4(hp[0], hp[1], hp[2], hp[3]);
        *(uint4*)(wlo + off) = make_uint4(lp[0], lp[1], lp[2], lp[3]);
      }
      // generic-proxy stores -> visible to the tensor core (async proxy)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&full_w[s]);
    }
  } else if (warp == TMA_WARP) {
    if (lane == 0) {
      for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % STAGES;
        if (kt >= STAGES && !mbar_wait_bounded(&empty[s], ((kt / STAGES) - 1) & 1, a.status)) break;
        uint8_t* st = smem + s * STAGE_BYTES;
        mbar_expect_tx(&full_a[s], WT ? 2 * TILE_A + 2 * TILE_W : 2 * TILE_A);
        tma_load_2d(st, &tm_hi, (kt0 + kt) * BK, m0, &full_a[s]);
        tma_load_2d(st + TILE_A, &tm_lo, (kt0 + kt) * BK, m0, &full_a[s]);
        if (WT) {
          tma_load_2d(st + 2 * TILE_A, &tm_whi, (kt0 + kt) * BK, n0, &full_a[s]);
          tma_load_2d(st + 2 * TILE_A + TILE_W, &tm_wlo, (kt0 + kt) * BK, n0, &full_a[s]);
        }
      }
    }
  } else if (warp == TMA_WARP + 1) {  // the MMA issuer
    if (lane == 0) {
      bool ok = true;
      for (int kt = 0; kt < nk && ok; ++kt) {
        const int s = kt % STAGES;
        const uint32_t par = (kt / STAGES) & 1;
        ok = mbar_wait_bounded(&full_a[s], par, a.status) && (WT || mbar_wait_bounded(&full_w[s], par, a.status));
        if (!ok) break;
        tc_fence_after();
        const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
        const uint64_t dah = sw128_desc(base), dal = sw128_desc(base + TILE_A);
        const uint64_t dwh = sw128_desc(base + 2 * TILE_A), dwl = sw128_desc(base + 2 * TILE_A + TILE_W);
#pragma unroll
        for (int ks = 0; ks < BK / 16; ++ks) {
          const uint64_t adv = (uint64_t)((ks * 32) >> 4);  // 16 fp16 = 32 bytes along k
          mma_f16<NB>(tmem, dah + adv, dwh + adv, (kt | ks) != 0);
          mma_f16<NB>(tmem, dah + adv, dwl + adv, 1);
          mma_f16<NB>(tmem, dal + adv, dwh + adv, 1);
        }
        mma_commit(&empty[s]);  // stage s may be refilled once these MMAs have read it
      }
      mma_commit(done);
    }
  }

  if (warp < 4) {
    // ---- epilogue: TMEM lanes 32 warp .. 32 warp + 31 = x rows, columns = weight rows
    const bool ok = mbar_wait_bounded(done, 0, a.status);
    tc_fence_after();
    if (ok) {
      const bool part = a.kslices > 1;
      int sg = 0;
      while (sg + 1 < a.nseg && n0 >= a.seg_n0[sg + 1]) ++sg;
      const int nb = a.seg_n0[sg], ne = a.seg_n0[sg + 1];
      // partial sums: [slice][M][N total]; final: the segment's own output, column n - nb
      // The accumulator rows go through shared memory (the stage buffers are free
      // once `done` has fired) so that each store instruction writes one whole
      // 512-byte output row: lane = 4 consecutive columns, not lane = row.
      // Row stride 132 floats: the 8 rows of a quarter-warp's 16-byte writes
      // land in distinct bank groups.
      constexpr int SR = NB + 4;
      float* stile = (float*)smem + warp * 32 * SR;
#pragma unroll 1
      for (int c0 = 0; c0 < NB; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
        float4* d = (float4*)(stile + lane * SR + c0);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          d[e] = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]), __uint_as_float(v[4 * e + 2]),
                             __uint_as_float(v[4 * e + 3]));
      }
      __syncwarp();
      const bool rmw = a.accumulate && !part;
#pragma unroll 1
      for (int cb = 0; cb < NB; cb += 128) {
      const int nc = n0 + cb + 4 * lane;  // this lane's 4 columns
      const bool full = nc + 3 < ne;
#pragma unroll 1
      for (int rr = 0; rr < 32; ++rr) {
        const int mr = m0 + warp * 32 + rr;
        if (mr >= a.M) break;
        float* yrow = part ? a.partial + ((int64_t)blockIdx.z * a.M + mr) * a.N
                           : a.seg_y[sg] + (int64_t)mr * a.seg_ldy[sg] - nb;
        float4 t = *(const float4*)(stile + rr * SR + cb + 4 * lane);
        float* dst = yrow + nc;
        if (full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
          if (rmw) {
            const float4 o = *(const float4*)dst;
            t.x += o.x;
            t.y += o.y;
            t.z += o.z;
            t.w += o.w;
          }
          *(float4*)dst = t;
        } else {
          const float tv[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (nc + e < ne) dst[e] = rmw ? dst[e] + tv[e] : tv[e];
        }
      }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------- two-MMA Q4_K GEMM
// y (+)= sum_b d[n][b] sum_{k in b} (sc q)[n][k] x[m][k]  -  sum_j (dmin m_j)[n] X_j[m]
// where X_j is the sum of x over 32-element sub-block j.  The weight operand sc*q is
// an exact fp16 integer, so each 16-wide k step needs two MMAs (x_hi and x_lo)
// instead of three.  The block scale d changes every 256 k, so each block's
// accumulator is read from TMEM and added into registers times d; two TMEM buffers
// let the MMAs of the next block run meanwhile.  "Virtual block" 0 of k slice 0 is
// the -dmin m term: an fp16 hi / lo GEMM over the x sums (three MMAs per step,
// K = Kp), read back with scale 1.
// Warps 0..EW-1: epilogue (warp w: TMEM lanes 32 (w % 4).., 128 columns from 128 (w / 4)),
// warp EW: TMA, warp EW + 1: MMA issuer.  NB = 256 for GEMMs with several x-row
// tiles (half the L2 traffic per MAC), 128 otherwise (more CTAs to split K over).
template <int NB>
struct Q2 {
  static constexpr int EW = NB / 32;  // epilogue warps
  static constexpr int THREADS = (EW + 2) * 32;
  static constexpr int TILE_Q = NB * BK * 2;
  static constexpr int STAGE_BYTES = 2 * TILE_A + TILE_Q;
  static constexpr int STAGES = NB == 256 ? 3 : 4;
  static constexpr int MAX_NB = 24;  // 256-weight blocks per k slice (K <= 6144)
  static constexpr size_t SMEM_BYTES = (size_t)STAGES * STAGE_BYTES + (size_t)(MAX_NB + 1) * NB * 4 + 1024 + 256;
};
constexpr int Q2_MAX_K = 256 * Q2<256>::MAX_NB;

template <int NB>
__global__ void __launch_bounds__(Q2<NB>::THREADS, 1)
    gemm_q4k2_kernel(const __grid_constant__ CUtensorMap tm_hi, const __grid_constant__ CUtensorMap tm_lo,
                     const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_xh,
                     const __grid_constant__ CUtensorMap tm_xl, const __grid_constant__ CUtensorMap tm_mh,
                     const __grid_constant__ CUtensorMap tm_ml, const float* __restrict__ dv, int Kp,
                     const __grid_constant__ TcArgs a) {
  using G = Q2<NB>;
  constexpr int STAGES = G::STAGES, STAGE_BYTES = G::STAGE_BYTES, TILE_Q = G::TILE_Q, EW = G::EW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* dsm = (float*)(smem + STAGES * STAGE_BYTES);  // [virtual block][NB columns] read-back scales
  uint64_t* full = (uint64_t*)(dsm + (G::MAX_NB + 1) * NB);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint64_t* acce = accf + 2;
  uint32_t* tmem_slot = (uint32_t*)(acce + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.y * NB, m0 = blockIdx.x * BM;
  const int K = a.K, NBall = K >> 8;
  const int b0 = (int)((int64_t)NBall * blockIdx.z / a.kslices);
  const int nbs = (int)((int64_t)NBall * (blockIdx.z + 1) / a.kslices) - b0;
  const int nmin = blockIdx.z == 0 ? 1 : 0;  // virtual block 0: the -dmin m term
  const int nvb = nbs + nmin;
  const int nm = nmin * 2 * (Kp / BK);      // its stages: x sums hi + lo with mh, then hi with ml
  const int nk = nm + 4 * nbs;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], EW);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * NB)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  for (int i = tid; i < nvb * NB; i += G::THREADS) {
    const int vb = i / NB, c = i - vb * NB;
    dsm[i] = vb < nmin ? 1.f : (n0 + c < a.N ? dv[(int64_t)(n0 + c) * NBall + b0 + vb - nmin] : 0.f);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == EW) {
    if (lane == 0) {
      for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % STAGES;
        if (kt >= STAGES && !mbar_wait_bounded(&empty[s], ((kt / STAGES) - 1) & 1, a.status)) break;
        uint8_t* st = smem + s * STAGE_BYTES;
        if (kt < nm) {
          const int kc = (kt >> 1) * BK;
          if ((kt & 1) == 0) {
            mbar_expect_tx(&full[s], 2 * TILE_A + TILE_Q);
            tma_load_2d(st, &tm_xh, kc, m0, &full[s]);
            tma_load_2d(st + TILE_A, &tm_xl, kc, m0, &full[s]);
            tma_load_2d(st + 2 * TILE_A, &tm_mh, kc, n0, &full[s]);
          } else {
            mbar_expect_tx(&full[s], TILE_A + TILE_Q);
            tma_load_2d(st, &tm_xh, kc, m0, &full[s]);
            tma_load_2d(st + 2 * TILE_A, &tm_ml, kc, n0, &full[s]);
          }
        } else {
          const int kg = (4 * b0 + kt - nm) * BK;
          mbar_expect_tx(&full[s], 2 * TILE_A + TILE_Q);
          tma_load_2d(st, &tm_hi, kg, m0, &full[s]);
          tma_load_2d(st + TILE_A, &tm_lo, kg, m0, &full[s]);
          tma_load_2d(st + 2 * TILE_A, &tm_q, kg, n0, &full[s]);
        }
      }
    }
  } else if (warp == EW + 1) {
    if (lane == 0) {
      bool ok = true;
      int kt = 0;
      for (int vb = 0; vb < nvb && ok; ++vb) {
        const int b = vb & 1;
        if (vb >= 2) ok = mbar_wait_bounded(&acce[b], ((vb >> 1) - 1) & 1, a.status);
        tc_fence_after();
        const bool mt = vb < nmin;
        const int ns = mt ? nm : 4;
        for (int j = 0; j < ns && ok; ++j, ++kt) {
          const int s = kt % STAGES;
          ok = mbar_wait_bounded(&full[s], (kt / STAGES) & 1, a.status);
          if (!ok) break;
          tc_fence_after();
          const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
          const uint64_t dah = sw128_desc(base), dal = sw128_desc(base + TILE_A), dq = sw128_desc(base + 2 * TILE_A);
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
            const uint64_t adv = (uint64_t)((ks * 32) >> 4);
            mma_f16<NB>(tmem + b * NB, dah + adv, dq + adv, (j | ks) != 0);
            if (!mt || (j & 1) == 0) mma_f16<NB>(tmem + b * NB, dal + adv, dq + adv, 1);
          }
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&accf[b]);
      }
    }
  } else {
    // ---- epilogue: row m0 + 32 (warp % 4) + lane, columns 128 (warp / 4) .. + 127
    const int lq = warp & 3, ch = (warp >> 2) * 128;
    float y[128];
#pragma unroll
    for (int c = 0; c < 128; ++c) y[c] = 0.f;
    bool ok = true;
    for (int vb = 0; vb < nvb; ++vb) {
      const int b = vb & 1;
      ok = mbar_wait_bounded(&accf[b], (vb >> 1) & 1, a.status);
      if (!ok) break;
      tc_fence_after();
      const float* db = dsm + vb * NB + ch;
      // the read-back of a block gates the MMAs of the block after next: the 128-wide form
      // (few x rows, 192 threads) has the registers for 64 columns per wait
      constexpr int CW = NB == 128 ? 64 : 16;
#pragma unroll
      for (int c0 = 0; c0 < 128; c0 += CW) {
        uint32_t v[CW];
        const uint32_t ta = tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(b * NB + ch + c0);
        if (CW == 64) {
          tmem_ld32_nowait(ta, v);
          tmem_ld32_nowait(ta + 32, v + 32);
          tmem_wait_ld();
        } else {
          tmem_ld16(ta, *(uint32_t(*)[16])v);
        }
#pragma unroll
        for (int e = 0; e < CW; ++e) y[c0 + e] = fmaf(__uint_as_float(v[e]), db[c0 + e], y[c0 + e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);
    }
    // every MMA has completed (the last accumulator was read): the stage buffers are
    // free, rows go through shared memory for whole-row stores
    asm volatile("bar.sync 2, %0;" ::"n"(EW * 32) : "memory");
    if (ok) {
      const bool part = a.kslices > 1;
      int sg = 0;
      while (sg + 1 < a.nseg && n0 >= a.seg_n0[sg + 1]) ++sg;
      const int nb = a.seg_n0[sg], ne = a.seg_n0[sg + 1];
      constexpr int SR = 128 + 4;
      float* stile = (float*)smem + warp * 32 * SR;
#pragma unroll
      for (int c = 0; c < 128; c += 4)
        *(float4*)(stile + lane * SR + c) = make_float4(y[c], y[c + 1], y[c + 2], y[c + 3]);
      __syncwarp();
      const bool rmw = a.accumulate && !part;
      const int nc = n0 + ch + 4 * lane;
      const bool fullc = nc + 3 < ne;
#pragma unroll 1
      for (int rr = 0; rr < 32; ++rr) {
        const int mr = m0 + lq * 32 + rr;
        if (mr >= a.M) break;
        float* yrow = part ? a.partial + ((int64_t)blockIdx.z * a.M + mr) * a.N
                           : a.seg_y[sg] + (int64_t)mr * a.seg_ldy[sg] - nb;
        float4 t = *(const float4*)(stile + rr * SR + 4 * lane);
        float* dst = yrow + nc;
        if (fullc && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
          if (rmw) {
            const float4 o = *(const float4*)dst;
            t.x += o.x;
            t.y += o.y;
            t.z += o.z;
            t.w += o.w;
          }
          *(float4*)dst = t;
        } else {
          const float tv[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (nc + e < ne) dst[e] = rmw ? dst[e] + tv[e] : tv[e];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * NB) : "memory");
  }
}

// x (fp32, rows of K) -> fp16 hi and lo planes
__global__ void gemm_split_kernel(const float4* __restrict__ x, int64_t n4, uint2* __restrict__ hi,
                                  uint2* __restrict__ lo) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = x[i];
    const float f[4] = {v.x, v.y, v.z, v.w};
    uint32_t hp[2] = {0, 0}, lp[2] = {0, 0};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __half h = __float2half_rn(f[e]);
      const __half l = __float2half_rn(__fsub_rn(f[e], __half2float(h)));
      hp[e >> 1] |= (uint32_t)__half_as_ushort(h) << (16 * (e & 1));
      lp[e >> 1] |= (uint32_t)__half_as_ushort(l) << (16 * (e & 1));
    }
    hi[i] = make_uint2(hp[0], hp[1]);
    lo[i] = make_uint2(lp[0], lp[1]);
  }
}

// The prologue of four consecutive elements f of a row (elements 4 q4 .. 4 q4 + 3):
// RMSNorm (gamma (x inv)) or the SiLU gate (silu(x) up), with the element arithmetic of
// rmsnorm_kernel / silu_mul_kernel (ops.cu).
__device__ __forceinline__ void prep4(float (&f)[4], const XPro& pro, float inv, const float* ur, int q4) {
  if (pro.kind == XPRO_RMSNORM) {
    const float4 g = ((const float4*)pro.gamma)[q4];
    const float gv[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) f[e] = __fmul_rn(gv[e], __fmul_rn(f[e], inv));
  } else if (pro.kind == XPRO_SILU) {
    const float4 uu = ((const float4*)ur)[q4];
    const float uv[4] = {uu.x, uu.y, uu.z, uu.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float c = fmaxf(-20.f, fminf(f[e], 20.f));
      const float sig = __fdiv_rn(1.f, __fadd_rn(1.f, expf(-c)));
      f[e] = __fmul_rn(__fmul_rn(f[e], sig), uv[e]);
    }
  }
}

// fp16 pair (hi, lo) of v: hi = fp16(v), lo = fp16(v - hi)
__device__ __forceinline__ void split_half(float v, uint32_t& h, uint32_t& l) {
  const __half hh = __float2half_rn(v);
  h = __half_as_ushort(hh);
  l = __half_as_ushort(__float2half_rn(__fsub_rn(v, __half2float(hh))));
}

// One row of x per block: the prologue (RMSNorm over the row, or the SiLU gate)
// and the fp16 hi / lo split, so the planes hold the values rmsnorm_kernel /
// silu_mul_kernel would produce.  xsh / xsl (optional): fp16 hi / lo of the sums of
// the values over each 32-element sub-block, [M][Kp].
// TILED (the skinny GEMM's x operand, gemm_sk_kernel): hi_ receives [K / 64 chunks][hi, lo
// plane][nbt rows][64 k] of fp16, each plane in the 128-byte-swizzled K-major layout the MMA
// reads, so one contiguous copy brings in whole stages; within each group of 8 elements the
// k order is 0,4,1,5,2,6,3,7 (the order of the weight operand).  The grid has nbt blocks;
// rows M .. nbt-1 are written as zeros.
template <bool TILED>
__global__ void __launch_bounds__(256) gemm_prep_kernel(const float* __restrict__ x, int K, const XPro pro,
                                                        void* __restrict__ hi_, void* __restrict__ lo_,
                                                        __half* __restrict__ xsh, __half* __restrict__ xsl, int Kp,
                                                        int M = 0, int nbt = 0) {
  const int row = blockIdx.x;
  if (TILED && row >= M) {
    uint4* t = (uint4*)hi_;
    for (int q = threadIdx.x; q < K / 8; q += blockDim.x) {
      const int64_t base = (int64_t)(q >> 3) * 2 * nbt * 8;
      const uint32_t c = sw_off(row, q & 7) >> 4;
      t[base + c] = make_uint4(0u, 0u, 0u, 0u);
      t[base + nbt * 8 + c] = make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }
  const float* xr = x + (int64_t)row * K;
  float inv = 1.f;
  if (pro.kind == XPRO_RMSNORM) {
    // sum of squares from 16-byte loads, several in flight per thread (K % 4 == 0)
    float s = 0.f;
#pragma unroll 4
    for (int q = threadIdx.x; q < K / 4; q += blockDim.x) {
      const float4 v = ((const float4*)xr)[q];
      s = fmaf(v.x, v.x, s);
      s = fmaf(v.y, v.y, s);
      s = fmaf(v.z, v.z, s);
      s = fmaf(v.w, v.w, s);
    }
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
    inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(red[0], (float)K), pro.eps)));
  }
  const float* ur = pro.u ? pro.u + (int64_t)row * K : nullptr;
  if (!TILED) {
    uint2* hi = (uint2*)hi_;
    uint2* lo = (uint2*)lo_;
#pragma unroll 4
    for (int q = threadIdx.x; q < K / 4; q += blockDim.x) {
      const float4 v = ((const float4*)xr)[q];
      float f[4] = {v.x, v.y, v.z, v.w};
      prep4(f, pro, inv, ur, q);
      uint32_t hp[2] = {0, 0}, lp[2] = {0, 0};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        uint32_t h, l;
        split_half(f[e], h, l);
        hp[e >> 1] |= h << (16 * (e & 1));
        lp[e >> 1] |= l << (16 * (e & 1));
      }
      const int64_t o = (int64_t)row * (K / 4) + q;
      hi[o] = make_uint2(hp[0], hp[1]);
      lo[o] = make_uint2(lp[0], lp[1]);
      if (xsh) {
        // sums of the values over each 32-element sub-block (8 consecutive threads)
        float sm = (f[0] + f[1]) + (f[2] + f[3]);
        const unsigned act = __activemask();
        sm += __shfl_xor_sync(act, sm, 1);
        sm += __shfl_xor_sync(act, sm, 2);
        sm += __shfl_xor_sync(act, sm, 4);
        if ((q & 7) == 0) {
          uint32_t h, l;
          split_half(sm, h, l);
          xsh[(int64_t)row * Kp + (q >> 3)] = __ushort_as_half((unsigned short)h);
          xsl[(int64_t)row * Kp + (q >> 3)] = __ushort_as_half((unsigned short)l);
        }
      }
    }
  } else {
    uint4* t = (uint4*)hi_;
    for (int q = threadIdx.x; q < K / 8; q += blockDim.x) {
      const float4 v0 = ((const float4*)xr)[2 * q], v1 = ((const float4*)xr)[2 * q + 1];
      float f0[4] = {v0.x, v0.y, v0.z, v0.w}, f1[4] = {v1.x, v1.y, v1.z, v1.w};
      prep4(f0, pro, inv, ur, 2 * q);
      prep4(f1, pro, inv, ur, 2 * q + 1);
      uint32_t hp[4], lp[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {  // pair e: elements e and e + 4 of the group
        uint32_t h0, l0, h1, l1;
        split_half(f0[e], h0, l0);
        split_half(f1[e], h1, l1);
        hp[e] = h0 | (h1 << 16);
        lp[e] = l0 | (l1 << 16);
      }
      const int64_t base = (int64_t)(q >> 3) * 2 * nbt * 8;  // 64-k chunk q / 8, in 16-byte units
      const uint32_t c = sw_off(row, q & 7) >> 4;
      t[base + c] = make_uint4(hp[0], hp[1], hp[2], hp[3]);
      t[base + nbt * 8 + c] = make_uint4(lp[0], lp[1], lp[2], lp[3]);
      if (xsh) {
        // sums over each 32-element sub-block (4 consecutive threads)
        float sm = ((f0[0] + f0[1]) + (f0[2] + f0[3])) + ((f1[0] + f1[1]) + (f1[2] + f1[3]));
        const unsigned act = __activemask();
        sm += __shfl_xor_sync(act, sm, 1);
        sm += __shfl_xor_sync(act, sm, 2);
        if ((q & 3) == 0) {
          uint32_t h, l;
          split_half(sm, h, l);
          xsh[(int64_t)row * Kp + (q >> 2)] = __ushort_as_half((unsigned short)h);
          xsl[(int64_t)row * Kp + (q >> 2)] = __ushort_as_half((unsigned short)l);
        }
      }
    }
  }
}

// ---------------------------------------------------------------- skinny GEMM from packed weights
// Batched decode (M <= 64 rows of x) on Q4_K / Q6_K weights read as their packed bytes
// (0.5625 / 0.8125 B per weight; no resident planes).  The MMA is transposed: A = 128
// weight rows (TMEM lanes), B = the NB (16 / 32 / 64) rows of x (TMEM columns), so the
// tensor work follows the batch instead of a 128-row x tile.
// Weight operand per 256-weight block b, from the element formulas of
// Q4KTensor.cs:129-147 (w = d sc_j q - dmin m_j) and Q6KTensor.cs:105-124 (w = d sc q):
//   Q4_K: A = sc_j q, an exact fp16 integer (<= 945), written as fma(1024 + q, sc, -1024 sc)
//         from the magic-number fp16 1024 + q; the block's d is applied as its accumulator is
//         read from TMEM; the -dmin m_j term is a separate fp16 hi / lo GEMM over the sums of
//         x per 32-element sub-block (three MMAs per k step, from the block headers).
//   Q6_K: A = hi + lo of sc q (|sc q| <= 4096): hi = fp16(sc q), lo = sc q - hi, exact;
//         d on the read-back; MMAs hi (x_hi | x_lo) and lo x_hi per k step.
// x comes as fp16 hi / lo planes (gemm_prep_kernel<true>) whose k order inside each group
// of 8 is 0,4,1,5,2,6,3,7: the order in which the two 16-bit lanes of a 32-bit code word,
// shifted by 0, 4, 8 and 12 bits, hold the nibbles of elements (0, 4), (1, 5), (2, 6), (3, 7).
// Warps 0..7: dequantize (thread = weight row, 32 k of each 64-k stage) from the packed
// block in shared memory into the 128-byte-swizzled A tile; 8..11: epilogue (TMEM lanes
// 32 (w % 4)..); 12: TMA of the packed blocks (one 2D box of 128 rows x 144 / 208 bytes per
// block); 13: bulk copies of x (two stages per copy, from the pre-tiled planes); 14: MMA.
// Split K in whole blocks over blockIdx.y.  Waits poll with test_wait (bounded).
// Measured on B200 (4096 x 11008, M = 64): ~70 us, of which a pipeline with no MMA, no
// dequantization and no loads still takes ~45 us: each 64-k stage costs ~0.55-0.65 us of
// hand-over between the roles, about inversely proportional to the ring depth.  The
// resident-plane GEMMs are faster at the bench shapes, so this kernel is opt-in
// (SMALLMIND_GEMM_SK=1): it needs no resident planes (0.56 - 0.81 B per weight in HBM
// instead of 2 - 4 B more).
// Wait of a whole warp: lane 0 polls (bounded, with a short back-off so the pollers leave
// the shared-memory pipe to the MMA issuer), then every lane takes the completed phase once
// for itself (its own acquire).  All lanes return the same result.
__device__ __forceinline__ bool sk_warp_wait(uint64_t* bar, uint32_t parity, int* status) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0 && !mbar_test_wait(bar, parity)) {
    const long long t0 = clock64();
    while (!mbar_test_wait(bar, parity)) {
      __nanosleep(32);
      if (clock64() - t0 > 4000000000LL) {
        if (status) atomicExch(status, SM_ERR_TIMEOUT);
        ok = false;
        break;
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) mbar_test_wait(bar, parity);
  return ok;
}

template <int NB>
struct Sk {
  static constexpr int A_BYTES = 128 * BK * 2;  // one fp16 plane of the weight tile (16 KB)
  static constexpr int B_BYTES = NB * BK * 2;   // one fp16 plane of the x tile
  static constexpr int XU_BYTES = 4 * B_BYTES;  // x unit: two 64-k stages x (hi, lo)
  static constexpr int ARENA = 212 * 1024;      // weight stages, x units and packed block slots
  static constexpr int MAX_NBS = 32;            // blocks per k slice (the block scales' table)
  static constexpr int DV_BYTES = MAX_NBS * 128 * 2;  // fp16 d of each (block, row) of the slice
  static constexpr int MAX_ST = 4, MAX_XS = 8, MAX_PK = 8;
  static constexpr int DW = 8;  // dequantizing warps
  static constexpr int PKW = DW + 4, XW = DW + 5, MW = DW + 6;
  static constexpr int THREADS = (DW + 7) * 32;
  // accumulators of 2 NB columns (x_hi products | x_lo products): 2 block buffers + the min term
  static constexpr int TMEM_COLS = NB == 16 ? 128 : NB == 32 ? 256 : 512;
  static constexpr size_t SMEM_BYTES = (size_t)ARENA + DV_BYTES + 1024 + 512;
  // Weight stages hold one plane (Q4_K; its -dmin m term comes as separate hi and lo stages)
  // or two (Q6_K).  x has its own ring of units of two stages, each one contiguous bulk copy
  // (a TMA operation costs a few hundred nanoseconds of its issuing warp whatever its size,
  // so x comes in few, large pieces).  What is left of the arena holds packed blocks.
  __host__ __device__ static constexpr int stages(bool q4) { return q4 ? (NB == 64 ? 3 : 4) : 2; }
  __host__ __device__ static constexpr int a_bytes(bool q4) { return (q4 ? 1 : 2) * A_BYTES; }
  __host__ __device__ static constexpr int xslots(bool q4) { return NB == 64 ? (q4 ? 4 : 3) : NB == 32 ? 6 : 8; }
  __host__ __device__ static constexpr int pk_room(bool q4) {
    return (ARENA - stages(q4) * a_bytes(q4) - xslots(q4) * XU_BYTES) / (128 * (q4 ? Q4K_BLOCK_BYTES : Q6K_BODY_BYTES));
  }
  __host__ __device__ static constexpr int slots(bool q4) { return pk_room(q4) > MAX_PK ? MAX_PK : pk_room(q4); }
};

// fp16 pair (1024 + a, 1024 + b) from a word holding a in bits 0-9 and b in bits 16-25
__device__ __forceinline__ uint32_t magic_pair(uint32_t v) { return v | 0x64006400u; }

// the two high bits of Q6_K elements (e, e + 4) of a group of 8 at bits 4-5 / 20-21, from
// the sub-block's re-packed high word (byte bb: elements 2bb, 2bb+1, 8+2bb, 9+2bb)
template <int S4, bool ODD>
__device__ __forceinline__ uint32_t q6_high(uint32_t hw) {
  constexpr int sh = ODD ? (S4 == 0 ? 0 : S4 == 1 ? 2 : S4 == 2 ? 8 : 10) : (S4 == 0 ? -4 : S4 == 1 ? -2 : S4 == 2 ? 4 : 6);
  return (sh >= 0 ? (hw >> sh) : (hw << -sh)) & 0x00300030u;
}

template <int NB>
__global__ void __launch_bounds__(Sk<NB>::THREADS, 1)
    gemm_sk_kernel(const uint8_t* __restrict__ xt, const __grid_constant__ CUtensorMap tm_sh,
                   const __grid_constant__ CUtensorMap tm_sl, const __grid_constant__ CUtensorMap tm_w0,
                   const __grid_constant__ CUtensorMap tm_w1, const __grid_constant__ CUtensorMap tm_w2,
                   const __grid_constant__ TcArgs a) {
  using G = Sk<NB>;
  constexpr int DW = G::DW, A_BYTES = G::A_BYTES, B_BYTES = G::B_BYTES, XU = G::XU_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __half* dvs = (__half*)(smem + G::ARENA);  // [slice block][row] block scales d
  uint64_t* full_a = (uint64_t*)(smem + G::ARENA + G::DV_BYTES);
  uint64_t* empty = full_a + G::MAX_ST;
  uint64_t* full_b = empty + G::MAX_ST;
  uint64_t* empty_b = full_b + G::MAX_XS;
  uint64_t* pk_full = empty_b + G::MAX_XS;
  uint64_t* pk_empty = pk_full + G::MAX_PK;
  uint64_t* accf = pk_empty + G::MAX_PK;
  uint64_t* acce = accf + 2;
  uint32_t* tmem_slot = (uint32_t*)(acce + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * 128;
  int sg = 0;
  while (sg + 1 < a.nseg && n0 >= a.seg_n0[sg + 1]) ++sg;
  const DevWeight& W = a.W[sg];
  const bool q4 = W.scheme == SM_Q4_K;
  const int nl0 = n0 - a.seg_n0[sg];  // the tile's first row inside its segment's weight
  const int NBall = a.K >> 8;
  const int b0 = (int)((int64_t)NBall * blockIdx.y / a.kslices);
  const int nbs = (int)((int64_t)NBall * (blockIdx.y + 1) / a.kslices) - b0;
  // -dmin m term (Q4_K): per 64 sub-blocks of the slice one stage with its hi plane (one MMA
  // over the x sums' hi and lo planes) and one with its lo plane (x sums hi)
  const int nms = q4 ? 2 * ((nbs * 8 + 63) / 64) : 0;
  const int rb = q4 ? Q4K_BLOCK_BYTES : Q6K_BODY_BYTES;  // packed bytes of one row's block
  // Every CTA reads the same x tiles; each walks the slice's blocks from its own starting
  // block, so the CTAs do not all read one tile at the same moment.
  const int rot = nbs > 1 ? (int)((blockIdx.x * 7u) % (unsigned)nbs) : 0;
  auto blk = [&](int vb) { return b0 + (vb + rot >= nbs ? vb + rot - nbs : vb + rot); };
  const int ST = G::stages(q4), SB = G::a_bytes(q4), XS = G::xslots(q4), PK = G::slots(q4);
  uint8_t* xr = smem + ST * SB;  // x ring: XS units of two stages x (hi | lo planes)
  uint8_t* pk = xr + XS * XU;    // packed block slots
  // x units: nms / 2 of the -dmin m term (the x sums' hi | lo tile, used by a hi and a lo
  // stage), then two per block (stages 0-1 and 2-3)
  const int nxu = nms / 2 + 2 * nbs;

  if (tid == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full_a[s], DW);  // one arrive per dequantizing warp
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < XS; ++s) {
      mbar_init(&full_b[s], 1);
      mbar_init(&empty_b[s], 1);
    }
    for (int p = 0; p < PK; ++p) {
      mbar_init(&pk_full[p], 1);
      mbar_init(&pk_empty[p], DW);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(G::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < DW) {
    // ---- dequantize: thread = (row r, 32-k half h of each 64-k stage)
    const int r = tid & 127, h = tid >> 7;
    const int n = nl0 + r;
    const bool live = n < W.rows;  // INTENDED layout: rows = N
    int kt = 0;
    bool ok = true;
    // (1) -dmin m_j, k' = 64 i .. 64 i + 63 of the slice (8 blocks x 8 sub-blocks): this
    //     thread writes blocks 8 i + 4 h + t (t < 4), one 16-byte chunk each, hi plane in
    //     stage 2 i and lo plane in stage 2 i + 1
    for (int i = 0; 2 * i < nms && ok; ++i) {
      uint32_t hv[4][4], lv[4][4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int lb = 8 * i + 4 * h + t;
        uint4 hd = make_uint4(0u, 0u, 0u, 0u);
        if (live && lb < nbs)
          hd = __ldg((const uint4*)((const uint8_t*)W.data + ((int64_t)n * NBall + b0 + lb) * Q4K_BLOCK_BYTES));
        const float dmin = half_bits_to_float((uint16_t)(hd.x >> 16));
        const uint64_t mb = (uint64_t)(hd.z >> 16) | ((uint64_t)hd.w << 16);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t h0, l0, h1, l1;
          split_half(-__fmul_rn(dmin, (float)(int)((mb >> (12 * e)) & 63)), h0, l0);
          split_half(-__fmul_rn(dmin, (float)(int)((mb >> (12 * e + 6)) & 63)), h1, l1);
          hv[t][e] = h0 | (h1 << 16);
          lv[t][e] = l0 | (l1 << 16);
        }
      }
#pragma unroll
      for (int pl = 0; pl < 2; ++pl, ++kt) {
        const int s = kt % ST;
        // every lane waits (bounded); the warp leaves together when any lane gave up
        if (kt >= ST && !sk_warp_wait(&empty[s], ((kt / ST) - 1) & 1, a.status)) {
          ok = false;
          break;
        }
        uint8_t* ah = smem + s * SB;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint32_t* v = pl ? lv[t] : hv[t];
          *(uint4*)(ah + sw_off(r, 4 * h + t)) = make_uint4(v[0], v[1], v[2], v[3]);
        }
        // generic-proxy stores -> visible to the tensor core; the warp's lanes then meet
        // and one of them arrives (256 arrivals on one barrier would serialize)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[s]);
      }
    }
    // (2) the blocks: four 64-k stages each, sub-block j = 2 qq + h of stage qq
    for (int vb = 0; vb < nbs && ok; ++vb) {
      const int p = vb % PK;
      if (!sk_warp_wait(&pk_full[p], (vb / PK) & 1, a.status)) {
        ok = false;
        break;
      }
      const uint8_t* row = pk + p * (128 * rb) + r * rb;
      uint64_t sb = 0;
      if (q4) {
        const uint4 hd = *(const uint4*)row;
        sb = (uint64_t)hd.y | ((uint64_t)(hd.z & 0xFFFFu) << 32);
      }
      for (int qq = 0; qq < 4; ++qq, ++kt) {
        const int s = kt % ST;
        const int j = 2 * qq + h;
        uint32_t hv[16], lv[16];
        if (q4) {
          const int sc = (int)((sb >> (6 * j)) & 63);
          const __half2 sc2 = __half2half2(__int2half_rn(sc));
          const __half2 off2 = __half2half2(__int2half_rn(-1024 * sc));
          const uint4 cw = *(const uint4*)(row + 16 + 16 * j);
          const uint32_t w4[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi)
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4) {
              const uint32_t m = magic_pair((w4[wi] >> (4 * s4)) & 0x000F000Fu);
              const __half2 v = __hfma2(*(const __half2*)&m, sc2, off2);
              hv[4 * wi + s4] = *(const uint32_t*)&v;
            }
        } else {
          const uint4 ql = *(const uint4*)(row + 16 * j);
          const uint2 qh = *(const uint2*)(row + 128 + 8 * j);
          const uint32_t scw = *(const uint16_t*)(row + 192 + 2 * j);
          const __half2 s0 = __half2half2(__int2half_rn((int)(int8_t)(scw & 0xFF)));
          const __half2 s1 = __half2half2(__int2half_rn((int)(int8_t)(scw >> 8)));
          const __half2 c1056 = __half2half2(__int2half_rn(1056));
          const uint32_t w4[4] = {ql.x, ql.y, ql.z, ql.w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const uint32_t hw = wi < 2 ? qh.x : qh.y;
            const __half2 sc2 = wi < 2 ? s0 : s1;
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4) {
              uint32_t hb;
              if (wi & 1) {
                hb = s4 == 0 ? q6_high<0, true>(hw) : s4 == 1 ? q6_high<1, true>(hw)
                   : s4 == 2 ? q6_high<2, true>(hw) : q6_high<3, true>(hw);
              } else {
                hb = s4 == 0 ? q6_high<0, false>(hw) : s4 == 1 ? q6_high<1, false>(hw)
                   : s4 == 2 ? q6_high<2, false>(hw) : q6_high<3, false>(hw);
              }
              const uint32_t m = magic_pair(((w4[wi] >> (4 * s4)) & 0x000F000Fu) | hb);
              const __half2 q = __hsub2(*(const __half2*)&m, c1056);  // q = u - 32, exact
              const __half2 hi = __hmul2_rn(q, sc2);
              const __half2 lo = __hfma2(q, sc2, __hneg2(hi));  // sc q - hi, exact
              hv[4 * wi + s4] = *(const uint32_t*)&hi;
              lv[4 * wi + s4] = *(const uint32_t*)&lo;
            }
          }
        }
        // every lane waits (bounded); the warp leaves together when any lane gave up
        if (kt >= ST && !sk_warp_wait(&empty[s], ((kt / ST) - 1) & 1, a.status)) {
          ok = false;
          break;
        }
        
        uint8_t* ah = smem + s * SB;
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          const uint32_t off = sw_off(r, 4 * h + wi);
          *(uint4*)(ah + off) = make_uint4(hv[4 * wi], hv[4 * wi + 1], hv[4 * wi + 2], hv[4 * wi + 3]);
          if (!q4) *(uint4*)(ah + A_BYTES + off) = make_uint4(lv[4 * wi], lv[4 * wi + 1], lv[4 * wi + 2], lv[4 * wi + 3]);
        }
        // generic-proxy stores -> visible to the tensor core; the warp's lanes then meet
        // and one of them arrives (256 arrivals on one barrier would serialize)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[s]);
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&pk_empty[p]);
    }
  } else if (warp < DW + 4) {
    // ---- epilogue: weight row r = TMEM lane 32 (warp % 4) + lane, x rows = columns
    const int lq = warp & 3, r = 32 * lq + lane;
    const int n = nl0 + r;
    const bool live = n < W.rows;
    // this row's block scales for the whole slice, loaded once (each thread reads back only
    // its own entries)
    for (int vb = 0; vb < nbs; ++vb) {
      unsigned short dbits = 0;
      if (live) {
        const int64_t b = (int64_t)n * NBall + blk(vb);
        dbits = q4 ? __ldg((const unsigned short*)((const uint8_t*)W.data + b * Q4K_BLOCK_BYTES))
                   : __ldg((const unsigned short*)W.aux + aux_idx(b, W.aux_bpr, W.aux_stride));
      }
      dvs[vb * 128 + r] = __ushort_as_half(dbits);
    }
    float y[NB];
#pragma unroll
    for (int c = 0; c < NB; ++c) y[c] = 0.f;
    bool ok = true;
    const uint32_t tl = (uint32_t)(lq * 32) << 16;
    for (int vb = 0; vb < nbs; ++vb) {
      const int buf = vb & 1;
      const float dc = __half2float(dvs[vb * 128 + r]);
      if (!sk_warp_wait(&accf[buf], (vb >> 1) & 1, a.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // columns c0 .. c0+31 of the x_hi and the x_lo products, one wait for both loads
#pragma unroll
      for (int c0 = 0; c0 < NB; c0 += 32) {
        uint32_t v[32], u[32];
        if (NB >= 32) {
          tmem_ld32_nowait(tl + (uint32_t)(buf * 2 * NB + c0), v);
          tmem_ld32_nowait(tl + (uint32_t)(buf * 2 * NB + NB + c0), u);
        } else {
          tmem_ld16_nowait(tl + (uint32_t)(buf * 2 * NB + c0), v);
          tmem_ld16_nowait(tl + (uint32_t)(buf * 2 * NB + NB + c0), u);
        }
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (c0 + e < NB) y[c0 + e] = fmaf(__uint_as_float(v[e]) + __uint_as_float(u[e]), dc, y[c0 + e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[buf]);
    }
    if (ok && q4) {
      // the -dmin m term (its MMAs were issued before the blocks' and completed with them)
#pragma unroll
      for (int c0 = 0; c0 < NB; c0 += 32) {
        uint32_t v[32], u[32];
        if (NB >= 32) {
          tmem_ld32_nowait(tl + (uint32_t)(4 * NB + c0), v);
          tmem_ld32_nowait(tl + (uint32_t)(4 * NB + NB + c0), u);
        } else {
          tmem_ld16_nowait(tl + (uint32_t)(4 * NB + c0), v);
          tmem_ld16_nowait(tl + (uint32_t)(4 * NB + NB + c0), u);
        }
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (c0 + e < NB) y[c0 + e] += __uint_as_float(v[e]) + __uint_as_float(u[e]);
      }
    }
    if (ok && live) {
      const bool part = a.kslices > 1;
      const bool rmw = a.accumulate && !part;
#pragma unroll
      for (int m = 0; m < NB; ++m) {
        if (m < a.M) {
          float* dst = part ? a.partial + ((int64_t)blockIdx.y * a.M + m) * a.N + n0 + r
                            : a.seg_y[sg] + (int64_t)m * a.seg_ldy[sg] + n;
          *dst = rmw ? *dst + y[m] : y[m];
        }
      }
    }
  } else if (warp == G::PKW) {
    if (lane == 0) {
      const CUtensorMap* tmw = sg == 0 ? &tm_w0 : sg == 1 ? &tm_w1 : &tm_w2;
      for (int vb = 0; vb < nbs; ++vb) {
        const int p = vb % PK;
        if (vb >= PK && !mbar_wait_spin(&pk_empty[p], ((vb / PK) - 1) & 1, a.status)) break;
        mbar_expect_tx(&pk_full[p], 128 * rb);
        tma_load_2d(pk + p * (128 * rb), tmw, blk(vb) * rb, nl0, &pk_full[p]);
      }
    }
  } else if (warp == G::XW) {
    if (lane == 0) {
      for (int u = 0; u < nxu; ++u) {
        const int s = u % XS;
        if (u >= XS && !mbar_wait_spin(&empty_b[s], ((u / XS) - 1) & 1, a.status)) break;
        uint8_t* bh = xr + s * XU;
        if (2 * u < nms) {
          mbar_expect_tx(&full_b[s], 2 * B_BYTES);
          const int kx = 8 * b0 + 64 * u;
          tma_load_2d(bh, &tm_sh, kx, 0, &full_b[s]);
          tma_load_2d(bh + B_BYTES, &tm_sl, kx, 0, &full_b[s]);
        } else {
          const int h2 = u - nms / 2;  // half block: stages 2 (h2 & 1), +1 of block h2 / 2
          const int kc = 4 * blk(h2 >> 1) + 2 * (h2 & 1);  // first 64-k chunk
          mbar_expect_tx(&full_b[s], XU);
          bulk_g2s(bh, xt + (size_t)kc * 2 * B_BYTES, XU, &full_b[s]);
        }
      }
    }
  } else if (warp == G::MW) {
    if (lane == 0) {
      bool ok = true;
      int kt = 0;
      for (; kt < nms && ok; ++kt) {
        const int s = kt % ST, u = kt >> 1, sx = u % XS;
        ok = mbar_wait_spin(&full_b[sx], (u / XS) & 1, a.status);
        ok = ok && mbar_wait_spin(&full_a[s], (kt / ST) & 1, a.status);
        if (!ok) break;
        tc_fence_after();
        const uint64_t da = sw128_desc(smem_u32(smem + s * SB));
        const uint64_t dbh = sw128_desc(smem_u32(xr + sx * XU));
        const uint32_t tmin = tmem + 4 * NB;
#pragma unroll
        for (int ks = 0; ks < BK / 16; ++ks) {
          const uint64_t adv = (uint64_t)((ks * 32) >> 4);
          // hi stage: one MMA over the x sums' hi and lo planes (2 NB rows of B, adjacent in
          // shared memory); lo stage: the hi plane only
          if ((kt & 1) == 0)
            mma_f16<2 * NB>(tmin, da + adv, dbh + adv, (kt | ks) != 0);
          else
            mma_f16<NB>(tmin, da + adv, dbh + adv, 1);
        }
        mma_commit(&empty[s]);
        if (kt & 1) mma_commit(&empty_b[sx]);  // after the unit's lo stage
      }
      for (int vb = 0; vb < nbs && ok; ++vb) {
        const int buf = vb & 1;
        if (vb >= 2 && !mbar_wait_spin(&acce[buf], ((vb >> 1) - 1) & 1, a.status)) break;
        tc_fence_after();
        const uint32_t tacc = tmem + buf * 2 * NB;
        for (int qq = 0; qq < 4 && ok; ++qq, ++kt) {
          const int s = kt % ST, u = nms / 2 + 2 * vb + (qq >> 1), sx = u % XS;
          ok = mbar_wait_spin(&full_b[sx], (u / XS) & 1, a.status);
          ok = ok && mbar_wait_spin(&full_a[s], (kt / ST) & 1, a.status);
          if (!ok) break;
          tc_fence_after();
          const uint32_t base = smem_u32(smem + s * SB);
          const uint64_t dah = sw128_desc(base), dal = sw128_desc(base + A_BYTES);
          const uint64_t dbh = sw128_desc(smem_u32(xr + sx * XU + (qq & 1) * 2 * B_BYTES));
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
            const uint64_t adv = (uint64_t)((ks * 32) >> 4);
            // columns 0..NB-1: w x_hi, NB..2NB-1: w x_lo (B = the two x planes, adjacent)
            mma_f16<2 * NB>(tacc, dah + adv, dbh + adv, (qq | ks) != 0);
            if (!q4) mma_f16<NB>(tacc, dal + adv, dbh + adv, 1);  // Q6_K: w_lo x_hi
          }
          mma_commit(&empty[s]);
          if (qq & 1) mma_commit(&empty_b[sx]);  // after the unit's second stage
        }
        if (ok) mma_commit(&accf[buf]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G::TMEM_COLS) : "memory");
  }
}

// W -> fp16 hi / lo planes [N][K] (one thread per 32-weight unit), for GEMMs
// with enough x rows that dequantizing each weight once up front is cheaper than
// once per 128-row tile of x.
__global__ void weight_split_kernel(const DevWeight W, int N, int K, uint4* __restrict__ hi, uint4* __restrict__ lo) {
  const int upr = K >> 5;
  const int64_t units = (int64_t)N * upr;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(u / upr), k0 = (int)(u - (int64_t)n * upr) * 32;
    float w[32];
    if (raw_prefetchable(W)) {
      RawUnit r;
      load_raw(W, n, k0, K, r);
      decode_raw(W.scheme, k0, r, w);
    } else {
      weight_unit(W, n, k0, K, w);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t hp[4], lp[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float v0 = w[8 * c + 2 * e], v1 = w[8 * c + 2 * e + 1];
        const __half2 hh = __floats2half2_rn(v0, v1);
        const float2 hf = __half22float2(hh);
        const __half2 ll = __floats2half2_rn(__fsub_rn(v0, hf.x), __fsub_rn(v1, hf.y));
        hp[e] = *(const uint32_t*)&hh;
        lp[e] = *(const uint32_t*)&ll;
      }
      hi[u * 4 + c] = make_uint4(hp[0], hp[1], hp[2], hp[3]);
      lo[u * 4 + c] = make_uint4(lp[0], lp[1], lp[2], lp[3]);
    }
  }
}

// Q4_K weight [N][K] -> the three arrays of the two-MMA path (one thread per
// 32-weight sub-block j of block b of row n; Q4KTensor.cs:129-147 element formula
// w = (d sc_j) q - dmin m_j, regrouped as d (sc_j q) - dmin m_j):
//   qp[n][k]   = fp16(sc_j q_k), an integer <= 945, exact in fp16;
//   dv[n][b]   = d of block b;
//   mh / ml[n][32b + j] = fp16 hi / lo of -(dmin m_j) (the reference's own fp32
//                product), columns past K / 32 up to Kp left as they are (zero).
__global__ void q4k2_weight_kernel(const DevWeight W, int N, int K, int Kp, __half* __restrict__ qp,
                                   float* __restrict__ dv, __half* __restrict__ mh, __half* __restrict__ ml) {
  const int NB = K >> 8;
  const int64_t units = (int64_t)N * NB * 8;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(u & 7);
    const int64_t nb = u >> 3;
    const int n = (int)(nb / NB), b = (int)(nb - (int64_t)n * NB);
    const uint8_t* blk = (const uint8_t*)W.data + ((int64_t)n * NB + b) * Q4K_BLOCK_BYTES;
    const uint32_t h0 = *(const uint32_t*)blk;
    const float d = half_bits_to_float((uint16_t)(h0 & 0xFFFF)), dmin = half_bits_to_float((uint16_t)(h0 >> 16));
    int sc, mn;
    unpack_q4k_scales(blk + 4, j, sc, mn);
    if (j == 0) dv[(int64_t)n * NB + b] = d;
    {
      const float mv = -__fmul_rn(dmin, (float)mn);
      const __half h = __float2half_rn(mv);
      mh[(int64_t)n * Kp + 8 * b + j] = h;
      ml[(int64_t)n * Kp + 8 * b + j] = __float2half_rn(__fsub_rn(mv, __half2float(h)));
    }
    const uint4 q = *(const uint4*)(blk + 16 + 16 * j);
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    uint32_t hv[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t by = (qw[i >> 2] >> (8 * (i & 3))) & 0xFF;
      const __half lo = __int2half_rn(sc * (int)(by & 0xF)), hi = __int2half_rn(sc * (int)(by >> 4));
      hv[i] = (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
    }
    uint4* dst = (uint4*)(qp + (int64_t)n * K + 256 * b + 32 * j);
#pragma unroll
    for (int c = 0; c < 4; ++c) dst[c] = make_uint4(hv[4 * c], hv[4 * c + 1], hv[4 * c + 2], hv[4 * c + 3]);
  }
}

// y (+)= sum over the k slices of the partial tiles, in slice order
__global__ void gemm_reduce_kernel(const float* __restrict__ part, int S, const __grid_constant__ TcArgs a) {
  const int64_t MN = (int64_t)a.M * a.N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < MN; i += (int64_t)gridDim.x * blockDim.x) {
    // the slices' loads are independent: unrolled so several are in flight (added in slice order)
    float s = 0.f;
#pragma unroll 8
    for (int z = 0; z < S; ++z) s += part[z * MN + i];
    const int64_t m = i / a.N;
    const int n = (int)(i - m * a.N);
    int sg = 0;
    while (sg + 1 < a.nseg && n >= a.seg_n0[sg + 1]) ++sg;
    float* d = a.seg_y[sg] + m * a.seg_ldy[sg] + (n - a.seg_n0[sg]);
    *d = a.accumulate ? *d + s : s;
  }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// the driver entry point is resolved at run time, so the library loads (and its
// symbols can be checked) on machines without a CUDA driver
EncodeTiled tensor_map_encoder() {
  static EncodeTiled encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess && fn)
      encode = (EncodeTiled)fn;
  }
  return encode;
}

int make_plane_map(CUtensorMap* map, void* base, int M, int K, int box_rows = BM) {
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  EncodeTiled encode = tensor_map_encoder();
  if (!encode) return fail(SM_ERR_CUDA, "gemm: cuTensorMapEncodeTiled is not available");
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SM_OK : fail(SM_ERR_CUDA, "gemm: tensor map encoding failed");
}

// Packed weight bytes as a 2D byte array [rows][row_bytes]; one box = 128 rows x box_bytes
// (one 256-weight block of each row), no swizzle.
int make_bytes_map(CUtensorMap* map, const void* base, int rows, int64_t row_bytes, int box_bytes) {
  const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)box_bytes, 128};
  const cuuint32_t estr[2] = {1, 1};
  EncodeTiled encode = tensor_map_encoder();
  if (!encode) return fail(SM_ERR_CUDA, "gemm: cuTensorMapEncodeTiled is not available");
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SM_OK : fail(SM_ERR_CUDA, "gemm: packed-weight tensor map encoding failed");
}

// Resident fp16 planes of weight groups.  A GEMM with more than one 128-row tile
// of x reads the weights as fp16 hi / lo planes; splitting them costs a pass over
// every weight per call (~11 us per TinyLlama weight).  The first such call for
// a weight group (outside stream capture, when free HBM stays above an eighth of
// the device after the allocation) keeps the planes, 4 bytes per weight, until
// one of the group's weights is destroyed.  SMALLMIND_WEIGHT_PLANES=0 disables it.
struct PlaneEntry {
  std::vector<const void*> keys;
  int dev;
  __half* hi;
  __half* lo;
};
std::mutex g_plane_mu;
std::vector<PlaneEntry> g_planes;

// Two-MMA Q4_K data of a weight group (q4k2_weight_kernel): the sc*q plane, the
// block d values and the -(dmin m) matrix as an fp32 weight per segment.
struct Q4k2Entry {
  std::vector<const void*> keys;
  int dev;
  int N, K, Kp;
  __half* qp;
  float* dv;
  __half* mh;  // fp16 hi / lo of -(dmin m), [N][Kp]
  __half* ml;
};
std::vector<Q4k2Entry> g_q4k2;

bool planes_enabled() {
  const char* e = std::getenv("SMALLMIND_WEIGHT_PLANES");
  return !(e && e[0] == '0');
}

// the group's planes (nullptr when not resident); creates them when allowed
int resident_planes(const DevWeight* const* Ws, int nw, int N, int K, int dev, cudaStream_t st, __half** hi,
                    __half** lo, int* n_launch) {
  *hi = *lo = nullptr;
  std::vector<const void*> keys(nw);
  for (int i = 0; i < nw; ++i) keys[i] = Ws[i]->data;
  std::lock_guard<std::mutex> g(g_plane_mu);
  for (const auto& e : g_planes)
    if (e.dev == dev && e.keys == keys) {
      *hi = e.hi;
      *lo = e.lo;
      return SM_OK;
    }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return SM_OK;
  const size_t bytes = (size_t)N * K * 4;
  size_t free_b = 0, total_b = 0;
  if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess || free_b < bytes + total_b / 8) return SM_OK;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return SM_OK;
  }
  __half* whi = (__half*)p;
  __half* wlo = whi + (size_t)N * K;
  int64_t row0 = 0;
  for (int i = 0; i < nw; ++i) {
    const int Ni = Ws[i]->N();
    const int64_t units = (int64_t)Ni * K / 32;
    weight_split_kernel<<<(int)std::min<int64_t>((units + 255) / 256, 148 * 16), 256, 0, st>>>(
        *Ws[i], Ni, K, (uint4*)(whi + row0 * K), (uint4*)(wlo + row0 * K));
    if (n_launch) ++*n_launch;
    row0 += Ni;
  }
  SM_CUDA_TRY(cudaGetLastError());
  SM_CUDA_TRY(cudaStreamSynchronize(st));  // complete before any other stream can find the entry
  g_planes.push_back(PlaneEntry{keys, dev, whi, wlo});
  *hi = whi;
  *lo = wlo;
  return SM_OK;
}

// the group's two-MMA Q4_K data (entry nullptr when not resident); creates it when allowed
int resident_q4k2(const DevWeight* const* Ws, int nw, int N, int K, int dev, cudaStream_t st, Q4k2Entry* out,
                  bool* found, int* n_launch) {
  *found = false;
  std::vector<const void*> keys(nw);
  for (int i = 0; i < nw; ++i) keys[i] = Ws[i]->data;
  std::lock_guard<std::mutex> g(g_plane_mu);
  for (const auto& e : g_q4k2)
    if (e.dev == dev && e.keys == keys) {
      *out = e;
      *found = true;
      return SM_OK;
    }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return SM_OK;
  const int NB = K / 256, Kp = (K / 32 + 63) / 64 * 64;
  const size_t bytes = (size_t)N * K * 2 + (size_t)N * NB * 4 + (size_t)N * Kp * 4;  // qp, dv, mh + ml
  size_t free_b = 0, total_b = 0;
  if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess || free_b < bytes + total_b / 8) return SM_OK;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return SM_OK;
  }
  Q4k2Entry e;
  e.keys = keys;
  e.dev = dev;
  e.N = N;
  e.K = K;
  e.Kp = Kp;
  e.qp = (__half*)p;
  e.dv = (float*)(e.qp + (size_t)N * K);
  e.mh = (__half*)(e.dv + (size_t)N * NB);
  e.ml = e.mh + (size_t)N * Kp;
  SM_CUDA_TRY(cudaMemsetAsync(e.mh, 0, (size_t)N * Kp * 4, st));
  int64_t row0 = 0;
  for (int i = 0; i < nw; ++i) {
    const int Ni = Ws[i]->N();
    const int64_t units = (int64_t)Ni * NB * 8;
    q4k2_weight_kernel<<<(int)std::min<int64_t>((units + 255) / 256, 148 * 16), 256, 0, st>>>(
        *Ws[i], Ni, K, Kp, e.qp + row0 * K, e.dv + row0 * NB, e.mh + row0 * Kp, e.ml + row0 * Kp);
    if (n_launch) ++*n_launch;
    row0 += Ni;
  }
  SM_CUDA_TRY(cudaGetLastError());
  SM_CUDA_TRY(cudaStreamSynchronize(st));
  g_q4k2.push_back(e);
  *out = e;
  *found = true;
  return SM_OK;
}

}  // namespace

void gemm_tc_release_weight(const void* data) {
  std::lock_guard<std::mutex> g(g_plane_mu);
  for (size_t i = 0; i < g_q4k2.size();) {
    const auto& k = g_q4k2[i].keys;
    if (std::find(k.begin(), k.end(), data) != k.end()) {
      int prev = -1;
      cudaGetDevice(&prev);
      if (prev != g_q4k2[i].dev) cudaSetDevice(g_q4k2[i].dev);
      cudaFree(g_q4k2[i].qp);
      if (prev >= 0 && prev != g_q4k2[i].dev) cudaSetDevice(prev);
      g_q4k2.erase(g_q4k2.begin() + i);
    } else {
      ++i;
    }
  }
  for (size_t i = 0; i < g_planes.size();) {
    const auto& k = g_planes[i].keys;
    if (std::find(k.begin(), k.end(), data) != k.end()) {
      int prev = -1;
      cudaGetDevice(&prev);
      if (prev != g_planes[i].dev) cudaSetDevice(g_planes[i].dev);
      cudaFree(g_planes[i].hi);
      if (prev >= 0 && prev != g_planes[i].dev) cudaSetDevice(prev);
      g_planes.erase(g_planes.begin() + i);
    } else {
      ++i;
    }
  }
}

bool gemm_tc_supports(const DevWeight& W, int M) {
  if (W.layout != SM_LAYOUT_INTENDED || M < 5) return false;
  const int K = W.K();
  if (K % BK) return false;
  switch (W.scheme) {
    case SM_Q4_K:
    case SM_Q6_K:
      return K % 256 == 0;
    case SM_Q8_0:
    case SM_Q4_0:
      return W.block_size > 0;
    case SM_Q4_1:
    case SM_Q5_0:
    case SM_F32:
      return true;
  }
  return false;
}

bool gemm_tc_supports_multi(const DevWeight* const* W, int nw, int M) {
  if (nw < 1 || nw > MAX_SEG) return false;
  for (int i = 0; i < nw; ++i) {
    if (!gemm_tc_supports(*W[i], M) || W[i]->K() != W[0]->K()) return false;
    if (i + 1 < nw && W[i]->N() % BN) return false;  // segments meet on tile boundaries
  }
  return true;
}

namespace {
// Every segment Q4_K with K a whole number of blocks (at most 8192): the two-MMA path applies.
bool q4k2_ok(const DevWeight* const* Ws, int nw) {
  for (int i = 0; i < nw; ++i)
    if (Ws[i]->scheme != SM_Q4_K || Ws[i]->layout != SM_LAYOUT_INTENDED || Ws[i]->K() % 256 ||
        Ws[i]->K() > Q2_MAX_K)
      return false;
  return true;
}

int launch_gemm_q4k2(const Q4k2Entry& e, const DevWeight* const* Ws, float* const* ys, const int* ldys, int nw,
                     const float* x, int M, int N, int K, int accumulate, int* status, cudaStream_t st,
                     int* n_launch, const XPro* pro, int dev) {
  static bool attr_set[64] = {};
  if (dev < 64 && !attr_set[dev]) {
    SM_CUDA_TRY(cudaFuncSetAttribute(gemm_q4k2_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)Q2<128>::SMEM_BYTES));
    SM_CUDA_TRY(cudaFuncSetAttribute(gemm_q4k2_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)Q2<256>::SMEM_BYTES));
    attr_set[dev] = true;
  }
  // 256-wide tiles with several x-row tiles, when the stacked segments meet on 256 rows
  bool wide = M > BM;
  for (int i = 0; i + 1 < nw; ++i) wide = wide && Ws[i]->N() % 256 == 0;
  const int nbw = wide ? 256 : BN;
  const int Kp = e.Kp;
  const int64_t n = (int64_t)M * K;
  void* buf = nullptr;
  SM_CUDA_TRY(cudaMallocAsync(&buf, (size_t)n * 4 + (size_t)M * Kp * 4, st));
  __half* hi = (__half*)buf;
  __half* lo = hi + n;
  __half* xsh = lo + n;  // x sums per 32 (fp16 hi / lo), [M][Kp]
  __half* xsl = xsh + (size_t)M * Kp;
  int rc = SM_OK;
  if (Kp > K / 32) SM_CUDA_TRY(cudaMemsetAsync(xsh, 0, (size_t)M * Kp * 4, st));
  XPro none;
  gemm_prep_kernel<false><<<M, 256, 0, st>>>(x, K, pro ? *pro : none, hi, lo, xsh, xsl, Kp);
  if (n_launch) ++*n_launch;
  CUtensorMap mh, ml, mq, mxh, mxl, mmh, mml;
  rc = make_plane_map(&mh, hi, M, K);
  if (rc == SM_OK) rc = make_plane_map(&ml, lo, M, K);
  if (rc == SM_OK) rc = make_plane_map(&mq, e.qp, N, K, nbw);
  if (rc == SM_OK) rc = make_plane_map(&mxh, xsh, M, Kp);
  if (rc == SM_OK) rc = make_plane_map(&mxl, xsl, M, Kp);
  if (rc == SM_OK) rc = make_plane_map(&mmh, e.mh, N, Kp, nbw);
  if (rc == SM_OK) rc = make_plane_map(&mml, e.ml, N, Kp, nbw);
  if (rc == SM_OK) {
    TcArgs a;
    a.nseg = nw;
    a.seg_n0[0] = 0;
    for (int i = 0; i < nw; ++i) {
      a.W[i] = *Ws[i];
      a.seg_y[i] = ys[i];
      a.seg_ldy[i] = ldys[i];
      a.seg_n0[i + 1] = a.seg_n0[i] + Ws[i]->N();
    }
    a.M = M;
    a.N = N;
    a.K = K;
    a.accumulate = accumulate;
    a.status = status;
    const int gn = (N + nbw - 1) / nbw, gm = (M + BM - 1) / BM;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int S = 1;
    if (gn * gm < sms) S = std::max(1, std::min(sms / (gn * gm), K / 256));
    void* pbuf = nullptr;
    if (S > 1 && cudaMallocAsync(&pbuf, (size_t)S * M * N * 4, st) != cudaSuccess) {
      cudaGetLastError();
      S = 1;
      pbuf = nullptr;
    }
    a.kslices = S;
    a.partial = (float*)pbuf;
    if (wide)
      gemm_q4k2_kernel<256><<<dim3(gm, gn, S), Q2<256>::THREADS, Q2<256>::SMEM_BYTES, st>>>(
          mh, ml, mq, mxh, mxl, mmh, mml, e.dv, Kp, a);
    else
      gemm_q4k2_kernel<128><<<dim3(gm, gn, S), Q2<128>::THREADS, Q2<128>::SMEM_BYTES, st>>>(
          mh, ml, mq, mxh, mxl, mmh, mml, e.dv, Kp, a);
    if (cudaGetLastError() != cudaSuccess) rc = fail(SM_ERR_CUDA, "gemm: launch failed");
    if (n_launch) ++*n_launch;
    if (S > 1) {
      if (rc == SM_OK) {
        const int64_t MN = (int64_t)M * N;
        gemm_reduce_kernel<<<(int)std::min<int64_t>((MN + 255) / 256, 148 * 8), 256, 0, st>>>(a.partial, S, a);
        if (n_launch) ++*n_launch;
      }
      cudaFreeAsync(pbuf, st);
    }
  }
  cudaFreeAsync(buf, st);
  return rc;
}
}  // namespace

namespace {
// Every segment Q4_K or Q6_K (INTENDED, K a whole number of blocks) and at most 64 rows of x:
// the skinny GEMM on the packed bytes applies when SMALLMIND_GEMM_SK=1 selects it.
bool sk_ok(const DevWeight* const* Ws, int nw, int M) {
  if (M < 1 || M > 64) return false;
  const char* e = std::getenv("SMALLMIND_GEMM_SK");
  if (!(e && e[0] == '1')) return false;
  for (int i = 0; i < nw; ++i) {
    const DevWeight& W = *Ws[i];
    if ((W.scheme != SM_Q4_K && W.scheme != SM_Q6_K) || W.layout != SM_LAYOUT_INTENDED || W.K() % 256 ||
        W.K() != Ws[0]->K())
      return false;
    if (W.scheme == SM_Q6_K && !W.aux) return false;
  }
  return true;
}

template <int NB>
int launch_sk_nb(const uint8_t* xt, const CUtensorMap* m, const TcArgs& a, dim3 grid, cudaStream_t st, int dev) {
  static bool attr_set[64] = {};
  if (dev < 64 && !attr_set[dev]) {
    SM_CUDA_TRY(cudaFuncSetAttribute(gemm_sk_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)Sk<NB>::SMEM_BYTES));
    attr_set[dev] = true;
  }
  gemm_sk_kernel<NB><<<grid, Sk<NB>::THREADS, Sk<NB>::SMEM_BYTES, st>>>(xt, m[0], m[1], m[2], m[3], m[4], a);
  return cudaGetLastError() == cudaSuccess ? SM_OK : fail(SM_ERR_CUDA, "gemm_sk: launch failed");
}

int launch_gemm_sk(const DevWeight* const* Ws, float* const* ys, const int* ldys, int nw, const float* x, int M, int N,
                   int K, int accumulate, int* status, cudaStream_t st, int* n_launch, const XPro* pro, int dev) {
  const int nb = M <= 16 ? 16 : M <= 32 ? 32 : 64;
  const int NBall = K / 256, Kp = (K / 32 + 63) / 64 * 64;
  const size_t xt_bytes = (size_t)K * nb * 4;  // tiled x planes: K / 64 chunks x 2 planes x nb x 128 B
  void* buf = nullptr;
  SM_CUDA_TRY(cudaMallocAsync(&buf, xt_bytes + (size_t)M * Kp * 4, st));
  uint8_t* xt = (uint8_t*)buf;
  __half* xsh = (__half*)(xt + xt_bytes);  // x sums per 32 (fp16 hi / lo), [M][Kp]
  __half* xsl = xsh + (size_t)M * Kp;
  int rc = SM_OK;
  if (Kp > K / 32) SM_CUDA_TRY(cudaMemsetAsync(xsh, 0, (size_t)M * Kp * 4, st));
  XPro none;
  gemm_prep_kernel<true><<<nb, 256, 0, st>>>(x, K, pro ? *pro : none, xt, nullptr, xsh, xsl, Kp, M, nb);
  if (n_launch) ++*n_launch;
  CUtensorMap maps[5];
  rc = make_plane_map(&maps[0], xsh, M, Kp, nb);
  if (rc == SM_OK) rc = make_plane_map(&maps[1], xsl, M, Kp, nb);
  for (int i = 0; i < 3 && rc == SM_OK; ++i) {
    const DevWeight& W = *Ws[std::min(i, nw - 1)];
    const int rbytes = W.scheme == SM_Q4_K ? Q4K_BLOCK_BYTES : Q6K_BODY_BYTES;
    rc = make_bytes_map(&maps[2 + i], W.data, W.N(), (int64_t)NBall * rbytes, rbytes);
  }
  if (rc == SM_OK) {
    TcArgs a;
    a.nseg = nw;
    a.seg_n0[0] = 0;
    for (int i = 0; i < nw; ++i) {
      a.W[i] = *Ws[i];
      a.seg_y[i] = ys[i];
      a.seg_ldy[i] = ldys[i];
      a.seg_n0[i + 1] = a.seg_n0[i] + Ws[i]->N();
    }
    a.M = M;
    a.N = N;
    a.K = K;
    a.accumulate = accumulate;
    a.status = status;
    const int gn = (N + 127) / 128;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int S = 1;
    if (gn < sms) S = std::max(1, std::min(sms / gn, NBall));
    S = std::max(S, (NBall + Sk<64>::MAX_NBS - 1) / Sk<64>::MAX_NBS);  // the d table holds 32 blocks
    void* pbuf = nullptr;
    if (S > 1 && cudaMallocAsync(&pbuf, (size_t)S * M * N * 4, st) != cudaSuccess) {
      cudaGetLastError();
      S = 1;
      pbuf = nullptr;
    }
    a.kslices = S;
    a.partial = (float*)pbuf;
    const dim3 grid(gn, S);
    rc = nb == 16 ? launch_sk_nb<16>(xt, maps, a, grid, st, dev)
         : nb == 32 ? launch_sk_nb<32>(xt, maps, a, grid, st, dev)
                    : launch_sk_nb<64>(xt, maps, a, grid, st, dev);
    if (n_launch) ++*n_launch;
    if (S > 1) {
      if (rc == SM_OK) {
        const int64_t MN = (int64_t)M * N;
        gemm_reduce_kernel<<<(int)std::min<int64_t>((MN + 255) / 256, 148 * 8), 256, 0, st>>>(a.partial, S, a);
        if (n_launch) ++*n_launch;
      }
      cudaFreeAsync(pbuf, st);
    }
  }
  cudaFreeAsync(buf, st);
  return rc;
}
}  // namespace

int launch_gemm_tc_multi(const DevWeight* const* Ws, float* const* ys, const int* ldys, int nw, const float* x, int M,
                         int accumulate, int* status, cudaStream_t st, int* n_launch, const XPro* pro) {
  if (!gemm_tc_supports_multi(Ws, nw, M)) return SM_ERR_UNSUPPORTED;
  const int K = Ws[0]->K();
  int N = 0;
  for (int i = 0; i < nw; ++i) N += Ws[i]->N();
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  // batched decode on Q4_K / Q6_K from the packed bytes (opt-in), transposed MMA
  if (sk_ok(Ws, nw, M)) return launch_gemm_sk(Ws, ys, ldys, nw, x, M, N, K, accumulate, status, st, n_launch, pro, dev);
  if (dev < 64 && !attr_set[dev]) {
    SM_CUDA_TRY(
        cudaFuncSetAttribute(gemm_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
    SM_CUDA_TRY(
        cudaFuncSetAttribute(gemm_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
    SM_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<true, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)Geo<256>::SMEM_BYTES));
    attr_set[dev] = true;
  }
  // Q4_K weights: the two-MMA path on its resident sc*q plane, when it exists or can be made
  if (planes_enabled() && q4k2_ok(Ws, nw)) {
    Q4k2Entry e;
    bool found = false;
    SM_TRY(resident_q4k2(Ws, nw, N, K, dev, st, &e, &found, n_launch));
    if (found) return launch_gemm_q4k2(e, Ws, ys, ldys, nw, x, M, N, K, accumulate, status, st, n_launch, pro, dev);
  }
  // More than one 128-row tile of x: the weights come as fp16 planes (resident, or split for this
  // call).  One tile (M <= 128): resident planes when they exist or can be made, since reading
  // 4 B per weight by TMA (~1.6 T weights/s) beats dequantizing in the loader warps (~0.5 T/s);
  // otherwise the loaders dequantize.
  __half *rhi = nullptr, *rlo = nullptr;
  if (planes_enabled()) SM_TRY(resident_planes(Ws, nw, N, K, dev, st, &rhi, &rlo, n_launch));
  const bool resident = rhi != nullptr;
  const bool wt = M > BM || resident;
  const int64_t n = (int64_t)M * K, nw_el = wt && !resident ? (int64_t)N * K : 0;
  void* planes = nullptr;
  SM_CUDA_TRY(cudaMallocAsync(&planes, (size_t)(n + nw_el) * 4, st));
  __half* hi = (__half*)planes;
  __half* lo = hi + n;
  __half* whi = resident ? rhi : lo + n;
  __half* wlo = resident ? rlo : whi + nw_el;
  int rc = SM_OK;
  {
    if (pro && pro->kind != XPRO_NONE) {
      gemm_prep_kernel<false><<<M, 256, 0, st>>>(x, K, *pro, hi, lo, nullptr, nullptr, 0);
    } else {
      const int64_t n4 = n / 4;
      const int blocks = (int)std::min<int64_t>((n4 + 255) / 256, 148 * 16);
      gemm_split_kernel<<<blocks, 256, 0, st>>>((const float4*)x, n4, (uint2*)hi, (uint2*)lo);
    }
    if (n_launch) ++*n_launch;
    if (wt && !resident) {
      int64_t row0 = 0;
      for (int i = 0; i < nw; ++i) {
        const int Ni = Ws[i]->N();
        const int64_t units = (int64_t)Ni * K / 32;
        weight_split_kernel<<<(int)std::min<int64_t>((units + 255) / 256, 148 * 16), 256, 0, st>>>(
            *Ws[i], Ni, K, (uint4*)(whi + row0 * K), (uint4*)(wlo + row0 * K));
        if (n_launch) ++*n_launch;
        row0 += Ni;
      }
    }
    CUtensorMap mh, ml, mwh, mwl;
    rc = make_plane_map(&mh, hi, M, K);
    if (rc == SM_OK) rc = make_plane_map(&ml, lo, M, K);
    // 256-wide weight tiles for GEMMs with several x-row tiles (prefill, large batches),
    // when the stacked segments meet on 256-row boundaries
    bool wide = wt && M > BM;
    for (int i = 0; i + 1 < nw; ++i) wide = wide && Ws[i]->N() % 256 == 0;
    const int nbw = wide ? 256 : BN;
    if (rc == SM_OK) rc = make_plane_map(&mwh, wt ? (void*)whi : (void*)hi, wt ? N : M, K, nbw);
    if (rc == SM_OK) rc = make_plane_map(&mwl, wt ? (void*)wlo : (void*)lo, wt ? N : M, K, nbw);
    if (rc == SM_OK) {
      TcArgs a;
      a.nseg = nw;
      a.seg_n0[0] = 0;
      for (int i = 0; i < nw; ++i) {
        a.W[i] = *Ws[i];
        a.seg_y[i] = ys[i];
        a.seg_ldy[i] = ldys[i];
        a.seg_n0[i + 1] = a.seg_n0[i] + Ws[i]->N();
      }
      a.M = M;
      a.N = N;
      a.K = K;
      a.accumulate = accumulate;
      a.status = status;
      const int gn = (N + nbw - 1) / nbw, gm = (M + BM - 1) / BM;
      // split K when the output tiles alone cannot fill the SMs
      int sms = 148;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      const int nk = K / BK;
      int S = 1;
      // (one wave: at most one CTA per SM)
      if (gn * gm < sms) S = std::max(1, std::min(sms / (gn * gm), nk / 2));
      a.kslices = S;
      a.partial = nullptr;
      void* pbuf = nullptr;
      if (S > 1) {
        if (cudaMallocAsync(&pbuf, (size_t)S * M * N * 4, st) != cudaSuccess) {
          S = 1;
          a.kslices = 1;
          pbuf = nullptr;
        }
        a.partial = (float*)pbuf;
      }
      dim3 grid(gm, gn, S);
      if (wt && wide)
        gemm_tc_kernel<true, 256><<<grid, Roles<true>::THREADS, Geo<256>::SMEM_BYTES, st>>>(mh, ml, mwh, mwl, a);
      else if (wt)
        gemm_tc_kernel<true><<<grid, Roles<true>::THREADS, SMEM_BYTES, st>>>(mh, ml, mwh, mwl, a);
      else
        gemm_tc_kernel<false><<<grid, Roles<false>::THREADS, SMEM_BYTES, st>>>(mh, ml, mwh, mwl, a);
      if (cudaGetLastError() != cudaSuccess) rc = fail(SM_ERR_CUDA, "gemm: launch failed");
      if (n_launch) ++*n_launch;
      if (S > 1) {
        if (rc == SM_OK) {
          const int64_t MN = (int64_t)M * N;
          const int blocks = (int)std::min<int64_t>((MN + 255) / 256, 148 * 8);
          gemm_reduce_kernel<<<blocks, 256, 0, st>>>(a.partial, S, a);
          if (n_launch) ++*n_launch;
        }
        cudaFreeAsync(pbuf, st);
      }
    }
  }
  cudaFreeAsync(planes, st);
  return rc;
}

int launch_gemm_tc(const DevWeight& W, const float* x, float* y, int M, int ldy, int accumulate, int* status,
                   cudaStream_t st, int* n_launch) {
  const DevWeight* ws[1] = {&W};
  float* ys[1] = {y};
  const int ld[1] = {ldy};
  return launch_gemm_tc_multi(ws, ys, ld, 1, x, M, accumulate, status, st, n_launch);
}

}  // namespace sm
