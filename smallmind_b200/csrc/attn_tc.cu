// Causal GQA prefill attention on the tcgen05 tensor cores.
//
// Semantics (MultiHeadAttention.cs:676-744, 810-844; OptimizedOps.cs:39-95):
// query row i of T new rows sits at absolute position off + i (off = S - T
// cached keys before it) and sees keys 0 .. off + i.  With s = q . k (unscaled)
// and scale = 1/sqrt(hd):  m = max_j (s_j * scale),  e_j = FastExp(s_j * scale - m),
// out = (sum_j e_j v_j) / (sum_j e_j).  FastExp is the reference's Padé form
// (MathUtils.cs:20-32), which is not multiplicative, so the exact row max is
// found first (pass 1) and the exponentials are formed against it (pass 2) —
// no online rescaling.
//
// Precision: q, k, v and the probabilities e are each split into fp16 pairs
// hi + lo and every product is formed as hi*hi + hi*lo + lo*hi (three kind::f16
// MMAs into an fp32 TMEM accumulator), ~2^-22 relative.  The Padé quotient uses
// the hardware reciprocal (a few ulp), far inside the 1e-4 attention tolerance.
//
// Structure: one CTA per (q head, 128-query block), 576 threads.
//   warps 0..15 softmax: TMEM lane = query row (warp % 4 selects the lane
//               quarter), warp / 4 selects 32 of the 128 key columns of each
//               block; key blocks wholly below the diagonal skip the mask; they
//               also run the epilogue (16 of the 64 output dims each);
//   warp 16     TMA: the q tile once, then per key block the k tile (pass 1)
//               or the k and v^T tiles (pass 2), 128-byte swizzle, no multicast;
//   warp 17     one lane issues the MMAs: S = Q K^T (M 128, N 128, K 64) and
//               O += P V (M 128, N 64, K 128).
// TMEM: S in columns 0..127, O in 128..191.  All waits are bounded.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>

#include "common.cuh"
#include "mbar.cuh"

namespace sm {
namespace {

constexpr int QB = 128;  // queries per CTA
constexpr int KB = 128;  // keys per block
constexpr int HD = 64;
constexpr int SOFT_WARPS = 16;
constexpr int NQ = SOFT_WARPS / 4;  // key-column quarters of a block, one per warp set
constexpr int CW = KB / NQ;         // key columns per softmax thread (32)
constexpr int TMA_WARP = SOFT_WARPS;
constexpr int MMA_WARP = SOFT_WARPS + 1;
constexpr int THREADS = (SOFT_WARPS + 2) * 32;
// shared memory (bytes); every tile 1024-aligned for the 128-byte swizzle
constexpr int Q_PLANE = QB * HD * 2;         // 16 KB
constexpr int K_PLANE = KB * HD * 2;         // 16 KB
constexpr int V_PLANE = HD * KB * 2;         // 16 KB (v^T: 64 rows x 128 keys, two 64-key atom columns)
constexpr int P_PLANE = QB * KB * 2;         // 32 KB (two 64-key atom columns)
constexpr int STAGE = 2 * K_PLANE + 2 * V_PLANE;  // k hi/lo + v^T hi/lo
constexpr int NSTAGE = 2;
constexpr int OFF_Q = 0;
constexpr int OFF_ST = OFF_Q + 2 * Q_PLANE;
constexpr int OFF_P = OFF_ST + NSTAGE * STAGE;
constexpr int OFF_BAR = OFF_P + 2 * P_PLANE;
constexpr size_t SMEM = (size_t)OFF_BAR + 256 + 1024;  // + barriers and alignment slack
constexpr int TMEM_COLS = 256;
constexpr uint32_t TM_S = 0, TM_O = 128;

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// kind::f16, fp32 accumulator, fp16 A/B, both K-major, M = 128, N = n
__host__ __device__ constexpr uint32_t idesc(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma3(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// byte offset of 16-byte chunk c (8 fp16) of row r in one 128B-swizzled atom column
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Padé exp of the reference with a hardware-reciprocal quotient
__device__ __forceinline__ float pade_exp_fast(float x) {
  x = fminf(fmaxf(x, -87.3f), 88.7f);
  const float x2 = x * x;
  const float num = fmaf(x2, 1.f / 12.f, fmaf(x, 0.5f, 1.f));
  const float den = fmaf(x2, 1.f / 12.f, fmaf(x, -0.5f, 1.f));
  return __fdividef(num, den);
}

struct AttnArgs {
  int T, S, nH, nKv, nqb;
  float scale;
  float* out;
  int out_stride;
  int* status;
};

__global__ void __launch_bounds__(THREADS, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tq_hi, const __grid_constant__ CUtensorMap tq_lo,
                           const __grid_constant__ CUtensorMap tk_hi, const __grid_constant__ CUtensorMap tk_lo,
                           const __grid_constant__ CUtensorMap tv_hi, const __grid_constant__ CUtensorMap tv_lo,
                           const __grid_constant__ AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = (uint64_t*)(smem + OFF_BAR);
  uint64_t* q_full = bar;           // 1
  uint64_t* st_full = bar + 1;      // [NSTAGE]
  uint64_t* st_empty = bar + 3;     // [NSTAGE]
  uint64_t* s_full = bar + 5;       // S written by the MMAs
  uint64_t* s_free = bar + 6;       // S read by the softmax warps (count 256)
  uint64_t* p_full = bar + 7;       // P written (count 256)
  uint64_t* p_free = bar + 8;       // P consumed by the PV MMAs
  uint64_t* o_done = bar + 9;
  uint32_t* tmem_slot = (uint32_t*)(bar + 10);
  // [2][QB] row max / sum exchange between the column halves, in the P tile while it is idle
  float* xrow = (float*)(smem + OFF_P);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // the heaviest (last) query blocks of every head first
  const int qb = a.nqb - 1 - (int)(blockIdx.x / a.nH), h = (int)(blockIdx.x % a.nH);
  const int g = h / (a.nH / a.nKv);
  const int off = a.S - a.T;
  const int q0 = qb * QB;
  const int kend = off + min(a.T, q0 + QB);  // keys [0, kend)
  const int nkb = (kend + KB - 1) / KB;

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&st_full[s], 1);
      mbar_init(&st_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, SOFT_WARPS * 32);
    mbar_init(p_full, SOFT_WARPS * 32);
    mbar_init(p_free, 1);
    mbar_init(o_done, 1);
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
  const int total = 2 * nkb;  // key blocks over both passes

  if (warp == TMA_WARP) {
    if (lane == 0) {
      mbar_expect_tx(q_full, 2 * Q_PLANE);
      tma3(smem + OFF_Q, &tq_hi, 0, q0, h, q_full);
      tma3(smem + OFF_Q + Q_PLANE, &tq_lo, 0, q0, h, q_full);
      for (int it = 0; it < total; ++it) {
        const int s = it % NSTAGE, jb = it % nkb;
        const bool pass2 = it >= nkb;
        if (it >= NSTAGE && !mbar_wait_bounded(&st_empty[s], ((it / NSTAGE) - 1) & 1, a.status)) break;
        uint8_t* st = smem + OFF_ST + s * STAGE;
        mbar_expect_tx(&st_full[s], pass2 ? STAGE : 2 * K_PLANE);
        tma3(st, &tk_hi, 0, jb * KB, g, &st_full[s]);
        tma3(st + K_PLANE, &tk_lo, 0, jb * KB, g, &st_full[s]);
        if (pass2) {
          uint8_t* vt = st + 2 * K_PLANE;
          tma3(vt, &tv_hi, jb * KB, 0, g, &st_full[s]);
          tma3(vt + V_PLANE / 2, &tv_hi, jb * KB + 64, 0, g, &st_full[s]);
          tma3(vt + V_PLANE, &tv_lo, jb * KB, 0, g, &st_full[s]);
          tma3(vt + V_PLANE + V_PLANE / 2, &tv_lo, jb * KB + 64, 0, g, &st_full[s]);
        }
      }
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      bool ok = mbar_wait_bounded(q_full, 0, a.status);
      tc_fence_after();
      const uint32_t qa = smem_u32(smem + OFF_Q);
      const uint64_t dqh = sw128_desc(qa), dql = sw128_desc(qa + Q_PLANE);
      const uint32_t pa = smem_u32(smem + OFF_P);
      for (int it = 0; it < total && ok; ++it) {
        const int s = it % NSTAGE;
        const bool pass2 = it >= nkb;
        const int j = pass2 ? it - nkb : it;
        ok = mbar_wait_bounded(&st_full[s], (it / NSTAGE) & 1, a.status);
        // S may be overwritten once the softmax warps have read the previous one
        if (ok && it > 0) ok = mbar_wait_bounded(s_free, (it - 1) & 1, a.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t ka = smem_u32(smem + OFF_ST + s * STAGE);
        const uint64_t dkh = sw128_desc(ka), dkl = sw128_desc(ka + K_PLANE);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const uint64_t adv = (uint64_t)((ks * 32) >> 4);
          mma_f16(tmem + TM_S, dqh + adv, dkh + adv, idesc(KB), ks != 0);
          mma_f16(tmem + TM_S, dqh + adv, dkl + adv, idesc(KB), 1);
          mma_f16(tmem + TM_S, dql + adv, dkh + adv, idesc(KB), 1);
        }
        mma_commit(s_full);
        if (!pass2) {
          mma_commit(&st_empty[s]);
          continue;
        }
        // O += P V once the softmax warps have written P for this block
        ok = mbar_wait_bounded(p_full, j & 1, a.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t va = ka + 2 * K_PLANE;
#pragma unroll
        for (int ks = 0; ks < KB / 16; ++ks) {
          // k step ks: atom column ks / 4, 32-byte step ks % 4 inside it
          const uint32_t col = (uint32_t)(ks >> 2), step = (uint32_t)((ks & 3) * 32);
          const uint64_t ph = sw128_desc(pa + col * (P_PLANE / 2) + step);
          const uint64_t pl = sw128_desc(pa + P_PLANE + col * (P_PLANE / 2) + step);
          const uint64_t vh = sw128_desc(va + col * (V_PLANE / 2) + step);
          const uint64_t vl = sw128_desc(va + V_PLANE + col * (V_PLANE / 2) + step);
          mma_f16(tmem + TM_O, ph, vh, idesc(HD), (j | ks) != 0);
          mma_f16(tmem + TM_O, ph, vl, idesc(HD), 1);
          mma_f16(tmem + TM_O, pl, vh, idesc(HD), 1);
        }
        mma_commit(p_free);
        mma_commit(&st_empty[s]);
      }
      mma_commit(o_done);
    }
  } else {
    // ---- softmax warps: row r, key columns [c0, c0 + 32) of each block
    const int r = (warp & 3) * 32 + lane;
    const int qt = warp >> 2, c0 = qt * CW;
    const int qi = q0 + r;               // query row
    const bool live = qi < a.T;
    const int pos = off + qi;            // keys 0 .. pos
    const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    float m = -FLT_MAX;
    bool ok = true;
    // pass 1: row max of s * scale
    for (int j = 0; j < nkb && ok; ++j) {
      ok = mbar_wait_bounded(s_full, j & 1, a.status);
      tc_fence_after();
      uint32_t v[2][16];
      tmem_ld16(trow + TM_S + c0, v[0]);
      tmem_ld16(trow + TM_S + c0 + 16, v[1]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(s_free);
      // every key of this block is visible to every row of the CTA: no mask
      const bool open = j * KB + KB - 1 <= off + q0;
      if (open) {
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) m = fmaxf(m, __fmul_rn(__uint_as_float(v[c][e]), a.scale));
      } else {
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int key = j * KB + c0 + 16 * c + e;
            if (key <= pos) m = fmaxf(m, __fmul_rn(__uint_as_float(v[c][e]), a.scale));
          }
      }
    }
    xrow[qt * QB + r] = m;
    asm volatile("bar.sync 1, %0;" ::"n"(SOFT_WARPS * 32) : "memory");
#pragma unroll
    for (int o = 0; o < NQ; ++o) m = fmaxf(m, xrow[o * QB + r]);
    asm volatile("bar.sync 1, %0;" ::"n"(SOFT_WARPS * 32) : "memory");  // before P overwrites the exchange
    // pass 2: e = FastExp(s * scale - m) -> P (fp16 hi / lo), row sums
    float sum = 0.f;
    // columns [c0, c0 + 32): atom column qt / 2, 16-byte chunks 4 (qt % 2) .. + 3
    uint8_t* ph = smem + OFF_P + (qt >> 1) * (P_PLANE / 2);
    uint8_t* pl = ph + P_PLANE;
    const int chunk0 = 4 * (qt & 1);
    for (int j = 0; j < nkb && ok; ++j) {
      ok = mbar_wait_bounded(s_full, (nkb + j) & 1, a.status);
      tc_fence_after();
      uint32_t v[2][16];
      tmem_ld16(trow + TM_S + c0, v[0]);
      tmem_ld16(trow + TM_S + c0 + 16, v[1]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(s_free);
      const bool open = live && j * KB + KB - 1 <= off + q0;
      float ev[32];
      if (open) {
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e)
            ev[16 * c + e] = pade_exp_fast(__fsub_rn(__fmul_rn(__uint_as_float(v[c][e]), a.scale), m));
      } else {
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int key = j * KB + c0 + 16 * c + e;
            ev[16 * c + e] = (live && key <= pos)
                                 ? pade_exp_fast(__fsub_rn(__fmul_rn(__uint_as_float(v[c][e]), a.scale), m))
                                 : 0.f;
          }
      }
#pragma unroll
      for (int e = 0; e < 32; ++e) sum += ev[e];
      // the previous block's P must have been consumed before it is overwritten
      if (j > 0 && ok) ok = mbar_wait_bounded(p_free, (j - 1) & 1, a.status);
#pragma unroll
      for (int hc = 0; hc < 4; ++hc) {  // 16-byte chunks of 8 keys
        uint32_t hp[4], lp[4];
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          const float v0 = ev[8 * hc + 2 * e2], v1 = ev[8 * hc + 2 * e2 + 1];
          const __half2 hh = __floats2half2_rn(v0, v1);
          const float2 hf = __half22float2(hh);
          const __half2 ll = __floats2half2_rn(v0 - hf.x, v1 - hf.y);
          hp[e2] = *(const uint32_t*)&hh;
          lp[e2] = *(const uint32_t*)&ll;
        }
        const uint32_t o = sw_off(r, chunk0 + hc);
        *(uint4*)(ph + o) = make_uint4(hp[0], hp[1], hp[2], hp[3]);
        *(uint4*)(pl + o) = make_uint4(lp[0], lp[1], lp[2], lp[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(p_full);
    }
    // ---- epilogue: O row r, dims [16 qt, 16 qt + 16); after o_done no MMA reads P
    ok = ok && mbar_wait_bounded(o_done, 0, a.status);
    tc_fence_after();
    xrow[qt * QB + r] = sum;
    asm volatile("bar.sync 1, %0;" ::"n"(SOFT_WARPS * 32) : "memory");
    sum = 0.f;
#pragma unroll
    for (int o = 0; o < NQ; ++o) sum += xrow[o * QB + r];
    uint32_t ov[16];
    tmem_ld16(trow + TM_O + 16 * qt, ov);
    tmem_wait_ld();
    if (ok && live) {
      const float inv = __fdiv_rn(1.f, sum);
      float* o = a.out + (int64_t)qi * a.out_stride + h * HD + 16 * qt;
#pragma unroll
      for (int e = 0; e < 16; e += 4)
        *(float4*)(o + e) = make_float4(__uint_as_float(ov[e]) * inv, __uint_as_float(ov[e + 1]) * inv,
                                        __uint_as_float(ov[e + 2]) * inv, __uint_as_float(ov[e + 3]) * inv);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// q rows [T][q_stride] (head h at column h * 64) -> planes [nH][T][64];
// k / v cache rows (kv head g at base + g * head_stride, position j at
// + j * row_stride) -> k planes [nKv][S][64] and v^T planes [nKv][64][Sp].
// q, k and v^T -> fp16 hi / lo planes.  Block (x, y): 64 rows (tokens / keys) of
// head y (q heads, then k heads, then v heads); v is transposed through shared
// memory to [kv head][d][key] (keys padded to Sp with zeros).
__device__ __forceinline__ void split_store(float x, __half* dh, __half* dl, int64_t di) {
  const __half hi = __float2half_rn(x);
  dh[di] = hi;
  dl[di] = __float2half_rn(x - __half2float(hi));
}

__global__ void __launch_bounds__(256) attn_split_kernel(const float* __restrict__ q, int q_stride,
                                                         const float* __restrict__ k, const float* __restrict__ v,
                                                         int64_t row_stride, int64_t head_stride, int T, int S, int Sp,
                                                         int nH, int nKv, __half* qh, __half* ql, __half* kh,
                                                         __half* kl, __half* vh, __half* vl) {
  const int y = blockIdx.y, r0 = blockIdx.x * 64, d = threadIdx.x & 63, rs = threadIdx.x >> 6;
  if (y < nH) {
    if (r0 >= T) return;
    for (int r = r0 + rs; r < min(T, r0 + 64); r += 4)
      split_store(q[(int64_t)r * q_stride + y * HD + d], qh, ql, ((int64_t)y * T + r) * HD + d);
  } else if (y < nH + nKv) {
    const int g = y - nH;
    if (r0 >= S) return;
    for (int r = r0 + rs; r < min(S, r0 + 64); r += 4)
      split_store(k[g * head_stride + r * row_stride + d], kh, kl, ((int64_t)g * S + r) * HD + d);
  } else {
    const int g = y - nH - nKv;
    if (r0 >= Sp) return;
    __shared__ float tile[64][65];
    for (int r = rs; r < 64; r += 4) tile[r][d] = r0 + r < S ? v[g * head_stride + (r0 + r) * row_stride + d] : 0.f;
    __syncthreads();
    // thread: key j = threadIdx & 63 (contiguous in the output), dims dd = rs, rs + 4, ...
    for (int dd = rs; dd < HD; dd += 4)
      split_store(tile[d][dd], vh, vl, ((int64_t)g * HD + dd) * Sp + r0 + d);
  }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 3-D fp16 plane [d2][d1][d0] with a box of {b0, b1, 1}, 128-byte swizzle
int make_map3(CUtensorMap* map, void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t b0, uint32_t b1) {
  static EncodeTiled encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) != cudaSuccess ||
        qr != cudaDriverEntryPointSuccess || !fn)
      return fail(SM_ERR_CUDA, "attention: cuTensorMapEncodeTiled is not available");
    encode = (EncodeTiled)fn;
  }
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
  const cuuint32_t box[3] = {b0, b1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SM_OK : fail(SM_ERR_CUDA, "attention: tensor map encoding failed");
}

}  // namespace

int launch_attention_prefill_tc(const float* q, int q_stride, const float* k, const float* v, int64_t row_stride,
                                int64_t head_stride, float* out, int out_stride, int T, int S, int nH, int nKv, int hd,
                                int* status, cudaStream_t st, int* n_launch) {
  if (hd != HD || nH % nKv || T <= 0 || S < T) return SM_ERR_UNSUPPORTED;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    SM_CUDA_TRY(cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM));
    attr_set[dev] = true;
  }
  const int Sp = (S + 63) / 64 * 64;
  const int64_t nq = (int64_t)nH * T * HD, nk = (int64_t)nKv * S * HD, nv = (int64_t)nKv * HD * Sp;
  void* buf = nullptr;
  SM_CUDA_TRY(cudaMallocAsync(&buf, (size_t)(nq + nk + nv) * 4, st));
  __half* qh = (__half*)buf;
  __half* ql = qh + nq;
  __half* kh = ql + nq;
  __half* kl = kh + nk;
  __half* vh = kl + nk;
  __half* vl = vh + nv;
  int rc = SM_OK;
  {
    dim3 grid((std::max(T, Sp) + 63) / 64, nH + 2 * nKv);
    attn_split_kernel<<<grid, 256, 0, st>>>(q, q_stride, k, v, row_stride, head_stride, T, S, Sp, nH, nKv, qh, ql,
                                            kh, kl, vh, vl);
    if (n_launch) ++*n_launch;
    CUtensorMap mqh, mql, mkh, mkl, mvh, mvl;
    rc = make_map3(&mqh, qh, HD, T, nH, HD, QB);
    if (rc == SM_OK) rc = make_map3(&mql, ql, HD, T, nH, HD, QB);
    if (rc == SM_OK) rc = make_map3(&mkh, kh, HD, S, nKv, HD, KB);
    if (rc == SM_OK) rc = make_map3(&mkl, kl, HD, S, nKv, HD, KB);
    if (rc == SM_OK) rc = make_map3(&mvh, vh, Sp, HD, nKv, 64, HD);
    if (rc == SM_OK) rc = make_map3(&mvl, vl, Sp, HD, nKv, 64, HD);
    if (rc == SM_OK) {
      AttnArgs a;
      a.T = T;
      a.S = S;
      a.nH = nH;
      a.nKv = nKv;
      a.nqb = (T + QB - 1) / QB;
      a.scale = 1.0f / sqrtf((float)hd);
      a.out = out;
      a.out_stride = out_stride;
      a.status = status;
      attn_prefill_tc_kernel<<<a.nqb * nH, THREADS, SMEM, st>>>(mqh, mql, mkh, mkl, mvh, mvl, a);
      if (cudaGetLastError() != cudaSuccess) rc = fail(SM_ERR_CUDA, "attention: launch failed");
      if (n_launch) ++*n_launch;
    }
  }
  cudaFreeAsync(buf, st);
  return rc;
}

}  // namespace sm
