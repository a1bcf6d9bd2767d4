// Decode GEMV (M = 1) for Q4_K on the integer tensor-core path.
//
// One mma.sync.m16n8k32 (u8 x s8 -> s32) covers one 32-weight unit (one Q4_K
// sub-block) of 16 rows.  Lane (g, tig) owns code word tig of the unit for rows
// g and g + 8: byte i of the word holds the codes of elements 8 tig + 2i (low
// nibble, lo) and 8 tig + 2i + 1 (high nibble, hi).  The A fragment takes the
// word twice: masked to its low nibbles at k = 4 tig + i, and unchanged
// (lo + 16 hi) at k = 16 + 4 tig + i, so no unpacking beyond one AND.  The
// matching B values are, with x in fixed point relative to the largest |x| of
// its 256-element block (one power-of-two exponent e per block),
//   at k = 16 + 4 tig + i:  H = round(x_hi * 2^(17-e))
//   at k =      4 tig + i:  L - H,  L = round(x_lo * 2^(21-e))
// so that lo (L - H) + (lo + 16 hi) H = lo L + hi (16 H): the exact integer
// dot of the codes with x at 21 bits (low elements) and 17 bits (high).  The
// B values are split into three signed 8-bit digits v = a*2^16 + b*2^8 + c
// held in B columns 0..2, giving integer sums A_j, B_j, C_j per row and unit j.
// The reference element formula (Q4KTensor.cs:129-147), w = d s_j q - dmin m_j,
// then gives per row and block
//   sum_k w_k x_k ~= d 2^(e-21) sum_j s_j (A_j 65536 + B_j 256 + C_j)
//                    - dmin sum_j m_j (sum of x over unit j),
// with the six-bit s_j multiplying the digit sums in integer arithmetic.
// The x rounding stays far inside the 1e-4 GEMV tolerance.  (The 4-bit
// m16n8k64 form would take the code words as they are, but runs at half this
// speed on sm_100a.)
//
// One persistent CTA per SM owns a contiguous range of 16-row tiles: warp 15
// brings each tile (one bulk copy per row, rows padded apart so the fragment
// loads are free of bank conflicts) into a shared-memory ring, issued before
// the PDL wait.  The other warps take the (tile, 256-weight block) items in turn
// with no CTA-wide barrier; each writes its block partials and arrives on the
// slot's empty barrier, and the producer warp, once all have arrived, sums the
// partials in block order (deterministic), stores y and refills the slot.
#include <algorithm>

#include "common.cuh"
#include "gemv1.cuh"
#include "mbar.cuh"
#include "mma_i8.cuh"

namespace sm {
namespace {

constexpr int MM_THREADS = 768;
constexpr int MM_CWARPS = MM_THREADS / 32 - 1;
constexpr int MM_CT = MM_CWARPS * 32;
constexpr int ROWS = 16;  // rows per stage (one MMA tile)

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(MM_CT) : "memory"); }


struct MmaArgs {
  const uint8_t* w = nullptr;  // Q4_K rows (INTENDED layout)
  const float* x = nullptr;
  float* y = nullptr;
  int N = 0, K = 0, accumulate = 0;
  int nslots = 2;
  int row_stride = 0;  // bytes between rows in a ring slot (row bytes + 16 or 32: no bank conflicts)
  int64_t slot_bytes = 0;
  int plane_offset = 0, red_offset = 0, scw_offset = 0, ring_offset = 0;
  int* status = nullptr;
  // Q6_K: fp16 d values in rows of aux_stride elements (16-byte padded), copied
  // behind each staged row (abytes per row)
  const uint16_t* aux = nullptr;
  int aux_stride = 0, abytes = 0;
  // Q4_K with several x rows: M rows of x (stride K), y rows of stride ldy
  int M = 1, ldy = 0;
};

constexpr int SCW = 9;  // per-warp scale scratch row stride (floats): rows g = 0..7 on distinct banks

// MX x rows (1, 2 or 4): B holds three digit columns per x row (column 3 m + q),
// NMMA = ceil(3 MX / 8) MMAs per unit share one A fragment; columns past 3 M
// load a real column and meet a zero weight.
template <int MX>
__global__ void __launch_bounds__(MM_THREADS, 1) gemv_mma_q4k_kernel(const __grid_constant__ MmaArgs a) {
  constexpr int NC = 3 * MX;            // digit columns stored per unit
  constexpr int NMMA = (NC + 7) / 8;    // MMAs per unit
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = (uint64_t*)smem;  // [8]
  uint64_t* empty = full + 8;        // [8]
  uint2* planes = (uint2*)(smem + a.plane_offset);  // [U][NC][4 tig] (k 4 tig + i, k 16 + 4 tig + i) words
  float* red = (float*)(smem + a.red_offset);       // [nslots][NB][MX][ROWS] block partials
  float* scw_all = (float*)(smem + a.scw_offset);   // per warp: int [ROWS][SCW], msum [MX][ROWS], fdv [MX][ROWS]
  uint8_t* ring = smem + a.ring_offset;
  const int K = a.K, U = K >> 5, NB = K >> 8, M = a.M;
  const uint32_t rbytes = (uint32_t)NB * Q4K_BLOCK_BYTES;
  const int rs = a.row_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ngroups = (a.N + ROWS - 1) / ROWS;
  const int g0 = (int)((int64_t)ngroups * blockIdx.x / gridDim.x);
  const int g1 = (int)((int64_t)ngroups * (blockIdx.x + 1) / gridDim.x);
  const int nst = g1 - g0;
  float* usum = (float*)(planes + U * NC * 4);  // [MX][U] sum of x over the unit
  float* bexp = usum + MX * U;                  // [MX][NB] 2^(e-21) of the block
  if (tid == 0) {
    for (int i = 0; i < a.nslots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NB);  // one arrival per (tile, block) item
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == MM_CWARPS) {
    // producer: one bulk copy per row into the padded slot (the weights do not
    // depend on the previous kernel, so this starts before the PDL wait); once
    // every block item of a tile has arrived on the slot's empty barrier, sum
    // the block partials in block order (deterministic), store y, refill.
    auto issue = [&](int k) {
      const int slot = k % a.nslots;
      const int row = (g0 + k) * ROWS;
      const int n = min(ROWS, a.N - row);
      if (lane == 0) mbar_expect_tx(&full[slot], (uint32_t)n * rbytes);
      __syncwarp();
      if (lane < n)
        bulk_g2s(ring + slot * a.slot_bytes + lane * rs, a.w + (int64_t)(row + lane) * rbytes, rbytes, &full[slot]);
    };
    int next = 0;
    for (; next < min(nst, a.nslots); ++next) issue(next);
    if (lane == 0) asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // y may be the previous kernel's output
    int slot = 0;
    uint32_t phase = 0;
    for (int k = 0; k < nst; ++k) {
      if (!mbar_wait_bounded(&empty[slot], phase, a.status)) return;
      const int row0 = (g0 + k) * ROWS;
      const int n = min(ROWS, a.N - row0);
      for (int t = lane; t < M * ROWS; t += 32) {
        const int m = t / ROWS, r = t - m * ROWS;
        if (r < n) {
          const float* rd = red + (slot * NB * MX + m) * ROWS + r;
          float s = 0.f;
          for (int b = 0; b < NB; ++b) s += rd[b * MX * ROWS];
          float* dst = a.y + (int64_t)m * a.ldy + row0 + r;
          *dst = a.accumulate ? *dst + s : s;
        }
      }
      __syncwarp();
      if (next < nst) issue(next++);
      if (++slot == a.nslots) slot = 0, phase ^= 1;
    }
    return;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // ---- digit planes of x: one warp per (x row, 256-element block), four lanes
  // per unit, eight elements per lane; one exponent per (row, block)
  for (int it = warp; it < M * NB; it += MM_CWARPS) {
    const int m = it / NB, blk = it - m * NB;
    const int u = blk * 8 + (lane >> 2), p = lane & 3;
    const float4* xp = (const float4*)(a.x + (int64_t)m * K + 32 * u + 8 * p);
    const float4 v0 = __ldcg(xp), v1 = __ldcg(xp + 1);
    const float xv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float amax = 0.f, sx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      amax = fmaxf(amax, fabsf(xv[i]));
      sx += xv[i];
    }
    sx += __shfl_xor_sync(0xffffffffu, sx, 1);
    sx += __shfl_xor_sync(0xffffffffu, sx, 2);
    amax = warp_max(amax);
    int ex = 0;
    frexpf(amax, &ex);  // amax < 2^ex
    const float up = ldexpf(1.f, 21 - ex), uph = ldexpf(1.f, 17 - ex);
    // B fragment of lane (column q, tig): word 0 = values at k = 4 tig + i,
    // word 1 = values at k = 16 + 4 tig + i
    uint32_t pw[2][3] = {};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int L = amax > 0.f ? __float2int_rn(xv[2 * i] * up) : 0;       // |L| <= 2^21
      const int H = amax > 0.f ? __float2int_rn(xv[2 * i + 1] * uph) : 0;  // |H| <= 2^17
      const int v2[2] = {L - H, H};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int X = v2[h];
        const int c = ((X + 128) & 255) - 128;
        const int X1 = (X - c) >> 8;
        const int b = ((X1 + 128) & 255) - 128;
        const int hi = (X1 - b) >> 8;
        pw[h][0] |= (uint32_t)(hi & 255) << (8 * i);
        pw[h][1] |= (uint32_t)(b & 255) << (8 * i);
        pw[h][2] |= (uint32_t)(c & 255) << (8 * i);
      }
    }
    uint2* d = planes + (u * NC + 3 * m) * 4 + p;
#pragma unroll
    for (int q = 0; q < 3; ++q) d[4 * q] = make_uint2(pw[0][q], pw[1][q]);
    if (p == 0) usum[m * U + u] = sx;
    if (lane == 0) bexp[m * NB + blk] = ldexpf(1.f, ex - 21);
  }
  csync();
  const int g = lane >> 2, tig = lane & 3;
  // lane (g, tig), MMA mi: B column 8 mi + g (a real column when past 3 M);
  // C columns 8 mi + 2 tig + {0, 1} = x row c / 3, digit c % 3 (x 65536, 256, 1)
  const uint2* pl[NMMA];
#pragma unroll
  for (int mi = 0; mi < NMMA; ++mi) {
    const int c = 8 * mi + g;
    pl[mi] = planes + (c < 3 * M ? c : 0) * 4 + tig;
  }
  float* scw = scw_all + warp * (ROWS * SCW + 2 * MX * ROWS);
  float* msum = scw + ROWS * SCW;  // [MX][ROWS]
  float* fdv = msum + MX * ROWS;   // [MX][ROWS]
  const int sr = lane >> 1, sh = lane & 1;  // scale decode: row, half of the sub-blocks
  // item (tile k, block kb) = warp, warp + MM_CWARPS, ... of nst * NB, walked without divisions
  int k = 0, kb = warp, slot = 0;
  uint32_t phase = 0;
  while (kb >= NB) {
    kb -= NB;
    ++k;
    if (++slot == a.nslots) slot = 0, phase ^= 1;
  }
  for (; k < nst;) {
    if (!mbar_wait_bounded(&full[slot], phase, a.status)) return;
    const uint8_t* st = ring + slot * a.slot_bytes + kb * Q4K_BLOCK_BYTES;
    const int row0 = (g0 + k) * ROWS;
    const int n = min(ROWS, a.N - row0);
    {
      // sub-block scales and mins of row sr, sub-blocks 4 sh .. 4 sh + 3
      // (Q4KTensor.cs:109-132): six-bit scales kept as integers, the mins
      // folded with each x row's unit sums, d with the row's block exponent
      const int4 hdr = *(const int4*)(st + min(sr, n - 1) * rs);
      const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFF)));
      const float dmin = __half2float(__ushort_as_half((unsigned short)((uint32_t)hdr.x >> 16)));
      const uint64_t sb = (uint32_t)hdr.y | ((uint64_t)((uint32_t)hdr.z & 0xFFFFu) << 32);
      const uint64_t mb = ((uint32_t)hdr.z >> 16) | ((uint64_t)(uint32_t)hdr.w << 16);
      const uint32_t s24 = (uint32_t)(sb >> (24 * sh)), m24 = (uint32_t)(mb >> (24 * sh));
      int* si = (int*)scw + sr * SCW + 4 * sh;
#pragma unroll
      for (int j = 0; j < 4; ++j) si[j] = (s24 >> (6 * j)) & 63;
      const float m0 = (float)(m24 & 63), m1 = (float)((m24 >> 6) & 63), m2 = (float)((m24 >> 12) & 63),
                  m3 = (float)((m24 >> 18) & 63);
#pragma unroll
      for (int m = 0; m < MX; ++m) {
        if (m >= M) break;
        const float4 q = *(const float4*)(usum + m * U + kb * 8 + 4 * sh);
        float mpart = m0 * q.x;
        mpart = fmaf(m1, q.y, mpart);
        mpart = fmaf(m2, q.z, mpart);
        mpart = fmaf(m3, q.w, mpart);
        mpart = dmin * (mpart + __shfl_xor_sync(0xffffffffu, mpart, 1));
        if (sh == 0) {
          msum[m * ROWS + sr] = mpart;
          fdv[m * ROWS + sr] = d * bexp[m * NB + kb];
        }
      }
    }
    __syncwarp();
    const uint8_t* rg = st + min(g, n - 1) * rs + 16 + 4 * tig;
    const uint8_t* rg8 = st + min(g + 8, n - 1) * rs + 16 + 4 * tig;
    const int ustride = NC * 4;  // uint2 per unit
    const int ub = kb * 8 * ustride;
    const int* si = (const int*)scw;
    int t[NMMA][4];
#pragma unroll
    for (int mi = 0; mi < NMMA; ++mi) t[mi][0] = t[mi][1] = t[mi][2] = t[mi][3] = 0;
    // four units in flight, then their epilogues
#pragma unroll
    for (int j0 = 0; j0 < 8; j0 += 4) {
      int dd[4][NMMA][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t w0 = *(const uint32_t*)(rg + 16 * (j0 + j));
        const uint32_t w1 = *(const uint32_t*)(rg8 + 16 * (j0 + j));
        const uint32_t lo0 = w0 & 0x0F0F0F0Fu, lo1 = w1 & 0x0F0F0F0Fu;
#pragma unroll
        for (int mi = 0; mi < NMMA; ++mi) {
          const uint2 b = pl[mi][ub + (j0 + j) * ustride];
          mma_u8s8(dd[j][mi][0], dd[j][mi][1], dd[j][mi][2], dd[j][mi][3], lo0, lo1, w0, w1, b.x, b.y);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int s0 = si[g * SCW + j0 + j], s1 = si[(g + 8) * SCW + j0 + j];
#pragma unroll
        for (int mi = 0; mi < NMMA; ++mi) {
          t[mi][0] += s0 * dd[j][mi][0];
          t[mi][1] += s0 * dd[j][mi][1];
          t[mi][2] += s1 * dd[j][mi][2];
          t[mi][3] += s1 * dd[j][mi][3];
        }
      }
    }
    // per x row: digit columns weighted (x 65536, 256, 1), then summed over the quad
    float v0[MX], v1[MX];
#pragma unroll
    for (int m = 0; m < MX; ++m) v0[m] = v1[m] = 0.f;
#pragma unroll
    for (int mi = 0; mi < NMMA; ++mi)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = 8 * mi + 2 * tig + e;
        const float wgt = (c % 3 == 0) ? 65536.f : (c % 3 == 1 ? 256.f : 1.f);
#pragma unroll
        for (int m = 0; m < MX; ++m)
          if (c / 3 == m && c < 3 * M) {
            v0[m] = fmaf((float)t[mi][e], wgt, v0[m]);
            v1[m] = fmaf((float)t[mi][2 + e], wgt, v1[m]);
          }
      }
    float* rd = red + (slot * NB + kb) * MX * ROWS;
#pragma unroll
    for (int m = 0; m < MX; ++m) {
      if (m >= M) break;
      float a0 = v0[m], a1 = v1[m];
      a0 += __shfl_xor_sync(0xffffffffu, a0, 1);
      a1 += __shfl_xor_sync(0xffffffffu, a1, 1);
      a0 += __shfl_xor_sync(0xffffffffu, a0, 2);
      a1 += __shfl_xor_sync(0xffffffffu, a1, 2);
      if (tig == 0) {
        rd[m * ROWS + g] = fmaf(fdv[m * ROWS + g], a0, -msum[m * ROWS + g]);
        rd[m * ROWS + g + 8] = fmaf(fdv[m * ROWS + g + 8], a1, -msum[m * ROWS + g + 8]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    __syncwarp();
    kb += MM_CWARPS;
    while (kb >= NB) {
      kb -= NB;
      ++k;
      if (++slot == a.nslots) slot = 0, phase ^= 1;
    }
  }
}

// ---------------------------------------------------------------- Q6_K
// Q6_K on the same integer tensor-core path.  The 6-bit codes of a 32-weight
// unit (Q6KTensor.cs:105-124: low nibble from ql, 2 high bits from qh) are
// rebuilt per A fragment from the ql word and the re-packed high-bit plane of
// the device layout: lane tig owns ql word tig (elements 8 tig .. 8 tig + 7),
// even elements at k = 4 tig + i, odd at k = 16 + 4 tig + i.  A unit carries two
// int8 scales (elements 0..15 and 16..31, lanes tig 0-1 and 2-3), so the B
// operand holds six digit columns: columns 0..2 the digits of x for the first
// half (zero at the second half's k positions), 3..5 for the second half.  One
// MMA gives both halves' integer sums, each multiplied by its integer scale:
//   sum_k w_k x_k = d 2^(e-22) sum_h sc_h (A_h 65536 + B_h 256 + C_h)
//                   - 32 d sum_h sc_h (sum of x over half h).
// x is 22-bit fixed point relative to its 256-element block's largest |x|.
constexpr int SCW2 = 9;  // int2 per scale row (8 units + 1): rows g = 0..7 on distinct banks

// MX x rows (1, 2 or 4): six digit columns per x row (column 6 m + 3 h + q),
// NMMA = ceil(6 MX / 8) MMAs per unit share the A fragments.
template <int MX>
__global__ void __launch_bounds__(MM_THREADS, 1) gemv_mma_q6k_kernel(const __grid_constant__ MmaArgs a) {
  constexpr int NC = 6 * MX;                // B columns: 6 per x row
  // stored columns per unit: one row keeps all six (the other half's zeros
  // included, no selects); more rows keep each lane's own half (3 per row)
  constexpr int NS = MX == 1 ? 6 : 3 * MX;
  constexpr int NMMA = (NC + 7) / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = (uint64_t*)smem;  // [8]
  uint64_t* empty = full + 8;        // [8]
  uint2* planes = (uint2*)(smem + a.plane_offset);  // [U][NS][4 tig] (even, odd) digit words, then hsum, bexp
  float* red = (float*)(smem + a.red_offset);       // [nslots][NB][MX][ROWS] block partials
  uint8_t* scw_all = smem + a.scw_offset;           // per warp: int2 [ROWS][SCW2], msum [MX][ROWS], fdv [MX][ROWS]
  uint8_t* ring = smem + a.ring_offset;
  const int K = a.K, U = K >> 5, NB = K >> 8, M = a.M;
  const uint32_t rbytes = (uint32_t)NB * Q6K_BODY_BYTES;
  const int rs = a.row_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ngroups = (a.N + ROWS - 1) / ROWS;
  const int g0 = (int)((int64_t)ngroups * blockIdx.x / gridDim.x);
  const int g1 = (int)((int64_t)ngroups * (blockIdx.x + 1) / gridDim.x);
  const int nst = g1 - g0;
  float* hsum = (float*)(planes + U * NS * 4);  // [MX][U][2] sum of x over each 16-element half
  float* bexp = hsum + MX * 2 * U;              // [MX][NB] 2^(e-22) of the block
  if (tid == 0) {
    for (int i = 0; i < a.nslots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NB);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == MM_CWARPS) {
    auto issue = [&](int k) {
      const int slot = k % a.nslots;
      const int row = (g0 + k) * ROWS;
      const int n = min(ROWS, a.N - row);
      if (lane == 0) mbar_expect_tx(&full[slot], (uint32_t)n * (rbytes + a.abytes));
      __syncwarp();
      if (lane < n) {
        uint8_t* dst = ring + slot * a.slot_bytes + lane * rs;
        bulk_g2s(dst, a.w + (int64_t)(row + lane) * rbytes, rbytes, &full[slot]);
        bulk_g2s(dst + rbytes, a.aux + (int64_t)(row + lane) * a.aux_stride, a.abytes, &full[slot]);
      }
    };
    int next = 0;
    for (; next < min(nst, a.nslots); ++next) issue(next);
    if (lane == 0) asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // y may be the previous kernel's output
    int slot = 0;
    uint32_t phase = 0;
    for (int k = 0; k < nst; ++k) {
      if (!mbar_wait_bounded(&empty[slot], phase, a.status)) return;
      const int row0 = (g0 + k) * ROWS;
      const int n = min(ROWS, a.N - row0);
      for (int t = lane; t < M * ROWS; t += 32) {
        const int m = t / ROWS, r = t - m * ROWS;
        if (r < n) {
          const float* rd = red + (slot * NB * MX + m) * ROWS + r;
          float s = 0.f;
          for (int b = 0; b < NB; ++b) s += rd[b * MX * ROWS];
          float* dst = a.y + (int64_t)m * a.ldy + row0 + r;
          *dst = a.accumulate ? *dst + s : s;
        }
      }
      __syncwarp();
      if (next < nst) issue(next++);
      if (++slot == a.nslots) slot = 0, phase ^= 1;
    }
    return;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // ---- digit columns of x: one warp per (x row, 256-element block), four lanes per unit
  for (int it = warp; it < M * NB; it += MM_CWARPS) {
    const int m = it / NB, blk = it - m * NB;
    const int u = blk * 8 + (lane >> 2), p = lane & 3;
    const float4* xp = (const float4*)(a.x + (int64_t)m * K + 32 * u + 8 * p);
    const float4 v0 = __ldcg(xp), v1 = __ldcg(xp + 1);
    const float xv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float amax = 0.f, sx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      amax = fmaxf(amax, fabsf(xv[i]));
      sx += xv[i];
    }
    sx += __shfl_xor_sync(0xffffffffu, sx, 1);  // the lane pair of one 16-element half
    amax = warp_max(amax);
    int ex = 0;
    frexpf(amax, &ex);  // amax < 2^ex
    const float up = ldexpf(1.f, 22 - ex);
    uint32_t pw[2][3] = {};  // [even / odd][digit]
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int X = amax > 0.f ? __float2int_rn(xv[i] * up) : 0;  // |X| <= 2^22
      const int c = ((X + 128) & 255) - 128;
      const int X1 = (X - c) >> 8;
      const int b = ((X1 + 128) & 255) - 128;
      const int hi = (X1 - b) >> 8;
      const int eo = i & 1, sh = 8 * (i >> 1);
      pw[eo][0] |= (uint32_t)(hi & 255) << sh;
      pw[eo][1] |= (uint32_t)(b & 255) << sh;
      pw[eo][2] |= (uint32_t)(c & 255) << sh;
    }
    // digit q of row m at stored column 3 m + q; the B column of the other half
    // is zero at this lane's k positions (applied by the consumer lanes)
    const int half = p >> 1;
    if (MX == 1) {
      uint2* d = planes + u * NS * 4 + p;
#pragma unroll
      for (int col = 0; col < 6; ++col)
        d[4 * col] = (col / 3) == half ? make_uint2(pw[0][col % 3], pw[1][col % 3]) : make_uint2(0u, 0u);
    } else {
      uint2* d = planes + (u * NS + 3 * m) * 4 + p;
#pragma unroll
      for (int q = 0; q < 3; ++q) d[4 * q] = make_uint2(pw[0][q], pw[1][q]);
    }
    if ((p & 1) == 0) hsum[(m * U + u) * 2 + half] = sx;
    if (lane == 0) bexp[m * NB + blk] = ldexpf(1.f, ex - 22);
  }
  csync();
  const int g = lane >> 2, tig = lane & 3;
  const int hshift = 4 * (tig & 1);  // high-bit byte fields of this lane's elements
  // lane (g, tig), MMA mi: B column 8 mi + g (a real column when past 6 M);
  // C column c = 8 mi + 2 tig + e: x row c / 6, half (c % 6) / 3, digit c % 3
  const uint2* pl[NMMA];
  bool bon[NMMA];  // this lane's half is the column's half (else the B words are zero)
#pragma unroll
  for (int mi = 0; mi < NMMA; ++mi) {
    const int c = 8 * mi + g;
    const bool real = c < 6 * M;
    if (MX == 1) {
      pl[mi] = planes + (real ? c : 0) * 4 + tig;
      bon[mi] = true;
    } else {
      pl[mi] = planes + (real ? 3 * (c / 6) + c % 3 : 0) * 4 + tig;
      bon[mi] = real && ((c % 6) / 3) == (tig >> 1);
    }
  }
  int2* scw = (int2*)(scw_all + warp * (ROWS * SCW2 * 8 + 2 * MX * ROWS * 4));
  float* msum = (float*)(scw + ROWS * SCW2);  // [MX][ROWS]
  float* fdv = msum + MX * ROWS;              // [MX][ROWS]
  const int sr = lane >> 1, shh = lane & 1;  // scale decode: row, half of the units
  int k = 0, kb = warp, slot = 0;
  uint32_t phase = 0;
  while (kb >= NB) {
    kb -= NB;
    ++k;
    if (++slot == a.nslots) slot = 0, phase ^= 1;
  }
  for (; k < nst;) {
    if (!mbar_wait_bounded(&full[slot], phase, a.status)) return;
    const uint8_t* st = ring + slot * a.slot_bytes;
    const uint8_t* blk0 = st + kb * Q6K_BODY_BYTES;
    const int row0 = (g0 + k) * ROWS;
    const int n = min(ROWS, a.N - row0);
    {
      // int8 scales of units 4 shh .. 4 shh + 3 of row sr, the x-sum correction and d
      const uint8_t* rp = st + min(sr, n - 1) * rs;
      const int2 sc8 = *(const int2*)(rp + kb * Q6K_BODY_BYTES + 192 + 8 * shh);
      const float d = __half2float(__ushort_as_half(*(const unsigned short*)(rp + rbytes + 2 * kb)));
      const uint32_t sw[2] = {(uint32_t)sc8.x, (uint32_t)sc8.y};
      float sa[4], sb[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int ia = (int)(int8_t)((sw[jj >> 1] >> (16 * (jj & 1))) & 0xFF);
        const int ib = (int)(int8_t)((sw[jj >> 1] >> (16 * (jj & 1) + 8)) & 0xFF);
        scw[sr * SCW2 + 4 * shh + jj] = make_int2(ia, ib);
        sa[jj] = (float)ia;
        sb[jj] = (float)ib;
      }
#pragma unroll
      for (int m = 0; m < MX; ++m) {
        if (m >= M) break;
        const float* hs = hsum + (m * U + kb * 8 + 4 * shh) * 2;
        float mpart = 0.f;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          mpart = fmaf(sa[jj], hs[2 * jj], mpart);
          mpart = fmaf(sb[jj], hs[2 * jj + 1], mpart);
        }
        mpart += __shfl_xor_sync(0xffffffffu, mpart, 1);
        if (shh == 0) {
          msum[m * ROWS + sr] = 32.f * d * mpart;
          fdv[m * ROWS + sr] = d * bexp[m * NB + kb];
        }
      }
    }
    __syncwarp();
    const uint8_t* rg = blk0 + min(g, n - 1) * rs;
    const uint8_t* rg8 = blk0 + min(g + 8, n - 1) * rs;
    const int ustride = NS * 4;
    const int ub = kb * 8 * ustride;
    int t[NMMA][4];
#pragma unroll
    for (int mi = 0; mi < NMMA; ++mi) t[mi][0] = t[mi][1] = t[mi][2] = t[mi][3] = 0;
#pragma unroll
    for (int j0 = 0; j0 < 8; j0 += 4) {
      int dd[4][NMMA][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int jj = j0 + j;
        const uint32_t w0 = *(const uint32_t*)(rg + 16 * jj + 4 * tig);
        const uint32_t w1 = *(const uint32_t*)(rg8 + 16 * jj + 4 * tig);
        const uint32_t W0 = *(const uint32_t*)(rg + 128 + 8 * jj + 4 * (tig >> 1)) >> hshift;
        const uint32_t W1 = *(const uint32_t*)(rg8 + 128 + 8 * jj + 4 * (tig >> 1)) >> hshift;
        // even elements: low nibbles + high bits at byte bits 4-5; odd: high nibbles + bits 6-7 of the field
        const uint32_t e0 = (w0 & 0x0F0F0F0Fu) | ((W0 << 4) & 0x30303030u);
        const uint32_t e1 = (w1 & 0x0F0F0F0Fu) | ((W1 << 4) & 0x30303030u);
        const uint32_t o0 = ((w0 >> 4) & 0x0F0F0F0Fu) | ((W0 << 2) & 0x30303030u);
        const uint32_t o1 = ((w1 >> 4) & 0x0F0F0F0Fu) | ((W1 << 2) & 0x30303030u);
#pragma unroll
        for (int mi = 0; mi < NMMA; ++mi) {
          const uint2 b = pl[mi][ub + jj * ustride];
          mma_u8s8(dd[j][mi][0], dd[j][mi][1], dd[j][mi][2], dd[j][mi][3], e0, e1, o0, o1, bon[mi] ? b.x : 0u,
                   bon[mi] ? b.y : 0u);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int2 s0 = scw[g * SCW2 + j0 + j], s1 = scw[(g + 8) * SCW2 + j0 + j];
#pragma unroll
        for (int mi = 0; mi < NMMA; ++mi)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const bool hb = (((8 * mi + 2 * tig + e) % 6) / 3) != 0;  // second half's scale
            t[mi][e] += (hb ? s0.y : s0.x) * dd[j][mi][e];
            t[mi][2 + e] += (hb ? s1.y : s1.x) * dd[j][mi][2 + e];
          }
      }
    }
    float v0[MX], v1[MX];
#pragma unroll
    for (int m = 0; m < MX; ++m) v0[m] = v1[m] = 0.f;
#pragma unroll
    for (int mi = 0; mi < NMMA; ++mi)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = 8 * mi + 2 * tig + e;
        const float wgt = (c % 3 == 0) ? 65536.f : (c % 3 == 1 ? 256.f : 1.f);
#pragma unroll
        for (int m = 0; m < MX; ++m)
          if (c / 6 == m && c < 6 * M) {
            v0[m] = fmaf((float)t[mi][e], wgt, v0[m]);
            v1[m] = fmaf((float)t[mi][2 + e], wgt, v1[m]);
          }
      }
    float* rd = red + (slot * NB + kb) * MX * ROWS;
#pragma unroll
    for (int m = 0; m < MX; ++m) {
      if (m >= M) break;
      float a0 = v0[m], a1 = v1[m];
      a0 += __shfl_xor_sync(0xffffffffu, a0, 1);
      a1 += __shfl_xor_sync(0xffffffffu, a1, 1);
      a0 += __shfl_xor_sync(0xffffffffu, a0, 2);
      a1 += __shfl_xor_sync(0xffffffffu, a1, 2);
      if (tig == 0) {
        rd[m * ROWS + g] = fmaf(fdv[m * ROWS + g], a0, -msum[m * ROWS + g]);
        rd[m * ROWS + g + 8] = fmaf(fdv[m * ROWS + g + 8], a1, -msum[m * ROWS + g + 8]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    __syncwarp();
    kb += MM_CWARPS;
    while (kb >= NB) {
      kb -= NB;
      ++k;
      if (++slot == a.nslots) slot = 0, phase ^= 1;
    }
  }
}

}  // namespace

namespace {
template <int MX>
int launch_q4k_mx(const DevWeight& W, const float* x, int M, float* y, int ldy, int accumulate, int* status,
                  cudaStream_t st, int* n_launch) {
  const int K = W.K(), N = W.N(), U = K / 32;
  MmaArgs a;
  a.w = (const uint8_t*)W.data;
  a.x = x;
  a.y = y;
  a.N = N;
  a.K = K;
  a.M = M;
  a.ldy = ldy;
  a.accumulate = accumulate;
  a.status = status;
  const int NB = K / 256;
  const int64_t rbytes = (int64_t)NB * Q4K_BLOCK_BYTES;
  // row stride in 16-byte units odd modulo 8 words-per-row quads: rows g = 0..7
  // land on distinct bank quads
  a.row_stride = (int)rbytes + ((NB % 2 == 0) ? 16 : 32);
  a.slot_bytes = (int64_t)ROWS * a.row_stride;
  a.plane_offset = 256;
  a.red_offset = a.plane_offset + U * 3 * MX * 4 * 8 + MX * (U + NB) * 4;
  a.red_offset = (a.red_offset + 15) / 16 * 16;
  int optin = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const int64_t fixed = a.red_offset + MM_CWARPS * (ROWS * SCW + 2 * MX * ROWS) * 4 + 128;
  const int64_t per_slot = a.slot_bytes + (int64_t)NB * MX * ROWS * 4;
  const int nslots = (int)std::min<int64_t>(8, (optin - 1024 - fixed) / per_slot);
  if (nslots < 2) return SM_ERR_UNSUPPORTED;
  a.nslots = nslots;
  a.scw_offset = a.red_offset + nslots * NB * MX * ROWS * 4;
  a.ring_offset = a.scw_offset + MM_CWARPS * (ROWS * SCW + 2 * MX * ROWS) * 4;
  a.ring_offset = (a.ring_offset + 127) / 128 * 128;
  const size_t smem = (size_t)a.ring_offset + (size_t)a.nslots * a.slot_bytes;
  if ((int64_t)smem > optin - 1024) return SM_ERR_UNSUPPORTED;
  static bool attr_set[64] = {};
  if (dev < 64 && !attr_set[dev]) {
    SM_CUDA_TRY(
        cudaFuncSetAttribute(gemv_mma_q4k_kernel<MX>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - 1024));
    attr_set[dev] = true;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int ngroups = (N + ROWS - 1) / ROWS;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(sms, ngroups));
  cfg.blockDim = dim3(MM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SM_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_mma_q4k_kernel<MX>, a));
  if (n_launch) ++*n_launch;
  return SM_OK;
}
}  // namespace

int launch_gemv_mma_q4k_rows(const DevWeight& W, const float* x, int M, float* y, int ldy, int accumulate,
                             int* status, cudaStream_t st, int* n_launch) {
  if (W.scheme != SM_Q4_K || W.layout != SM_LAYOUT_INTENDED || M < 1) return SM_ERR_UNSUPPORTED;
  const int K = W.K();
  if (K % 256 || K / 32 > 1024) return SM_ERR_UNSUPPORTED;
  // passes of up to four x rows (the digit planes of four rows fit shared memory)
  // the widest pass whose digit planes and two ring slots fit shared memory
  int width = 4;
  for (int m0 = 0; m0 < M;) {
    const int mm = std::min(width, M - m0);
    const float* xm = x + (int64_t)m0 * K;
    float* ym = y + (int64_t)m0 * ldy;
    int rc;
    if (mm == 1)
      rc = launch_q4k_mx<1>(W, xm, 1, ym, ldy, accumulate, status, st, n_launch);
    else if (mm == 2)
      rc = launch_q4k_mx<2>(W, xm, 2, ym, ldy, accumulate, status, st, n_launch);
    else
      rc = launch_q4k_mx<4>(W, xm, mm, ym, ldy, accumulate, status, st, n_launch);
    if (rc == SM_ERR_UNSUPPORTED && mm > 1) {
      width = mm > 2 ? 2 : 1;
      continue;
    }
    if (rc != SM_OK) return rc;
    m0 += mm;
  }
  return SM_OK;
}

int launch_gemv_mma_q4k(const DevWeight& W, const float* x, float* y, int accumulate, int* status, cudaStream_t st,
                        int* n_launch) {
  return launch_gemv_mma_q4k_rows(W, x, 1, y, W.N(), accumulate, status, st, n_launch);
}

namespace {
template <int MX>
int launch_q6k_mx(const DevWeight& W, const float* x, int M, float* y, int ldy, int accumulate, int* status,
                  cudaStream_t st, int* n_launch) {
  const int K = W.K(), N = W.N(), U = K / 32;
  MmaArgs a;
  a.w = (const uint8_t*)W.data;
  a.aux = (const uint16_t*)W.aux;
  a.aux_stride = W.aux_stride;
  a.abytes = W.aux_stride * 2;
  if (a.abytes % 16) return SM_ERR_UNSUPPORTED;
  a.x = x;
  a.y = y;
  a.N = N;
  a.K = K;
  a.M = M;
  a.ldy = ldy;
  a.accumulate = accumulate;
  a.status = status;
  const int NB = K / 256;
  const int64_t rbytes = (int64_t)NB * Q6K_BODY_BYTES;
  // staged row = body + d row; stride an odd number of 16-byte units so rows
  // g = 0..7 of a fragment load fall on distinct bank quads
  int rs = (int)(rbytes + a.abytes);
  if ((rs / 16) % 2 == 0) rs += 16;
  a.row_stride = rs;
  a.slot_bytes = (int64_t)ROWS * a.row_stride;
  a.plane_offset = 256;
  a.red_offset = a.plane_offset + U * (MX == 1 ? 6 : 3 * MX) * 4 * 8 + MX * (2 * U + NB) * 4;
  a.red_offset = (a.red_offset + 15) / 16 * 16;
  int optin = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const int64_t scw_bytes = (int64_t)MM_CWARPS * (ROWS * SCW2 * 8 + 2 * MX * ROWS * 4);
  const int64_t fixed = a.red_offset + scw_bytes + 128;
  const int64_t per_slot = a.slot_bytes + (int64_t)NB * MX * ROWS * 4;
  const int nslots = (int)std::min<int64_t>(8, (optin - 1024 - fixed) / per_slot);
  if (nslots < 2) return SM_ERR_UNSUPPORTED;
  a.nslots = nslots;
  a.scw_offset = a.red_offset + nslots * NB * MX * ROWS * 4;
  a.ring_offset = a.scw_offset + (int)scw_bytes;
  a.ring_offset = (a.ring_offset + 127) / 128 * 128;
  const size_t smem = (size_t)a.ring_offset + (size_t)a.nslots * a.slot_bytes;
  if ((int64_t)smem > optin - 1024) return SM_ERR_UNSUPPORTED;
  static bool attr_set[64] = {};
  if (dev < 64 && !attr_set[dev]) {
    SM_CUDA_TRY(
        cudaFuncSetAttribute(gemv_mma_q6k_kernel<MX>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - 1024));
    attr_set[dev] = true;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int ngroups = (N + ROWS - 1) / ROWS;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(sms, ngroups));
  cfg.blockDim = dim3(MM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SM_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_mma_q6k_kernel<MX>, a));
  if (n_launch) ++*n_launch;
  return SM_OK;
}
}  // namespace

int launch_gemv_mma_q6k_rows(const DevWeight& W, const float* x, int M, float* y, int ldy, int accumulate,
                             int* status, cudaStream_t st, int* n_launch) {
  if (W.scheme != SM_Q6_K || W.layout != SM_LAYOUT_INTENDED || W.aux_stride <= 0 || M < 1)
    return SM_ERR_UNSUPPORTED;
  const int K = W.K();
  if (K % 256 || K / 32 > 1024) return SM_ERR_UNSUPPORTED;
  // the widest pass whose digit planes and two ring slots fit shared memory
  int width = 4;
  for (int m0 = 0; m0 < M;) {
    const int mm = std::min(width, M - m0);
    const float* xm = x + (int64_t)m0 * K;
    float* ym = y + (int64_t)m0 * ldy;
    int rc;
    if (mm == 1)
      rc = launch_q6k_mx<1>(W, xm, 1, ym, ldy, accumulate, status, st, n_launch);
    else if (mm == 2)
      rc = launch_q6k_mx<2>(W, xm, 2, ym, ldy, accumulate, status, st, n_launch);
    else
      rc = launch_q6k_mx<4>(W, xm, mm, ym, ldy, accumulate, status, st, n_launch);
    if (rc == SM_ERR_UNSUPPORTED && mm > 1) {
      width = mm > 2 ? 2 : 1;
      continue;
    }
    if (rc != SM_OK) return rc;
    m0 += mm;
  }
  return SM_OK;
}

int launch_gemv_mma_q6k(const DevWeight& W, const float* x, float* y, int accumulate, int* status, cudaStream_t st,
                        int* n_launch) {
  return launch_gemv_mma_q6k_rows(W, x, 1, y, W.N(), accumulate, status, st, n_launch);
}

}  // namespace sm
