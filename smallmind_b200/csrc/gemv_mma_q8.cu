// Decode GEMV (M = 1) for Q8_0 and Q4_0 on the integer tensor-core path.
//
// Weights: int8 codes (Q8_0) or two's-complement nibbles packed by index (Q4_0,
// Q4Tensor.cs:119-143), fp32 scales per block of `block_size` elements
// (a multiple of 32) in row-padded aux rows.  w = q * scale (Q8Tensor.cs:151,
// Q4Tensor.cs:150-179).
//
// One mma.sync.m16n8k32 (s8 x s8 -> s32) covers one 32-element unit of 16
// rows.  Lane (g, tig) supplies 8 elements of the unit for rows g and g + 8:
//   Q8_0: elements 8 tig .. 8 tig + 7 (8 contiguous code bytes): the first four
//         at k = 4 tig + i, the last four at k = 16 + 4 tig + i;
//   Q4_0: the 4 code bytes 4 tig .. 4 tig + 3 = elements 8 tig .. 8 tig + 7:
//         even elements (low nibbles, sign-extended to bytes) at k = 4 tig + i,
//         odd elements (high nibbles) at k = 16 + 4 tig + i.
// The B operand holds x in the same k order as three signed 8-bit digits of a
// 22-bit fixed-point value relative to its 256-element block's largest |x|
// (columns 0..2), so the digit sums are exact integers.  Per unit and row the
// fp32 scale multiplies the combined digit sums; the 256-element block's power
// of two is applied once per item.
//
// Schedule as in gemv_mma.cu: one persistent CTA per SM owns a range of 16-row
// tiles; warp 15 (of 24) bulk-copies each row and its scale row into a padded
// ring slot and later sums the tile's block partials in block order
// (deterministic); the other warps take (tile, 256-element block) items.
#include <algorithm>

#include "common.cuh"
#include "gemv1.cuh"
#include "mbar.cuh"
#include "mma_i8.cuh"

namespace sm {
namespace {

constexpr int Q8_THREADS = 768;
constexpr int Q8_CWARPS = Q8_THREADS / 32 - 1;
constexpr int Q8_CT = Q8_CWARPS * 32;
constexpr int Q8_ROWS = 16;

__device__ __forceinline__ void q8_csync() { asm volatile("bar.sync 1, %0;" ::"n"(Q8_CT) : "memory"); }

// D = A B, m16n8k32, A s8 (row), B s8 (col), zero accumulator input
__device__ __forceinline__ void mma_s8s8(int& d0, int& d1, int& d2, int& d3, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  const int z = 0;
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(z));
}

// four two's-complement nibbles (one per byte, in bits 0-3) -> four int8
__device__ __forceinline__ uint32_t sext_nibbles(uint32_t v) {
  // per byte: (v ^ 8 | 128) - 8 stays in [120, 135] (no borrow), ^ 128 gives v - 8 mod 256
  return (((v & 0x0F0F0F0Fu) ^ 0x88888888u) - 0x08080808u) ^ 0x80808080u;
}

struct Q8Args {
  const uint8_t* w = nullptr;
  const float* aux = nullptr;  // row-padded scales
  const float* x = nullptr;
  float* y = nullptr;
  int N = 0, K = 0, accumulate = 0, block_size = 32;
  int aux_stride = 0, abytes = 0;
  int nslots = 2, row_stride = 0;
  int64_t slot_bytes = 0;
  int plane_offset = 0, red_offset = 0, ring_offset = 0;
  int* status = nullptr;
};

template <int FMT>
__global__ void __launch_bounds__(Q8_THREADS, 1) gemv_mma_q80_kernel(const __grid_constant__ Q8Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = (uint64_t*)smem;  // [8]
  uint64_t* empty = full + 8;        // [8]
  uint2* planes = (uint2*)(smem + a.plane_offset);  // [U][3][4 tig] digit words (k lo, k hi)
  float* red = (float*)(smem + a.red_offset);       // [nslots][NB][ROWS] block partials
  uint8_t* ring = smem + a.ring_offset;
  const int K = a.K, U = K >> 5, NB = K >> 8;
  constexpr int UB = FMT == SM_Q8_0 ? 32 : 16;  // code bytes per unit
  const uint32_t rbytes = (uint32_t)U * UB;
  const int rs = a.row_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ngroups = (a.N + Q8_ROWS - 1) / Q8_ROWS;
  const int g0 = (int)((int64_t)ngroups * blockIdx.x / gridDim.x);
  const int g1 = (int)((int64_t)ngroups * (blockIdx.x + 1) / gridDim.x);
  const int nst = g1 - g0;
  float* bexp = (float*)(planes + U * 3 * 4);  // [NB] 2^(e-22) of each block
  if (tid == 0) {
    for (int i = 0; i < a.nslots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NB);  // one arrival per (tile, block) item
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == Q8_CWARPS) {
    // producer: rows and their scale rows into the padded ring (before the PDL
    // wait: the weights do not depend on the previous kernel); once a tile's
    // items have all arrived, its block partials are summed in block order
    auto issue = [&](int k) {
      const int slot = k % a.nslots;
      const int row = (g0 + k) * Q8_ROWS;
      const int n = min(Q8_ROWS, a.N - row);
      if (lane == 0) mbar_expect_tx(&full[slot], (uint32_t)n * (rbytes + a.abytes));
      __syncwarp();
      if (lane < n) {
        uint8_t* dst = ring + slot * a.slot_bytes + lane * rs;
        bulk_g2s(dst, a.w + (int64_t)(row + lane) * rbytes, rbytes, &full[slot]);
        bulk_g2s(dst + rbytes, (const uint8_t*)a.aux + (int64_t)(row + lane) * a.abytes, a.abytes, &full[slot]);
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
      const int row0 = (g0 + k) * Q8_ROWS;
      const int n = min(Q8_ROWS, a.N - row0);
      if (lane < n) {
        const float* rd = red + slot * NB * Q8_ROWS + lane;
        float s = 0.f;
        for (int b = 0; b < NB; ++b) s += rd[b * Q8_ROWS];
        float* dst = a.y + row0 + lane;
        *dst = a.accumulate ? *dst + s : s;
      }
      __syncwarp();
      if (next < nst) issue(next++);
      if (++slot == a.nslots) slot = 0, phase ^= 1;
    }
    return;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // ---- digit columns of x: one warp per 256-element block, four lanes per unit
  for (int blk = warp; blk < NB; blk += Q8_CWARPS) {
    const int u = blk * 8 + (lane >> 2), p = lane & 3;
    const float4* xp = (const float4*)(a.x + 32 * u + 8 * p);
    const float4 v0 = __ldcg(xp), v1 = __ldcg(xp + 1);
    const float xv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(xv[i]));
    amax = warp_max(amax);
    const int ex = block_exp(amax);  // amax < 2^ex
    const float up = pow2i(22 - ex);
    int X[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) X[i] = __float2int_rn(xv[i] * up);  // |X| <= 2^22
    uint32_t pw[2][3];  // [k lo / k hi][digit hi, b, c]
    if (FMT == SM_Q8_0) {
      digits4(X[0], X[1], X[2], X[3], pw[0][0], pw[0][1], pw[0][2]);
      digits4(X[4], X[5], X[6], X[7], pw[1][0], pw[1][1], pw[1][2]);
    } else {
      digits4(X[0], X[2], X[4], X[6], pw[0][0], pw[0][1], pw[0][2]);  // even elements
      digits4(X[1], X[3], X[5], X[7], pw[1][0], pw[1][1], pw[1][2]);  // odd elements
    }
    uint2* d = planes + (u * 3) * 4 + p;
#pragma unroll
    for (int q = 0; q < 3; ++q) d[4 * q] = make_uint2(pw[0][q], pw[1][q]);
    if (lane == 0) bexp[blk] = pow2i(ex - 22);
  }
  q8_csync();
  const int g = lane >> 2, tig = lane & 3;
  // C columns 2 tig, 2 tig + 1: digit hi, b (tig 0), c (tig 1); tig 2, 3 hold no column
  const float fA = tig == 0 ? 65536.f : (tig == 1 ? 1.f : 0.f);
  const float fB = tig == 0 ? 256.f : 0.f;
  const uint2* pl = planes + (g < 3 ? g : 0) * 4 + tig;
  const int spb = a.block_size >> 5;  // units per scale block
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
    const int row0 = (g0 + k) * Q8_ROWS;
    const int n = min(Q8_ROWS, a.N - row0);
    const uint8_t* r0 = st + min(g, n - 1) * rs;
    const uint8_t* r1 = st + min(g + 8, n - 1) * rs;
    const float* sc0 = (const float*)(r0 + rbytes);
    const float* sc1 = (const float*)(r1 + rbytes);
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int j0 = 0; j0 < 8; j0 += 4) {
      int dd[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int u = kb * 8 + j0 + j;
        const uint2 b = pl[u * 12];
        uint32_t a0, a1, a2, a3;
        if (FMT == SM_Q8_0) {
          const uint2 w0 = *(const uint2*)(r0 + u * 32 + 8 * tig);
          const uint2 w1 = *(const uint2*)(r1 + u * 32 + 8 * tig);
          a0 = w0.x, a2 = w0.y, a1 = w1.x, a3 = w1.y;
        } else {
          const uint32_t w0 = *(const uint32_t*)(r0 + u * 16 + 4 * tig);
          const uint32_t w1 = *(const uint32_t*)(r1 + u * 16 + 4 * tig);
          a0 = sext_nibbles(w0), a2 = sext_nibbles(w0 >> 4);
          a1 = sext_nibbles(w1), a3 = sext_nibbles(w1 >> 4);
        }
        mma_s8s8(dd[j][0], dd[j][1], dd[j][2], dd[j][3], a0, a1, a2, a3, b.x, b.y);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int si = (kb * 8 + j0 + j) / spb;
        acc0 = fmaf(sc0[si], fmaf((float)dd[j][0], fA, (float)dd[j][1] * fB), acc0);
        acc1 = fmaf(sc1[si], fmaf((float)dd[j][2], fA, (float)dd[j][3] * fB), acc1);
      }
    }
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    if (tig == 0) {
      const float e = bexp[kb];
      float* rd = red + (slot * NB + kb) * Q8_ROWS;
      rd[g] = acc0 * e;
      rd[g + 8] = acc1 * e;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    __syncwarp();
    kb += Q8_CWARPS;
    while (kb >= NB) {
      kb -= NB;
      ++k;
      if (++slot == a.nslots) slot = 0, phase ^= 1;
    }
  }
}

template <int FMT>
int launch_q80(const DevWeight& W, const float* x, float* y, int accumulate, int* status, cudaStream_t st,
               int* n_launch) {
  const int K = W.K(), N = W.N(), U = K / 32, NB = K / 256;
  Q8Args a;
  a.w = (const uint8_t*)W.data;
  a.aux = (const float*)W.aux;
  a.aux_stride = W.aux_stride;
  a.abytes = W.aux_stride * 4;
  a.block_size = W.block_size;
  a.x = x;
  a.y = y;
  a.N = N;
  a.K = K;
  a.accumulate = accumulate;
  a.status = status;
  const int64_t rbytes = (int64_t)U * (FMT == SM_Q8_0 ? 32 : 16);
  int rs = (int)(rbytes + a.abytes);  // an odd number of 16-byte units: rows g = 0..7 on distinct bank quads
  if ((rs / 16) % 2 == 0) rs += 16;
  a.row_stride = rs;
  a.slot_bytes = (int64_t)Q8_ROWS * rs;
  a.plane_offset = 256;
  a.red_offset = (a.plane_offset + U * 3 * 4 * 8 + NB * 4 + 15) / 16 * 16;
  int optin = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const int64_t per_slot = a.slot_bytes + (int64_t)NB * Q8_ROWS * 4;
  const int nslots = (int)std::min<int64_t>(8, (optin - 1024 - a.red_offset - 128) / per_slot);
  if (nslots < 2) return SM_ERR_UNSUPPORTED;
  a.nslots = nslots;
  a.ring_offset = (a.red_offset + nslots * NB * Q8_ROWS * 4 + 127) / 128 * 128;
  const size_t smem = (size_t)a.ring_offset + (size_t)nslots * a.slot_bytes;
  if ((int64_t)smem > optin - 1024) return SM_ERR_UNSUPPORTED;
  static bool attr_set[64] = {};
  if (dev < 64 && !attr_set[dev]) {
    SM_CUDA_TRY(cudaFuncSetAttribute(gemv_mma_q80_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     optin - 1024));
    attr_set[dev] = true;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int ngroups = (N + Q8_ROWS - 1) / Q8_ROWS;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(sms, ngroups));
  cfg.blockDim = dim3(Q8_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SM_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_mma_q80_kernel<FMT>, a));
  if (n_launch) ++*n_launch;
  return SM_OK;
}

}  // namespace

int launch_gemv_mma_q80(const DevWeight& W, const float* x, float* y, int accumulate, int* status, cudaStream_t st,
                        int* n_launch) {
  if ((W.scheme != SM_Q8_0 && W.scheme != SM_Q4_0) || W.layout != SM_LAYOUT_INTENDED) return SM_ERR_UNSUPPORTED;
  const int K = W.K();
  // whole 256-element blocks; scale blocks of whole units that divide the row;
  // 16-byte-padded scale rows (one bulk copy each)
  if (K % 256 || K / 32 > 1024 || W.block_size % 32 || K % W.block_size || W.aux_stride <= 0 ||
      (W.aux_stride * 4) % 16 || W.aux_bpr != K / W.block_size)
    return SM_ERR_UNSUPPORTED;
  if (W.scheme == SM_Q8_0) return launch_q80<SM_Q8_0>(W, x, y, accumulate, status, st, n_launch);
  return launch_q80<SM_Q4_0>(W, x, y, accumulate, status, st, n_launch);
}

}  // namespace sm
