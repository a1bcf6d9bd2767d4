// Causal GQA attention with the reference's Pade softmax.
//
// The reference normalises with FastExp(s*scale - rowmax) (OptimizedOps.cs:48-94,
// MathUtils.cs:20-32).  That rational function is not multiplicative, so the
// usual online-softmax rescaling (exp(a-b) = exp(a)/exp(b)) would change the
// result.  Both kernels therefore find the exact row max first and only then
// exponentiate: decode = scores pass (split over the context) + exp/PV pass
// + combine; prefill = a max pass and an exp/PV pass over key tiles.
#include <cfloat>

#include <cooperative_groups.h>

#include <cstdlib>

#include "common.cuh"

namespace sm {
namespace {

constexpr int DEC_CHUNK = 64;   // keys per decode CTA
constexpr int DEC_THREADS = 128;
constexpr int MAXG = 16;        // max q heads per kv head handled by the decode kernels

// K/V addressing: element d of key j of kv head g = base + j*row_stride + g*head_stride + d.

// ---------------------------------------------------------------- decode
// grid (chunks, nKv, B).  8 lanes per key (8 dims each), 16 keys per CTA pass.
template <int HD>
__global__ void __launch_bounds__(DEC_THREADS) decode_scores_kernel(
    const float* __restrict__ q, int q_stride, const float* __restrict__ kc, int64_t seq_stride, int64_t row_stride,
    int64_t head_stride, const int* __restrict__ lens, const int* __restrict__ seq_map, int nH, int nKv,
    float scale, float* __restrict__ scores, int max_ctx, float* __restrict__ cmax, int nchunks) {
  const int chunk = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int len = lens[b];
  const int j0 = chunk * DEC_CHUNK;
  const int G = nH / nKv;
  if (j0 >= len) return;
  const int j1 = min(len, j0 + DEC_CHUNK);
  __shared__ float qs[MAXG][HD];
  for (int t = threadIdx.x; t < G * HD; t += DEC_THREADS) {
    const int h = t / HD, d = t - h * HD;
    qs[h][d] = q[(int64_t)b * q_stride + (g * G + h) * HD + d];
  }
  __syncthreads();
  const int sub = threadIdx.x & 7;          // dims sub*8 .. +8 (HD=64)
  const int kslot = threadIdx.x >> 3;       // 16 key slots
  constexpr int DPL = HD / 8;
  float lmax[MAXG];
#pragma unroll
  for (int h = 0; h < MAXG; ++h) lmax[h] = -FLT_MAX;
  const float* kb = kc + (int64_t)(seq_map ? seq_map[b] : b) * seq_stride + (int64_t)g * head_stride;
  for (int j = j0 + kslot; j < j1 + ((j1 - j0 + 15) / 16) * 16 - (j1 - j0); j += 16) {
    const bool valid = j < j1;
    float kv[DPL];
    if (valid) {
      const float4* kp = (const float4*)(kb + (int64_t)j * row_stride + sub * DPL);
#pragma unroll
      for (int i = 0; i < DPL / 4; ++i) {
        float4 t = __ldg(kp + i);
        kv[4 * i] = t.x; kv[4 * i + 1] = t.y; kv[4 * i + 2] = t.z; kv[4 * i + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < DPL; ++i) kv[i] = 0.f;
    }
    for (int h = 0; h < G; ++h) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) s = fmaf(qs[h][sub * DPL + i], kv[i], s);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      if (valid) {
        if (sub == 0) scores[((int64_t)b * nH + g * G + h) * max_ctx + j] = s;
        lmax[h] = fmaxf(lmax[h], __fmul_rn(s, scale));
      }
    }
  }
  // chunk max per head
  __shared__ float red[MAXG][DEC_THREADS / 32];
  for (int h = 0; h < G; ++h) {
    float m = warp_max(lmax[h]);
    if ((threadIdx.x & 31) == 0) red[h][threadIdx.x >> 5] = m;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    float m = -FLT_MAX;
    for (int w = 0; w < DEC_THREADS / 32; ++w) m = fmaxf(m, red[threadIdx.x][w]);
    cmax[((int64_t)b * nH + g * G + threadIdx.x) * nchunks + chunk] = m;
  }
}

// grid (chunks, nKv, B): e_j = FastExp(s_j*scale - max) and partial sum / e.V.
template <int HD>
__global__ void __launch_bounds__(DEC_THREADS) decode_pv_kernel(
    const float* __restrict__ vc, int64_t seq_stride, int64_t row_stride, int64_t head_stride,
    const int* __restrict__ lens, const int* __restrict__ seq_map, int nH, int nKv, float scale,
    const float* __restrict__ scores, int max_ctx,
    const float* __restrict__ cmax, int nchunks, float* __restrict__ pacc, float* __restrict__ psum) {
  const int chunk = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int len = lens[b];
  const int j0 = chunk * DEC_CHUNK;
  const int G = nH / nKv;
  if (j0 >= len) return;
  const int j1 = min(len, j0 + DEC_CHUNK);
  const int used = (len + DEC_CHUNK - 1) / DEC_CHUNK;
  __shared__ float es[MAXG][DEC_CHUNK];
  __shared__ float gmax[MAXG];
  if (threadIdx.x < G) {
    float m = -FLT_MAX;
    const float* cm = cmax + ((int64_t)b * nH + g * G + threadIdx.x) * nchunks;
    for (int c = 0; c < used; ++c) m = fmaxf(m, cm[c]);
    gmax[threadIdx.x] = m;
  }
  __syncthreads();
  for (int t = threadIdx.x; t < G * DEC_CHUNK; t += DEC_THREADS) {
    const int h = t / DEC_CHUNK, jj = t - h * DEC_CHUNK;
    const int j = j0 + jj;
    float e = 0.f;
    if (j < j1) {
      const float s = scores[((int64_t)b * nH + g * G + h) * max_ctx + j];
      e = pade_exp(__fsub_rn(__fmul_rn(s, scale), gmax[h]));
    }
    es[h][jj] = e;
  }
  __syncthreads();
  // PV: thread -> (dim d = tid % HD, key phase = tid / HD)
  constexpr int PH = DEC_THREADS / HD;
  const int d = threadIdx.x % HD, ph = threadIdx.x / HD;
  float acc[MAXG];
#pragma unroll
  for (int h = 0; h < MAXG; ++h) acc[h] = 0.f;
  const float* vb = vc + (int64_t)(seq_map ? seq_map[b] : b) * seq_stride + (int64_t)g * head_stride;
  for (int j = j0 + ph; j < j1; j += PH) {
    const float v = __ldg(vb + (int64_t)j * row_stride + d);
    for (int h = 0; h < G; ++h) acc[h] = fmaf(es[h][j - j0], v, acc[h]);
  }
  __shared__ float part[PH][MAXG][HD];
  for (int h = 0; h < G; ++h) part[ph][h][d] = acc[h];
  __syncthreads();
  for (int t = threadIdx.x; t < G * HD; t += DEC_THREADS) {
    const int h = t / HD, dd = t - h * HD;
    float s = 0.f;
    for (int p = 0; p < PH; ++p) s += part[p][h][dd];
    pacc[(((int64_t)b * nH + g * G + h) * nchunks + chunk) * HD + dd] = s;
  }
  if (threadIdx.x < G) {
    float s = 0.f;
    for (int jj = 0; jj < j1 - j0; ++jj) s += es[threadIdx.x][jj];
    psum[((int64_t)b * nH + g * G + threadIdx.x) * nchunks + chunk] = s;
  }
}

// grid (nH, B): out = (sum_c pacc) * (1 / sum_c psum).
template <int HD>
__global__ void decode_combine_kernel(const int* __restrict__ lens, int nH, const float* __restrict__ pacc,
                                      const float* __restrict__ psum, int nchunks, float* __restrict__ out,
                                      int out_stride) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int used = (lens[b] + DEC_CHUNK - 1) / DEC_CHUNK;
  const int64_t bh = (int64_t)b * nH + h;
  float tot = 0.f;
  for (int c = 0; c < used; ++c) tot += psum[bh * nchunks + c];
  const float inv = __fdiv_rn(1.f, tot);
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float s = 0.f;
    for (int c = 0; c < used; ++c) s += pacc[(bh * nchunks + c) * HD + d];
    out[(int64_t)b * out_stride + h * HD + d] = s * inv;
  }
}

// ---------------------------------------------------------------- prefill
// One CTA per (64-query tile, q head); 256 threads as 16x16, 4x4 micro-tiles.
constexpr int PT = 64;

template <int HD>
__global__ void __launch_bounds__(256) prefill_attention_kernel(
    const float* __restrict__ q, int q_stride, const float* __restrict__ k, const float* __restrict__ v,
    int64_t row_stride, int64_t head_stride, float* __restrict__ out, int out_stride, int T, int S, int nH, int nKv,
    float scale) {
  const int tile = blockIdx.x, h = blockIdx.y;
  const int g = h / (nH / nKv);
  const int i0 = tile * PT;
  const int off = S - T;  // absolute position of query row 0
  extern __shared__ float sm_[];
  float* Qs = sm_;                    // [HD][PT+1]  (transposed: d-major)
  float* Ks = Qs + HD * (PT + 1);     // [HD][PT+1]
  float* Vs = Ks + HD * (PT + 1);     // [PT][HD]
  float* Ps = Vs + PT * HD;           // [PT][PT+1]
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  // load Q tile transposed
  for (int t = threadIdx.x; t < PT * HD; t += 256) {
    const int r = t / HD, d = t - r * HD;
    const int i = i0 + r;
    Qs[d * (PT + 1) + r] = i < T ? q[(int64_t)i * q_stride + h * HD + d] : 0.f;
  }
  const float* kb = k + (int64_t)g * head_stride;
  const float* vb = v + (int64_t)g * head_stride;
  const int last_row = min(T, i0 + PT) - 1;
  const int kend = off + last_row + 1;  // keys [0, kend)
  float rmax[4] = {-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX};
  // ---- pass 1: row max of s*scale over the causal range
  for (int j0 = 0; j0 < kend; j0 += PT) {
    __syncthreads();
    for (int t = threadIdx.x; t < PT * HD; t += 256) {
      const int r = t / HD, d = t - r * HD;
      const int j = j0 + r;
      Ks[d * (PT + 1) + r] = j < kend ? kb[(int64_t)j * row_stride + d] : 0.f;
    }
    __syncthreads();
    float s[4][4] = {};
#pragma unroll 8
    for (int d = 0; d < HD; ++d) {
      float a[4], bb[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) a[x] = Qs[d * (PT + 1) + ty * 4 + x];
#pragma unroll
      for (int x = 0; x < 4; ++x) bb[x] = Ks[d * (PT + 1) + tx * 4 + x];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[r][c] = fmaf(a[r], bb[c], s[r][c]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int pos = off + i0 + ty * 4 + r;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = j0 + tx * 4 + c;
        if (j <= pos) rmax[r] = fmaxf(rmax[r], __fmul_rn(s[r][c], scale));
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) rmax[r] = fmaxf(rmax[r], __shfl_xor_sync(0xffffffffu, rmax[r], o));
  // ---- pass 2: e = FastExp(s*scale - max); O += e V; sum += e
  float o[4][4] = {};
  float rsum[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j0 = 0; j0 < kend; j0 += PT) {
    __syncthreads();
    for (int t = threadIdx.x; t < PT * HD; t += 256) {
      const int r = t / HD, d = t - r * HD;
      const int j = j0 + r;
      Ks[d * (PT + 1) + r] = j < kend ? kb[(int64_t)j * row_stride + d] : 0.f;
      Vs[r * HD + d] = j < kend ? vb[(int64_t)j * row_stride + d] : 0.f;
    }
    __syncthreads();
    float s[4][4] = {};
#pragma unroll 8
    for (int d = 0; d < HD; ++d) {
      float a[4], bb[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) a[x] = Qs[d * (PT + 1) + ty * 4 + x];
#pragma unroll
      for (int x = 0; x < 4; ++x) bb[x] = Ks[d * (PT + 1) + tx * 4 + x];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[r][c] = fmaf(a[r], bb[c], s[r][c]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int pos = off + i0 + ty * 4 + r;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = j0 + tx * 4 + c;
        const float e = (j <= pos) ? pade_exp(__fsub_rn(__fmul_rn(s[r][c], scale), rmax[r])) : 0.f;
        rsum[r] += e;
        Ps[(ty * 4 + r) * (PT + 1) + tx * 4 + c] = e;
      }
    }
    __syncthreads();
    // O[rows ty*4..][dims tx*4..] += P[rows][j] * V[j][dims]
#pragma unroll 8
    for (int jj = 0; jj < PT; ++jj) {
      float p[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) p[r] = Ps[(ty * 4 + r) * (PT + 1) + jj];
      const float4 vv = *(const float4*)(Vs + jj * HD + tx * 4);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        o[r][0] = fmaf(p[r], vv.x, o[r][0]);
        o[r][1] = fmaf(p[r], vv.y, o[r][1]);
        o[r][2] = fmaf(p[r], vv.z, o[r][2]);
        o[r][3] = fmaf(p[r], vv.w, o[r][3]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int o2 = 8; o2 > 0; o2 >>= 1) rsum[r] += __shfl_xor_sync(0xffffffffu, rsum[r], o2);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = i0 + ty * 4 + r;
    if (i >= T) continue;
    const float inv = __fdiv_rn(1.f, rsum[r]);
    float4 res = make_float4(o[r][0] * inv, o[r][1] * inv, o[r][2] * inv, o[r][3] * inv);
    *(float4*)(out + (int64_t)i * out_stride + h * HD + tx * 4) = res;
  }
}

// ---------------------------------------------------------------- decode, one launch
// A thread-block cluster of CL CTAs per (sequence, kv head).  Each CTA scores
// its slice of the context for the G query heads of the group (scores stay in
// shared memory), the CTAs exchange their slice maxima through distributed
// shared memory so every CTA exponentiates against the exact global row max
// (the Pade exp of the reference is not multiplicative), and the partial sums
// and e.V accumulators are reduced into CTA rank 0 the same way.  No global
// scratch, one launch.
// CL CTAs per cluster (1..16; 16 is a non-portable size): many CTAs per
// sequence for long contexts at small batch, one CTA per (sequence, kv head)
// when the batch alone fills the GPU.
constexpr int CT = 256;         // threads per CTA
constexpr int CMAXG = 8;        // q heads per kv head

template <int HD, int CL>
__global__ void __launch_bounds__(CT) decode_cluster_kernel(
    const float* __restrict__ q, int q_stride, const float* __restrict__ kc, const float* __restrict__ vc,
    int64_t seq_stride, int64_t row_stride, int64_t head_stride, const int* __restrict__ lens,
    const int* __restrict__ seq_map, int nH, int nKv, float scale, float* __restrict__ out, int out_stride,
    int chunk_cap) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int g = blockIdx.y, b = blockIdx.z;
  const int G = nH / nKv;
  extern __shared__ float sm_[];
  float* qs = sm_;                        // [CMAXG][HD]
  float* sc = qs + CMAXG * HD;            // [chunk_cap][CMAXG]: a key's scores of the group's heads side by side
  float* pacc = sc + CMAXG * chunk_cap;   // [CMAXG][HD]  this CTA's e.V
  float* stat = pacc + CMAXG * HD;        // [CMAXG] slice max, [CMAXG] slice sum
  float* part = stat + 2 * CMAXG;         // [CT/32][CMAXG][HD]
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int len = lens[b];
  const int per = (len + CL - 1) / CL;
  const int j0 = min(len, rank * per), j1 = min(len, j0 + per);
  const int n = j1 - j0;
  for (int t = threadIdx.x; t < G * HD; t += CT) {
    const int h = t / HD, d = t - h * HD;
    qs[h * HD + d] = q[(int64_t)b * q_stride + (g * G + h) * HD + d];
  }
  __syncthreads();
  const int64_t sbase = (int64_t)(seq_map ? seq_map[b] : b) * seq_stride + (int64_t)g * head_stride;
  const float* kb = kc + sbase;
  const float* vb = vc + sbase;
  // scores: 8 lanes per key (8 dims each), 32 keys per pass
  const int sub = threadIdx.x & 7, slot = threadIdx.x >> 3;
  constexpr int DPL = HD / 8;
  float lmax[CMAXG];
#pragma unroll
  for (int h = 0; h < CMAXG; ++h) lmax[h] = -FLT_MAX;
  const int passes = (n + 31) / 32;
  // the next pass's key slice is loaded before this pass's dot products (two passes in flight)
  float kn[DPL];
  auto load_k = [&](int pp, float (&dst)[DPL]) {
    const int j = pp * 32 + slot;
    if (j < n) {
      const float4* kp = (const float4*)(kb + (int64_t)(j0 + j) * row_stride + sub * DPL);
#pragma unroll
      for (int i = 0; i < DPL / 4; ++i) {
        const float4 t = __ldg(kp + i);
        dst[4 * i] = t.x; dst[4 * i + 1] = t.y; dst[4 * i + 2] = t.z; dst[4 * i + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < DPL; ++i) dst[i] = 0.f;
    }
  };
  if (passes > 0) load_k(0, kn);
  for (int p = 0; p < passes; ++p) {
    const int jj = p * 32 + slot;
    const bool valid = jj < n;
    float kv[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) kv[i] = kn[i];
    if (p + 1 < passes) load_k(p + 1, kn);
#pragma unroll
    for (int h = 0; h < CMAXG; ++h) {
      if (h >= G) break;
      const float4 qa = *(const float4*)&qs[h * HD + sub * DPL];
      const float4 qb = *(const float4*)&qs[h * HD + sub * DPL + 4];
      float s = 0.f;
      s = fmaf(qa.x, kv[0], s);
      s = fmaf(qa.y, kv[1], s);
      s = fmaf(qa.z, kv[2], s);
      s = fmaf(qa.w, kv[3], s);
      s = fmaf(qb.x, kv[4], s);
      s = fmaf(qb.y, kv[5], s);
      s = fmaf(qb.z, kv[6], s);
      s = fmaf(qb.w, kv[7], s);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      if (valid) {
        if (sub == 0) sc[jj * CMAXG + h] = s;
        lmax[h] = fmaxf(lmax[h], __fmul_rn(s, scale));
      }
    }
  }
  // slice max per head
  {
    float* wred = part;  // reuse [CT/32][CMAXG]
#pragma unroll
    for (int h = 0; h < CMAXG; ++h) {
      const float m = warp_max(lmax[h]);
      if ((threadIdx.x & 31) == 0) wred[(threadIdx.x >> 5) * CMAXG + h] = m;
    }
    __syncthreads();
    if (threadIdx.x < CMAXG) {
      float m = -FLT_MAX;
      for (int w = 0; w < CT / 32; ++w) m = fmaxf(m, wred[w * CMAXG + threadIdx.x]);
      stat[threadIdx.x] = m;
    }
  }
  cluster.sync();
  // global max of each head from every CTA's slice max (distributed shared memory)
  __shared__ float gmax[CMAXG];
  if (threadIdx.x < G) {
    float m = -FLT_MAX;
    for (int r = 0; r < CL; ++r) m = fmaxf(m, cluster.map_shared_rank(stat, r)[threadIdx.x]);
    gmax[threadIdx.x] = m;
  }
  __syncthreads();
  // e = FastExp(s*scale - max) in place (each thread keeps one head: CT is a multiple of CMAXG),
  // with this thread's share of the slice sum of its head
  float esum = 0.f;
  {
    const int h = threadIdx.x & (CMAXG - 1);
    if (h < G) {
      const float gm = gmax[h];
      for (int t = threadIdx.x; t < CMAXG * n; t += CT) {
        const float e = pade_exp(__fsub_rn(__fmul_rn(sc[t], scale), gm));
        sc[t] = e;
        esum += e;
      }
    }
  }
  __syncthreads();
  // e.V: 16 lanes per value row (4 dims each, one 16-byte load), 16 rows per pass;
  // lanes l and l + 16 of a warp hold the same dims and are merged by a shuffle
  constexpr int PH = CT / 32;
  static_assert(HD == 64, "e.V lane layout assumes head_dim 64");
  const int d4 = threadIdx.x & 15, pr = threadIdx.x >> 4;
  float4 acc[CMAXG];
#pragma unroll
  for (int h = 0; h < CMAXG; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int jj = pr; jj < n; jj += CT / 16) {
    const float4 v = __ldg((const float4*)(vb + (int64_t)(j0 + jj) * row_stride) + d4);
    const float4 ea = *(const float4*)&sc[jj * CMAXG], eb = *(const float4*)&sc[jj * CMAXG + 4];
    const float ev[CMAXG] = {ea.x, ea.y, ea.z, ea.w, eb.x, eb.y, eb.z, eb.w};
#pragma unroll
    for (int h = 0; h < CMAXG; ++h)
      if (h < G) {
        const float e = ev[h];
        acc[h].x = fmaf(e, v.x, acc[h].x);
        acc[h].y = fmaf(e, v.y, acc[h].y);
        acc[h].z = fmaf(e, v.z, acc[h].z);
        acc[h].w = fmaf(e, v.w, acc[h].w);
      }
  }
  {
    const int ph = threadIdx.x >> 5;
#pragma unroll
    for (int h = 0; h < CMAXG; ++h)
      if (h < G) {
        acc[h].x += __shfl_xor_sync(0xffffffffu, acc[h].x, 16);
        acc[h].y += __shfl_xor_sync(0xffffffffu, acc[h].y, 16);
        acc[h].z += __shfl_xor_sync(0xffffffffu, acc[h].z, 16);
        acc[h].w += __shfl_xor_sync(0xffffffffu, acc[h].w, 16);
        if ((threadIdx.x & 31) < 16) *(float4*)&part[(ph * CMAXG + h) * HD + 4 * d4] = acc[h];
      }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < G * HD; t += CT) {
    const int h = t / HD, dd = t - h * HD;
    float s = 0.f;
    for (int p = 0; p < PH; ++p) s += part[(p * CMAXG + h) * HD + dd];
    pacc[h * HD + dd] = s;
  }
  {
    // slice sum of each head: lanes of one head (lane & 7) merged by shuffles, then the warps
    esum += __shfl_xor_sync(0xffffffffu, esum, 8);
    esum += __shfl_xor_sync(0xffffffffu, esum, 16);
    __syncthreads();  // every thread is done reading part (the e.V partials)
    const int w = threadIdx.x >> 5, ln = threadIdx.x & 31;
    if (ln < CMAXG) part[w * CMAXG + ln] = esum;
    __syncthreads();
    if (threadIdx.x < G) {
      float s = 0.f;
      for (int ww = 0; ww < CT / 32; ++ww) s += part[ww * CMAXG + threadIdx.x];
      stat[CMAXG + threadIdx.x] = s;
    }
  }
  cluster.sync();
  // rank 0 reduces the slices and writes out = (sum e.V) / (sum e)
  if (rank == 0) {
    for (int t = threadIdx.x; t < G * HD; t += CT) {
      const int h = t / HD, dd = t - h * HD;
      float s = 0.f, tot = 0.f;
      for (int r = 0; r < CL; ++r) {
        s += cluster.map_shared_rank(pacc, r)[h * HD + dd];
        tot += cluster.map_shared_rank(stat, r)[CMAXG + h];
      }
      out[(int64_t)b * out_stride + (g * G + h) * HD + dd] = s * __fdiv_rn(1.f, tot);
    }
  }
  cluster.sync();  // keep every CTA's shared memory alive until rank 0 has read it
}

}  // namespace

size_t attention_decode_scratch_floats(int B, int nH, int max_ctx) {
  const int nchunks = (max_ctx + DEC_CHUNK - 1) / DEC_CHUNK;
  return (size_t)B * nH * max_ctx + (size_t)B * nH * nchunks * (2 + 64);
}

int launch_attention_decode(const float* q, int q_stride, const float* kc, const float* vc, int64_t seq_stride,
                            int64_t row_stride, int64_t head_stride, int max_ctx, float* out, int out_stride,
                            const int* lens, const int* seq_map, int B, int nH, int nKv, int hd, float* scratch,
                            size_t scratch_floats, cudaStream_t st, int* n_launch) {
  if (hd != 64) return fail(SM_ERR_UNSUPPORTED, "attention: head_dim must be 64");
  if (nH % nKv || nH / nKv > MAXG) return fail(SM_ERR_UNSUPPORTED, "attention: unsupported GQA group size");
  if (scratch_floats < attention_decode_scratch_floats(B, nH, max_ctx))
    return fail(SM_ERR_INVALID_ARG, "attention: scratch too small");
  const int nchunks = (max_ctx + DEC_CHUNK - 1) / DEC_CHUNK;
  float* scores = scratch;
  float* cmax = scores + (size_t)B * nH * max_ctx;
  float* psum = cmax + (size_t)B * nH * nchunks;
  float* pacc = psum + (size_t)B * nH * nchunks;
  const float scale = 1.0f / sqrtf((float)hd);
  dim3 grid(nchunks, nKv, B);
  decode_scores_kernel<64><<<grid, DEC_THREADS, 0, st>>>(q, q_stride, kc, seq_stride, row_stride, head_stride, lens,
                                                         seq_map, nH, nKv, scale, scores, max_ctx, cmax, nchunks);
  decode_pv_kernel<64><<<grid, DEC_THREADS, 0, st>>>(vc, seq_stride, row_stride, head_stride, lens, seq_map, nH, nKv, scale,
                                                     scores, max_ctx, cmax, nchunks, pacc, psum);
  decode_combine_kernel<64><<<dim3(nH, B), 64, 0, st>>>(lens, nH, pacc, psum, nchunks, out, out_stride);
  SM_CUDA_TRY(cudaGetLastError());
  if (n_launch) *n_launch += 3;
  return SM_OK;
}

// Single-launch cluster variant (no scratch).  Returns SM_ERR_UNSUPPORTED when
// the shape does not fit it (caller falls back to launch_attention_decode).
namespace {

template <int CL>
int launch_decode_cluster_cl(const float* q, int q_stride, const float* kc, const float* vc, int64_t seq_stride,
                             int64_t row_stride, int64_t head_stride, int max_ctx, float* out, int out_stride,
                             const int* lens, const int* seq_map, int B, int nH, int nKv, int hd, cudaStream_t st,
                             int* n_launch) {
  const int chunk_cap = (max_ctx + CL - 1) / CL;
  const size_t smem = sizeof(float) * (CMAXG * 64 * 2 + CMAXG * (size_t)chunk_cap + 2 * CMAXG + (CT / 32) * CMAXG * 64);
  if (smem > 200 * 1024 / 4) return SM_ERR_UNSUPPORTED;
  auto kern = decode_cluster_kernel<64, CL>;
  static bool attr_set[64] = {};
  static int cluster_ok[64] = {};  // 0 unknown, 1 usable, -1 not schedulable on this device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return SM_ERR_UNSUPPORTED;
  if (!attr_set[dev]) {
    if (CL > 8) SM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    SM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_set[dev] = true;
  }
  if (cluster_ok[dev] == 0) {
    cudaLaunchConfig_t probe = {};
    probe.gridDim = dim3(CL, 1, 1);
    probe.blockDim = dim3(CT);
    probe.dynamicSmemBytes = 200 * 1024 / 4;
    cudaLaunchAttribute pa[1];
    pa[0].id = cudaLaunchAttributeClusterDimension;
    pa[0].val.clusterDim.x = CL;
    pa[0].val.clusterDim.y = 1;
    pa[0].val.clusterDim.z = 1;
    probe.attrs = pa;
    probe.numAttrs = 1;
    int nclusters = 0;
    cudaError_t oe = cudaOccupancyMaxActiveClusters(&nclusters, (void*)kern, &probe);
    cluster_ok[dev] = (oe == cudaSuccess && nclusters > 0) ? 1 : -1;
    if (oe != cudaSuccess) cudaGetLastError();
  }
  if (cluster_ok[dev] < 0) return SM_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, nKv, B);
  cfg.blockDim = dim3(CT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const float scale = 1.0f / sqrtf((float)hd);
  SM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, q, q_stride, kc, vc, seq_stride, row_stride, head_stride, lens,
                                 seq_map, nH, nKv, scale, out, out_stride, chunk_cap));
  if (n_launch) *n_launch += 1;
  return SM_OK;
}

}  // namespace

// Single-launch cluster variant (no scratch).  Returns SM_ERR_UNSUPPORTED when
// the shape does not fit it (caller falls back to launch_attention_decode).
// Cluster size: as many CTAs per (sequence, kv head) as keep about two waves of
// CTAs on the GPU (16 for one sequence, 1 once the batch fills the SMs), and at
// least as many as the context's score rows need to fit shared memory.
int launch_attention_decode_cluster(const float* q, int q_stride, const float* kc, const float* vc,
                                    int64_t seq_stride, int64_t row_stride, int64_t head_stride, int max_ctx,
                                    float* out, int out_stride, const int* lens, const int* seq_map, int B, int nH,
                                    int nKv, int hd, cudaStream_t st, int* n_launch) {
  if (hd != 64 || nH % nKv || nH / nKv > CMAXG) return SM_ERR_UNSUPPORTED;
  {
    // SMALLMIND_ATTN_CLUSTER=0 selects the three-kernel split-context path
    const char* e = std::getenv("SMALLMIND_ATTN_CLUSTER");
    if (e && e[0] == '0') return SM_ERR_UNSUPPORTED;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int cl = 16;
  while (cl > 1 && (int64_t)cl * nKv * B > 2 * sms) cl >>= 1;
  auto fits = [&](int c) {
    const int64_t cap = (max_ctx + c - 1) / c;
    return sizeof(float) * (CMAXG * 64 * 2 + CMAXG * cap + 2 * CMAXG + (CT / 32) * CMAXG * 64) <= 200 * 1024 / 4;
  };
  while (cl < 16 && !fits(cl)) cl <<= 1;
  switch (cl) {
    case 1: return launch_decode_cluster_cl<1>(q, q_stride, kc, vc, seq_stride, row_stride, head_stride, max_ctx, out,
                                               out_stride, lens, seq_map, B, nH, nKv, hd, st, n_launch);
    case 2: return launch_decode_cluster_cl<2>(q, q_stride, kc, vc, seq_stride, row_stride, head_stride, max_ctx, out,
                                               out_stride, lens, seq_map, B, nH, nKv, hd, st, n_launch);
    case 4: return launch_decode_cluster_cl<4>(q, q_stride, kc, vc, seq_stride, row_stride, head_stride, max_ctx, out,
                                               out_stride, lens, seq_map, B, nH, nKv, hd, st, n_launch);
    case 8: return launch_decode_cluster_cl<8>(q, q_stride, kc, vc, seq_stride, row_stride, head_stride, max_ctx, out,
                                               out_stride, lens, seq_map, B, nH, nKv, hd, st, n_launch);
    default: return launch_decode_cluster_cl<16>(q, q_stride, kc, vc, seq_stride, row_stride, head_stride, max_ctx,
                                                 out, out_stride, lens, seq_map, B, nH, nKv, hd, st, n_launch);
  }
}

int launch_attention_prefill(const float* q, int q_stride, const float* k, const float* v, int64_t row_stride,
                             int64_t head_stride, float* out, int out_stride, int T, int S, int nH, int nKv, int hd,
                             cudaStream_t st, int* n_launch) {
  if (hd != 64) return fail(SM_ERR_UNSUPPORTED, "attention: head_dim must be 64");
  if (nH % nKv) return fail(SM_ERR_UNSUPPORTED, "attention: n_heads must be a multiple of n_kv_heads");
  if (T <= 0 || S < T) return fail(SM_ERR_SHAPE, "attention: need 0 < T <= S");
  {
    // tensor-core kernel (SMALLMIND_ATTN_TC=0 selects the CUDA-core one below)
    const char* e = std::getenv("SMALLMIND_ATTN_TC");
    if (!(e && e[0] == '0')) {
      const int rc = launch_attention_prefill_tc(q, q_stride, k, v, row_stride, head_stride, out, out_stride, T, S, nH,
                                                 nKv, hd, nullptr, st, n_launch);
      if (rc != SM_ERR_UNSUPPORTED) return rc;
    }
  }
  const size_t smem = sizeof(float) * (2 * 64 * (PT + 1) + PT * 64 + PT * (PT + 1));
  auto kern = prefill_attention_kernel<64>;
  SM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(ceil_div(T, PT), nH);
  const float scale = 1.0f / sqrtf((float)hd);
  kern<<<grid, 256, smem, st>>>(q, q_stride, k, v, row_stride, head_stride, out, out_stride, T, S, nH, nKv, scale);
  SM_CUDA_TRY(cudaGetLastError());
  if (n_launch) *n_launch += 1;
  return SM_OK;
}

}  // namespace sm
