// Streaming decode GEMV (M = 1): one persistent CTA per SM walks a contiguous
// range of weight rows, which TMA bulk copies (cp.async.bulk + mbarrier) bring
// into a ring of shared-memory stages while the CTA computes on earlier
// stages.  The first stages are requested before waiting on the previous
// kernel (programmatic dependent launch), so weight streaming overlaps that
// kernel's tail.
//
// Thread t owns one 32-weight unit u = t % U of K (U = K/32) for every row,
// and keeps the matching 32 activations (RMS-normalised when a gamma is given)
// in registers for the whole launch.  Threads t / U = 0..P-1 split the rows of
// a stage.  Each thread writes one partial per (row, unit); a warp then sums a
// row's U partials in a fixed order (deterministic) and applies the epilogue.
//
// Dequant arithmetic per unit is the exact byte-permute form of gemv1.cu
// (Unit<FMT>::dot), reading the packed unit from shared memory.
#include <algorithm>

#include "common.cuh"
#include "gemv1.cuh"
#include "gemv_units.cuh"
#include "mbar.cuh"

namespace sm {
namespace {

constexpr int ST_THREADS = 512;
constexpr int ST_WARPS = ST_THREADS / 32;
constexpr int MAX_STAGE_ROWS = 16;  // rows in one stage (GLU: gate + up rows)

__device__ __forceinline__ int64_t row_bytes_of(int fmt, int K) {
  switch (fmt) {
    case SM_Q4_K: return (int64_t)(K >> 8) * Q4K_BLOCK_BYTES;
    case SM_Q6_K: return (int64_t)(K >> 8) * Q6K_BODY_BYTES;
    case SM_Q8_0: return K;
    default: return K >> 1;
  }
}

struct CtaWork {
  int si;          // segment
  int r0, r1;      // rows [r0, r1) of the segment (GLU: output rows)
  int rb;          // rows per stage (GLU: output rows per stage)
  int nstages;
  int64_t rbytes;  // bytes of one weight row
};

__device__ __forceinline__ CtaWork cta_work(const StreamArgs& a) {
  CtaWork w;
  int si = 0;
  while (si + 1 < a.g.nseg && (int)blockIdx.x >= a.cta_begin[si + 1]) ++si;
  const GemvSeg& s = a.g.seg[si];
  const int nct = a.cta_count[si], i = blockIdx.x - a.cta_begin[si];
  // even row boundaries (RoPE pairs stay in one CTA and one stage)
  const int pairs = (s.rows + 1) / 2;
  w.si = si;
  w.r0 = min(s.rows, 2 * (int)((int64_t)pairs * i / nct));
  w.r1 = min(s.rows, 2 * (int)((int64_t)pairs * (i + 1) / nct));
  w.rb = a.stage_rows[si];
  w.nstages = (w.r1 - w.r0 + w.rb - 1) / w.rb;
  w.rbytes = row_bytes_of(s.fmt, a.g.K);
  return w;
}

__device__ __forceinline__ void issue_stage(const StreamArgs& a, const CtaWork& w, int k, uint8_t* slot,
                                            uint64_t* bar) {
  const GemvSeg& s = a.g.seg[w.si];
  const int row = w.r0 + k * w.rb;
  const int n = min(w.rb, w.r1 - row);
  const uint32_t bytes = (uint32_t)(n * w.rbytes);
  const bool glu = s.mode == GEMV_GLU;
  mbar_expect_tx(bar, glu ? 2 * bytes : bytes);
  bulk_g2s(slot, s.data + row * w.rbytes, bytes, bar);
  if (glu) bulk_g2s(slot + w.rb * w.rbytes, s.data2 + row * w.rbytes, bytes, bar);
}

template <int FMT>
__device__ __forceinline__ float unit_dot_smem(const GemvSeg& s, const uint8_t* rowp, int grow, int u, int K,
                                               bool up, const float* xr, float xa, float xb) {
  typename Unit<FMT>::Raw raw;
  Unit<FMT>::load_row(s, rowp, grow, u, K, up, raw);
  return Unit<FMT>::dot(raw, u & 7, xr, xa, xb);
}

// Warp 15 produces (bulk copies into the ring), warps 0..14 consume.  full[s]
// completes when a stage's bytes have landed; empty[s] when every consumer
// warp is done with it.  Partials of every row of the CTA stay in shared
// memory and are reduced once at the end.
template <int FA, int FB>
__global__ void __launch_bounds__(ST_THREADS, 1) gemv_stream_kernel(const __grid_constant__ StreamArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int CONS_WARPS = ST_WARPS - 1, CONS = CONS_WARPS * 32;
  const int K = a.g.K, U = K >> 5, P = CONS / U;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const CtaWork w = cta_work(a);
  const GemvSeg& s = a.g.seg[w.si];
  const bool glu = s.mode == GEMV_GLU;
  const int srows = glu ? 2 * w.rb : w.rb;  // weight rows held by one stage
  const int64_t stage_bytes = (int64_t)srows * w.rbytes;
  const int NS = a.nslots;
  const int nout = w.r1 - w.r0;             // output rows of this CTA
  uint64_t* full = (uint64_t*)smem;         // [8]
  uint64_t* empty = full + 8;               // [8]
  float* red = (float*)(smem + 128);        // [ST_WARPS + 4]
  float* part = red + ST_WARPS + 4;         // [(glu ? 2 : 1) * rows of this CTA][U]
  uint8_t* ring = smem + a.ring_offset;
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CONS_WARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == CONS_WARPS) {
    // ---------------- producer: weights do not depend on the previous kernel
    if (lane == 0)
      for (int k = 0; k < min(NS, w.nstages); ++k) issue_stage(a, w, k, ring + k * stage_bytes, &full[k]);
    if (s.aux) {  // block scales / Q6_K d of this CTA's rows into L2
      const int64_t per_row = (s.fmt == SM_Q6_K) ? (K >> 8) * 2 : (int64_t)K / s.bs * 4;
      for (int m = 0; m < (glu ? 2 : 1); ++m) {
        const uint8_t* base = (const uint8_t*)(m ? s.aux2 : s.aux) + w.r0 * per_row;
        for (int64_t off = lane * 128; off < nout * per_row; off += 32 * 128)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(base + off));
      }
    }
  }
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // this thread's unit of x in registers (RMS-normalised if gamma is set)
  const int u = tid % U, ph = tid / U;
  float xr[32];
  {
    const float4* xp = (const float4*)(a.g.x + 32 * u);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 v = xp[c];
      xr[4 * c] = v.x; xr[4 * c + 1] = v.y; xr[4 * c + 2] = v.z; xr[4 * c + 3] = v.w;
    }
  }
  if (a.g.gamma) {
    float ss = 0.f;
    if (ph == 0 && warp < CONS_WARPS)
#pragma unroll
      for (int i = 0; i < 32; ++i) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < ST_WARPS; ++i) tot += red[i];
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), a.g.eps)));
    const float4* gp = (const float4*)(a.g.gamma + 32 * u);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 gv = gp[c];
      xr[4 * c] = __fmul_rn(gv.x, __fmul_rn(xr[4 * c], inv));
      xr[4 * c + 1] = __fmul_rn(gv.y, __fmul_rn(xr[4 * c + 1], inv));
      xr[4 * c + 2] = __fmul_rn(gv.z, __fmul_rn(xr[4 * c + 2], inv));
      xr[4 * c + 3] = __fmul_rn(gv.w, __fmul_rn(xr[4 * c + 3], inv));
    }
  }
  float xa = 0.f, xb = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    xa += xr[i];
    xb += xr[16 + i];
  }
  bool ok = true;
  if (warp == CONS_WARPS) {
    // ---------------- producer, steady state: refill a slot once every consumer warp released it
    if (lane == 0)
      for (int k = NS; k < w.nstages; ++k) {
        const int slot = k % NS;
        if (!mbar_wait_bounded(&empty[slot], ((k / NS) - 1) & 1, a.status)) {
          ok = false;
          break;
        }
        issue_stage(a, w, k, ring + slot * stage_bytes, &full[slot]);
      }
  } else {
    // ---------------- consumers
    for (int k = 0; k < w.nstages; ++k) {
      const int slot = k % NS;
      if (!mbar_wait_bounded(&full[slot], (k / NS) & 1, a.status)) {
        ok = false;
        break;
      }
      const uint8_t* st = ring + slot * stage_bytes;
      const int row0 = w.r0 + k * w.rb;
      const int n = min(w.rb, w.r1 - row0);
      const int nrows = glu ? 2 * n : n;
      if (ph < P) {
        for (int sr = ph; sr < nrows; sr += P) {
          const bool up = glu && sr >= n;
          const int lr = up ? sr - n : sr;
          const uint8_t* rowp = st + (int64_t)(up ? w.rb + lr : lr) * w.rbytes;
          float v;
          if (FA == FB || s.fmt == FA)
            v = unit_dot_smem<FA>(s, rowp, row0 + lr, u, K, up, xr, xa, xb);
          else
            v = unit_dot_smem<FB>(s, rowp, row0 + lr, u, K, up, xr, xa, xb);
          // part rows: output row (row0 - r0 + lr), up rows after all gate rows
          part[((up ? nout : 0) + (row0 - w.r0) + lr) * U + u] = v;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
  }
  if (!ok) red[ST_WARPS] = 1.f;
  __syncthreads();
  if (red[ST_WARPS] == 1.f) return;  // a stage timed out (status already set)
  // ---------------- reduction (fixed order) and epilogue
  const bool pairs = s.mode == GEMV_ROPE_Q || s.mode == GEMV_ROPE_K_CACHE;
  const int nitems = pairs ? (nout + 1) / 2 : nout;
  for (int it = warp; it < nitems; it += ST_WARPS) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    int rows_in[2] = {it, 0};
    int nr = 1;
    if (glu) {
      rows_in[1] = nout + it;
      nr = 2;
    } else if (pairs) {
      rows_in[0] = 2 * it;
      rows_in[1] = 2 * it + 1;
      nr = (2 * it + 1 < nout) ? 2 : 1;
    }
    for (int q = 0; q < nr; ++q) {
      float t = 0.f;
      for (int uu = lane; uu < U; uu += 32) t += part[rows_in[q] * U + uu];
      v[q] = warp_sum(t);
    }
    if (lane == 0) {
      if (glu)
        group_store<2>(a.g, s, w.r0 + it, v);  // v = {gate, up}
      else if (pairs)
        group_store<2>(a.g, s, (w.r0 >> 1) + it, v);
      else
        group_store<1>(a.g, s, w.r0 + it, v);
    }
  }
}

}  // namespace

int launch_gemv_stream(const GemvArgs& g, int* status, cudaStream_t st, int* n_launch) {
  StreamArgs a;
  a.g = g;
  a.status = status;
  const int K = g.K, U = K / 32;
  if (U > ST_THREADS - 32 || U < 1) return SM_ERR_UNSUPPORTED;
  for (int i = 0; i < g.nseg; ++i)
    if (g.seg[i].mode == GEMV_ROPE_Q || g.seg[i].mode == GEMV_ROPE_K_CACHE)
      if (g.head_dim % 2) return SM_ERR_UNSUPPORTED;
  // formats
  int fa = g.seg[0].fmt, fb = fa;
  for (int i = 1; i < g.nseg; ++i) {
    if (g.seg[i].fmt == fa || g.seg[i].fmt == fb) continue;
    if (fb != fa) return SM_ERR_UNSUPPORTED;
    fb = g.seg[i].fmt;
  }
  if (fb == SM_Q4_K && fa == SM_Q6_K) std::swap(fa, fb);
  void* kern = nullptr;
  if (fa == fb) {
    switch (fa) {
      case SM_Q4_K: kern = (void*)gemv_stream_kernel<SM_Q4_K, SM_Q4_K>; break;
      case SM_Q6_K: kern = (void*)gemv_stream_kernel<SM_Q6_K, SM_Q6_K>; break;
      case SM_Q8_0: kern = (void*)gemv_stream_kernel<SM_Q8_0, SM_Q8_0>; break;
      case SM_Q4_0: kern = (void*)gemv_stream_kernel<SM_Q4_0, SM_Q4_0>; break;
    }
  } else if (fa == SM_Q4_K && fb == SM_Q6_K) {
    kern = (void*)gemv_stream_kernel<SM_Q4_K, SM_Q6_K>;
  }
  if (!kern) return SM_ERR_UNSUPPORTED;
  // CTAs per segment in proportion to its bytes; stage rows sized to ~12 KB
  int64_t bytes[GEMV_MAX_SEG], total = 0;
  for (int i = 0; i < g.nseg; ++i) {
    const GemvSeg& s = g.seg[i];
    int64_t rb;
    switch (s.fmt) {
      case SM_Q4_K: rb = (int64_t)(K / 256) * Q4K_BLOCK_BYTES; break;
      case SM_Q6_K: rb = (int64_t)(K / 256) * Q6K_BODY_BYTES; break;
      case SM_Q8_0: rb = K; break;
      default: rb = K / 2; break;
    }
    if (rb % 16) return SM_ERR_UNSUPPORTED;
    const int mult = s.mode == GEMV_GLU ? 2 : 1;
    bytes[i] = rb * s.rows * mult;
    total += bytes[i];
    int r = (int)std::max<int64_t>(1, 12288 / (rb * mult));
    r = std::min(r, MAX_STAGE_ROWS / mult);
    if (s.mode == GEMV_ROPE_Q || s.mode == GEMV_ROPE_K_CACHE) r = std::max(2, r & ~1);
    a.stage_rows[i] = r;
  }
  const int nct = 148;
  int used = 0;
  for (int i = 0; i < g.nseg; ++i) {
    int c = (int)std::max<int64_t>(1, (int64_t)nct * bytes[i] / std::max<int64_t>(1, total));
    c = std::min(c, (g.seg[i].rows + 1) / 2);
    a.cta_begin[i] = used;
    a.cta_count[i] = c;
    used += c;
  }
  // ring: as many stages as fit in ~150 KB
  int64_t max_stage = 0, max_part = 0;
  for (int i = 0; i < g.nseg; ++i) {
    const int mult = g.seg[i].mode == GEMV_GLU ? 2 : 1;
    const int64_t rbytes = bytes[i] / g.seg[i].rows / mult;
    max_stage = std::max<int64_t>(max_stage, rbytes * a.stage_rows[i] * mult);
    const int pairs = (g.seg[i].rows + 1) / 2;
    const int cta_rows = 2 * ((pairs + a.cta_count[i] - 1) / a.cta_count[i]) + 2;
    max_part = std::max<int64_t>(max_part, (int64_t)cta_rows * mult * U * 4);
  }
  a.ring_offset = (int)(((128 + 4 * (ST_WARPS + 4) + max_part) + 127) / 128 * 128);
  const int64_t ring_budget = 200 * 1024 - a.ring_offset;
  if (ring_budget < 2 * max_stage) return SM_ERR_UNSUPPORTED;
  a.nslots = (int)std::min<int64_t>(8, ring_budget / max_stage);
  const size_t smem = (size_t)a.ring_offset + (size_t)a.nslots * max_stage;
  static bool attr_set[64][8][8] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev][fa][fb]) {
    SM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_set[dev][fa][fb] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(used);
  cfg.blockDim = dim3(ST_THREADS);
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
