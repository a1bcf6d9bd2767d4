// Persistent one-launch decode step for one sequence (bs1).
//
// A decode step is ~30 MB of weights per layer read once.  Launching a kernel
// per GEMV costs ~2 us of ramp-up and drain each on B200, which at these
// sizes is as long as the transfer itself, so this kernel runs the whole step
// (22 layers + LM head + argmax) as one launch: one CTA per SM, co-resident.
//
//  * Warp 15 of every CTA is a producer.  It walks the fixed schedule of the
//    step's GEMV rows assigned to this CTA (Q|K|V, O, gate/up, down for every
//    layer, then the head) and streams them into a ring of shared-memory
//    stages with cp.async.bulk + mbarrier.  It never waits for other CTAs, so
//    while the consumers sit in a grid barrier or do attention, the next
//    phases' weights keep arriving.
//  * Warps 0..14 consume: per phase they build their 32-element slice of the
//    input vector in registers (RMSNorm fused), compute per-(row, unit)
//    partials from the staged bytes (exact byte-permute dequant of
//    gemv_units.cuh), reduce rows in a fixed order and run the epilogue (RoPE
//    + KV append, residual add, SiLU gate).
//  * There is no grid-wide barrier.  Every vector one CTA hands to others (the
//    residual stream after each residual add, q, this token's K/V rows, the
//    attention chunk maxima / partials / output, the SiLU-gate output) is
//    written as 64-bit words {value, tag}, tag = (launch epoch, layer), and a
//    reader polls exactly the words it needs until their tags match.  A wait
//    therefore costs one L2 round trip after the last producer's store instead
//    of a release fence, an arrival, a counter poll and the reload of the data.
//    Single buffers suffice: a word is rewritten one layer later only by a CTA
//    whose own inputs needed (transitively) every reader's output of the layer
//    before; a CTA with no output rows in a phase does not read its input.
//  * Attention is three steps per (kv head, chunk) item: scores + chunk max,
//    Pade exp against the exact row max (all chunk maxima polled) and partial
//    e.V, then the combine of this CTA's slice of the outputs.
//  * Every wait is bounded (~2 s of clock64); on timeout the kernel records
//    SM_ERR_TIMEOUT in the context status word and returns.
#include <algorithm>
#include <cfloat>
#include <cstdlib>

#include "common.cuh"
#include "decode_mega.cuh"
#include "gemv_units.cuh"
#include "mbar.cuh"
#include "mma_i8.cuh"

namespace sm {
namespace {

constexpr int MT = 512;              // threads per CTA
constexpr int MW = MT / 32;          // warps
constexpr int CWARPS = MW - 1;       // consumer warps
constexpr int CT = CWARPS * 32;      // consumer threads
constexpr int MGMAX = 8;             // q heads per kv head
constexpr long long kSpin = 4000000000LL;

__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory"); }

// ---- tagged exchange words {float value (low 32 bits), uint32 tag (high 32 bits)}.
// An aligned 8-byte access is single-copy atomic, so a reader that sees the tag it
// expects also sees the value stored with it; gpu-scope relaxed accesses are served
// by L2, where every SM's stores meet.
typedef unsigned long long u64;
__device__ __forceinline__ u64 ll_ld(const u64* p) {
  u64 v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// two consecutive words (16-byte aligned): each 8-byte half is single-copy atomic
__device__ __forceinline__ ulonglong2 ll_ld2(const u64* p) {
  ulonglong2 v;
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void ll_st(u64* p, float v, unsigned tag) {
  const u64 w = ((u64)tag << 32) | (u64)__float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ bool ll_ok(u64 w, unsigned tag) { return (unsigned)(w >> 32) == tag; }
__device__ __forceinline__ float ll_val(u64 w) { return __uint_as_float((unsigned)w); }
__device__ __forceinline__ unsigned ll_tag(unsigned epoch, int layer) {
  return ((epoch + 1u) << 8) | ((unsigned)layer & 255u);
}

__host__ __device__ __forceinline__ int64_t row_bytes_fmt(int fmt, int K) {
  switch (fmt) {
    case SM_Q4_K: return (int64_t)(K >> 8) * Q4K_BLOCK_BYTES;
    case SM_Q6_K: return (int64_t)(K >> 8) * Q6K_BODY_BYTES;
    case SM_Q8_0: return K;
    default: return K >> 1;
  }
}

// bytes of one padded row of scales / d (0: the format has none)
__host__ __device__ __forceinline__ int64_t aux_row_bytes(const MegaSeg& s) {
  if (s.fmt == SM_Q4_K) return 0;
  return (int64_t)s.aux_stride * (s.fmt == SM_Q6_K ? 2 : 4);
}

// output rows per stage: as many as fit one ring slot (weights + scales, gate + up for GLU)
__device__ __forceinline__ int stage_rows(const MegaSeg& s, int K, int64_t slot_bytes) {
  const int mult = s.mode == GEMV_GLU ? 2 : 1;
  const unsigned per = (unsigned)(mult * (row_bytes_fmt(s.fmt, K) + aux_row_bytes(s)));
  return (int)max(1u, min(64u, (unsigned)slot_bytes / per));  // a slot and a row are far below 2^32 bytes
}

// rows of a segment for CTA i of n: whole row pairs, balanced
__device__ __forceinline__ void seg_rows(int rows, int i, int n, int& r0, int& r1) {
  const int pairs = (rows + 1) / 2;
  // pairs * (i + 1) stays far below 2^31 (rows < 2^20, at most 1024 CTAs)
  r0 = min(rows, 2 * (int)((unsigned)(pairs * i) / (unsigned)n));
  r1 = min(rows, 2 * (int)((unsigned)(pairs * (i + 1)) / (unsigned)n));
}

// MMA segments (Q4_K, Q6_K with row-padded d): the GEMV runs on the int8
// tensor-core path of gemv_mma.cu.  A stage is one 16-row tile of the CTA's rows
// (a gate and an up tile for GLU) over a range of 256-weight blocks; every row
// is its own bulk copy into a padded slot row (an odd number of 16-byte units,
// so the 8 rows of a fragment load fall on distinct bank quads), with the
// Q6_K d row after the largest block range.
struct MGeo {
  int nT, bb, abytes, NB, nkbs, rs, nch;
};

__device__ __forceinline__ bool mma_seg(const MegaArgs& a, const MegaSeg& s) {
  if (!a.use_mma) return false;
  return s.fmt == SM_Q4_K || (s.fmt == SM_Q6_K && s.aux_stride > 0 && (s.aux_stride * 2) % 16 == 0);
}

__device__ __forceinline__ MGeo mgeo(const MegaSeg& s, int K, int64_t slot_bytes) {
  MGeo m;
  m.nT = s.mode == GEMV_GLU ? 2 : 1;
  m.bb = s.fmt == SM_Q4_K ? Q4K_BLOCK_BYTES : Q6K_BODY_BYTES;
  m.abytes = s.fmt == SM_Q6_K ? s.aux_stride * 2 : 0;
  m.NB = K >> 8;
  auto stride = [&](int nk) {
    int rs = nk * m.bb + m.abytes;
    if (((rs >> 4) & 1) == 0) rs += 16;
    return rs;
  };
  for (m.nkbs = m.NB; m.nkbs > 1; --m.nkbs)
    if ((int64_t)m.nT * 16 * stride(m.nkbs) <= slot_bytes) break;
  m.rs = stride(m.nkbs);
  m.nch = (m.NB + m.nkbs - 1) / m.nkbs;
  return m;
}

// Q|K|V: CTAs [cb[s], cb[s+1]) take segment s, in proportion to its bytes, so
// every CTA runs one segment (one stage stream, one epilogue) per phase.
// segment rows of CTA `i` when CTAs [c0, c1) share the segment (none outside)
__device__ __forceinline__ void seg_rows_in(int rows, int i, int c0, int c1, int& r0, int& r1) {
  if (i < c0 || i >= c1) {
    r0 = r1 = 0;
    return;
  }
  seg_rows(rows, i - c0, c1 - c0, r0, r1);
}

// What a GEMV phase of the consumers needs besides the data: worked out by one
// thread while the CTA waits at the grid barrier before the phase.
struct SegPlan {
  const MegaSeg* s;
  const float* src;    // input vector
  const float* gamma;  // RMSNorm weight (null: none)
  float* amax_v;       // LM head: this CTA's argmax slot
  int* amax_i;
  int K, rb, r0, r1;   // inputs, dp4a stage rows, this CTA's output rows
  int mma;             // the int8 tensor-core path
  MGeo mg;
  int nst, red_n, red_off;  // MMA: stages, block partials, their offset in part
  int slot0, par0;          // ring slot and parity of the segment's first stage
  // tagged exchange: the input vector (null: `src` is a plain array), the residual
  // rows (ADD; null: res_plain), the output words (null: plain stores to s->y)
  const u64* src_ll;
  const u64* res_ll;
  const float* res_plain;
  u64* dst;
  unsigned src_tag, res_tag, dst_tag;
};

struct Shared {
  uint64_t full[16];
  uint64_t empty[16];
  MegaLayer lay[2];  // the consumers' copies of the layer table (layer l in lay[l & 1])
  SegPlan plan;      // the next GEMV phase
  float red[MW * MGMAX];
  float vec[4 * MGMAX];
  __align__(16) float kvrow[64];  // this token's K row of the attention item's kv head
  int flag[4];
  int consumed;
  int abort;
  volatile int phase;  // consumers' current GEMV phase (no-lookahead mode)
};

// ---------------------------------------------------------------- producer
// AM: every segment is on the tensor-core path (no dp4a staging code compiled in)
template <bool AM>
struct Producer {
  const MegaArgs& a;
  Shared& sh;
  uint8_t* ring;
  int64_t slot_bytes;
  int k = 0;  // stages issued
  bool ok = true;

  // MMA segment: 16-row tiles x block ranges, one bulk copy per row (and per d row)
  __device__ void mseg(const MegaSeg& s, int K, int r0, int r1) {
    const MGeo m = mgeo(s, K, slot_bytes);
    const int64_t rbytes = (int64_t)m.NB * m.bb;
    for (int row = r0; row < r1; row += 16) {
      const int n = min(16, r1 - row);
      for (int c = 0; c < m.nch; ++c) {
        const int kb0 = c * m.nkbs, nkb = min(m.nkbs, m.NB - kb0);
        const int slot = k % a.nslots;
        if (k >= a.nslots) {
          if (!mbar_wait_bounded(&sh.empty[slot], ((k / a.nslots) - 1) & 1, a.status) || sh.abort) {
            ok = false;
            return;
          }
        }
        uint8_t* dst = ring + slot * slot_bytes;
        const uint32_t per_row = (uint32_t)(nkb * m.bb + m.abytes);
        mbar_expect_tx(&sh.full[slot], (uint32_t)(m.nT * n) * per_row);
        for (int tt = 0; tt < m.nT; ++tt) {
          const uint8_t* src = tt ? s.data2 : s.data;
          const uint8_t* asrc = (const uint8_t*)(tt ? s.aux2 : s.aux);
          for (int r = 0; r < n; ++r) {
            uint8_t* d = dst + (tt * 16 + r) * m.rs;
            bulk_g2s(d, src + (row + r) * rbytes + kb0 * m.bb, (uint32_t)(nkb * m.bb), &sh.full[slot]);
            if (m.abytes) bulk_g2s(d + m.nkbs * m.bb, asrc + (int64_t)(row + r) * m.abytes, m.abytes, &sh.full[slot]);
          }
        }
        ++k;
      }
    }
  }

  __device__ void seg(const MegaSeg& s, int K, int /*rb*/, int phase, int c0 = 0, int c1 = -1) {
    if (!ok) return;
    const int rb = stage_rows(s, K, slot_bytes);
    if (!a.lookahead) {
      const long long t0 = clock64();
      while (sh.phase < phase && !sh.abort)
        if (clock64() - t0 > kSpin) {
          ok = false;
          return;
        }
    }
    int r0, r1;
    seg_rows_in(s.rows, blockIdx.x, c0, c1 < 0 ? (int)gridDim.x : c1, r0, r1);
    if (AM || mma_seg(a, s)) {
      mseg(s, K, r0, r1);
      return;
    }
    const int64_t rbytes = row_bytes_fmt(s.fmt, K);
    const bool glu = s.mode == GEMV_GLU;
    for (int row = r0; row < r1; row += rb) {
      const int n = min(rb, r1 - row);
      const int slot = k % a.nslots;
      if (k >= a.nslots) {
        if (!mbar_wait_bounded(&sh.empty[slot], ((k / a.nslots) - 1) & 1, a.status) || sh.abort) {
          ok = false;
          return;
        }
      }
      uint8_t* dst = ring + slot * slot_bytes;
      const uint32_t bytes = (uint32_t)(n * rbytes);
      const int64_t arb = aux_row_bytes(s);
      const uint32_t abytes = (uint32_t)(n * arb);
      const int nw = glu ? 2 : 1;
      mbar_expect_tx(&sh.full[slot], nw * (bytes + abytes));
      bulk_g2s(dst, s.data + row * rbytes, bytes, &sh.full[slot]);
      if (glu) bulk_g2s(dst + rb * rbytes, s.data2 + row * rbytes, bytes, &sh.full[slot]);
      if (abytes) {
        uint8_t* adst = dst + nw * rb * rbytes;
        bulk_g2s(adst, (const uint8_t*)s.aux + row * arb, abytes, &sh.full[slot]);
        if (glu) bulk_g2s(adst + rb * arb, (const uint8_t*)s.aux2 + row * arb, abytes, &sh.full[slot]);
      }
      ++k;
    }
  }
};

// ---------------------------------------------------------------- consumers
// AM: every GEMV segment runs on the tensor-core path (the dp4a path is not compiled in,
// which keeps the kernel's code small)
template <bool AM>
struct Consumer {
  const MegaArgs& a;
  Shared& sh;
  uint8_t* ring;
  int64_t slot_bytes;
  float* part;
  GemvArgs ep;  // epilogue context (RoPE / cache)
  int tid;
  int k = 0;  // stages consumed
  unsigned epoch = 0;  // this launch's exchange epoch (read once at the start)
  int ev = 0;
  int seq_v = 0;  // the sequence id (read once)
  int lx = 0;  // load_x calls (trace: the sub-steps of calls 4..11 go to events 900..)
  // Phase timestamps (SMALLMIND_MEGA_TRACE) exist only in a build with
  // -DSMALLMIND_MEGA_TRACE_BUILD: the kernel's code is kept small, because every
  // layer runs all of it once and what does not fit the SM's instruction cache
  // is fetched again each layer.
  __device__ void stamp_at(int e) {
#ifdef SMALLMIND_MEGA_TRACE_BUILD
    if (a.trace && tid == 0 && e < MEGA_TRACE_EVENTS) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      a.trace[(size_t)blockIdx.x * MEGA_TRACE_EVENTS + e] = t;
    }
#else
    (void)e;
#endif
  }
  __device__ void stamp() {
#ifdef SMALLMIND_MEGA_TRACE_BUILD
    if (a.trace && tid == 0 && ev < MEGA_TRACE_EVENTS) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      a.trace[(size_t)blockIdx.x * MEGA_TRACE_EVENTS + ev] = t;
    }
    ++ev;
#endif
  }
  // this thread's slice of the current input vector, as dp4a byte planes
  XPlanes xp;
  // MMA segments: the staged vector as the B operand of the int8 tensor-core path
  int mfmt = 0;            // SM_Q4_K / SM_Q6_K: mpl holds that format's digit columns
  const uint2* mpl = nullptr;  // [U][3 (Q4_K) or 6 (Q6_K)][4 tig] word pairs
  const float* msx = nullptr;  // Q4_K: [U] unit sums; Q6_K: [U][2] half sums
  const float* mbx = nullptr;  // [NB] 2^(e-21) (Q4_K) or 2^(e-22) (Q6_K) of each block
  int mend = 0;                // first float of part past the digit planes
  float x_inv = 1.f;           // RMSNorm scale of the staged vector (not folded into the planes)
  bool pair = true;  // plane packing (PAIR for K-quants / Q4_0, NATURAL for Q8_0)
  const float* x_src = nullptr;
  const float* x_gamma = nullptr;
  int x_K = 0;
  int U = 1, u = 0, ph = 0, P = 1, nwpp = 1;
  bool u_ok = false;

  // Plan GEMV phase ph (layer ph / 4; kind Q|K|V, O, gate|up, down; the last one
  // is the LM head) into sh.plan.  Runs on one thread.
  __device__ void prepare(int ph, const float* emb) {
    SegPlan& P = sh.plan;
    const int l = ph >> 2, kind = ph & 3;
    const bool head = l == a.n_layers;
    const MegaLayer& L = sh.lay[l & 1];
    int si = 0, c0 = 0, c1 = (int)gridDim.x;
    if (kind == 0 && !head) {
      si = blockIdx.x < L.qkv_cb[1] ? 0 : (blockIdx.x < L.qkv_cb[2] ? 1 : 2);
      c0 = L.qkv_cb[si];
      c1 = L.qkv_cb[si + 1];
    }
    const MegaSeg& sg = head ? a.head : (kind == 0 ? L.qkv[si] : (kind == 1 ? L.o : (kind == 2 ? L.gu : L.down)));
    P.s = &sg;
    // RMSNorm (Q|K|V, gate|up, head) on the residual stream; O reads the attention output, down the GLU.
    // Exchange words: Q|K|V (and the head) read x1 of the previous layer, O reads att and adds x1,
    // gate|up reads x0, down reads act and adds x0.
    P.src = ph == 0 ? emb : nullptr;
    const unsigned tl = ll_tag(epoch, l), tp = ll_tag(epoch, l - 1);
    P.src_ll = nullptr;
    P.res_ll = nullptr;
    P.res_plain = nullptr;
    P.dst = nullptr;
    P.src_tag = P.res_tag = P.dst_tag = tl;
    if (head) {
      P.src_ll = a.ll_x1;
      P.src_tag = tp;
    } else if (kind == 0) {
      if (ph > 0) P.src_ll = a.ll_x1;
      P.src_tag = tp;
      P.dst = si == 0 ? a.ll_q : (si == 1 ? a.ll_kv : a.ll_kv + a.kd);
    } else if (kind == 1) {
      P.src_ll = a.ll_att;
      if (l == 0) P.res_plain = emb;
      else P.res_ll = a.ll_x1;
      P.res_tag = tp;
      P.dst = a.ll_x0;
    } else if (kind == 2) {
      P.src_ll = a.ll_x0;
      P.dst = a.ll_act;
    } else {
      P.src_ll = a.ll_act;
      P.res_ll = a.ll_x0;
      P.dst = a.ll_x1;
    }
    P.gamma = head ? a.out_norm : (kind == 0 ? L.attn_norm : (kind == 2 ? L.ffn_norm : nullptr));
    P.amax_v = head ? &a.amax_val[blockIdx.x] : nullptr;
    P.amax_i = head ? &a.amax_idx[blockIdx.x] : nullptr;
    const int K = (kind == 1 && !head) ? a.qd : ((kind == 3 && !head) ? a.F : a.H);
    P.K = K;
    P.rb = stage_rows(sg, K, slot_bytes);
    seg_rows_in(sg.rows, blockIdx.x, c0, c1, P.r0, P.r1);
    P.mma = mma_seg(a, sg);
    P.slot0 = k % a.nslots;
    P.par0 = (k / a.nslots) & 1;
    if (P.mma) {
      const MGeo m = mgeo(sg, K, slot_bytes);
      P.mg = m;
      const int ntiles = (P.r1 - P.r0 + 15) / 16;
      P.nst = ntiles * m.nch;
      P.red_n = ntiles * m.nT * m.NB * 16;
      // block partials and the warp scratch: below the digit planes when they fit, else after them
      const int mend = K + 50 * (K >> 5) + (K >> 8);
      P.red_off = (P.red_n + CWARPS * WS <= K) ? 0 : ((mend + 3) & ~3);
    }
  }

  // ---- polling the exchange words (bounded: ~2 s of clock64, then SM_ERR_TIMEOUT)
  // One tick of a poll loop: false once the CTA has given up (its own timeout or
  // another thread's); the loop then stops and the caller's values are garbage,
  // which is harmless: the CTA leaves at its next phase transition.
  __device__ bool poll_tick(long long& t0) {
    if (*(volatile int*)&sh.abort) return false;
    const long long now = clock64();
    if (t0 == 0) {
      t0 = now;
    } else if (now - t0 > kSpin) {
      atomicExch(a.status, SM_ERR_TIMEOUT);
      *(volatile int*)&sh.abort = 1;
      return false;
    }
    __nanosleep(32);
    return true;
  }

  // Consumer threads gather n exchange words: value i (word at addr(i)) goes to
  // put(i, v) once its tag is `tag`.  Up to B words per thread are in flight at a
  // time; only the words not yet tagged are loaded again.
  template <int B, class Addr, class Put>
  __device__ void ll_gather(int n, unsigned tag, Addr addr, Put put) {
    for (int base = 0; base < n; base += B * CT) {
      u64 w[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int i = base + b * CT + tid;
        w[b] = i < n ? ll_ld(addr(i)) : 0ull;
      }
      long long t0 = 0;
      while (true) {
        bool all = true;
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const int i = base + b * CT + tid;
          if (i < n && !ll_ok(w[b], tag)) {
            all = false;
            w[b] = ll_ld(addr(i));
          }
        }
        if (all || !poll_tick(t0)) break;
      }
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int i = base + b * CT + tid;
        if (i < n) put(i, ll_val(w[b]));
      }
    }
  }

  // Consumer threads gather n (even) consecutive exchange words from src (16-byte
  // aligned) into dst[0, n): two words per 16-byte load, up to 2B words per thread
  // in flight.
  template <int B>
  __device__ void ll_gather2(int n, unsigned tag, const u64* src, float* dst) {
    const int np = n >> 1;
    for (int base = 0; base < np; base += B * CT) {
      ulonglong2 w[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int i = base + b * CT + tid;
        w[b] = i < np ? ll_ld2(src + 2 * i) : make_ulonglong2(0ull, 0ull);
      }
      long long t0 = 0;
      while (true) {
        bool all = true;
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const int i = base + b * CT + tid;
          if (i < np && !(ll_ok(w[b].x, tag) && ll_ok(w[b].y, tag))) {
            all = false;
            w[b] = ll_ld2(src + 2 * i);
          }
        }
        if (all || !poll_tick(t0)) break;
      }
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int i = base + b * CT + tid;
        if (i < np) *(float2*)&dst[2 * i] = make_float2(ll_val(w[b].x), ll_val(w[b].y));
      }
    }
  }

  // two words, polled together by the calling thread alone
  __device__ void ll_wait2(const u64* p0, const u64* p1, unsigned tag, float& v0, float& v1) {
    u64 w0 = ll_ld(p0), w1 = ll_ld(p1);
    long long t0 = 0;
    while (!(ll_ok(w0, tag) && ll_ok(w1, tag)) && poll_tick(t0)) {
      w0 = ll_ld(p0);
      w1 = ll_ld(p1);
    }
    v0 = ll_val(w0);
    v1 = ll_val(w1);
  }

  // one word, polled by the calling thread alone
  __device__ float ll_wait1(const u64* p, unsigned tag) {
    u64 w = ll_ld(p);
    long long t0 = 0;
    while (!ll_ok(w, tag) && poll_tick(t0)) w = ll_ld(p);
    return ll_val(w);
  }

  // Phase transition inside the CTA (no grid-wide barrier: data readiness travels
  // in the exchange words).  `next`: a layer table entry to bring on chip into
  // lay[next_slot]; `prep`: the GEMV phase to plan (thread 64); `kvl`: the layer
  // whose attention rows of this CTA are prefetched into L2.  False (uniformly
  // across the consumer threads) once the CTA has given up.
  __device__ bool transition(const MegaLayer* next = nullptr, int next_slot = 0, int prep = -1,
                             const float* emb = nullptr, const MegaLayer* kvl = nullptr, int chunks = 0,
                             int len = 0) {
    cons_sync();
    stamp();
    if (kvl) {
      for (int it = blockIdx.x; it < a.nKv * chunks; it += gridDim.x) {
        const int per = (len + chunks - 1) / chunks, cc = it % chunks, gg = it / chunks;
        const int j0 = min(len, cc * per), j1 = min(len, j0 + per);
        const int64_t off = ((int64_t)seq_v * a.nKv + gg) * a.max_ctx * 64 + (int64_t)j0 * 64;
        const int lines = (j1 - j0) * 2;  // 256-byte rows
        for (int t = tid; t < 2 * lines; t += CT) {
          const float* base = (t < lines ? kvl->kc : kvl->vc) + off;
          asm volatile("prefetch.global.L2 [%0];" ::"l"(base + (t % lines) * 32));
        }
      }
    }
    if (next && tid >= 32 && tid < 32 + (int)(sizeof(MegaLayer) / 4))
      ((int*)&sh.lay[next_slot])[tid - 32] = __ldg((const int*)next + (tid - 32));
    if (prep >= 0 && tid == 64) prepare(prep, emb);
    if (tid == 0) sh.flag[0] = !*(volatile int*)&sh.abort;
    cons_sync();
    stamp();
    return sh.flag[0] != 0;
  }

  // x slice for a phase with K inputs (optionally RMS-normalised with gamma)
  // need: this CTA has output rows in the phase.  A CTA without any does not wait
  // for the vector (nothing downstream waits for it, so it could fall a layer
  // behind and see the words of the next one); its planes hold zeros.
  __device__ void load_x(const float* src, const u64* src_ll, unsigned src_tag, const float* gamma, int K,
                         bool want_pair, int mma, bool need) {
    x_src = src;
    x_gamma = gamma;
    x_K = K;
    pair = want_pair;
    mfmt = 0;
    const int lxe = (lx >= 4 && lx < 12) ? 900 + 8 * (lx - 4) : -1;
    ++lx;
    if (lxe >= 0) stamp_at(lxe);
    // warp w covers units (w % nwpp)*32 + lane of row phase w / nwpp, so a warp's
    // partials for one row can be reduced with shuffles inside the compute loop
    U = K >> 5;
    nwpp = (U + 31) / 32;
    P = CWARPS / nwpp;
    ph = (tid >> 5) / nwpp;
    const int u_raw = ((tid >> 5) % nwpp) * 32 + (tid & 31);
    u_ok = u_raw < U && ph < P;
    u = u_ok ? u_raw : 0;
    // one coalesced pass per CTA (the vector was written by other CTAs: bypass L1).
    // 16-byte chunk c of unit w is stored at chunk (c + w) % 8 of that unit, so the
    // 8 lanes of a quarter-warp reading chunk c of 8 consecutive units hit 8
    // different bank groups.
    if (AM || mma) {
      // the tensor-core path needs no staged copy: each lane reads its own elements
      build_mma_planes(src, src_ll, src_tag, K, gamma, mma, lxe, need);
      return;
    }
    float4* xs = (float4*)part;        // [K/4]
    float4* gs = (float4*)part + K / 4; // [K/4]
    uint32_t* pls = (uint32_t*)(part + 2 * K);  // [U][28]: planes a, b, c (8 words each), inv, x16a, x16b
    for (int t = tid; t < K / 4; t += CT) {
      const int w = t >> 3, p = (w << 3) + (((t & 7) + w) & 7);
      if (!src_ll) xs[p] = __ldcg((const float4*)src + t);
      if (gamma) gs[p] = __ldg((const float4*)gamma + t);
    }
    if (src_ll && !need) {
      for (int t = tid; t < K / 4; t += CT) xs[t] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else if (src_ll) {
      // element i: float4 t = i / 4 of the staging order above, lane i % 4
      float* xf = (float*)xs;
      ll_gather<12>(K, src_tag, [&](int i) { return src_ll + i; }, [&](int i, float v) {
        const int t = i >> 2, w = t >> 3;
        xf[4 * ((w << 3) + (((t & 7) + w) & 7)) + (i & 3)] = v;
      });
    }
    if (lxe >= 0) stamp_at(lxe + 1);
    cons_sync();
    if (lxe >= 0) stamp_at(lxe + 2);
    // The byte planes of every unit, built once per CTA: four threads per unit,
    // eight elements each, from y = gamma * x (the RMS scale is a per-vector
    // scalar and is folded into each unit's factor below); the same pass
    // accumulates sum(x^2) for RMSNorm.
    float sq = 0.f;
    for (int t0 = (tid >> 5) * 32; t0 < 4 * U; t0 += CT) {
      const int t = t0 + (tid & 31);
      const bool on = t < 4 * U;
      const int uu = on ? t >> 2 : 0, pp = t & 3;
      const float4 v0 = xs[(uu << 3) + ((2 * pp + uu) & 7)], v1 = xs[(uu << 3) + ((2 * pp + 1 + uu) & 7)];
      float y[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      if (gamma) {
        const float4 g0 = gs[(uu << 3) + ((2 * pp + uu) & 7)], g1 = gs[(uu << 3) + ((2 * pp + 1 + uu) & 7)];
        const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (on) sq = fmaf(y[i], y[i], sq);
          y[i] = __fmul_rn(gv[i], y[i]);
        }
      }
      float am = 0.f, sp = 0.f;
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        am = fmaxf(am, fmaxf(fabsf(y[i]), fabsf(y[i + 1])));
        sp += y[i] + y[i + 1];
      }
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
      sp += __shfl_xor_sync(0xffffffffu, sp, 1);  // elements 0..15 (parts 0, 1) or 16..31 (2, 3)
      int ex = 0;
      frexpf(am, &ex);  // am < 2^ex
      const float up = ldexpf(1.f, 23 - ex);
      uint32_t X[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) X[i] = am > 0.f ? (uint32_t)__float2int_rn(y[i] * up) : 0u;
      // PAIR: word pp = elements 8pp + 0, 2, 4, 6; word 4 + pp = 8pp + 1, 3, 5, 7.
      // NATURAL: words 2pp, 2pp + 1 = elements 8pp .. 8pp + 3, 8pp + 4 .. + 7.
      const int w0 = pair ? pp : 2 * pp, w1 = pair ? 4 + pp : 2 * pp + 1;
      const uint32_t e0 = pair ? X[0] : X[0], e1 = pair ? X[2] : X[1], e2 = pair ? X[4] : X[2], e3 = pair ? X[6] : X[3];
      const uint32_t o0 = pair ? X[1] : X[4], o1 = pair ? X[3] : X[5], o2 = pair ? X[5] : X[6], o3 = pair ? X[7] : X[7];
      if (on) {
        uint32_t* d = pls + uu * 28;
        d[w0] = __byte_perm(__byte_perm(e0, e1, 0x0062), __byte_perm(e2, e3, 0x0062), 0x5410);
        d[8 + w0] = __byte_perm(__byte_perm(e0, e1, 0x0051), __byte_perm(e2, e3, 0x0051), 0x5410);
        d[16 + w0] = __byte_perm(__byte_perm(e0, e1, 0x0040), __byte_perm(e2, e3, 0x0040), 0x5410);
        d[w1] = __byte_perm(__byte_perm(o0, o1, 0x0062), __byte_perm(o2, o3, 0x0062), 0x5410);
        d[8 + w1] = __byte_perm(__byte_perm(o0, o1, 0x0051), __byte_perm(o2, o3, 0x0051), 0x5410);
        d[16 + w1] = __byte_perm(__byte_perm(o0, o1, 0x0040), __byte_perm(o2, o3, 0x0040), 0x5410);
        if (pp == 0) {
          d[24] = __float_as_uint(ldexpf(1.f, ex - 23));
          d[25] = __float_as_uint(sp);
        }
        if (pp == 2) d[26] = __float_as_uint(sp);
      }
    }
    if (gamma) {
      sq = warp_sum(sq);
      if ((tid & 31) == 0) sh.red[tid >> 5] = sq;
    }
    if (lxe >= 0) stamp_at(lxe + 3);
    cons_sync();
    if (lxe >= 0) stamp_at(lxe + 4);
    float inv = 1.f;
    if (gamma) {
      float tot = 0.f;
      for (int w = 0; w < CWARPS; ++w) tot += sh.red[w];
      inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), a.eps)));
    }
    const uint4* q4 = (const uint4*)(pls + u * 28);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint4 va = q4[c], vb = q4[2 + c], vc = q4[4 + c];
      xp.a[4 * c] = va.x; xp.a[4 * c + 1] = va.y; xp.a[4 * c + 2] = va.z; xp.a[4 * c + 3] = va.w;
      xp.b[4 * c] = vb.x; xp.b[4 * c + 1] = vb.y; xp.b[4 * c + 2] = vb.z; xp.b[4 * c + 3] = vb.w;
      xp.c[4 * c] = vc.x; xp.c[4 * c + 1] = vc.y; xp.c[4 * c + 2] = vc.z; xp.c[4 * c + 3] = vc.w;
    }
    const uint4 hd4 = q4[6];
    xp.inv = __uint_as_float(hd4.x) * inv;
    xp.x16a = __uint_as_float(hd4.y) * inv;
    xp.x16b = __uint_as_float(hd4.z) * inv;
    cons_sync();  // staging area (part) and sh.red are reused next
    if (lxe >= 0) stamp_at(lxe + 5);
  }

  // Digit columns of the staged vector for the int8 tensor-core path, built once
  // per CTA: four threads per 32-element unit, a warp per 256-element block (one
  // power-of-two exponent per block).  y = gamma * x; the RMS scale is a scalar
  // kept in x_inv.  Q4_K: B holds L - H at the low-nibble positions and H at the
  // raw-byte positions (L: 21-bit low elements, H: 17-bit high elements), see
  // gemv_mma.cu; Q6_K: 22-bit values, six columns (three per 16-element half,
  // zero at the other half's positions).
  __device__ void build_mma_planes(const float* src, const u64* src_ll, unsigned src_tag, int K,
                                   const float* gamma, int fmt, int lxe, bool need) {
    const int U = K >> 5, NB = K >> 8, lane = tid & 31;
    const int pbase = K;  // part [0, K) stays free for the block partials
    uint2* mp = (uint2*)(part + pbase);        // [U][6][4] at most
    float* sx = part + pbase + 48 * U;         // [U][2] at most
    float* bx = sx + 2 * U;                    // [NB]
    mend = pbase + 50 * U + NB;
    // this thread's first 8 RMSNorm weights, loaded before the exchange wait so the two
    // round trips overlap
    float4 gpre0 = make_float4(0.f, 0.f, 0.f, 0.f), gpre1 = gpre0;
    const int t_first = (tid >> 5) * 32 + lane;
    if (gamma && t_first < 4 * U) {
      const float4* gg = (const float4*)(gamma + 8 * t_first);
      gpre0 = __ldg(gg);
      gpre1 = __ldg(gg + 1);
    }
    if (src_ll) {
      // the vector arrives in exchange words: gathered into part [0, K) first (the
      // block partials are written there only after the planes are built)
      if (need)
        ll_gather2<6>(K, src_tag, src_ll, part);
      else
        for (int i = tid; i < K; i += CT) part[i] = 0.f;
      if (lxe >= 0) stamp_at(lxe + 1);
      cons_sync();
      if (lxe >= 0) stamp_at(lxe + 2);
      src = part;
    }
    float sq = 0.f;
    for (int t0 = (tid >> 5) * 32; t0 < 4 * U; t0 += CT) {  // 4U is a multiple of 32: whole warps
      const int t = t0 + lane, uu = t >> 2, pp = t & 3;
      // the vector was written by other CTAs (or gathered above): bypass L1
      const float4* xg = (const float4*)(src + 32 * uu + 8 * pp);
      const float4 v0 = src_ll ? xg[0] : __ldcg(xg), v1 = src_ll ? xg[1] : __ldcg(xg + 1);
      float y[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      if (gamma) {
        const float4* gg = (const float4*)(gamma + 32 * uu + 8 * pp);
        const bool first = t == t_first;
        const float4 g0 = first ? gpre0 : __ldg(gg), g1 = first ? gpre1 : __ldg(gg + 1);
        const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          sq = fmaf(y[i], y[i], sq);
          y[i] = __fmul_rn(gv[i], y[i]);
        }
      }
      float am = 0.f, su = 0.f;
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        am = fmaxf(am, fmaxf(fabsf(y[i]), fabsf(y[i + 1])));
        su += y[i] + y[i + 1];
      }
      am = warp_max(am);  // the warp's 8 units are one block
      const int ex = block_exp(am);  // am < 2^ex
      uint32_t pw[2][3];  // [low / high positions][digit hi, b, c]
      if (fmt == SM_Q4_K) {
        const float up = pow2i(21 - ex), uph = pow2i(17 - ex);
        int X[2][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int L = __float2int_rn(y[2 * i] * up);
          const int H = __float2int_rn(y[2 * i + 1] * uph);
          X[0][i] = L - H;
          X[1][i] = H;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) digits4(X[h][0], X[h][1], X[h][2], X[h][3], pw[h][0], pw[h][1], pw[h][2]);
#pragma unroll
        for (int q = 0; q < 3; ++q) mp[(uu * 3 + q) * 4 + pp] = make_uint2(pw[0][q], pw[1][q]);
        su += __shfl_xor_sync(0xffffffffu, su, 1);
        su += __shfl_xor_sync(0xffffffffu, su, 2);
        if (pp == 0) sx[uu] = su;
        if (lane == 0) bx[uu >> 3] = pow2i(ex - 21);
      } else {
        const float up = pow2i(22 - ex);
        int X[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) X[i] = __float2int_rn(y[i] * up);
        digits4(X[0], X[2], X[4], X[6], pw[0][0], pw[0][1], pw[0][2]);  // even elements
        digits4(X[1], X[3], X[5], X[7], pw[1][0], pw[1][1], pw[1][2]);  // odd elements
        const int half = pp >> 1;
#pragma unroll
        for (int col = 0; col < 6; ++col)
          mp[(uu * 6 + col) * 4 + pp] =
              (col / 3) == half ? make_uint2(pw[0][col % 3], pw[1][col % 3]) : make_uint2(0u, 0u);
        su += __shfl_xor_sync(0xffffffffu, su, 1);
        if ((pp & 1) == 0) sx[uu * 2 + half] = su;
        if (lane == 0) bx[uu >> 3] = pow2i(ex - 22);
      }
    }
    if (gamma) {
      sq = warp_sum(sq);
      if (lane == 0) sh.red[tid >> 5] = sq;
    }
    if (lxe >= 0) stamp_at(lxe + 3);
    cons_sync();
    if (lxe >= 0) stamp_at(lxe + 4);
    float inv = 1.f;
    if (gamma) {
      float tot = 0.f;
      for (int w = 0; w < CWARPS; ++w) tot += sh.red[w];
      inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), a.eps)));
    }
    x_inv = inv;
    mpl = mp;
    msx = sx;
    mbx = bx;
    mfmt = fmt;
    (void)NB;
    if (lxe >= 0) stamp_at(lxe + 5);
  }

  // per-warp scratch of an MMA item: int2 scales [16][9], msum [16], fdv [16]
  static constexpr int WS = 16 * 9 * 2 + 32;

  // One (16-row tile, 256-weight block) item of a Q4_K MMA segment: the
  // tile's rows start at tb with stride rs; the block is staged at kbl, global
  // block kb.  Returns rows g and g + 8 on lanes with tig == 0.
  __device__ void item_q4k(const uint8_t* tb, int rs, int kbl, int kb, int n, float* ws, float& out0, float& out1) {
    const int lane = tid & 31, g = lane >> 2, tig = lane & 3, sr = lane >> 1, sh2 = lane & 1;
    int* si = (int*)ws;  // [16][9]
    float* msum = ws + 16 * 9 * 2;
    float* fdv = msum + 16;
    {
      const int4 hdr = *(const int4*)(tb + min(sr, n - 1) * rs + kbl * Q4K_BLOCK_BYTES);
      const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFF)));
      const float dmin = __half2float(__ushort_as_half((unsigned short)((uint32_t)hdr.x >> 16)));
      const uint64_t sb = (uint32_t)hdr.y | ((uint64_t)((uint32_t)hdr.z & 0xFFFFu) << 32);
      const uint64_t mb = ((uint32_t)hdr.z >> 16) | ((uint64_t)(uint32_t)hdr.w << 16);
      const uint32_t s24 = (uint32_t)(sb >> (24 * sh2)), m24 = (uint32_t)(mb >> (24 * sh2));
#pragma unroll
      for (int j = 0; j < 4; ++j) si[sr * 9 + 4 * sh2 + j] = (s24 >> (6 * j)) & 63;
      const float* q = msx + kb * 8 + 4 * sh2;
      float mpart = (float)(m24 & 63) * q[0];
      mpart = fmaf((float)((m24 >> 6) & 63), q[1], mpart);
      mpart = fmaf((float)((m24 >> 12) & 63), q[2], mpart);
      mpart = fmaf((float)((m24 >> 18) & 63), q[3], mpart);
      mpart = dmin * x_inv * (mpart + __shfl_xor_sync(0xffffffffu, mpart, 1));
      if (sh2 == 0) {
        msum[sr] = mpart;
        fdv[sr] = d * mbx[kb] * x_inv;
      }
    }
    __syncwarp();
    const float fA = tig == 0 ? 65536.f : (tig == 1 ? 1.f : 0.f);
    const float fB = tig == 0 ? 256.f : 0.f;
    const uint8_t* rg = tb + min(g, n - 1) * rs + kbl * Q4K_BLOCK_BYTES + 16 + 4 * tig;
    const uint8_t* rg8 = tb + min(g + 8, n - 1) * rs + kbl * Q4K_BLOCK_BYTES + 16 + 4 * tig;
    const uint2* plu = mpl + (kb * 8 * 3 + (g % 3)) * 4 + tig;
    int t0 = 0, t1 = 0, t2 = 0, t3 = 0;
#pragma unroll
    for (int j0 = 0; j0 < 8; j0 += 4) {
      int dd[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t w0 = *(const uint32_t*)(rg + 16 * (j0 + j));
        const uint32_t w1 = *(const uint32_t*)(rg8 + 16 * (j0 + j));
        const uint2 b = plu[12 * (j0 + j)];
        mma_u8s8(dd[j][0], dd[j][1], dd[j][2], dd[j][3], w0 & 0x0F0F0F0Fu, w1 & 0x0F0F0F0Fu, w0, w1, b.x, b.y);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int s0 = si[g * 9 + j0 + j], s1 = si[(g + 8) * 9 + j0 + j];
        t0 += s0 * dd[j][0];
        t1 += s0 * dd[j][1];
        t2 += s1 * dd[j][2];
        t3 += s1 * dd[j][3];
      }
    }
    float acc0 = fmaf((float)t0, fA, (float)t1 * fB);
    float acc1 = fmaf((float)t2, fA, (float)t3 * fB);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    out0 = fmaf(fdv[g], acc0, -msum[g]);
    out1 = fmaf(fdv[g + 8], acc1, -msum[g + 8]);
    __syncwarp();
  }

  // Q6_K item: as item_q4k; the d row sits at dofs in every staged row.
  __device__ void item_q6k(const uint8_t* tb, int rs, int kbl, int kb, int n, int dofs, float* ws, float& out0,
                           float& out1) {
    const int lane = tid & 31, g = lane >> 2, tig = lane & 3, sr = lane >> 1, sh2 = lane & 1;
    int2* scw = (int2*)ws;  // [16][9]
    float* msum = ws + 16 * 9 * 2;
    float* fdv = msum + 16;
    {
      const uint8_t* rp = tb + min(sr, n - 1) * rs;
      const int2 sc8 = *(const int2*)(rp + kbl * Q6K_BODY_BYTES + 192 + 8 * sh2);
      const float d = __half2float(__ushort_as_half(*(const unsigned short*)(rp + dofs + 2 * kb)));
      const uint32_t sw[2] = {(uint32_t)sc8.x, (uint32_t)sc8.y};
      const float* hs = msx + 2 * (kb * 8 + 4 * sh2);
      float mpart = 0.f;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int sa = (int)(int8_t)((sw[jj >> 1] >> (16 * (jj & 1))) & 0xFF);
        const int sb = (int)(int8_t)((sw[jj >> 1] >> (16 * (jj & 1) + 8)) & 0xFF);
        scw[sr * 9 + 4 * sh2 + jj] = make_int2(sa, sb);
        mpart = fmaf((float)sa, hs[2 * jj], mpart);
        mpart = fmaf((float)sb, hs[2 * jj + 1], mpart);
      }
      mpart += __shfl_xor_sync(0xffffffffu, mpart, 1);
      if (sh2 == 0) {
        msum[sr] = 32.f * d * x_inv * mpart;
        fdv[sr] = d * mbx[kb] * x_inv;
      }
    }
    __syncwarp();
    const float fA = tig == 0 ? 65536.f : (tig == 1 ? 1.f : (tig == 2 ? 256.f : 0.f));
    const float fB = tig == 0 ? 256.f : (tig == 1 ? 65536.f : (tig == 2 ? 1.f : 0.f));
    const bool s0_first = tig < 2, s1_first = tig == 0;
    const int hshift = 4 * (tig & 1);
    const uint8_t* rg = tb + min(g, n - 1) * rs + kbl * Q6K_BODY_BYTES;
    const uint8_t* rg8 = tb + min(g + 8, n - 1) * rs + kbl * Q6K_BODY_BYTES;
    const uint2* plu = mpl + (kb * 8 * 6 + (g < 6 ? g : 0)) * 4 + tig;
    int t0 = 0, t1 = 0, t2 = 0, t3 = 0;
#pragma unroll
    for (int j0 = 0; j0 < 8; j0 += 4) {
      int dd[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int jj = j0 + j;
        const uint32_t w0 = *(const uint32_t*)(rg + 16 * jj + 4 * tig);
        const uint32_t w1 = *(const uint32_t*)(rg8 + 16 * jj + 4 * tig);
        const uint32_t W0 = *(const uint32_t*)(rg + 128 + 8 * jj + 4 * (tig >> 1)) >> hshift;
        const uint32_t W1 = *(const uint32_t*)(rg8 + 128 + 8 * jj + 4 * (tig >> 1)) >> hshift;
        const uint32_t e0 = (w0 & 0x0F0F0F0Fu) | ((W0 << 4) & 0x30303030u);
        const uint32_t e1 = (w1 & 0x0F0F0F0Fu) | ((W1 << 4) & 0x30303030u);
        const uint32_t o0 = ((w0 >> 4) & 0x0F0F0F0Fu) | ((W0 << 2) & 0x30303030u);
        const uint32_t o1 = ((w1 >> 4) & 0x0F0F0F0Fu) | ((W1 << 2) & 0x30303030u);
        const uint2 b = plu[24 * jj];
        mma_u8s8(dd[j][0], dd[j][1], dd[j][2], dd[j][3], e0, e1, o0, o1, b.x, b.y);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int2 s0 = scw[g * 9 + j0 + j], s1 = scw[(g + 8) * 9 + j0 + j];
        t0 += (s0_first ? s0.x : s0.y) * dd[j][0];
        t1 += (s1_first ? s0.x : s0.y) * dd[j][1];
        t2 += (s0_first ? s1.x : s1.y) * dd[j][2];
        t3 += (s1_first ? s1.x : s1.y) * dd[j][3];
      }
    }
    float acc0 = fmaf((float)t0, fA, (float)t1 * fB);
    float acc1 = fmaf((float)t2, fA, (float)t3 * fB);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    out0 = fmaf(fdv[g], acc0, -msum[g]);
    out1 = fmaf(fdv[g + 8], acc1, -msum[g + 8]);
    __syncwarp();
  }

  // MMA segment body: the CTA's (tile, block) items, round-robin over the warps
  // and in stage order; every warp arrives on each stage's empty barrier once,
  // after its last item there.  Block partials go to red [tiles][nT][NB][16].
  __device__ bool seg_mma_body(const MegaSeg& s, const SegPlan& PL, float*& red_out) {
    const MGeo m = PL.mg;
    const int nout = PL.r1 - PL.r0, nst = PL.nst, red_n = PL.red_n;
    float* base = part + PL.red_off;
    if (PL.red_off + red_n + CWARPS * WS > a.part_floats) {  // host sizing covers every phase
      if (tid == 0) atomicExch(a.status, SM_ERR_UNSUPPORTED);
      sh.abort = 1;
      return false;
    }
    float* red = base;
    float* ws = base + red_n + (tid >> 5) * WS;
    const int lane = tid & 31, warp = tid >> 5;
    // walk the stages without divisions: stage st = (tile t, block chunk c) holds
    // per = nT * nkb items; this warp's items are warp, warp + CWARPS, ...
    int st = 0, t = 0, c = 0, nkb = min(m.nkbs, m.NB), per = m.nT * nkb, loc = warp;
    int slot = PL.slot0;
    uint32_t par = (uint32_t)PL.par0;
    bool waited = false;
    while (true) {
      while (st < nst && loc >= per) {
        // leave stage st: a stage this warp had no item in is released only once it
        // has filled, so the arrival cannot reach the slot's previous use
        if (!waited && !mbar_wait_spin(&sh.full[slot], par, a.status)) {
          sh.abort = 1;
          return false;
        }
        if (lane == 0) mbar_arrive(&sh.empty[slot]);
        waited = false;
        loc -= per;
        ++st;
        if (++c == m.nch) c = 0, ++t;
        nkb = min(m.nkbs, m.NB - c * m.nkbs);
        per = m.nT * nkb;
        if (++slot == a.nslots) slot = 0, par ^= 1u;
      }
      if (st >= nst) break;
      if (!waited) {
        if (!mbar_wait_spin(&sh.full[slot], par, a.status)) {
          sh.abort = 1;
          return false;
        }
        waited = true;
      }
      const int tt = loc >= nkb ? 1 : 0, kbl = loc - tt * nkb, kb = c * m.nkbs + kbl;
      const int n = min(16, nout - 16 * t);
      const uint8_t* tb = ring + slot * slot_bytes + tt * 16 * m.rs;
      float o0, o1;
      if (s.fmt == SM_Q4_K)
        item_q4k(tb, m.rs, kbl, kb, n, ws, o0, o1);
      else
        item_q6k(tb, m.rs, kbl, kb, n, m.nkbs * m.bb, ws, o0, o1);
      if ((lane & 3) == 0) {
        float* rd = red + ((t * m.nT + tt) * m.NB + kb) * 16;
        rd[lane >> 2] = o0;
        rd[(lane >> 2) + 8] = o1;
      }
      loc += CWARPS;
    }
    __syncwarp();
    k += nst;
    red_out = red;
    return true;
  }

  // one unit of a staged row (integer dot path); `auxp` is the row's staged scales / d
  __device__ float dot(int fmt, int bs, const uint8_t* rowp, const uint8_t* auxp) {
    switch (fmt) {
      case SM_Q4_K: {
        Unit<SM_Q4_K>::Raw r;
        const uint8_t* blk = rowp + (u >> 3) * Q4K_BLOCK_BYTES;
        r.hdr = *(const int4*)blk;
        r.qs = *(const int4*)(blk + 16 + 16 * (u & 7));
        return dot_i8_q4k(r, u & 7, xp);
      }
      case SM_Q6_K: {
        Unit<SM_Q6_K>::Raw r;
        const uint8_t* blk = rowp + (u >> 3) * Q6K_BODY_BYTES;
        const int j = u & 7;
        r.ql = *(const int4*)(blk + 16 * j);
        r.qh = *(const int2*)(blk + 128 + 8 * j);
        r.sc = *(const unsigned short*)(blk + 192 + 2 * j);
        r.d = ((const unsigned short*)auxp)[u >> 3];
        return dot_i8_q6k(r, xp);
      }
      case SM_Q8_0: {
        Unit<SM_Q8_0>::Raw r;
        r.a = *(const int4*)(rowp + 32 * u);
        r.b = *((const int4*)(rowp + 32 * u) + 1);
        r.sc = ((const float*)auxp)[(32 * u) / bs];
        return dot_i8_q8(r, xp);
      }
      default: {
        Unit<SM_Q4_0>::Raw r;
        r.q = *(const int4*)(rowp + 16 * u);
        r.sc = ((const float*)auxp)[(32 * u) / bs];
        return dot_i8_q4_0(r, xp);
      }
    }
  }

  static __device__ GemvSeg to_gemv(const MegaSeg& s) {
    GemvSeg g;
    g.fmt = s.fmt;
    g.rows = s.rows;
    g.bs = s.bs;
    g.aux_bpr = s.aux_bpr;
    g.aux_stride = s.aux_stride;
    g.mode = s.mode;
    g.data = s.data;
    g.aux = s.aux;
    g.data2 = s.data2;
    g.aux2 = s.aux2;
    g.y = s.y;
    return g;
  }

  // GEMV rows of this CTA for one segment; `amax` (head only) tracks the local argmax.
  __device__ bool seg(const SegPlan& PL) {
    const MegaSeg& s = *PL.s;
    const int K = PL.K, rb = PL.rb, r0 = PL.r0, r1 = PL.r1;
    float* amax_v = PL.amax_v;
    int* amax_i = PL.amax_i;
    const int nout = r1 - r0;
    const int64_t rbytes = row_bytes_fmt(s.fmt, K);
    const bool glu = s.mode == GEMV_GLU;
    const GemvSeg g = to_gemv(s);
    const bool use_mma = PL.mma;
    float* mred = nullptr;
    // ADD: this thread's residual row, read before the GEMV rather than after it
    const bool addm = s.mode == GEMV_ADD;
    float resid = 0.f;
    if (addm && tid < nout)
      resid = PL.res_ll ? ll_wait1(PL.res_ll + r0 + tid, PL.res_tag) : __ldg(&PL.res_plain[r0 + tid]);
    const MGeo mg = PL.mg;
    // the caller staged the vector for this segment's path (one staging call site
    // keeps the kernel small): a mismatch is a scheduling error
    if ((AM && !use_mma) || (use_mma ? mfmt != s.fmt : (mfmt != 0 || (s.fmt != SM_Q8_0) != pair))) {
      if (tid == 0) atomicExch(a.status, SM_ERR_UNSUPPORTED);
      sh.abort = 1;
      return false;
    }
    if (AM || use_mma) {
      stamp();
      stamp();
      // a failed wait leaves the loop early; the warp still meets the CTA barriers
      // below and the epilogue is skipped (the CTA leaves at its next transition)
      if (!seg_mma_body(s, PL, mred)) *(volatile int*)&sh.abort = 1;
    } else {
    stamp();
    for (int row = r0; row < r1; row += rb) {
      const int n = min(rb, r1 - row);
      const int slot = k % a.nslots;
      if (!mbar_wait_bounded(&sh.full[slot], (k / a.nslots) & 1, a.status)) {
        *(volatile int*)&sh.abort = 1;
        break;
      }
      if (row == r0) stamp();
      const uint8_t* st = ring + slot * slot_bytes;
      const uint8_t* sa = st + (glu ? 2 : 1) * rb * rbytes;  // staged scales / d
      const int64_t arb = aux_row_bytes(s);
      const int nrows = glu ? 2 * n : n;
      if (ph < P)  // warp-uniform; four independent rows per pass for instruction-level parallelism
        for (int sr0 = ph; sr0 < nrows; sr0 += 4 * P) {
          float v[4];
          int pidx[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int sr = sr0 + q * P;
            v[q] = 0.f;
            pidx[q] = -1;
            if (sr < nrows) {
              const bool up = glu && sr >= n;
              const int lr = up ? sr - n : sr;
              const int srow = up ? rb + lr : lr;
              if (u_ok) v[q] = dot(s.fmt, s.bs, st + (int64_t)srow * rbytes, sa + (int64_t)srow * arb);
              pidx[q] = ((up ? nout : 0) + (row - r0) + lr) * nwpp + ((tid >> 5) % nwpp);
            }
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) v[q] = warp_sum(v[q]);
          if ((tid & 31) == 0)
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (pidx[q] >= 0) part[pidx[q]] = v[q];
        }
      __syncwarp();
      if ((tid & 31) == 0) mbar_arrive(&sh.empty[slot]);
      ++k;
    }
    if (r0 == r1) stamp();
    }
    stamp();
    cons_sync();
    const bool pairs = s.mode == GEMV_ROPE_Q || s.mode == GEMV_ROPE_K_CACHE;
    if (tid == 0) sh.flag[1] = *(volatile int*)&sh.abort;
    cons_sync();
    // after a failed wait nothing is stored: readers of these rows time out too
    const int nitems = sh.flag[1] ? 0 : (pairs ? (nout + 1) / 2 : nout);
    const int lane = tid & 31, warp = tid >> 5;
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int it = tid; it < nitems; it += CT) {
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      int rin[2] = {it, 0};
      int nr = 1;
      if (glu) {
        rin[1] = nout + it;
        nr = 2;
      } else if (pairs) {
        rin[0] = 2 * it;
        rin[1] = 2 * it + 1;
        nr = (2 * it + 1 < nout) ? 2 : 1;
      }
      for (int q = 0; q < nr; ++q) {
        float t = 0.f;
        if (mred) {
          // MMA partials: row rin of the gate (or, past nout, the up) tiles, blocks in order
          const int tt = rin[q] >= nout ? 1 : 0, lr = rin[q] - tt * nout;
          const float* rd = mred + (((lr >> 4) * mg.nT + tt) * mg.NB) * 16 + (lr & 15);
          for (int b = 0; b < mg.NB; ++b) t += rd[b * 16];
        } else {
          for (int j = 0; j < nwpp; ++j) t += part[rin[q] * nwpp + j];
        }
        v[q] = t;
      }
      // one epilogue for every mode: GLU (gate row it, up row nout + it -> row r0 + it),
      // RoPE pairs (rows r0 + 2it, + 1), residual add, plain store
      const int row0 = r0 + (pairs ? 2 * it : it);
      int nst = 1;
      float o0 = v[0], o1 = v[1];
      if (glu) {
        const float c = fmaxf(-20.f, fminf(v[0], 20.f));
        const float sig = __fdiv_rn(1.f, __fadd_rn(1.f, expf(-c)));  // ActivationOps.cs:304-309
        o0 = __fmul_rn(__fmul_rn(v[0], sig), v[1]);
      } else if (pairs) {
        rope_pair(o0, o1, ep, *ep.pos, row0 % ep.head_dim);
        nst = nr;
      } else if (addm) {
        o0 += it == tid ? resid
                        : (PL.res_ll ? ll_wait1(PL.res_ll + row0, PL.res_tag) : __ldg(&PL.res_plain[row0]));
      }
      for (int q = 0; q < nst; ++q) {
        const int row = row0 + q;
        const float val = q ? o1 : o0;
        if (s.mode == GEMV_ROPE_K_CACHE || s.mode == GEMV_V_CACHE) {
          // head-major cache [seq][kv_head][pos][hd] (MultiHeadAttention.cs:262-274) for later
          // steps; this step's attention reads the row from the exchange words
          const int64_t seq = *ep.seq, pos = *ep.pos;
          const int h = row / ep.head_dim, d = row - h * ep.head_dim;
          s.y[((seq * ep.n_kv + h) * ep.max_ctx + pos) * ep.head_dim + d] = val;
        }
        if (PL.dst)
          ll_st(PL.dst + row, val, PL.dst_tag);
        else
          s.y[row] = val;
      }
      if (amax_v && (v[0] > bv || (v[0] == bv && r0 + it < bi))) {
        bv = v[0];
        bi = r0 + it;
      }
    }
    if (amax_v) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        sh.red[warp] = bv;
        ((int*)sh.vec)[warp] = bi;
      }
    }
    cons_sync();
    if (amax_v && tid == 0) {
      for (int w = 0; w < CWARPS; ++w) {
        const float ov = sh.red[w];
        const int oi = ((int*)sh.vec)[w];
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      *amax_v = bv;
      *amax_i = bi;
    }
    return true;
  }

  // Shared-memory layout of the two attention phases (floats): the same CTA
  // runs item (kv head g, chunk c) in both, so the scores and the chunk's V rows
  // stay on chip across the barrier between them.
  //   es [MGMAX][per]        scores of the chunk (phase A), exponentials (B)
  //   pp [PH][MGMAX][64]     P.V partials (B); the q rows in phase A
  //   cm [chunks][G]         chunk maxima (B)
  //   vs [per][64]           V rows of the chunk (cp.async in A, read in B)
  static constexpr int PH = CT / 64;
  __device__ float* att_es() { return part; }
  __device__ float* att_pp(int per) { return part + MGMAX * per; }
  __device__ float* att_cm(int per) { return att_pp(per) + PH * MGMAX * 64; }
  __device__ float* att_vs(int per, int chunks) {
    float* v = att_cm(per) + chunks * MGMAX;
    return (float*)(((uintptr_t)v + 15) & ~(uintptr_t)15);
  }

  // ---- attention, phase A: scores and slice max of item (kv head g, chunk c)
  __device__ void attn_scores(const MegaLayer& L, int lay_idx, int g, int c, int chunks, int len) {
    const int G = a.nH / a.nKv, HD = 64;
    const int per = (len + chunks - 1) / chunks;
    const int j0 = min(len, c * per), j1 = min(len, j0 + per), n = j1 - j0;
    float* qs = att_pp(per);  // [G][64]
    float* es = att_es();
    const int64_t seq = seq_v;
    const float* kb = L.kc + (seq * a.nKv + g) * (int64_t)a.max_ctx * HD;
    const int sub = tid & 7, slot = tid >> 3;  // 60 key slots
    constexpr int SLOTS = CT / 8;
    const unsigned tag = ll_tag(epoch, lay_idx);
    // key row j: the cache for earlier tokens; this token's row (j = len - 1) comes
    // from the exchange words its Q|K|V CTA wrote this step, staged in sh.kvrow
    const int jn = len - 1 - j0;  // local index of this token's row (>= n: not in this chunk)
    // the first pass's key rows load together with the queries (one round trip)
    float4 k0 = make_float4(0.f, 0.f, 0.f, 0.f), k1 = k0;
    if (slot < n && slot != jn) {
      const float4* kp = (const float4*)(kb + (int64_t)(j0 + slot) * HD + sub * 8);
      k0 = __ldcg(kp);
      k1 = __ldcg(kp + 1);
    }
    if (jn < n && tid < HD) sh.kvrow[tid] = ll_wait1(a.ll_kv + g * HD + tid, tag);
    ll_gather2<1>(G * HD, tag, a.ll_q + g * G * HD, qs);
    cons_sync();
    if (slot == jn) {
      k0 = *(const float4*)&sh.kvrow[sub * 8];
      k1 = *(const float4*)&sh.kvrow[sub * 8 + 4];
    }
    float lmax[MGMAX];
#pragma unroll
    for (int h = 0; h < MGMAX; ++h) lmax[h] = -FLT_MAX;
    const float scale = 1.0f / sqrtf((float)HD);
    for (int p = 0; p < (n + SLOTS - 1) / SLOTS; ++p) {
      const int jj = p * SLOTS + slot;
      const bool valid = jj < n;
      if (p > 0) {
        k0 = k1 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (valid) {
          const float4* kp = jj == jn ? (const float4*)&sh.kvrow[sub * 8]
                                      : (const float4*)(kb + (int64_t)(j0 + jj) * HD + sub * 8);
          k0 = jj == jn ? kp[0] : __ldcg(kp);
          k1 = jj == jn ? kp[1] : __ldcg(kp + 1);
        }
      }
      const float kv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
      for (int h = 0; h < MGMAX; ++h) {
        if (h >= G) break;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) s = fmaf(qs[h * HD + sub * 8 + i], kv[i], s);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        if (valid) {
          if (sub == 0) es[h * per + jj] = s;
          lmax[h] = fmaxf(lmax[h], __fmul_rn(s, scale));
        }
      }
    }
#pragma unroll
    for (int h = 0; h < MGMAX; ++h) {
      const float m = warp_max(lmax[h]);
      if ((tid & 31) == 0) sh.red[(tid >> 5) * MGMAX + h] = m;
    }
    cons_sync();
    if (tid < G) {
      float m = -FLT_MAX;
      for (int w = 0; w < CWARPS; ++w) m = fmaxf(m, sh.red[w * MGMAX + tid]);
      ll_st(a.ll_cmax + (g * chunks + c) * G + tid, m, tag);
    }
    // the chunk's V rows (contiguous in the head-major cache) into shared memory
    // with asynchronous copies that land while this CTA waits for the other chunks'
    // maxima; this token's row comes from the exchange words in phase B
    const float* vb = L.vc + ((seq * a.nKv + g) * (int64_t)a.max_ctx + j0) * HD;
    float* vs = att_vs(per, chunks);
    const int ncp = j1 == len ? n - 1 : n;
    for (int t = tid; t < ncp * (HD / 4); t += CT)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(vs + 4 * t)), "l"(vb + 4 * t)
                   : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
    cons_sync();
  }

  // ---- attention, phase B: e = FastExp(s*scale - max), partial sums, last CTA of the head combines
  __device__ void attn_pv(const MegaLayer& L, int lay_idx, int g, int c, int chunks, int len) {
    const int G = a.nH / a.nKv, HD = 64;
    const int per = (len + chunks - 1) / chunks;
    const int j0 = min(len, c * per), j1 = min(len, j0 + per), n = j1 - j0;
    const float scale = 1.0f / sqrtf((float)HD);
    const unsigned tag = ll_tag(epoch, lay_idx);
    float* es = att_es();         // [G][per] scores from phase A
    float* pp = att_pp(per);      // [PH][G][64]
    {
      // exact row max of every head of the group: all chunk maxima, gathered in parallel
      float* cm = att_cm(per);  // [chunks][G]
      ll_gather<1>(chunks * G, tag, [&](int i) { return a.ll_cmax + g * chunks * G + i; },
                   [&](int i, float v) { cm[i] = v; });
      cons_sync();
      if (tid < G) {
        float m = -FLT_MAX;
        for (int cc = 0; cc < chunks; ++cc) m = fmaxf(m, cm[cc * G + tid]);
        sh.vec[tid] = m;
      }
      cons_sync();
    }
    for (int t = tid; t < G * n; t += CT) {
      const int h = t / n, jj = t - h * n;
      es[h * per + jj] = pade_exp(__fsub_rn(__fmul_rn(es[h * per + jj], scale), sh.vec[h]));
    }
    // the V rows copied in phase A, and this token's row from the exchange words
    if (j1 == len && tid < HD)
      att_vs(per, chunks)[(n - 1) * HD + tid] = ll_wait1(a.ll_kv + a.kd + g * HD + tid, tag);
    asm volatile("cp.async.wait_all;" ::: "memory");
    cons_sync();
    (void)L;
    const float* vs = att_vs(per, chunks);
    const int d = tid % 64, kp = tid / 64;
    if (kp < PH) {
      float acc[MGMAX];
#pragma unroll
      for (int h = 0; h < MGMAX; ++h) acc[h] = 0.f;
      // unrolled so the shared-memory loads of several keys are in flight together
#pragma unroll 4
      for (int jj = kp; jj < n; jj += PH) {
        const float v = vs[jj * HD + d];
#pragma unroll
        for (int h = 0; h < MGMAX; ++h)
          if (h < G) acc[h] = fmaf(es[h * per + jj], v, acc[h]);
      }
#pragma unroll
      for (int h = 0; h < MGMAX; ++h)
        if (h < G) pp[(kp * MGMAX + h) * 64 + d] = acc[h];
    }
    cons_sync();
    const int base = (g * chunks + c) * G;
    for (int t = tid; t < G * 64; t += CT) {
      const int h = t / 64, dd = t - h * 64;
      float s = 0.f;
      for (int p = 0; p < PH; ++p) s += pp[(p * MGMAX + h) * 64 + dd];
      ll_st(a.ll_pacc + (int64_t)(base + h) * 64 + dd, s, tag);
    }
    {
      const int w = tid >> 5, ln = tid & 31;
      if (w < G) {
        float s = 0.f;
        for (int jj = ln; jj < n; jj += 32) s += es[w * per + jj];
        s = warp_sum(s);
        if (ln == 0) ll_st(a.ll_psum + base + w, s, tag);
      }
    }
    cons_sync();
  }

  // ---- attention, phase C: out[o] = sum_c pacc / sum_c psum for this CTA's slice of the outputs.
  // Output o's partials over the chunks are split into P interleaved parts (one thread
  // each, two chunks polled per round trip); the parts are then added in part order.
  // The last two warps add each spanned head's psum over the chunks.
  __device__ void attn_combine(int lay_idx, int chunks) {
    const int G = a.nH / a.nKv, NO = a.nH * 64;
    const int o0 = (int)((int64_t)NO * blockIdx.x / gridDim.x), o1 = (int)((int64_t)NO * (blockIdx.x + 1) / gridDim.x);
    const int n = o1 - o0;
    if (n <= 0) return;
    const unsigned tag = ll_tag(epoch, lay_idx);
    const int h0 = o0 >> 6, nh = ((o1 - 1) >> 6) - h0 + 1;
    const int P = max(1, min(chunks, (CT - 64) / n));
    float* sums = part;           // [P][n]
    float* tots = part + P * n;   // [nh]
    const int64_t cstride = (int64_t)G * 64;
    if (tid < P * n) {
      const int r = tid % n, pp = tid / n;
      const int o = o0 + r, h = o >> 6, g = h / G;
      const u64* base = a.ll_pacc + (int64_t)g * chunks * cstride + (int64_t)(h - g * G) * 64 + (o & 63);
      float sm = 0.f;
      for (int c = pp; c < chunks; c += 2 * P) {
        const bool two = c + P < chunks;
        float v0, v1;
        ll_wait2(base + c * cstride, base + (two ? c + P : c) * cstride, tag, v0, v1);
        sm += v0;
        if (two) sm += v1;
      }
      sums[pp * n + r] = sm;
    }
    const int w = tid >> 5, ln = tid & 31;
    if (w >= CWARPS - 2) {
      for (int hi = CWARPS - 1 - w; hi < nh; hi += 2) {
        const int h = h0 + hi, g = h / G;
        const u64* base = a.ll_psum + (int64_t)g * chunks * G + (h - g * G);
        float sm = 0.f;
        for (int c = ln; c < chunks; c += 64) {
          float v0, v1;
          ll_wait2(base + (int64_t)c * G, base + (int64_t)min(c + 32, chunks - 1) * G, tag, v0, v1);
          sm += v0;
          if (c + 32 < chunks) sm += v1;
        }
        sm = warp_sum(sm);
        if (ln == 0) tots[hi] = sm;
      }
    }
    cons_sync();
    for (int t = tid; t < n; t += CT) {
      float sm = 0.f;
      for (int pp = 0; pp < P; ++pp) sm += sums[pp * n + t];
      ll_st(a.ll_att + o0 + t, sm * __fdiv_rn(1.f, tots[((o0 + t) >> 6) - h0]), tag);
    }
    cons_sync();
  }
};

template <bool AM>
__global__ void __launch_bounds__(MT, 1) decode_mega_kernel(const __grid_constant__ MegaArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Shared& sh = *(Shared*)smem_raw;
  float* part = (float*)(smem_raw + ((sizeof(Shared) + 127) / 128) * 128);
  uint8_t* ring = smem_raw + a.ring_offset;
  const int64_t slot_bytes = (int64_t)(((a.smem_bytes - a.ring_offset) / a.nslots) / 128 * 128);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < a.nslots; ++i) {
      mbar_init(&sh.full[i], 1);
      mbar_init(&sh.empty[i], CWARPS);
    }
    sh.abort = 0;
    sh.consumed = 0;
    sh.phase = -1;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // the sequence id is read once: every later use (attention, KV append, the L2
  // prefetch of the layer's K/V rows) reads the shared copy
  __shared__ int seq_s;
  __shared__ unsigned epoch_s;
  if (tid == 0) {
    seq_s = *a.seq;
    epoch_s = __ldcg(a.epoch);
  }
  __syncthreads();
  const int seqv = seq_s;
  const int len = a.kv_len[seqv] + 1;  // context including this token
  if (len > a.max_ctx) {
    if (tid == 0 && blockIdx.x == 0) atomicExch(a.status, SM_ERR_SHAPE);
    return;
  }
  if (warp == CWARPS) {
    // ------------------------------------------------------------ producer
    if ((tid & 31) == 0) {
      Producer<AM> p{a, sh, ring, slot_bytes};
      // one call site per kind of work keeps the kernel's code small (phase p:
      // layer p / 4, Q|K|V, O, gate|up, down; the last one is the LM head)
      for (int ph = 0; ph <= 4 * a.n_layers; ++ph) {
        const int l = ph >> 2, kind = ph & 3;
        const bool head = l == a.n_layers;
        const MegaLayer& L = a.layers[head ? 0 : l];
        const int ns = (kind == 0 && !head) ? 3 : 1;
        for (int s = 0; s < ns; ++s) {
          const MegaSeg& sg = head ? a.head : (kind == 0 ? L.qkv[s] : (kind == 1 ? L.o : (kind == 2 ? L.gu : L.down)));
          const int K = (kind == 1 && !head) ? a.qd : ((kind == 3 && !head) ? a.F : a.H);
          const int rb = head ? a.stage_rows_v : (kind == 3 ? a.stage_rows_f : a.stage_rows_h);
          const int c0 = ns == 3 ? L.qkv_cb[s] : 0, c1 = ns == 3 ? L.qkv_cb[s + 1] : -1;
          p.seg(sg, K, rb, ph, c0, c1);
        }
      }
      // drain: wait (bounded) until every stage issued has landed before exiting
      if (!p.ok) {
        for (int kk = max(0, p.k - a.nslots); kk < p.k; ++kk)
          mbar_wait_bounded(&sh.full[kk % a.nslots], (kk / a.nslots) & 1, nullptr);
      }
    }
    return;
  }
  // -------------------------------------------------------------- consumers
  Consumer<AM> c{a, sh, ring, slot_bytes, part};
  c.tid = tid;
  c.epoch = epoch_s;
  c.seq_v = seqv;
  c.ep.pos = nullptr;
  c.ep.seq = &seq_s;
  c.ep.head_dim = a.hd;
  c.ep.n_kv = a.nKv;
  c.ep.max_ctx = a.max_ctx;
  // the position of this token = the sequence length before it: kv_len[seq]
  __shared__ int pos_s;
  __shared__ float rope_s[2][64];  // sin / cos row of this position (head_dim <= 128)
  if (tid == 0) pos_s = len - 1;
  const int half = a.hd / 2;
  for (int t = tid; t < half; t += CT) {
    rope_s[0][t] = a.sin_t[(int64_t)(len - 1) * half + t];
    rope_s[1][t] = a.cos_t[(int64_t)(len - 1) * half + t];
  }
  if (tid < (int)(sizeof(MegaLayer) / 4)) ((int*)&sh.lay[0])[tid] = __ldg((const int*)&a.layers[0] + tid);
  cons_sync();
  c.ep.pos = &pos_s;
  // epilogue reads table[pos * half + i]: point at the shared row shifted back by pos * half
  c.ep.sin_t = &rope_s[0][0] - (int64_t)(len - 1) * half;
  c.ep.cos_t = &rope_s[1][0] - (int64_t)(len - 1) * half;
  c.stamp();
  const float* emb = a.embd + (int64_t)(*a.token) * a.H;
  const int G = a.nH / a.nKv;
  const int chunks = max(1, (int)gridDim.x / a.nKv);
  (void)G;
  // one call site per kind of work keeps the kernel's code small: phase p is
  // layer p / 4, kind Q|K|V (attention follows), O, gate|up, down; the last
  // phase is the LM head
  // Steps of a layer: 0 Q|K|V, 1 attention scores, 2 exp / P.V, 3 combine, 4 O,
  // 5 gate|up, 6 down; the last step is the LM head.  One transition call site and
  // one call site per kind of work keep the kernel's code small (every layer runs
  // all of it once; what misses the instruction cache is fetched again).
  const int nsteps = 7 * a.n_layers + 1;
  for (int st = 0; st < nsteps; ++st) {
    const int l = st / 7, k = st - 7 * l;
    const bool attn = k >= 1 && k <= 3;
    // the GEMV phase of this step (layer l; kind Q|K|V, O, gate|up, down; the head)
    const int ph = attn ? -1 : 4 * l + (k == 0 ? 0 : k - 3);
    const MegaLayer& L = sh.lay[l & 1];
    // the transition before a GEMV step plans it; the one before gate|up brings the
    // next layer's table entry on chip; the one before Q|K|V prefetches this CTA's
    // attention K / V rows of the layer into L2 (they are read two steps later)
    const bool nx = k == 5 && l + 1 < a.n_layers;
    if (!c.transition(nx ? &a.layers[l + 1] : nullptr, (l + 1) & 1, ph, emb, k == 0 && l < a.n_layers ? &L : nullptr, chunks, len))
      return;
    if (attn) {
      // every wait on another CTA's result is a poll of its exchange words
      if (k == 3) {
        c.attn_combine(l, chunks);
      } else {
        for (int it = blockIdx.x; it < a.nKv * chunks; it += gridDim.x) {
          if (k == 1)
            c.attn_scores(L, l, it / chunks, it % chunks, chunks, len);
          else
            c.attn_pv(L, l, it / chunks, it % chunks, chunks, len);
        }
      }
      continue;
    }
    const SegPlan& P = sh.plan;
    if (c.lx >= 4 && c.lx < 12) c.stamp_at(900 + 8 * (c.lx - 4) + 6);
    c.load_x(P.src, P.src_ll, P.src_tag, P.gamma, P.K, P.s->fmt != SM_Q8_0, P.mma ? P.s->fmt : 0, P.r1 > P.r0);
    if (tid == 0) sh.phase = ph;
    if (!c.seg(P)) return;
  }
  c.stamp();
  // greedy argmax over the CTAs' partial maxima (lowest id on ties); the last CTA commits
  __threadfence();
  cons_sync();
  __shared__ int last_s;
  if (tid == 0) {
    const unsigned old = atomicAdd(&a.sync[63], 1u);
    last_s = old == gridDim.x - 1;
    __threadfence();
  }
  cons_sync();
  if (last_s && tid < 32) {
    // the CTA that arrives last reduces every CTA's (max, index) in one warp
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int b = tid; b < (int)gridDim.x; b += 32) {
      const float v = __ldcg(&a.amax_val[b]);
      const int i = __ldcg(&a.amax_idx[b]);
      if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (tid == 0) {
      *a.next_token = bi;
      a.kv_len[seqv] = len;
      // every CTA has read the epoch and finished its exchange (it arrived above):
      // the next launch tags its words with the next epoch
      *a.epoch = epoch_s + 1u;
    }
  }
}

}  // namespace

int mega_grid_size() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

size_t mega_scratch_floats(int nH, int nKv, int hd, int max_ctx, int grid) {
  const int chunks = std::max(1, grid / nKv);
  const int G = nH / nKv;
  return (size_t)nH * max_ctx + (size_t)nKv * chunks * G * (2 + hd) + 2 * (size_t)grid + 64;
}

namespace {
// region sizes in 64-bit words, each rounded up to a 16-byte multiple
struct LLLayout {
  size_t off[10];
  size_t total;
};
LLLayout ll_layout(int H, int qd, int kd, int F, int nH, int nKv, int hd, int grid) {
  const size_t chunks = std::max(1, grid / nKv), G = nH / nKv;
  const size_t n[10] = {2,  // epoch word (+ pad)
                        (size_t)H, (size_t)H, (size_t)qd, 2 * (size_t)kd, nKv * chunks * G, nKv * chunks * G * hd,
                        nKv * chunks * G, (size_t)qd, (size_t)F};
  LLLayout L;
  size_t o = 0;
  for (int i = 0; i < 10; ++i) {
    L.off[i] = o;
    o += (n[i] + 1) & ~(size_t)1;
  }
  L.total = o;
  return L;
}
}  // namespace

size_t mega_ll_words(int H, int qd, int kd, int F, int nH, int nKv, int hd, int grid) {
  return ll_layout(H, qd, kd, F, nH, nKv, hd, grid).total;
}

void mega_ll_assign(MegaArgs& a, unsigned long long* base, int grid) {
  const LLLayout L = ll_layout(a.H, a.qd, a.kd, a.F, a.nH, a.nKv, a.hd, grid);
  a.epoch = (unsigned*)base;
  a.ll_x0 = base + L.off[1];
  a.ll_x1 = base + L.off[2];
  a.ll_q = base + L.off[3];
  a.ll_kv = base + L.off[4];
  a.ll_cmax = base + L.off[5];
  a.ll_pacc = base + L.off[6];
  a.ll_psum = base + L.off[7];
  a.ll_att = base + L.off[8];
  a.ll_act = base + L.off[9];
}

bool mega_supported(const MegaArgs& a) {
  if (a.hd != 64 || a.nH % a.nKv || a.nH / a.nKv > MGMAX) return false;
  if ((a.H % 256) || (a.qd % 256) || (a.F % 32)) return false;
  if (a.H / 32 > CT || a.qd / 32 > CT || a.F / 32 > CT) return false;
  return true;
}

void mega_layer_split(MegaLayer& L, int K, int grid) {
  int64_t b[3], tot = 0;
  for (int i = 0; i < 3; ++i) {
    b[i] = (int64_t)L.qkv[i].rows * (row_bytes_fmt(L.qkv[i].fmt, K) + aux_row_bytes(L.qkv[i]));
    tot += b[i];
  }
  int* cb = L.qkv_cb;
  cb[0] = 0;
  cb[1] = (int)std::min<int64_t>(grid - 2, std::max<int64_t>(1, (grid * b[0] + tot / 2) / tot));
  cb[2] = (int)std::min<int64_t>(grid - 1, std::max<int64_t>(cb[1] + 1, cb[1] + (grid * b[1] + tot / 2) / tot));
  cb[3] = grid;
}

bool mega_seg_mma_ok(const MegaSeg& s) {
  return s.fmt == SM_Q4_K || (s.fmt == SM_Q6_K && s.aux_stride > 0 && (s.aux_stride * 2) % 16 == 0);
}

bool mega_seg_supported(const MegaSeg& s) {
  if (s.fmt == SM_Q4_K) return true;
  return (s.fmt == SM_Q6_K || s.fmt == SM_Q8_0 || s.fmt == SM_Q4_0) && s.aux_stride > 0;
}

int launch_decode_mega(MegaArgs& a, cudaStream_t st, int* n_launch) {
  const int grid = mega_grid_size();
  int optin = 0, dev0 = 0;
  cudaGetDevice(&dev0);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev0);
  const int smem_total = optin - 1024;  // leave room for the kernel's static shared memory
  a.smem_bytes = smem_total;
  // stage rows: ~24 KB per stage
  auto rb_for = [](int64_t row_bytes, int mult) {
    return (int)std::max<int64_t>(1, (40 * 1024) / (row_bytes * mult));
  };
  // largest staged row (weights + padded scales / d) over the formats
  auto max_row_bytes = [](int K) {
    return std::max<int64_t>((int64_t)K / 256 * Q6K_BODY_BYTES + ((int64_t)K / 256 * 2 + 15) / 16 * 16,
                             (int64_t)K + ((int64_t)K / 32 * 4 + 15) / 16 * 16);
  };
  const int64_t rb_h = max_row_bytes(a.H), rb_f = max_row_bytes(a.F);
  a.stage_rows_h = rb_for(rb_h, 2);
  a.stage_rows_f = rb_for(rb_f, 1);
  a.stage_rows_v = rb_for(rb_h, 1);
  const int64_t slot_need = std::max({rb_h * 2 * a.stage_rows_h, rb_f * a.stage_rows_f, rb_h * a.stage_rows_v});
  // partials: the most rows any CTA holds in one segment (GLU: gate + up) x units
  auto cta_rows = [&](int rows) { return 2 * (((rows + 1) / 2 + grid - 1) / grid); };
  auto nwpp = [](int K) { return (int64_t)((K / 32 + 31) / 32); };
  const int64_t part0 = std::max({(int64_t)2 * cta_rows(a.F) * nwpp(a.H), (int64_t)cta_rows(a.qd) * nwpp(a.H),
                                 (int64_t)cta_rows(a.H) * std::max(nwpp(a.qd), nwpp(a.F)),
                                 (int64_t)cta_rows(a.V) * nwpp(a.H), (int64_t)MGMAX * (a.max_ctx / 2 + 64) + 4096,
                                 (int64_t)(MGMAX + 64) * (a.max_ctx / std::max(1, grid / a.nKv) + 2) + 4096 +
                                     (int64_t)std::max(1, grid / a.nKv) * MGMAX,
                                 (int64_t)2 * std::max({a.H, a.qd, a.F}) + 28 * (std::max({a.H, a.qd, a.F}) / 32) + 64});
  // MMA segments: digit planes (50 floats per unit + 1 per block) after the
  // staged vector, then the block partials and the warps' scratch
  auto mma_part = [&](int K, int rows, int nT, bool gamma) {
    const int64_t tiles = (rows / nT + 15) / 16;
    return (int64_t)(gamma ? 2 : 1) * K + 50 * (K / 32) + K / 256 + 4 + tiles * nT * (K / 256) * 16 + (int64_t)CWARPS * 320;
  };
  const int64_t part = std::max({part0, mma_part(a.H, cta_rows(2 * a.F), 2, true),
                                 mma_part(a.H, cta_rows(4 * a.qd), 1, true), mma_part(a.H, cta_rows(a.V), 1, true),
                                 mma_part(a.qd, cta_rows(a.H), 1, false), mma_part(a.F, cta_rows(a.H), 1, false)});
  a.part_floats = (int)part;
  a.use_mma = 1;  // SMALLMIND_MEGA_MMA=0: Q4_K / Q6_K phases on the dp4a path
  if (const char* e = std::getenv("SMALLMIND_MEGA_MMA")) a.use_mma = atoi(e);
  const int shared_bytes = (int)((sizeof(Shared) + 127) / 128 * 128);
  a.ring_offset = (int)((shared_bytes + part * 4 + 127) / 128 * 128);
  const int64_t ring = smem_total - a.ring_offset;
  const int64_t slot = (slot_need + 127) / 128 * 128;
  a.nslots = (int)std::min<int64_t>(16, ring / slot);
  if (const char* e = std::getenv("SMALLMIND_MEGA_SLOTS")) a.nslots = std::max(2, std::min(a.nslots, atoi(e)));
  if (const char* e = std::getenv("SMALLMIND_MEGA_LOOKAHEAD")) a.lookahead = atoi(e);
  if (a.nslots < 2) return fail(SM_ERR_UNSUPPORTED, "decode_mega: shared memory too small for the stage ring");
  // the kernel recomputes the slot size as (227 KB - ring_offset) / nslots rounded down to 128 B
  if ((int64_t)(((smem_total - a.ring_offset) / a.nslots) / 128 * 128) < slot_need)
    return fail(SM_ERR_UNSUPPORTED, "decode_mega: stage slot too small");
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    SM_CUDA_TRY(cudaFuncSetAttribute(decode_mega_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_total));
    SM_CUDA_TRY(cudaFuncSetAttribute(decode_mega_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_total));
    attr_set[dev] = true;
  }
  SM_CUDA_TRY(cudaMemsetAsync(a.sync, 0, 64 * sizeof(unsigned), st));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(MT);
  cfg.dynamicSmemBytes = smem_total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barriers rely on it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.use_mma && a.mma_only)
    SM_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_mega_kernel<true>, a));
  else
    SM_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_mega_kernel<false>, a));
  if (n_launch) *n_launch += 1;
  return SM_OK;
}

}  // namespace sm
