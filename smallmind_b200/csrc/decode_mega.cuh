// Persistent one-launch decode step (bs1): interface.
#pragma once
#include "common.cuh"
#include "gemv1.cuh"

namespace sm {

// One GEMV of a phase: rows of an INTENDED-layout weight (GLU: gate rows with
// the matching up rows from data2/aux2).
struct MegaSeg {
  int fmt = 0, rows = 0, bs = 0, mode = 0;
  int aux_bpr = 0, aux_stride = 0;  // row-padded scales / d (required when the format has them)
  const uint8_t* data = nullptr;
  const void* aux = nullptr;
  const uint8_t* data2 = nullptr;
  const void* aux2 = nullptr;
  float* y = nullptr;  // output (STORE/ADD/GLU/ROPE_Q) or the layer's K/V cache base
};

struct MegaLayer {
  MegaSeg qkv[3];  // Q (ROPE_Q -> q), K (ROPE_K_CACHE -> k cache), V (V_CACHE -> v cache)
  MegaSeg o;       // ADD -> x
  MegaSeg gu;      // GLU -> act
  MegaSeg down;    // ADD -> x
  const float* attn_norm = nullptr;
  const float* ffn_norm = nullptr;
  const float* kc = nullptr;  // layer bases of the head-major cache
  const float* vc = nullptr;
  int qkv_cb[4] = {0, 0, 0, 0};  // CTAs [qkv_cb[s], qkv_cb[s + 1]) run segment s (mega_layer_split)
};

struct MegaArgs {
  int n_layers = 0, H = 0, qd = 0, kd = 0, F = 0, V = 0, nH = 0, nKv = 0, hd = 0, max_ctx = 0;
  float eps = 1e-5f;
  const MegaLayer* layers = nullptr;  // device array [n_layers]
  MegaSeg head;                       // STORE -> logits
  const float* out_norm = nullptr;
  const float* embd = nullptr;
  const float* sin_t = nullptr;
  const float* cos_t = nullptr;
  float* x = nullptr;       // residual stream [H]
  float* q = nullptr;       // rotated queries [qd]
  float* att = nullptr;     // attention output [qd]
  float* act = nullptr;     // silu(gate) * up [F]
  float* logits = nullptr;  // [V]
  int* next_token = nullptr;
  const int* token = nullptr;  // device scalar
  const int* seq = nullptr;    // device scalar
  int* kv_len = nullptr;       // per-sequence lengths (read, then +1 at the end)
  // scratch
  float* scores = nullptr;  // [nH][max_ctx]
  float* cmax = nullptr;    // [nKv][chunks][G]
  float* psum = nullptr;    // [nKv][chunks][G]
  float* pacc = nullptr;    // [nKv][chunks][G][hd]
  float* amax_val = nullptr;  // [grid]
  int* amax_idx = nullptr;    // [grid]
  unsigned* sync = nullptr;   // [63] argmax counter (zeroed per launch)
  // Tagged exchange words: the CTAs hand each other the step's vectors as 64-bit
  // words {float value, uint32 tag} (low / high half), stored and polled with
  // gpu-scope relaxed 8-byte accesses, so a word carries its own readiness and no
  // grid-wide barrier is needed.  tag = ((epoch + 1) << 8) | (layer & 255); the
  // epoch advances once per launch (last CTA), so no buffer is ever cleared.
  unsigned long long* ll_x0 = nullptr;    // [H] residual stream after attention (O + residual)
  unsigned long long* ll_x1 = nullptr;    // [H] residual stream after the MLP (down + residual)
  unsigned long long* ll_q = nullptr;     // [qd] rotated queries
  unsigned long long* ll_kv = nullptr;    // [2 kd] this token's rotated K row, then its V row
  unsigned long long* ll_cmax = nullptr;  // [nKv][chunks][G] chunk maxima of the scaled scores
  unsigned long long* ll_pacc = nullptr;  // [nKv][chunks][G][hd] chunk partials of e.V
  unsigned long long* ll_psum = nullptr;  // [nKv][chunks][G] chunk partial sums of e
  unsigned long long* ll_att = nullptr;   // [qd] attention output
  unsigned long long* ll_act = nullptr;   // [F] silu(gate) * up
  unsigned* epoch = nullptr;              // launch counter (device word, never reset)
  int* status = nullptr;
  unsigned long long* trace = nullptr;  // optional [grid][MEGA_TRACE_EVENTS] globaltimer stamps
  // schedule
  int nslots = 0, ring_offset = 0, part_floats = 0, smem_bytes = 0;
  int stage_rows_h = 1, stage_rows_f = 1, stage_rows_v = 1;
  int use_mma = 1;    // Q4_K / Q6_K phases on the int8 tensor-core path
  int mma_only = 0;   // every GEMV segment can take that path (mega_seg_mma_ok): the kernel without the dp4a path runs
  int lookahead = 1;  // 0: the producer only issues a phase's stages once the consumers entered it  // stage rows for K = H / qd, K = F, LM head
};

constexpr int MEGA_TRACE_EVENTS = 1024;

// Sizes of the scratch the launcher expects (floats / ints) for a given grid.
size_t mega_scratch_floats(int nH, int nKv, int hd, int max_ctx, int grid);
// 64-bit words of the tagged exchange buffer (epoch word + every ll_* region,
// each region starting on a 16-byte boundary)
size_t mega_ll_words(int H, int qd, int kd, int F, int nH, int nKv, int hd, int grid);
// points a's ll_* regions and epoch into `base` (mega_ll_words words)
void mega_ll_assign(MegaArgs& a, unsigned long long* base, int grid);
bool mega_supported(const MegaArgs& a);
// Q|K|V CTA ranges of a layer for a grid of `grid` CTAs, in proportion to each segment's bytes
void mega_layer_split(MegaLayer& L, int K, int grid);
// the segment's format has the int8 tensor-core path (Q4_K; Q6_K with a 16-byte multiple d row)
bool mega_seg_mma_ok(const MegaSeg& s);
bool mega_seg_supported(const MegaSeg& s);
int launch_decode_mega(MegaArgs& a, cudaStream_t st, int* n_launch);
int mega_grid_size();

}  // namespace sm
