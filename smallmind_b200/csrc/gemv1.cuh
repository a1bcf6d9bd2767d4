// Launch interface of the M = 1 decode GEMV (gemv1.cu).
#pragma once
#include "common.cuh"

namespace sm {

constexpr int GEMV_MAX_SEG = 4;
// STORE: y[row] = v; ADD: y[row] += v (residual); GLU: y[row] = silu(gate) * up;
// ROPE_Q: RoPE on pairs, then store; ROPE_K_CACHE / V_CACHE: (RoPE and) store into the
// head-major KV cache at (*seq, *pos).
enum { GEMV_STORE = 0, GEMV_ADD = 1, GEMV_GLU = 2, GEMV_ROPE_Q = 3, GEMV_ROPE_K_CACHE = 4, GEMV_V_CACHE = 5 };

struct GemvSeg {
  int fmt = 0, rows = 0, bs = 0, mode = 0;
  int aux_bpr = 0, aux_stride = 0;  // DevWeight::aux_bpr / aux_stride
  const uint8_t* data = nullptr;
  const void* aux = nullptr;
  const uint8_t* data2 = nullptr;  // GLU: the up-projection weight (same scheme and shape)
  const void* aux2 = nullptr;
  float* y = nullptr;
  int group_begin = 0;
};

struct GemvArgs {
  GemvSeg seg[GEMV_MAX_SEG];
  int nseg = 0, ngroups = 0, K = 0;
  const float* x = nullptr;
  const float* gamma = nullptr;  // non-null: RMSNorm x first (eps below)
  float eps = 1e-5f;
  int S = 1;  // warps per row group (set by the launcher)
  // RoPE / KV-cache epilogues
  const int* pos = nullptr;
  const int* seq = nullptr;
  const float* sin_t = nullptr;
  const float* cos_t = nullptr;
  int head_dim = 0, n_kv = 0, max_ctx = 0;
};


bool gemv1_supports(const DevWeight& w, int K);
// true when one gemv1 launch can mix segments of formats fa and fb (fa == fb, or Q4_K with Q6_K)
bool gemv1_mix_ok(int fa, int fb);
int gemv1_segment(GemvArgs& a, const DevWeight& w, const DevWeight* w2, float* y, int mode);
int launch_gemv1(const GemvArgs& a, cudaStream_t st, int* n_launch);
// y[M][N] (+)= x[M][K] W^T on tcgen05 (INTENDED layout, M >= 5, K % 64 == 0)
bool gemm_tc_supports(const DevWeight& W, int M);
int launch_gemm_tc(const DevWeight& W, const float* x, float* y, int M, int ldy, int accumulate, int* status,
                   cudaStream_t st, int* n_launch);
// up to 3 weights with the same K stacked along N, each with its own output (ys[i], row stride ldys[i]);
// every weight but the last must have N % 128 == 0
bool gemm_tc_supports_multi(const DevWeight* const* W, int nw, int M);
// Drops the resident fp16 planes of every weight group that contains this weight
// (called before the weight's memory is freed).
void gemm_tc_release_weight(const void* data);
// What the GEMM's x-split pass applies to x first (the producer of the fp16 planes):
// nothing, RMSNorm (RMSNormOps.cs:28-220, gamma / eps) or the SiLU gate
// silu(x) * u (ActivationOps.cs:565-580), so the block's norm / activation
// kernels and their fp32 round trip are not needed.
enum { XPRO_NONE = 0, XPRO_RMSNORM = 1, XPRO_SILU = 2 };
struct XPro {
  int kind = XPRO_NONE;
  const float* gamma = nullptr;
  float eps = 0.f;
  const float* u = nullptr;  // SILU: the up rows (same shape as x)
};
int launch_gemm_tc_multi(const DevWeight* const* Ws, float* const* ys, const int* ldys, int nw, const float* x, int M,
                         int accumulate, int* status, cudaStream_t st, int* n_launch, const XPro* pro = nullptr);
// Q4_K (INTENDED) y[m] (+)= W x[m] for M rows of x (stride K), y rows of stride ldy
int launch_gemv_mma_q4k_rows(const DevWeight& W, const float* x, int M, float* y, int ldy, int accumulate,
                             int* status, cudaStream_t st, int* n_launch);
// Q6_K (INTENDED, row-padded d) y[m] (+)= W x[m] for M rows of x
int launch_gemv_mma_q6k_rows(const DevWeight& W, const float* x, int M, float* y, int ldy, int accumulate,
                             int* status, cudaStream_t st, int* n_launch);
// Q6_K (INTENDED, row-padded d) y = W x on the int8 tensor-core path
int launch_gemv_mma_q6k(const DevWeight& W, const float* x, float* y, int accumulate, int* status, cudaStream_t st,
                        int* n_launch);
// Q4_K (INTENDED) y = W x on the int8 tensor-core path (mma.sync m16n8k32)
// Q8_0 / Q4_0, M = 1, on the int8 tensor cores (gemv_mma_q8.cu); SM_ERR_UNSUPPORTED when the shape does not fit
int launch_gemv_mma_q80(const DevWeight& W, const float* x, float* y, int accumulate, int* status, cudaStream_t st,
                        int* n_launch);
int launch_gemv_mma_q4k(const DevWeight& W, const float* x, float* y, int accumulate, int* status, cudaStream_t st,
                        int* n_launch);

}  // namespace sm
