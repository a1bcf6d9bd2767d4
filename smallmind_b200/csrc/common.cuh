// Shared definitions of the SmallMind.Cuda library (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/smallmind_cuda.h"

namespace sm {

// ---------------------------------------------------------------- errors
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

#define SM_CUDA_TRY(expr)                                                                        \
  do {                                                                                           \
    cudaError_t _e = (expr);                                                                     \
    if (_e != cudaSuccess)                                                                       \
      return ::sm::fail(SM_ERR_CUDA, std::string(#expr " failed: ") + cudaGetErrorString(_e)); \
  } while (0)

#define SM_TRY(expr)          \
  do {                        \
    int _rc = (expr);         \
    if (_rc != SM_OK) return _rc; \
  } while (0)

// ---------------------------------------------------------------- device weight
// Device layout of a packed weight.  Q8_0/Q4_0/Q4_K keep the reference bytes
// as uploaded.  Q6_K blocks (210 B, only 2-byte aligned) are re-laid for
// 128-bit loads: a 208 B body per block [ql 128 | qh' 64 | int8 scales 16] in
// `data` (qh' is the high-bit plane re-packed, see q6k_relayout_kernel), and
// the fp16 super-scale d of every block in `aux` (same block order).
struct DevWeight {
  int scheme = 0;
  int layout = 0;
  int rows = 0, cols = 0;  // reference Rows / Cols
  int block_size = 0;      // Q8_0 / Q4_0 scale block
  int64_t n = 0;           // rows * cols
  void* data = nullptr;
  void* aux = nullptr;     // Q8_0/Q4_0: float scales; Q6_K: half d[]
  size_t data_bytes = 0, aux_bytes = 0;
  // INTENDED-layout weights keep each row's scales (Q8_0/Q4_0) or d values (Q6_K)
  // in a row of `aux_stride` elements, padded to 16 bytes, so a row's packed
  // bytes and its scales can both be moved with 16-byte bulk copies.
  // aux_stride == 0: scales in plain linear block order.
  int aux_bpr = 0;     // scale blocks per row
  int aux_stride = 0;  // elements per padded row
  // matmul orientation view: N outputs, K inputs
  int N() const { return layout == SM_LAYOUT_INTENDED ? rows : cols; }
  int K() const { return layout == SM_LAYOUT_INTENDED ? cols : rows; }
};

// linear scale-block index -> index in the (possibly row-padded) aux array
__host__ __device__ __forceinline__ int64_t aux_idx(int64_t b, int bpr, int stride) {
  return stride ? (b / bpr) * stride + (b % bpr) : b;
}

// Q4_1 / Q5_0 (block 32): the aux array holds the block scales and, beside them,
// a second value per block (Q4_1: the min; Q5_0: the 32 high bits as a uint32).
// Row-padded aux (aux_stride > 0): a row is [scales (bpr) | second (bpr) | pad];
// plain aux: [scales (all blocks) | second (all blocks)].
__host__ __device__ __forceinline__ int64_t aux_second_idx(int64_t b, int bpr, int stride, int64_t nblocks) {
  return stride ? (b / bpr) * stride + bpr + (b % bpr) : nblocks + b;
}

// w of element li of a Q4_1 / Q5_0 weight (Q4_1Tensor.cs:153-156: q * scale + min;
// Q5_0Tensor.cs:157-172: (low | high << 4) - 16, times scale)
__device__ __forceinline__ float q41_q50_weight(int scheme, const void* data, const void* aux, int bpr, int stride,
                                                int64_t nblocks, int64_t li) {
  const int64_t b = li >> 5;
  const uint8_t p = ((const uint8_t*)data)[li >> 1];
  const int lo4 = (li & 1) ? (p >> 4) : (p & 0xF);
  const float* af = (const float*)aux;
  const float sc = af[aux_idx(b, bpr, stride)];
  if (scheme == 4 /* SM_Q4_1 */) return __fadd_rn(__fmul_rn((float)lo4, sc), af[aux_second_idx(b, bpr, stride, nblocks)]);
  const uint32_t hb = ((const uint32_t*)aux)[aux_second_idx(b, bpr, stride, nblocks)];
  const int q = (lo4 | (int)(((hb >> (li & 31)) & 1u) << 4)) - 16;
  return __fmul_rn((float)q, sc);
}

constexpr int Q4K_BLOCK_BYTES = 144;
constexpr int Q6K_BLOCK_BYTES = 210;
constexpr int Q6K_BODY_BYTES = 208;

// ---------------------------------------------------------------- device helpers
// Reference HalfToFloat (Q4KTensor.cs:155-191) is exact IEEE fp16->fp32, which
// is what the hardware conversion does.
__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ void unpack_q4k_scales(const uint8_t* s, int j, int& sc, int& mn) {
  // Q4KTensor.cs:109-126 sequential 6-bit packing; s = 12 scale bytes.
  const int base = (j < 4) ? 0 : 3;
  const int jj = j & 3;
  const uint8_t* t = s + base;
  const uint8_t* u = s + 6 + base;
  switch (jj) {
    case 0: sc = t[0] & 0x3F; mn = u[0] & 0x3F; break;
    case 1: sc = (t[0] >> 6) | ((t[1] & 0x0F) << 2); mn = (u[0] >> 6) | ((u[1] & 0x0F) << 2); break;
    case 2: sc = (t[1] >> 4) | ((t[2] & 0x03) << 4); mn = (u[1] >> 4) | ((u[2] & 0x03) << 4); break;
    default: sc = (t[2] >> 2) & 0x3F; mn = (u[2] >> 2) & 0x3F; break;
  }
}

// Pade exp of MathUtils.FastExp (MathUtils.cs:20-32), every op separately
// rounded (no FMA contraction), IEEE division: bit-exact with the reference.
__device__ __forceinline__ float pade_exp(float x) {
  x = fmaxf(-87.3f, fminf(x, 88.7f));
  float x2 = __fmul_rn(x, x);
  float hx = __fmul_rn(x, 0.5f);
  float cx = __fmul_rn(x2, 0.08333333f);
  float num = __fadd_rn(__fadd_rn(1.0f, hx), cx);
  float den = __fadd_rn(__fsub_rn(1.0f, hx), cx);
  return __fdiv_rn(num, den);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// ---------------------------------------------------------------- launch accounting
struct LaunchCounter {
  int64_t* counter = nullptr;
  void add(int64_t k = 1) const {
    if (counter) *counter += k;
  }
};

// capi.cu: device, stream and launch counter of a context
int ctx_view(sm_ctx* ctx, int* device, cudaStream_t* stream, int64_t** launches);

// ---------------------------------------------------------------- kernel entry points (host wrappers)
// quant.cu
int launch_dequant(const DevWeight& w, float* out, cudaStream_t st);
int launch_quantize(int scheme, const float* src, int64_t n, int bs, void* data, float* scales, cudaStream_t st);
int launch_q6k_relayout(const uint8_t* src, uint8_t* body, uint16_t* d, int64_t nblocks, int bpr, int stride,
                        cudaStream_t st);
// gemv.cu: y[m][n] (+)= x[m][k] . W^T over a row range; epilogue: 0 store, 1 add into y
int launch_matmul(const DevWeight& w, const float* x, float* y, int M, int ldy, int accumulate, cudaStream_t st,
                  int* n_launch);
// ops.cu
int launch_rmsnorm(const float* x, const float* gamma, float* y, int rows, int F, float eps, cudaStream_t st);
int launch_rope_rows(float* x, int rows, int row_stride, int n_heads, int hd, const int* positions,
                     const float* sin_t, const float* cos_t, cudaStream_t st);
int launch_silu_mul(const float* g, const float* u, float* out, int64_t n, cudaStream_t st);
int launch_embed(const float* table, const int* tokens, float* x, int n, int H, cudaStream_t st);
// Tensor-parallel group (tp.cu): NCCL loaded at run time
int tp_unique_id(void* out, size_t n);
int tp_comm_create(int size, int rank, const void* id, size_t n, void** comm);
void tp_comm_destroy(void* comm);
int tp_allreduce_sum(void* comm, float* buf, size_t n, cudaStream_t st);
int launch_add(float* x, const float* p, int64_t n, cudaStream_t st);
int launch_argmax(const float* logits, int rows, int V, int* out, cudaStream_t st);
// attention.cu  (K/V element d of key j, kv head g: base + j*row_stride + g*head_stride + d)
// causal GQA prefill attention on tcgen05 (hd 64); SM_ERR_UNSUPPORTED when the shape is not handled
int launch_attention_prefill_tc(const float* q, int q_stride, const float* k, const float* v, int64_t row_stride,
                                int64_t head_stride, float* out, int out_stride, int T, int S, int nH, int nKv, int hd,
                                int* status, cudaStream_t st, int* n_launch);
int launch_attention_prefill(const float* q, int q_stride, const float* k, const float* v, int64_t row_stride,
                             int64_t head_stride, float* out, int out_stride, int T, int S, int nH, int nKv, int hd,
                             cudaStream_t st, int* n_launch);
int launch_attention_decode(const float* q, int q_stride, const float* kc, const float* vc, int64_t seq_stride,
                            int64_t row_stride, int64_t head_stride, int max_ctx, float* out, int out_stride,
                            const int* lens, const int* seq_map, int B, int nH, int nKv, int hd, float* scratch,
                            size_t scratch_floats, cudaStream_t st, int* n_launch);
size_t attention_decode_scratch_floats(int B, int nH, int max_ctx);
int launch_attention_decode_cluster(const float* q, int q_stride, const float* kc, const float* vc,
                                    int64_t seq_stride, int64_t row_stride, int64_t head_stride, int max_ctx,
                                    float* out, int out_stride, const int* lens, const int* seq_map, int B, int nH,
                                    int nKv, int hd, cudaStream_t st, int* n_launch);
int launch_rope_qk_append(float* qkv, int rows, int qkv_stride, int nH, int nKv, int hd, const int* positions,
                          const int* seq_ids, const float* sin_t, const float* cos_t, float* kc, float* vc,
                          int max_ctx, cudaStream_t st);

}  // namespace sm
