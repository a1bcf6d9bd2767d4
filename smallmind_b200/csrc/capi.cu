// C-ABI implementation: contexts, weights, ops, the device-resident LLaMA
// model with its HBM KV cache, and the prefill / decode drivers.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <vector>

#include "common.cuh"
#include "gemv1.cuh"
#include "decode_mega.cuh"

// ---------------------------------------------------------------- errors
namespace sm {
static thread_local std::string g_last_error;
void set_error(const std::string& msg) { g_last_error = msg; }
int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
}  // namespace sm

using namespace sm;

struct sm_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int64_t launches = 0;
  int* dev_status = nullptr;  // device-side status word (bounded waits, range checks)
  void* tp_comm = nullptr;    // tensor-parallel group (NCCL communicator), sm_tp_init
  int tp_size = 1, tp_rank = 0;
};

struct sm_weight {
  sm_ctx* ctx = nullptr;
  int device = 0;  // destroy needs only this, so a weight may outlive its context
  DevWeight w;
};

namespace sm {
// Read-only view of a context for entry points defined in other files.
int ctx_view(sm_ctx* ctx, int* device, cudaStream_t* stream, int64_t** launches) {
  if (!ctx) return fail(SM_ERR_INVALID_ARG, "null ctx");
  *device = ctx->device;
  *stream = ctx->stream;
  *launches = &ctx->launches;
  return SM_OK;
}
}  // namespace sm

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

bool valid_scheme(int s) {
  return s == SM_F32 || s == SM_Q8_0 || s == SM_Q4_0 || s == SM_Q4_1 || s == SM_Q5_0 || s == SM_Q4_K || s == SM_Q6_K;
}

size_t packed_bytes(int scheme, int64_t n) {
  switch (scheme) {
    case SM_F32: return (size_t)n * 4;
    case SM_Q8_0: return (size_t)n;
    case SM_Q4_0: return (size_t)(n + 1) / 2;
    case SM_Q4_1: return (size_t)(n + 1) / 2;                          // nibbles
    case SM_Q5_0: return (size_t)(n + 1) / 2 + 4 * (size_t)((n + 31) / 32);  // low nibbles, then 32 high bits per block
    case SM_Q4_K: return (size_t)(n / 256) * Q4K_BLOCK_BYTES;
    case SM_Q6_K: return (size_t)(n / 256) * Q6K_BLOCK_BYTES;
  }
  return 0;
}

// Device scratch for a host-pointer call.
struct TempBuf {
  void* p = nullptr;
  cudaStream_t st = nullptr;
  TempBuf() = default;
  TempBuf(const TempBuf&) = delete;
  ~TempBuf() {
    if (p) cudaFreeAsync(p, st);
  }
  int alloc(size_t bytes, cudaStream_t s) {
    st = s;
    if (cudaMallocAsync(&p, bytes ? bytes : 16, s) != cudaSuccess) return fail(SM_ERR_OOM, "device allocation failed");
    return SM_OK;
  }
};

int upload_weight(sm_ctx* ctx, int scheme, int rows, int cols, int bs, const void* data, size_t nbytes,
                  const float* scales, size_t nscales, int layout, bool from_device, sm_weight** out) {
  if (!ctx || !out) return fail(SM_ERR_INVALID_ARG, "weight_upload: null argument");
  *out = nullptr;
  if (!valid_scheme(scheme)) return fail(SM_ERR_UNSUPPORTED, "weight_upload: unsupported QuantScheme");
  if (rows <= 0 || cols <= 0) return fail(SM_ERR_SHAPE, "weight_upload: rows and cols must be positive");
  if (layout != SM_LAYOUT_INTENDED && layout != SM_LAYOUT_REFERENCE)
    return fail(SM_ERR_INVALID_ARG, "weight_upload: unknown layout");
  const int64_t n = (int64_t)rows * cols;
  if ((scheme == SM_Q4_K || scheme == SM_Q6_K) && cols % 256)
    return fail(SM_ERR_SHAPE, "weight_upload: Columns must be divisible by block size (256)");
  // reference layout: Rows = K is also walked in 256-element blocks (FusedQ4KMatMul.cs:118)
  if ((scheme == SM_Q4_K || scheme == SM_Q6_K) && layout == SM_LAYOUT_REFERENCE && rows % 256)
    return fail(SM_ERR_SHAPE, "weight_upload: reference-layout K-quant needs K (rows) divisible by 256");
  if (nbytes != packed_bytes(scheme, n)) return fail(SM_ERR_SHAPE, "weight_upload: data length does not match shape");
  const bool q41_q50 = scheme == SM_Q4_1 || scheme == SM_Q5_0;
  if (q41_q50) {
    // block size fixed at 32 (Q4_1Tensor.cs:14, Q5_0Tensor.cs:14); Q4_1 scales = block scales then block mins
    const size_t nb = (size_t)((n + 31) / 32);
    if (bs != 32 && bs != 0) return fail(SM_ERR_INVALID_ARG, "weight_upload: Q4_1 / Q5_0 block size is 32");
    if (!scales || nscales != (scheme == SM_Q4_1 ? 2 * nb : nb))
      return fail(SM_ERR_SHAPE, "weight_upload: scales length does not match block count");
  }
  const bool has_scales = scheme == SM_Q8_0 || scheme == SM_Q4_0;
  if (has_scales) {
    if (bs <= 0) return fail(SM_ERR_INVALID_ARG, "weight_upload: block size must be positive");
    if (!scales || nscales != (size_t)((n + bs - 1) / bs))
      return fail(SM_ERR_SHAPE, "weight_upload: scales length does not match block count");
  }
  if (!data) return fail(SM_ERR_INVALID_ARG, "weight_upload: null data");
  DeviceGuard g(ctx->device);
  auto* w = new sm_weight();
  w->ctx = ctx;
  w->device = ctx->device;
  DevWeight& d = w->w;
  d.scheme = scheme;
  d.layout = layout;
  d.rows = rows;
  d.cols = cols;
  d.block_size = has_scales ? bs : (q41_q50 ? 32 : 256);
  d.n = n;
  const cudaMemcpyKind kind = from_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  cudaStream_t st = ctx->stream;
  auto cleanup = [&](int rc) {
    if (d.data) cudaFree(d.data);
    if (d.aux) cudaFree(d.aux);
    delete w;
    return rc;
  };
  if (scheme == SM_Q6_K) {
    const int64_t nb = n / 256;
    d.data_bytes = (size_t)nb * Q6K_BODY_BYTES;
    int64_t aux_elems = nb;
    if (layout == SM_LAYOUT_INTENDED) {  // one 16-byte-padded row of d values per weight row
      d.aux_bpr = cols / 256;
      d.aux_stride = (d.aux_bpr * 2 + 15) / 16 * 8;
      aux_elems = (int64_t)rows * d.aux_stride;
    }
    d.aux_bytes = (size_t)aux_elems * 2;
    if (cudaMalloc(&d.data, d.data_bytes) != cudaSuccess || cudaMalloc(&d.aux, d.aux_bytes) != cudaSuccess)
      return cleanup(fail(SM_ERR_OOM, "weight_upload: out of device memory"));
    cudaMemsetAsync(d.aux, 0, d.aux_bytes, st);
    void* staging = nullptr;
    if (cudaMallocAsync(&staging, nbytes, st) != cudaSuccess)
      return cleanup(fail(SM_ERR_OOM, "weight_upload: out of device memory"));
    cudaMemcpyAsync(staging, data, nbytes, kind, st);
    int rc = launch_q6k_relayout((const uint8_t*)staging, (uint8_t*)d.data, (uint16_t*)d.aux, nb, d.aux_bpr,
                                 d.aux_stride, st);
    cudaFreeAsync(staging, st);
    if (rc) return cleanup(rc);
  } else if (q41_q50) {
    // nibbles in data; the scales and the second per-block array (mins / high bits) in aux
    const int64_t nb = (n + 31) / 32;
    d.data_bytes = (size_t)(n + 1) / 2;
    if (cudaMalloc(&d.data, d.data_bytes) != cudaSuccess)
      return cleanup(fail(SM_ERR_OOM, "weight_upload: out of device memory"));
    cudaMemcpyAsync(d.data, data, d.data_bytes, kind, st);
    const void* second = scheme == SM_Q4_1 ? (const void*)(scales + nb) : (const void*)((const uint8_t*)data + d.data_bytes);
    if (layout == SM_LAYOUT_INTENDED && cols % 32 == 0) {  // [scales | second] rows, padded to 16 bytes
      d.aux_bpr = cols / 32;
      d.aux_stride = (2 * d.aux_bpr * 4 + 15) / 16 * 4;
      d.aux_bytes = (size_t)rows * d.aux_stride * 4;
      if (cudaMalloc(&d.aux, d.aux_bytes) != cudaSuccess)
        return cleanup(fail(SM_ERR_OOM, "weight_upload: out of device memory"));
      cudaMemsetAsync(d.aux, 0, d.aux_bytes, st);
      cudaMemcpy2DAsync(d.aux, (size_t)d.aux_stride * 4, scales, (size_t)d.aux_bpr * 4, (size_t)d.aux_bpr * 4, rows,
                        kind, st);
      cudaMemcpy2DAsync((float*)d.aux + d.aux_bpr, (size_t)d.aux_stride * 4, second, (size_t)d.aux_bpr * 4,
                        (size_t)d.aux_bpr * 4, rows, kind, st);
    } else {
      d.aux_bytes = (size_t)nb * 8;
      if (cudaMalloc(&d.aux, d.aux_bytes) != cudaSuccess)
        return cleanup(fail(SM_ERR_OOM, "weight_upload: out of device memory"));
      cudaMemcpyAsync(d.aux, scales, (size_t)nb * 4, kind, st);
      cudaMemcpyAsync((float*)d.aux + nb, second, (size_t)nb * 4, kind, st);
    }
  } else {
    d.data_bytes = nbytes;
    if (cudaMalloc(&d.data, nbytes) != cudaSuccess) return cleanup(fail(SM_ERR_OOM, "weight_upload: out of device memory"));
    cudaMemcpyAsync(d.data, data, nbytes, kind, st);
    if (has_scales) {
      if (layout == SM_LAYOUT_INTENDED && cols % bs == 0) {  // 16-byte-padded row of scales per weight row
        d.aux_bpr = cols / bs;
        d.aux_stride = (d.aux_bpr * 4 + 15) / 16 * 4;
        d.aux_bytes = (size_t)rows * d.aux_stride * sizeof(float);
        if (cudaMalloc(&d.aux, d.aux_bytes) != cudaSuccess)
          return cleanup(fail(SM_ERR_OOM, "weight_upload: out of device memory"));
        cudaMemsetAsync(d.aux, 0, d.aux_bytes, st);
        cudaMemcpy2DAsync(d.aux, (size_t)d.aux_stride * 4, scales, (size_t)d.aux_bpr * 4, (size_t)d.aux_bpr * 4, rows,
                          kind, st);
      } else {
        d.aux_bytes = nscales * sizeof(float);
        if (cudaMalloc(&d.aux, d.aux_bytes) != cudaSuccess)
          return cleanup(fail(SM_ERR_OOM, "weight_upload: out of device memory"));
        cudaMemcpyAsync(d.aux, scales, d.aux_bytes, kind, st);
      }
    }
  }
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cleanup(fail(SM_ERR_CUDA, std::string("weight_upload: ") + cudaGetErrorString(e)));
  *out = w;
  return SM_OK;
}

}  // namespace

extern "C" {

SM_API int sm_version(void) { return 1; }

SM_API int sm_last_error(char* buf, size_t n) {
  if (!buf || n == 0) return SM_ERR_INVALID_ARG;
  std::snprintf(buf, n, "%s", g_last_error.c_str());
  return SM_OK;
}

SM_API int sm_device_count(int* out) {
  if (!out) return fail(SM_ERR_INVALID_ARG, "null out");
  int c = 0;
  cudaError_t e = cudaGetDeviceCount(&c);
  if (e != cudaSuccess) {
    *out = 0;
    return fail(SM_ERR_CUDA, std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e));
  }
  *out = c;
  return SM_OK;
}

SM_API int sm_ctx_create(int device, sm_ctx** out) {
  if (!out) return fail(SM_ERR_INVALID_ARG, "ctx_create: null out");
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count)
    return fail(SM_ERR_INVALID_ARG, "ctx_create: no such CUDA device");
  SM_CUDA_TRY(cudaSetDevice(device));
  auto* c = new sm_ctx();
  c->device = device;
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete c;
    return fail(SM_ERR_CUDA, "ctx_create: stream creation failed");
  }
  c->own_stream = true;
  if (cudaMalloc(&c->dev_status, sizeof(int)) != cudaSuccess) {
    cudaStreamDestroy(c->stream);
    delete c;
    return fail(SM_ERR_OOM, "ctx_create: allocation failed");
  }
  cudaMemset(c->dev_status, 0, sizeof(int));
  {
    // the library's per-call temporaries come from this process's default stream-ordered
    // pool; keep freed blocks in it (the default threshold of 0 hands them back to the
    // driver at every synchronising call, and the next call maps them again)
    cudaMemPool_t pool = nullptr;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
      uint64_t keep = UINT64_MAX;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    cudaGetLastError();
  }
  *out = c;
  return SM_OK;
}

SM_API int sm_ctx_destroy(sm_ctx* ctx) {
  if (!ctx) return SM_OK;
  DeviceGuard g(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->dev_status) cudaFree(ctx->dev_status);
  if (ctx->tp_comm) tp_comm_destroy(ctx->tp_comm);
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return SM_OK;
}

SM_API int sm_ctx_set_stream(sm_ctx* ctx, void* stream) {
  if (!ctx) return fail(SM_ERR_INVALID_ARG, "null ctx");
  DeviceGuard g(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  if (stream) {
    ctx->stream = (cudaStream_t)stream;
    ctx->own_stream = false;
  } else {
    SM_CUDA_TRY(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking));
    ctx->own_stream = true;
  }
  return SM_OK;
}

SM_API int sm_stream_sync(sm_ctx* ctx) {
  if (!ctx) return fail(SM_ERR_INVALID_ARG, "null ctx");
  DeviceGuard g(ctx->device);
  SM_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return SM_OK;
}

SM_API int sm_ctx_device_status(sm_ctx* ctx) {
  if (!ctx) return fail(SM_ERR_INVALID_ARG, "null ctx");
  DeviceGuard g(ctx->device);
  int s = 0;
  SM_CUDA_TRY(cudaMemcpyAsync(&s, ctx->dev_status, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
  SM_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return s;
}

SM_API int sm_ctx_launch_count(sm_ctx* ctx, int64_t* out) {
  if (!ctx || !out) return fail(SM_ERR_INVALID_ARG, "null argument");
  *out = ctx->launches;
  return SM_OK;
}

SM_API int sm_weight_upload(sm_ctx* ctx, int scheme, int rows, int cols, int bs, const void* data, size_t nbytes,
                            const float* scales, size_t nscales, int layout, sm_weight** out) {
  return upload_weight(ctx, scheme, rows, cols, bs, data, nbytes, scales, nscales, layout, false, out);
}

SM_API int sm_weight_upload_device(sm_ctx* ctx, int scheme, int rows, int cols, int bs, const void* data,
                                   size_t nbytes, const float* scales, size_t nscales, int layout, sm_weight** out) {
  return upload_weight(ctx, scheme, rows, cols, bs, data, nbytes, scales, nscales, layout, true, out);
}

SM_API int sm_weight_destroy(sm_weight* w) {
  if (!w) return SM_OK;
  DeviceGuard g(w->device);
  cudaDeviceSynchronize();
  gemm_tc_release_weight(w->w.data);
  if (w->w.data) cudaFree(w->w.data);
  if (w->w.aux) cudaFree(w->w.aux);
  delete w;
  return SM_OK;
}

SM_API int sm_weight_info(const sm_weight* w, int* scheme, int* rows, int* cols, int* layout) {
  if (!w) return fail(SM_ERR_INVALID_ARG, "null weight");
  if (scheme) *scheme = w->w.scheme;
  if (rows) *rows = w->w.rows;
  if (cols) *cols = w->w.cols;
  if (layout) *layout = w->w.layout;
  return SM_OK;
}

SM_API int sm_weight_nbytes(const sm_weight* w, size_t* out) {
  if (!w || !out) return fail(SM_ERR_INVALID_ARG, "null argument");
  *out = w->w.data_bytes + w->w.aux_bytes;
  return SM_OK;
}

SM_API int sm_matmul(sm_weight* wt, const float* a, float* c, int m, int k, int n, int flags) {
  if (!wt || !a || !c) return fail(SM_ERR_INVALID_ARG, "matmul: null argument");
  const DevWeight& W = wt->w;
  // Q4KWeightTensor.cs:43-48 / NeuralNet.cs:89 shape rules, per orientation.
  if (k != W.K()) return fail(SM_ERR_SHAPE, "matmul: k does not match the weight");
  if (n != W.N()) return fail(SM_ERR_SHAPE, "matmul: n does not match the weight");
  if (m <= 0) return fail(SM_ERR_SHAPE, "matmul: m must be positive");
  sm_ctx* ctx = wt->ctx;
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  int nl = 0;
  if (flags == SM_PTR_DEVICE) {
    int rc = launch_matmul(W, a, c, m, n, 0, st, &nl);
    ctx->launches += nl;
    return rc;
  }
  TempBuf da, dc;
  SM_TRY(da.alloc(sizeof(float) * (size_t)m * k, st));
  SM_TRY(dc.alloc(sizeof(float) * (size_t)m * n, st));
  SM_CUDA_TRY(cudaMemcpyAsync(da.p, a, sizeof(float) * (size_t)m * k, cudaMemcpyHostToDevice, st));
  SM_TRY(launch_matmul(W, (const float*)da.p, (float*)dc.p, m, n, 0, st, &nl));
  ctx->launches += nl;
  SM_CUDA_TRY(cudaMemcpyAsync(c, dc.p, sizeof(float) * (size_t)m * n, cudaMemcpyDeviceToHost, st));
  SM_CUDA_TRY(cudaStreamSynchronize(st));
  return SM_OK;
}

SM_API int sm_dequant(sm_weight* wt, float* out, int flags) {
  if (!wt || !out) return fail(SM_ERR_INVALID_ARG, "dequant: null argument");
  sm_ctx* ctx = wt->ctx;
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  const size_t bytes = sizeof(float) * (size_t)wt->w.n;
  if (flags == SM_PTR_DEVICE) {
    ctx->launches += 1;
    return launch_dequant(wt->w, out, st);
  }
  TempBuf d;
  SM_TRY(d.alloc(bytes, st));
  SM_TRY(launch_dequant(wt->w, (float*)d.p, st));
  ctx->launches += 1;
  SM_CUDA_TRY(cudaMemcpyAsync(out, d.p, bytes, cudaMemcpyDeviceToHost, st));
  SM_CUDA_TRY(cudaStreamSynchronize(st));
  return SM_OK;
}

SM_API int sm_quantize(sm_ctx* ctx, int scheme, const float* src, int64_t n, int bs, void* data, float* scales) {
  if (!ctx || !src || !data) return fail(SM_ERR_INVALID_ARG, "quantize: null argument");
  if ((scheme == SM_Q8_0 || scheme == SM_Q4_0) && !scales) return fail(SM_ERR_INVALID_ARG, "quantize: null scales");
  DeviceGuard g(ctx->device);
  ctx->launches += (scheme == SM_Q8_0 || scheme == SM_Q4_0) ? 2 : 1;
  return launch_quantize(scheme, src, n, bs, data, scales, ctx->stream);
}

// ---------------------------------------------------------------- ops
SM_API int sm_op_rmsnorm(sm_ctx* ctx, const float* x, const float* gamma, float* y, int rows, int F, float eps,
                         int flags) {
  if (!ctx || !x || !gamma || !y) return fail(SM_ERR_INVALID_ARG, "rmsnorm: null argument");
  if (rows <= 0 || F <= 0) return fail(SM_ERR_SHAPE, "rmsnorm: rows and features must be positive");
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  ctx->launches += 1;
  if (flags == SM_PTR_DEVICE) return launch_rmsnorm(x, gamma, y, rows, F, eps, st);
  const size_t nb = sizeof(float) * (size_t)rows * F;
  TempBuf dx, dg, dy;
  SM_TRY(dx.alloc(nb, st));
  SM_TRY(dg.alloc(sizeof(float) * F, st));
  SM_TRY(dy.alloc(nb, st));
  SM_CUDA_TRY(cudaMemcpyAsync(dx.p, x, nb, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(dg.p, gamma, sizeof(float) * F, cudaMemcpyHostToDevice, st));
  SM_TRY(launch_rmsnorm((const float*)dx.p, (const float*)dg.p, (float*)dy.p, rows, F, eps, st));
  SM_CUDA_TRY(cudaMemcpyAsync(y, dy.p, nb, cudaMemcpyDeviceToHost, st));
  SM_CUDA_TRY(cudaStreamSynchronize(st));
  return SM_OK;
}

}  // extern "C"

namespace {
// RotaryEmbedding.cs:45-60, computed on the host with the C runtime's powf /
// sinf / cosf (what MathF.Pow/Sin/Cos call on Linux), then uploaded.
void host_rope_tables(int max_seq, int hd, float theta, std::vector<float>& s, std::vector<float>& c) {
  const int half = hd / 2;
  s.resize((size_t)max_seq * half);
  c.resize((size_t)max_seq * half);
  for (int pos = 0; pos < max_seq; ++pos)
    for (int i = 0; i < half; ++i) {
      volatile float e = (2.0f * (float)i) / (float)hd;
      float freq = 1.0f / powf(theta, e);
      float angle = (float)pos * freq;
      s[(size_t)pos * half + i] = sinf(angle);
      c[(size_t)pos * half + i] = cosf(angle);
    }
}
}  // namespace

extern "C" {

SM_API int sm_op_rope(sm_ctx* ctx, float* x, int rows, int n_heads, int hd, const int* positions, float theta,
                      int max_seq, int flags) {
  if (!ctx || !x || !positions) return fail(SM_ERR_INVALID_ARG, "rope: null argument");
  if (hd % 2) return fail(SM_ERR_INVALID_ARG, "rope: Head dimension must be even for RoPE");
  if (rows <= 0 || n_heads <= 0 || max_seq <= 0) return fail(SM_ERR_SHAPE, "rope: bad shape");
  if (flags != SM_PTR_HOST) return fail(SM_ERR_UNSUPPORTED, "rope: host pointers only");
  for (int r = 0; r < rows; ++r)
    if (positions[r] < 0 || positions[r] >= max_seq)
      return fail(SM_ERR_INVALID_ARG, "rope: Position exceeds max sequence length");
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  std::vector<float> hs, hc;
  host_rope_tables(max_seq, hd, theta, hs, hc);
  const size_t nb = sizeof(float) * (size_t)rows * n_heads * hd;
  TempBuf dx, ds, dc, dp;
  SM_TRY(dx.alloc(nb, st));
  SM_TRY(ds.alloc(hs.size() * 4, st));
  SM_TRY(dc.alloc(hc.size() * 4, st));
  SM_TRY(dp.alloc(sizeof(int) * rows, st));
  SM_CUDA_TRY(cudaMemcpyAsync(dx.p, x, nb, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(ds.p, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(dc.p, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(dp.p, positions, sizeof(int) * rows, cudaMemcpyHostToDevice, st));
  SM_TRY(launch_rope_rows((float*)dx.p, rows, n_heads * hd, n_heads, hd, (const int*)dp.p, (const float*)ds.p,
                          (const float*)dc.p, st));
  ctx->launches += 1;
  SM_CUDA_TRY(cudaMemcpyAsync(x, dx.p, nb, cudaMemcpyDeviceToHost, st));
  SM_CUDA_TRY(cudaStreamSynchronize(st));
  return SM_OK;
}

SM_API int sm_op_silu_mul(sm_ctx* ctx, const float* gate, const float* up, float* out, int n, int flags) {
  if (!ctx || !gate || !up || !out) return fail(SM_ERR_INVALID_ARG, "silu_mul: null argument");
  if (n <= 0) return fail(SM_ERR_SHAPE, "silu_mul: n must be positive");
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  ctx->launches += 1;
  if (flags == SM_PTR_DEVICE) return launch_silu_mul(gate, up, out, n, st);
  const size_t nb = sizeof(float) * (size_t)n;
  TempBuf a, b, c;
  SM_TRY(a.alloc(nb, st));
  SM_TRY(b.alloc(nb, st));
  SM_TRY(c.alloc(nb, st));
  SM_CUDA_TRY(cudaMemcpyAsync(a.p, gate, nb, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(b.p, up, nb, cudaMemcpyHostToDevice, st));
  SM_TRY(launch_silu_mul((const float*)a.p, (const float*)b.p, (float*)c.p, n, st));
  SM_CUDA_TRY(cudaMemcpyAsync(out, c.p, nb, cudaMemcpyDeviceToHost, st));
  SM_CUDA_TRY(cudaStreamSynchronize(st));
  return SM_OK;
}

SM_API int sm_attention(sm_ctx* ctx, const float* q, const float* k, const float* v, float* out, int T, int S,
                        int nH, int nKv, int hd, int flags) {
  if (!ctx || !q || !k || !v || !out) return fail(SM_ERR_INVALID_ARG, "attention: null argument");
  if (T <= 0 || S < T || nH <= 0 || nKv <= 0 || nH % nKv) return fail(SM_ERR_SHAPE, "attention: bad shape");
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  int nl = 0;
  const int64_t rs = (int64_t)nKv * hd;
  if (flags == SM_PTR_DEVICE) {
    int rc = launch_attention_prefill(q, nH * hd, k, v, rs, hd, out, nH * hd, T, S, nH, nKv, hd, st, &nl);
    ctx->launches += nl;
    return rc;
  }
  const size_t qb = sizeof(float) * (size_t)T * nH * hd, kb = sizeof(float) * (size_t)S * nKv * hd;
  TempBuf dq, dk, dv, dout;
  SM_TRY(dq.alloc(qb, st));
  SM_TRY(dk.alloc(kb, st));
  SM_TRY(dv.alloc(kb, st));
  SM_TRY(dout.alloc(qb, st));
  SM_CUDA_TRY(cudaMemcpyAsync(dq.p, q, qb, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(dk.p, k, kb, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(dv.p, v, kb, cudaMemcpyHostToDevice, st));
  SM_TRY(launch_attention_prefill((const float*)dq.p, nH * hd, (const float*)dk.p, (const float*)dv.p, rs, hd,
                                  (float*)dout.p, nH * hd, T, S, nH, nKv, hd, st, &nl));
  ctx->launches += nl;
  SM_CUDA_TRY(cudaMemcpyAsync(out, dout.p, qb, cudaMemcpyDeviceToHost, st));
  SM_CUDA_TRY(cudaStreamSynchronize(st));
  return SM_OK;
}

SM_API int sm_attention_decode(sm_ctx* ctx, const float* q, const float* kc, const float* vc, float* out,
                               const int* lens_dev, int B, int max_ctx, int nH, int nKv, int hd) {
  // shape first: a zero head count must come back as an error, never reach the modulo
  if (B <= 0 || max_ctx <= 0 || nH <= 0 || nKv <= 0 || hd <= 0 || nH % nKv)
    return fail(SM_ERR_SHAPE, "attention_decode: bad shape");
  if (!ctx || !q || !kc || !vc || !out || !lens_dev) return fail(SM_ERR_INVALID_ARG, "attention_decode: null argument");
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  int nl = 0;
  const int64_t hstride = (int64_t)max_ctx * hd;
  int crc = launch_attention_decode_cluster(q, nH * hd, kc, vc, hstride * nKv, hd, hstride, max_ctx, out, nH * hd,
                                            lens_dev, nullptr, B, nH, nKv, hd, st, &nl);
  if (crc != SM_ERR_UNSUPPORTED) {
    ctx->launches += nl;
    return crc;
  }
  const size_t sf = attention_decode_scratch_floats(B, nH, max_ctx);
  TempBuf scratch;
  SM_TRY(scratch.alloc(sf * sizeof(float), st));
  const int64_t head_stride = (int64_t)max_ctx * hd;
  int rc = launch_attention_decode(q, nH * hd, kc, vc, head_stride * nKv, hd, head_stride, max_ctx, out, nH * hd,
                                   lens_dev, nullptr, B, nH, nKv, hd, (float*)scratch.p, sf, st, &nl);
  ctx->launches += nl;
  return rc;
}

}  // extern "C"

// ================================================================ model
namespace {

constexpr int N_LAYER_ROLES = 9;

struct Work {
  int cap_rows = 0;
  float *x = nullptr, *h = nullptr, *qkv = nullptr, *att = nullptr, *g = nullptr, *u = nullptr;
  float* logits = nullptr;
  int cap_logit_rows = 0;
  int* ints = nullptr;  // tok | seq | pos | lens | argmax, each cap_rows
  float* attn_scratch = nullptr;
  size_t attn_scratch_floats = 0;
  int generation = 0;
  int* tok() const { return ints; }
  int* seq() const { return ints + cap_rows; }
  int* pos() const { return ints + 2 * cap_rows; }
  int* lens() const { return ints + 3 * cap_rows; }
  int* amax() const { return ints + 4 * cap_rows; }
};

}  // namespace

struct sm_model {
  sm_ctx* ctx = nullptr;
  int device = 0;  // destroy needs only this
  sm_model_config cfg{};
  struct Layer {
    const DevWeight* w[N_LAYER_ROLES] = {};
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
  };
  std::vector<Layer> layers;
  float* embd = nullptr;
  float* out_norm = nullptr;
  const DevWeight* output = nullptr;
  float* sin_t = nullptr;
  float* cos_t = nullptr;
  bool finalized = false;
  bool tp = false;  // a tensor-parallel shard: O / down outputs are all-reduced over ctx->tp_comm
  Work work;
  size_t own_bytes = 0;
  int qd() const { return cfg.n_heads * cfg.head_dim; }
  int kd() const { return cfg.n_kv_heads * cfg.head_dim; }
  int qkv_stride() const { return qd() + 2 * kd(); }
};

struct sm_kv {
  sm_model* m = nullptr;
  int device = 0;  // destroy needs only this
  int max_seqs = 0, max_tokens = 0;
  float* k = nullptr;
  float* v = nullptr;
  int* len_dev = nullptr;
  std::vector<int> len_host;
  bool host_stale = false;
  struct Graph {
    cudaGraphExec_t exec = nullptr;
    int generation = -1;
    int launches = 0;
    int eager_runs = 0;
  };
  std::map<int, Graph> graphs;  // decode batch size -> captured step
  int* pinned = nullptr;        // host staging for per-step inputs
  int pinned_cap = 0;
  // one-launch bs1 decode step (decode_mega.cu)
  MegaLayer* mega_layers = nullptr;  // device table of per-layer segments
  unsigned* mega_sync = nullptr;     // argmax arrival counter
  unsigned long long* mega_ll = nullptr;  // tagged exchange words of the one-launch decode (+ its epoch)
  size_t mega_ll_words = 0;
  unsigned long long* mega_trace = nullptr;  // SMALLMIND_MEGA_TRACE: per-CTA phase timestamps
  int mega_generation = -1;
  bool mega_mma_only = false;  // every segment of the layer table has the tensor-core path
  size_t layer_stride() const { return (size_t)max_seqs * m->cfg.n_kv_heads * max_tokens * m->cfg.head_dim; }
};

namespace {

int work_reserve(sm_model* m, int rows, int logit_rows, int attn_rows, int max_tokens) {
  Work& w = m->work;
  const auto& c = m->cfg;
  const size_t need_scratch =
      std::max(attention_decode_scratch_floats(std::max(1, attn_rows), c.n_heads, max_tokens),
               mega_scratch_floats(c.n_heads, c.n_kv_heads, c.head_dim, max_tokens, mega_grid_size()));
  if (rows <= w.cap_rows && logit_rows <= w.cap_logit_rows && need_scratch <= w.attn_scratch_floats) return SM_OK;
  cudaStreamSynchronize(m->ctx->stream);
  const int R = std::max(rows, w.cap_rows);
  const int LR = std::max(logit_rows, w.cap_logit_rows);
  const size_t S = std::max(need_scratch, w.attn_scratch_floats);
  for (void* p : {(void*)w.x, (void*)w.h, (void*)w.qkv, (void*)w.att, (void*)w.g, (void*)w.u, (void*)w.logits,
                  (void*)w.ints, (void*)w.attn_scratch})
    if (p) cudaFree(p);
  w = Work{};
  auto al = [&](void** p, size_t bytes) { return cudaMalloc(p, bytes) == cudaSuccess; };
  const size_t H = c.hidden, F = c.ffn_hidden;
  bool ok = al((void**)&w.x, 4 * R * H) && al((void**)&w.h, 4 * R * H) &&
            al((void**)&w.qkv, 4 * (size_t)R * m->qkv_stride()) && al((void**)&w.att, 4 * (size_t)R * m->qd()) &&
            al((void**)&w.g, 4 * R * F) && al((void**)&w.u, 4 * R * F) &&
            al((void**)&w.logits, 4 * (size_t)LR * c.vocab_size) && al((void**)&w.ints, 4 * 5 * (size_t)R) &&
            al((void**)&w.attn_scratch, 4 * S);
  if (!ok) return fail(SM_ERR_OOM, "model: workspace allocation failed");
  w.cap_rows = R;
  w.cap_logit_rows = LR;
  w.attn_scratch_floats = S;
  static int gen = 0;
  w.generation = ++gen;
  return SM_OK;
}

// ---- small device helpers for the decode step
__global__ void decode_prep_kernel(const int* __restrict__ seq, int* __restrict__ pos, int* __restrict__ lens,
                                   const int* __restrict__ kv_len, int n, int max_tokens, int* status) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n) return;
  int p = kv_len[seq[b]];
  if (p >= max_tokens) {  // context full: report, clamp so nothing is written out of range
    atomicExch(status, SM_ERR_SHAPE);
    p = max_tokens - 1;
  }
  pos[b] = p;
  lens[b] = p + 1;
}
__global__ void decode_commit_kernel(const int* __restrict__ seq, int* __restrict__ kv_len, int n, int max_tokens) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n) return;
  const int s = seq[b];
  if (kv_len[s] < max_tokens) kv_len[s] += 1;
}

// One-row step (bs1 decode): fused launches built on the M = 1 GEMV.  Per layer:
// [RMSNorm + Q|K|V] -> RoPE + KV append -> attention -> [O-proj + residual]
// -> [RMSNorm + gate/up + SiLU-gate] -> [down-proj + residual].
// warp-per-row-group GEMV
int launch_m1(const GemvArgs& a, sm_model* m, cudaStream_t st, int& nl) {
  (void)m;
  return launch_gemv1(a, st, &nl);
}

bool m1_supported(const sm_model* m) {
  const auto& c = m->cfg;
  for (const auto& L : m->layers) {
    for (int r : {SM_ROLE_WQ, SM_ROLE_WK, SM_ROLE_WV, SM_ROLE_W_GATE, SM_ROLE_W_UP})
      if (!gemv1_supports(*L.w[r], c.hidden)) return false;
    if (!gemv1_supports(*L.w[SM_ROLE_WO], m->qd()) || !gemv1_supports(*L.w[SM_ROLE_W_DOWN], c.ffn_hidden))
      return false;
    // one launch per Q|K|V and per gate|up: their formats must share a kernel
    const int fq = L.w[SM_ROLE_WQ]->scheme, fk = L.w[SM_ROLE_WK]->scheme, fv = L.w[SM_ROLE_WV]->scheme;
    int fa = fq, fb = fq;
    for (int f : {fk, fv}) {
      if (f == fa || f == fb) continue;
      if (fb != fa) return false;
      fb = f;
    }
    if (!gemv1_mix_ok(fa, fb) || L.w[SM_ROLE_W_GATE]->scheme != L.w[SM_ROLE_W_UP]->scheme) return false;
  }
  return gemv1_supports(*m->output, c.hidden);
}

// Tensor-parallel shard: the partial output of a row-split projection (rows x H in
// `partial`) is summed over the group in place, then added to the residual stream.
int tp_reduce_residual(sm_model* m, float* partial, int rows, int& nl) {
  const size_t n = (size_t)rows * m->cfg.hidden;
  SM_TRY(tp_allreduce_sum(m->ctx->tp_comm, partial, n, m->ctx->stream));
  SM_TRY(launch_add(m->work.x, partial, (int64_t)n, m->ctx->stream));
  nl += 2;
  return SM_OK;
}

int forward_m1(sm_model* m, sm_kv* kv, bool prefill_head_only, int& nl) {
  const auto& c = m->cfg;
  Work& w = m->work;
  cudaStream_t st = m->ctx->stream;
  const int H = c.hidden, qd = m->qd(), kd = m->kd(), QS = m->qkv_stride();
  const int hd = c.head_dim, mt = kv->max_tokens;
  const int64_t head_stride = (int64_t)mt * hd;
  const int64_t seq_stride = head_stride * c.n_kv_heads;
  if (!prefill_head_only) {
    SM_TRY(launch_embed(m->embd, w.tok(), w.x, 1, H, st));
    ++nl;
    for (int l = 0; l < c.n_layers; ++l) {
      const sm_model::Layer& L = m->layers[l];
      float* kc = kv->k + kv->layer_stride() * l;
      float* vc = kv->v + kv->layer_stride() * l;
      GemvArgs qkv;
      qkv.K = H;
      qkv.x = w.x;
      qkv.gamma = L.attn_norm;
      qkv.eps = c.norm_eps;
      // RoPE and the KV-cache append are fused into the Q|K|V epilogue
      qkv.pos = w.pos();
      qkv.seq = w.seq();
      qkv.sin_t = m->sin_t;
      qkv.cos_t = m->cos_t;
      qkv.head_dim = hd;
      qkv.n_kv = c.n_kv_heads;
      qkv.max_ctx = mt;
      SM_TRY(gemv1_segment(qkv, *L.w[SM_ROLE_WQ], nullptr, w.qkv, GEMV_ROPE_Q));
      SM_TRY(gemv1_segment(qkv, *L.w[SM_ROLE_WK], nullptr, kc, GEMV_ROPE_K_CACHE));
      SM_TRY(gemv1_segment(qkv, *L.w[SM_ROLE_WV], nullptr, vc, GEMV_V_CACHE));
      SM_TRY(launch_m1(qkv, m, st, nl));
      int arc = launch_attention_decode_cluster(w.qkv, QS, kc, vc, seq_stride, hd, head_stride, mt, w.att, qd,
                                                w.lens(), w.seq(), 1, c.n_heads, c.n_kv_heads, hd, st, &nl);
      if (arc == SM_ERR_UNSUPPORTED)
        arc = launch_attention_decode(w.qkv, QS, kc, vc, seq_stride, hd, head_stride, mt, w.att, qd, w.lens(),
                                      w.seq(), 1, c.n_heads, c.n_kv_heads, hd, w.attn_scratch, w.attn_scratch_floats,
                                      st, &nl);
      SM_TRY(arc);
      GemvArgs o;
      o.K = qd;
      o.x = w.att;
      SM_TRY(gemv1_segment(o, *L.w[SM_ROLE_WO], nullptr, m->tp ? w.h : w.x, m->tp ? GEMV_STORE : GEMV_ADD));
      SM_TRY(launch_m1(o, m, st, nl));
      if (m->tp) SM_TRY(tp_reduce_residual(m, w.h, 1, nl));
      GemvArgs gu;
      gu.K = H;
      gu.x = w.x;
      gu.gamma = L.ffn_norm;
      gu.eps = c.norm_eps;
      if (L.w[SM_ROLE_W_GATE]->scheme == L.w[SM_ROLE_W_UP]->scheme) {
        SM_TRY(gemv1_segment(gu, *L.w[SM_ROLE_W_GATE], L.w[SM_ROLE_W_UP], w.g, GEMV_GLU));
        SM_TRY(launch_m1(gu, m, st, nl));
      } else {
        SM_TRY(gemv1_segment(gu, *L.w[SM_ROLE_W_GATE], nullptr, w.g, GEMV_STORE));
        SM_TRY(gemv1_segment(gu, *L.w[SM_ROLE_W_UP], nullptr, w.u, GEMV_STORE));
        SM_TRY(launch_m1(gu, m, st, nl));
        SM_TRY(launch_silu_mul(w.g, w.u, w.g, c.ffn_hidden, st));
        ++nl;
      }
      GemvArgs dn;
      dn.K = c.ffn_hidden;
      dn.x = w.g;
      SM_TRY(gemv1_segment(dn, *L.w[SM_ROLE_W_DOWN], nullptr, m->tp ? w.h : w.x, m->tp ? GEMV_STORE : GEMV_ADD));
      SM_TRY(launch_m1(dn, m, st, nl));
      if (m->tp) SM_TRY(tp_reduce_residual(m, w.h, 1, nl));
    }
  }
  return SM_OK;
}

// LM head of one row x_row: RMSNorm fused into the GEMV, then argmax.
int head_m1(sm_model* m, const float* x_row, int& nl) {
  const auto& c = m->cfg;
  Work& w = m->work;
  cudaStream_t st = m->ctx->stream;
  GemvArgs hd;
  hd.K = c.hidden;
  hd.x = x_row;
  hd.gamma = m->out_norm;
  hd.eps = c.norm_eps;
  SM_TRY(gemv1_segment(hd, *m->output, nullptr, w.logits, GEMV_STORE));
  SM_TRY(launch_m1(hd, m, st, nl));
  SM_TRY(launch_argmax(w.logits, 1, c.vocab_size, w.amax(), st));
  ++nl;
  return SM_OK;
}

// Projections that share their input (Q|K|V, gate|up) run as one tensor-core GEMM
// over the stacked weights when it applies, else one launch per weight.  x first
// passes through a prologue (RMSNorm or the SiLU gate, XPro): on the tensor-core
// GEMM inside its x-split pass; other paths apply it into `tmp` (rows x K) and read that.
int matmul_multi_pro(const DevWeight* const* ws, float* const* ys, const int* ld, int nw, const float* x, int rows,
                     const XPro& pro, float* tmp, int accumulate, cudaStream_t st, int& nl) {
  const char* et = std::getenv("SMALLMIND_GEMM_TC");
  if (!(et && et[0] == '0') && gemm_tc_supports_multi(ws, nw, rows))
    return launch_gemm_tc_multi(ws, ys, ld, nw, x, rows, accumulate, nullptr, st, &nl, &pro);
  const int K = ws[0]->K();
  if (pro.kind == XPRO_RMSNORM) {
    SM_TRY(launch_rmsnorm(x, pro.gamma, tmp, rows, K, pro.eps, st));
  } else {
    SM_TRY(launch_silu_mul(x, pro.u, tmp, (int64_t)rows * K, st));
  }
  ++nl;
  for (int i = 0; i < nw; ++i) SM_TRY(launch_matmul(*ws[i], tmp, ys[i], rows, ld[i], accumulate, st, &nl));
  return SM_OK;
}

// One prompt of a prefill: its rows [r0, r0 + T) of the step, its slot and its first position.
struct PrefillSeg {
  int seq, pos0, r0, T;
};

// rows: the step's token rows.  Prefill: segs[0..nsegs) cover the rows (one or more prompts,
// each attending causally to its own slot); decode: segs is null (one row per sequence).
int forward(sm_model* m, sm_kv* kv, int rows, const PrefillSeg* segs, int nsegs, int& nl) {
  const bool prefill = segs != nullptr;
  const auto& c = m->cfg;
  Work& w = m->work;
  cudaStream_t st = m->ctx->stream;
  const bool m1 = m1_supported(m);
  if (m1 && rows == 1 && !prefill) {
    SM_TRY(forward_m1(m, kv, false, nl));
    return head_m1(m, w.x, nl);
  }
  const int H = c.hidden, F = c.ffn_hidden, qd = m->qd(), kd = m->kd(), QS = m->qkv_stride();
  const int hd = c.head_dim, mt = kv->max_tokens;
  SM_TRY(launch_embed(m->embd, w.tok(), w.x, rows, H, st));
  ++nl;
  const int64_t head_stride = (int64_t)mt * hd;
  const int64_t seq_stride = head_stride * c.n_kv_heads;
  for (int l = 0; l < c.n_layers; ++l) {
    const sm_model::Layer& L = m->layers[l];
    float* kc = kv->k + kv->layer_stride() * l;
    float* vc = kv->v + kv->layer_stride() * l;
    // RMSNorm, then the merged [Q | K | V] rows (MultiHeadAttention.cs:213, layout :395-462)
    {
      const DevWeight* ws[3] = {L.w[SM_ROLE_WQ], L.w[SM_ROLE_WK], L.w[SM_ROLE_WV]};
      float* ys[3] = {w.qkv, w.qkv + qd, w.qkv + qd + kd};
      const int ld[3] = {QS, QS, QS};
      XPro pro;
      pro.kind = XPRO_RMSNORM;
      pro.gamma = L.attn_norm;
      pro.eps = c.norm_eps;
      SM_TRY(matmul_multi_pro(ws, ys, ld, 3, w.x, rows, pro, w.h, 0, st, nl));
    }
    SM_TRY(launch_rope_qk_append(w.qkv, rows, QS, c.n_heads, c.n_kv_heads, hd, w.pos(), w.seq(), m->sin_t, m->cos_t,
                                 kc, vc, mt, st));
    ++nl;
    if (prefill) {
      for (int i = 0; i < nsegs; ++i) {
        const PrefillSeg& sg = segs[i];
        SM_TRY(launch_attention_prefill(w.qkv + (size_t)sg.r0 * QS, QS, kc + seq_stride * sg.seq,
                                        vc + seq_stride * sg.seq, hd, head_stride, w.att + (size_t)sg.r0 * qd, qd,
                                        sg.T, sg.pos0 + sg.T, c.n_heads, c.n_kv_heads, hd, st, &nl));
      }
    } else {
      int arc = launch_attention_decode_cluster(w.qkv, QS, kc, vc, seq_stride, hd, head_stride, mt, w.att, qd,
                                                w.lens(), w.seq(), rows, c.n_heads, c.n_kv_heads, hd, st, &nl);
      if (arc == SM_ERR_UNSUPPORTED)
        arc = launch_attention_decode(w.qkv, QS, kc, vc, seq_stride, hd, head_stride, mt, w.att, qd, w.lens(),
                                      w.seq(), rows, c.n_heads, c.n_kv_heads, hd, w.attn_scratch,
                                      w.attn_scratch_floats, st, &nl);
      SM_TRY(arc);
    }
    // o-proj with the residual add fused in its epilogue (TransformerBlock.cs:170); a
    // tensor-parallel shard all-reduces its partial output first
    if (m->tp) {
      SM_TRY(launch_matmul(*L.w[SM_ROLE_WO], w.att, w.h, rows, H, 0, st, &nl));
      SM_TRY(tp_reduce_residual(m, w.h, rows, nl));
    } else {
      SM_TRY(launch_matmul(*L.w[SM_ROLE_WO], w.att, w.x, rows, H, 1, st, &nl));
    }
    {
      const DevWeight* ws[2] = {L.w[SM_ROLE_W_GATE], L.w[SM_ROLE_W_UP]};
      float* ys[2] = {w.g, w.u};
      const int ld[2] = {F, F};
      XPro pro;
      pro.kind = XPRO_RMSNORM;
      pro.gamma = L.ffn_norm;
      pro.eps = c.norm_eps;
      SM_TRY(matmul_multi_pro(ws, ys, ld, 2, w.x, rows, pro, w.h, 0, st, nl));
    }
    {
      // down(silu(gate) * up) (GatedMLP.cs:51-93), + residual (TransformerBlock.cs:184); a
      // tensor-parallel shard all-reduces its partial output first
      const DevWeight* ws[1] = {L.w[SM_ROLE_W_DOWN]};
      float* ys[1] = {m->tp ? w.h : w.x};
      const int ld[1] = {H};
      XPro pro;
      pro.kind = XPRO_SILU;
      pro.u = w.u;
      SM_TRY(matmul_multi_pro(ws, ys, ld, 1, w.g, rows, pro, w.g, m->tp ? 0 : 1, st, nl));
      if (m->tp) SM_TRY(tp_reduce_residual(m, w.h, rows, nl));
    }
  }
  // final norm + LM head: each prompt's last row only for prefill (what the loop reads), every
  // row for decode
  const int nrows = prefill ? nsegs : rows;
  if (prefill && nsegs == 1 && m1) return head_m1(m, w.x + (size_t)(segs[0].r0 + segs[0].T - 1) * H, nl);
  if (!prefill && m1 && rows == 1) return head_m1(m, w.x, nl);
  if (prefill) {
    for (int i = 0; i < nsegs; ++i) {
      SM_TRY(launch_rmsnorm(w.x + (size_t)(segs[i].r0 + segs[i].T - 1) * H, m->out_norm, w.h + (size_t)i * H, 1, H,
                            c.norm_eps, st));
      ++nl;
    }
  } else {
    // decode rows: the final RMSNorm runs in the head GEMM's x-split pass when it takes the rows
    const DevWeight* ws[1] = {m->output};
    float* ys[1] = {w.logits};
    const int ld[1] = {c.vocab_size};
    XPro pro;
    pro.kind = XPRO_RMSNORM;
    pro.gamma = m->out_norm;
    pro.eps = c.norm_eps;
    SM_TRY(matmul_multi_pro(ws, ys, ld, 1, w.x, nrows, pro, w.h, 0, st, nl));
    SM_TRY(launch_argmax(w.logits, nrows, c.vocab_size, w.amax(), st));
    ++nl;
    return SM_OK;
  }
  SM_TRY(launch_matmul(*m->output, w.h, w.logits, nrows, c.vocab_size, 0, st, &nl));
  SM_TRY(launch_argmax(w.logits, nrows, c.vocab_size, w.amax(), st));
  ++nl;
  return SM_OK;
}

MegaSeg mega_seg(const DevWeight& w, const DevWeight* w2, int mode, float* y) {
  MegaSeg s;
  s.fmt = w.scheme;
  s.rows = w.rows;
  s.bs = w.block_size;
  s.aux_bpr = w.aux_bpr;
  s.aux_stride = w.aux_stride;
  s.mode = mode;
  s.data = (const uint8_t*)w.data;
  s.aux = w.aux;
  s.data2 = w2 ? (const uint8_t*)w2->data : nullptr;
  s.aux2 = w2 ? w2->aux : nullptr;
  s.y = y;
  return s;
}

bool mega_enabled(sm_model* m) {
  const char* e = std::getenv("SMALLMIND_MEGA");
  if (e && e[0] == '0') return false;
  if (m->tp) return false;  // the all-reduce between layers runs as NCCL calls
  if (!m1_supported(m)) return false;
  for (const auto& L : m->layers)
    if (L.w[SM_ROLE_W_GATE]->scheme != L.w[SM_ROLE_W_UP]->scheme) return false;
  return true;
}

// Fills the one-launch decode arguments for the current workspace and cache;
// returns SM_ERR_UNSUPPORTED if the shape does not fit the kernel.
int mega_args(sm_model* m, sm_kv* kv, MegaArgs& a) {
  const auto& c = m->cfg;
  Work& w = m->work;
  a.n_layers = c.n_layers;
  a.H = c.hidden;
  a.qd = m->qd();
  a.kd = m->kd();
  a.F = c.ffn_hidden;
  a.V = c.vocab_size;
  a.nH = c.n_heads;
  a.nKv = c.n_kv_heads;
  a.hd = c.head_dim;
  a.max_ctx = kv->max_tokens;
  a.eps = c.norm_eps;
  if (!mega_supported(a)) return SM_ERR_UNSUPPORTED;
  const int grid = mega_grid_size();
  if (mega_scratch_floats(a.nH, a.nKv, a.hd, a.max_ctx, grid) > w.attn_scratch_floats) return SM_ERR_UNSUPPORTED;
  if (!kv->mega_layers || kv->mega_generation != w.generation) {
    std::vector<MegaLayer> hl(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
      const auto& L = m->layers[l];
      float* kc = kv->k + kv->layer_stride() * l;
      float* vc = kv->v + kv->layer_stride() * l;
      MegaLayer& t = hl[l];
      t.qkv[0] = mega_seg(*L.w[SM_ROLE_WQ], nullptr, GEMV_ROPE_Q, w.qkv);
      t.qkv[1] = mega_seg(*L.w[SM_ROLE_WK], nullptr, GEMV_ROPE_K_CACHE, kc);
      t.qkv[2] = mega_seg(*L.w[SM_ROLE_WV], nullptr, GEMV_V_CACHE, vc);
      t.o = mega_seg(*L.w[SM_ROLE_WO], nullptr, GEMV_ADD, w.x);
      t.gu = mega_seg(*L.w[SM_ROLE_W_GATE], L.w[SM_ROLE_W_UP], GEMV_GLU, w.g);
      t.down = mega_seg(*L.w[SM_ROLE_W_DOWN], nullptr, GEMV_ADD, w.x);
      t.attn_norm = L.attn_norm;
      t.ffn_norm = L.ffn_norm;
      t.kc = kc;
      t.vc = vc;
      mega_layer_split(t, c.hidden, grid);
    }
    kv->mega_mma_only = mega_seg_mma_ok(mega_seg(*m->output, nullptr, GEMV_STORE, w.logits));
    for (const MegaLayer& t : hl)
      for (const MegaSeg* sg : {&t.qkv[0], &t.qkv[1], &t.qkv[2], &t.o, &t.gu, &t.down})
        kv->mega_mma_only = kv->mega_mma_only && mega_seg_mma_ok(*sg);
    if (!kv->mega_layers) SM_CUDA_TRY(cudaMalloc(&kv->mega_layers, sizeof(MegaLayer) * c.n_layers));
    if (!kv->mega_sync) SM_CUDA_TRY(cudaMalloc(&kv->mega_sync, 64 * sizeof(unsigned)));
    SM_CUDA_TRY(cudaMemcpy(kv->mega_layers, hl.data(), sizeof(MegaLayer) * c.n_layers, cudaMemcpyHostToDevice));
    kv->mega_generation = w.generation;
  }
  a.layers = kv->mega_layers;
  a.mma_only = kv->mega_mma_only ? 1 : 0;
  a.head = mega_seg(*m->output, nullptr, GEMV_STORE, w.logits);
  if (!mega_seg_supported(a.head)) return SM_ERR_UNSUPPORTED;
  for (const auto& L : m->layers)
    for (int r : {SM_ROLE_WQ, SM_ROLE_WK, SM_ROLE_WV, SM_ROLE_WO, SM_ROLE_W_GATE, SM_ROLE_W_UP, SM_ROLE_W_DOWN})
      if (!mega_seg_supported(mega_seg(*L.w[r], nullptr, GEMV_STORE, nullptr))) return SM_ERR_UNSUPPORTED;
  a.out_norm = m->out_norm;
  a.embd = m->embd;
  a.sin_t = m->sin_t;
  a.cos_t = m->cos_t;
  a.x = w.x;
  a.q = w.qkv;
  a.att = w.att;
  a.act = w.g;
  a.logits = w.logits;
  a.next_token = w.amax();
  a.token = w.tok();
  a.seq = w.seq();
  a.kv_len = kv->len_dev;
  const int chunks = std::max(1, grid / a.nKv);
  const int G = a.nH / a.nKv;
  float* sc = w.attn_scratch;
  a.scores = sc;
  sc += (size_t)a.nH * a.max_ctx;
  a.cmax = sc;
  sc += (size_t)a.nKv * chunks * G;
  a.psum = sc;
  sc += (size_t)a.nKv * chunks * G;
  a.pacc = sc;
  sc += (size_t)a.nKv * chunks * G * a.hd;
  a.amax_val = sc;
  sc += grid;
  a.amax_idx = (int*)sc;
  a.sync = kv->mega_sync;
  {
    const size_t words = mega_ll_words(a.H, a.qd, a.kd, a.F, a.nH, a.nKv, a.hd, grid);
    if (kv->mega_ll_words < words) {
      if (kv->mega_ll) cudaFree(kv->mega_ll);
      kv->mega_ll = nullptr;
      kv->mega_ll_words = 0;
      SM_CUDA_TRY(cudaMalloc(&kv->mega_ll, words * sizeof(unsigned long long)));
      // all-ones: no word carries a tag a launch waits for until it is written
      SM_CUDA_TRY(cudaMemset(kv->mega_ll, 0xff, words * sizeof(unsigned long long)));
      SM_CUDA_TRY(cudaMemset(kv->mega_ll, 0, sizeof(unsigned long long)));  // epoch 0
      kv->mega_ll_words = words;
    }
    mega_ll_assign(a, kv->mega_ll, grid);
  }
  a.status = m->ctx->dev_status;
  if (std::getenv("SMALLMIND_MEGA_TRACE")) {
    if (!kv->mega_trace)
      SM_CUDA_TRY(cudaMalloc(&kv->mega_trace, sizeof(unsigned long long) * MEGA_TRACE_EVENTS * grid));
    a.trace = kv->mega_trace;
  }
  return SM_OK;
}

bool use_graphs() {
  const char* e = std::getenv("SMALLMIND_CUDA_GRAPHS");
  return !(e && e[0] == '0');
}

}  // namespace

extern "C" {

SM_API int sm_model_create(sm_ctx* ctx, const sm_model_config* cfg, sm_model** out) {
  if (!ctx || !cfg || !out) return fail(SM_ERR_INVALID_ARG, "model_create: null argument");
  *out = nullptr;
  const auto& c = *cfg;
  if (c.vocab_size <= 0 || c.hidden <= 0 || c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 ||
      c.head_dim <= 0 || c.ffn_hidden <= 0 || c.max_context <= 0)
    return fail(SM_ERR_INVALID_ARG, "model_create: config fields must be positive");
  if (c.n_heads % c.n_kv_heads)
    return fail(SM_ERR_INVALID_ARG, "model_create: Number of query heads must be divisible by number of KV heads");
  if (c.head_dim != 64) return fail(SM_ERR_UNSUPPORTED, "model_create: head_dim 64 only");
  if (c.hidden % 4) return fail(SM_ERR_UNSUPPORTED, "model_create: hidden must be a multiple of 4");
  DeviceGuard g(ctx->device);
  auto* m = new sm_model();
  m->ctx = ctx;
  m->device = ctx->device;
  m->cfg = c;
  m->layers.resize(c.n_layers);
  std::vector<float> hs, hc;
  host_rope_tables(c.max_context, c.head_dim, c.rope_theta, hs, hc);
  bool ok = cudaMalloc(&m->sin_t, hs.size() * 4) == cudaSuccess && cudaMalloc(&m->cos_t, hc.size() * 4) == cudaSuccess;
  if (!ok) {
    delete m;
    return fail(SM_ERR_OOM, "model_create: allocation failed");
  }
  cudaMemcpy(m->sin_t, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(m->cos_t, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice);
  m->own_bytes += hs.size() * 8;
  *out = m;
  return SM_OK;
}

SM_API int sm_model_set_weight(sm_model* m, int layer, int role, sm_weight* w) {
  if (!m || !w) return fail(SM_ERR_INVALID_ARG, "model_set_weight: null argument");
  if (w->ctx != m->ctx) return fail(SM_ERR_INVALID_ARG, "model_set_weight: weight belongs to another context");
  if (w->w.layout != SM_LAYOUT_INTENDED)
    return fail(SM_ERR_INVALID_ARG, "model_set_weight: model weights use the intended (out x in) layout");
  const auto& c = m->cfg;
  int er = 0, ec = 0;
  const int qd = m->qd(), kd = m->kd();
  switch (role) {
    case SM_ROLE_WQ: er = qd; ec = c.hidden; break;
    case SM_ROLE_WK: case SM_ROLE_WV: er = kd; ec = c.hidden; break;
    case SM_ROLE_WO: er = c.hidden; ec = qd; break;
    case SM_ROLE_W_GATE: case SM_ROLE_W_UP: er = c.ffn_hidden; ec = c.hidden; break;
    case SM_ROLE_W_DOWN: er = c.hidden; ec = c.ffn_hidden; break;
    case SM_ROLE_OUTPUT: er = c.vocab_size; ec = c.hidden; break;
    default: return fail(SM_ERR_INVALID_ARG, "model_set_weight: role is not a weight");
  }
  // Linear.SetQuantizedWeight dimension rule (NeuralNet.cs:89): Rows == out, Cols == in.
  if (w->w.rows != er || w->w.cols != ec)
    return fail(SM_ERR_SHAPE, "model_set_weight: Quantized weight dimensions don't match layer dimensions");
  if (role == SM_ROLE_OUTPUT) {
    m->output = &w->w;
  } else {
    if (layer < 0 || layer >= c.n_layers) return fail(SM_ERR_INVALID_ARG, "model_set_weight: bad layer");
    m->layers[layer].w[role] = &w->w;
  }
  m->finalized = false;
  return SM_OK;
}

SM_API int sm_model_set_vector(sm_model* m, int layer, int role, const float* data, size_t n) {
  if (!m || !data) return fail(SM_ERR_INVALID_ARG, "model_set_vector: null argument");
  const auto& c = m->cfg;
  DeviceGuard g(m->ctx->device);
  float** dst = nullptr;
  size_t need = 0;
  if (role == SM_ROLE_TOKEN_EMBD) {
    dst = &m->embd;
    need = (size_t)c.vocab_size * c.hidden;
  } else if (role == SM_ROLE_OUT_NORM) {
    dst = &m->out_norm;
    need = c.hidden;
  } else if (role == SM_ROLE_ATTN_NORM || role == SM_ROLE_FFN_NORM) {
    if (layer < 0 || layer >= c.n_layers) return fail(SM_ERR_INVALID_ARG, "model_set_vector: bad layer");
    dst = role == SM_ROLE_ATTN_NORM ? &m->layers[layer].attn_norm : &m->layers[layer].ffn_norm;
    need = c.hidden;
  } else {
    return fail(SM_ERR_INVALID_ARG, "model_set_vector: role is not a vector");
  }
  if (n != need) return fail(SM_ERR_SHAPE, "model_set_vector: length does not match the config");
  if (!*dst) {
    SM_CUDA_TRY(cudaMalloc((void**)dst, need * 4));
    m->own_bytes += need * 4;
  }
  SM_CUDA_TRY(cudaMemcpy(*dst, data, need * 4, cudaMemcpyHostToDevice));
  m->finalized = false;
  return SM_OK;
}

SM_API int sm_tp_unique_id(void* id, size_t n) { return tp_unique_id(id, n); }

SM_API int sm_tp_init(sm_ctx* ctx, int tp_size, int tp_rank, const void* id, size_t n) {
  if (!ctx) return fail(SM_ERR_INVALID_ARG, "tp_init: null ctx");
  if (ctx->tp_comm) return fail(SM_ERR_STATE, "tp_init: the context already belongs to a group");
  if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) return fail(SM_ERR_INVALID_ARG, "tp_init: rank outside [0, size)");
  DeviceGuard g(ctx->device);
  void* comm = nullptr;
  SM_TRY(tp_comm_create(tp_size, tp_rank, id, n, &comm));
  ctx->tp_comm = comm;
  ctx->tp_size = tp_size;
  ctx->tp_rank = tp_rank;
  return SM_OK;
}

SM_API int sm_tp_allreduce(sm_ctx* ctx, float* buf, size_t n) {
  if (!ctx || !buf) return fail(SM_ERR_INVALID_ARG, "tp_allreduce: null argument");
  if (!ctx->tp_comm) return fail(SM_ERR_STATE, "tp_allreduce: the context has no group (sm_tp_init)");
  DeviceGuard g(ctx->device);
  SM_TRY(tp_allreduce_sum(ctx->tp_comm, buf, n, ctx->stream));
  ctx->launches += 1;
  return SM_OK;
}

SM_API int sm_model_set_tp(sm_model* m, int enable) {
  if (!m) return fail(SM_ERR_INVALID_ARG, "model_set_tp: null model");
  if (enable && !m->ctx->tp_comm) return fail(SM_ERR_STATE, "model_set_tp: the context has no group (sm_tp_init)");
  m->tp = enable != 0;
  m->work.generation += 1000000;  // captured steps of the other mode are rebuilt
  return SM_OK;
}

SM_API int sm_model_finalize(sm_model* m) {
  if (!m) return fail(SM_ERR_INVALID_ARG, "null model");
  if (!m->embd || !m->out_norm || !m->output) return fail(SM_ERR_STATE, "model_finalize: missing global tensor");
  for (int l = 0; l < m->cfg.n_layers; ++l) {
    const auto& L = m->layers[l];
    if (!L.attn_norm || !L.ffn_norm) return fail(SM_ERR_STATE, "model_finalize: missing norm");
    for (int r : {SM_ROLE_WQ, SM_ROLE_WK, SM_ROLE_WV, SM_ROLE_WO, SM_ROLE_W_GATE, SM_ROLE_W_UP, SM_ROLE_W_DOWN})
      if (!L.w[r]) return fail(SM_ERR_STATE, "model_finalize: missing weight");
  }
  m->finalized = true;
  return SM_OK;
}

SM_API int sm_model_destroy(sm_model* m) {
  if (!m) return SM_OK;
  DeviceGuard g(m->device);
  cudaDeviceSynchronize();
  Work& w = m->work;
  for (void* p : {(void*)w.x, (void*)w.h, (void*)w.qkv, (void*)w.att, (void*)w.g, (void*)w.u, (void*)w.logits,
                  (void*)w.ints, (void*)w.attn_scratch, (void*)m->embd, (void*)m->out_norm, (void*)m->sin_t,
                  (void*)m->cos_t})
    if (p) cudaFree(p);
  for (auto& L : m->layers)
    for (void* p : {(void*)L.attn_norm, (void*)L.ffn_norm})
      if (p) cudaFree(p);
  delete m;
  return SM_OK;
}

SM_API int sm_model_nbytes(const sm_model* m, size_t* out) {
  if (!m || !out) return fail(SM_ERR_INVALID_ARG, "null argument");
  const auto& c = m->cfg;
  const Work& w = m->work;
  *out = m->own_bytes + (size_t)w.cap_rows * 4 * (2 * c.hidden + m->qkv_stride() + m->qd() + 2 * c.ffn_hidden + 5) +
         (size_t)w.cap_logit_rows * 4 * c.vocab_size + w.attn_scratch_floats * 4;
  return SM_OK;
}

SM_API int sm_kv_create(sm_model* m, int max_seqs, int max_tokens, sm_kv** out) {
  if (!m || !out) return fail(SM_ERR_INVALID_ARG, "kv_create: null argument");
  *out = nullptr;
  if (max_seqs <= 0 || max_tokens <= 0) return fail(SM_ERR_INVALID_ARG, "kv_create: sizes must be positive");
  if (max_tokens > m->cfg.max_context) return fail(SM_ERR_INVALID_ARG, "kv_create: max_tokens exceeds max_context");
  DeviceGuard g(m->ctx->device);
  auto* kv = new sm_kv();
  kv->m = m;
  kv->device = m->device;
  kv->max_seqs = max_seqs;
  kv->max_tokens = max_tokens;
  const size_t bytes = kv->layer_stride() * m->cfg.n_layers * sizeof(float);
  bool ok = cudaMalloc(&kv->k, bytes) == cudaSuccess && cudaMalloc(&kv->v, bytes) == cudaSuccess &&
            cudaMalloc(&kv->len_dev, sizeof(int) * max_seqs) == cudaSuccess;
  if (!ok) {
    if (kv->k) cudaFree(kv->k);
    if (kv->v) cudaFree(kv->v);
    delete kv;
    return fail(SM_ERR_OOM, "kv_create: out of device memory");
  }
  cudaMemset(kv->len_dev, 0, sizeof(int) * max_seqs);
  kv->len_host.assign(max_seqs, 0);
  *out = kv;
  return SM_OK;
}

SM_API int sm_kv_destroy(sm_kv* kv) {
  if (!kv) return SM_OK;
  DeviceGuard g(kv->device);
  cudaDeviceSynchronize();
  for (auto& it : kv->graphs)
    if (it.second.exec) cudaGraphExecDestroy(it.second.exec);
  if (kv->mega_layers) cudaFree(kv->mega_layers);
  if (kv->mega_sync) cudaFree(kv->mega_sync);
  if (kv->mega_ll) cudaFree(kv->mega_ll);
  if (kv->mega_trace) cudaFree(kv->mega_trace);
  cudaFree(kv->k);
  cudaFree(kv->v);
  cudaFree(kv->len_dev);
  if (kv->pinned) cudaFreeHost(kv->pinned);
  delete kv;
  return SM_OK;
}

static int kv_sync_host(sm_kv* kv) {
  if (!kv->host_stale) return SM_OK;
  cudaStream_t st = kv->m->ctx->stream;
  SM_CUDA_TRY(cudaMemcpyAsync(kv->len_host.data(), kv->len_dev, sizeof(int) * kv->max_seqs, cudaMemcpyDeviceToHost,
                              st));
  SM_CUDA_TRY(cudaStreamSynchronize(st));
  kv->host_stale = false;
  return SM_OK;
}

SM_API int sm_kv_reset(sm_kv* kv, int seq) {
  if (!kv) return fail(SM_ERR_INVALID_ARG, "null kv");
  if (seq < 0 || seq >= kv->max_seqs) return fail(SM_ERR_INVALID_ARG, "kv_reset: bad sequence id");
  DeviceGuard g(kv->m->ctx->device);
  SM_TRY(kv_sync_host(kv));
  kv->len_host[seq] = 0;
  SM_CUDA_TRY(cudaMemsetAsync(kv->len_dev + seq, 0, sizeof(int), kv->m->ctx->stream));
  return SM_OK;
}

// KvCacheEntry.Slide (KvCacheEntry.cs:203-229): positions [start, start + keep)
// move to [0, keep) in every layer and KV head, K and V.  One CTA per (head,
// K|V, layer) walks the run front to back in chunks of at most `start` tokens,
// so a chunk's source never overlaps its destination or a later chunk's source.
__global__ void kv_slide_kernel(float* k, float* v, size_t layer_stride, int seq, int n_kv, int max_tokens, int hd,
                                int start, int keep) {
  float* base = (blockIdx.y ? v : k) + layer_stride * blockIdx.z + ((size_t)seq * n_kv + blockIdx.x) * max_tokens * hd;
  const int step = min(start, 64);
  for (int t0 = 0; t0 < keep; t0 += step) {
    const int n = min(step, keep - t0) * hd / 4;
    const float4* src = (const float4*)(base + (size_t)(t0 + start) * hd);
    float4* dst = (float4*)(base + (size_t)t0 * hd);
    float4 tmp[4];
    for (int i0 = 0; i0 < n; i0 += 4 * blockDim.x) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = i0 + j * blockDim.x + threadIdx.x;
        if (i < n) tmp[j] = src[i];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = i0 + j * blockDim.x + threadIdx.x;
        if (i < n) dst[i] = tmp[j];
      }
    }
    __syncthreads();
  }
}

static int kv_set_length(sm_kv* kv, int seq, int len) {
  kv->len_host[seq] = len;
  SM_CUDA_TRY(cudaMemcpyAsync(kv->len_dev + seq, &len, sizeof(int), cudaMemcpyHostToDevice, kv->m->ctx->stream));
  SM_CUDA_TRY(cudaStreamSynchronize(kv->m->ctx->stream));
  return SM_OK;
}

SM_API int sm_kv_truncate(sm_kv* kv, int seq, int len) {
  if (!kv) return fail(SM_ERR_INVALID_ARG, "null kv");
  if (seq < 0 || seq >= kv->max_seqs) return fail(SM_ERR_INVALID_ARG, "kv_truncate: bad sequence id");
  DeviceGuard g(kv->m->ctx->device);
  SM_TRY(kv_sync_host(kv));
  if (len < 0 || len > kv->len_host[seq]) return fail(SM_ERR_SHAPE, "kv_truncate: length outside [0, current length]");
  return kv_set_length(kv, seq, len);
}

SM_API int sm_kv_slide(sm_kv* kv, int seq, int window) {
  if (!kv) return fail(SM_ERR_INVALID_ARG, "null kv");
  if (seq < 0 || seq >= kv->max_seqs) return fail(SM_ERR_INVALID_ARG, "kv_slide: bad sequence id");
  // KvCacheEntry.cs:205-206
  if (window < 0) return fail(SM_ERR_INVALID_ARG, "kv_slide: window must be non-negative");
  DeviceGuard g(kv->m->ctx->device);
  SM_TRY(kv_sync_host(kv));
  const int cur = kv->len_host[seq];
  if (window >= cur) return SM_OK;  // nothing to slide (KvCacheEntry.cs:208-209)
  const auto& c = kv->m->cfg;
  if (window > 0) {
    if (c.head_dim % 4) return fail(SM_ERR_UNSUPPORTED, "kv_slide: head_dim must be a multiple of 4");
    dim3 grid(c.n_kv_heads, 2, c.n_layers);
    kv_slide_kernel<<<grid, 256, 0, kv->m->ctx->stream>>>(kv->k, kv->v, kv->layer_stride(), seq, c.n_kv_heads,
                                                         kv->max_tokens, c.head_dim, cur - window, window);
    SM_CUDA_TRY(cudaGetLastError());
  }
  return kv_set_length(kv, seq, window);
}

SM_API int sm_kv_read(sm_kv* kv, int layer, int seq, int start, int count, float* keys, float* values) {
  if (!kv || (!keys && !values)) return fail(SM_ERR_INVALID_ARG, "kv_read: null argument");
  const auto& c = kv->m->cfg;
  if (layer < 0 || layer >= c.n_layers) return fail(SM_ERR_INVALID_ARG, "kv_read: bad layer");
  if (seq < 0 || seq >= kv->max_seqs) return fail(SM_ERR_INVALID_ARG, "kv_read: bad sequence id");
  DeviceGuard g(kv->m->ctx->device);
  SM_TRY(kv_sync_host(kv));
  // KvCacheEntry.GetKeys / GetValues (KvCacheEntry.cs:155-189): the range must lie inside the cached tokens
  if (start < 0 || count < 0 || start + count > kv->len_host[seq]) return fail(SM_ERR_SHAPE, "kv_read: range outside the cached tokens");
  if (count == 0) return SM_OK;
  cudaStream_t st = kv->m->ctx->stream;
  const size_t hd = c.head_dim, row = hd * sizeof(float);
  for (int which = 0; which < 2; ++which) {
    float* out = which ? values : keys;
    if (!out) continue;
    const float* base = (which ? kv->v : kv->k) + kv->layer_stride() * layer;
    for (int h = 0; h < c.n_kv_heads; ++h) {
      const float* src = base + (((size_t)seq * c.n_kv_heads + h) * kv->max_tokens + start) * hd;
      SM_CUDA_TRY(cudaMemcpy2DAsync(out + h * hd, row * c.n_kv_heads, src, row, row, count, cudaMemcpyDeviceToHost, st));
    }
  }
  SM_CUDA_TRY(cudaStreamSynchronize(st));
  return SM_OK;
}

SM_API int sm_kv_length(sm_kv* kv, int seq, int* len) {
  if (!kv || !len) return fail(SM_ERR_INVALID_ARG, "null argument");
  if (seq < 0 || seq >= kv->max_seqs) return fail(SM_ERR_INVALID_ARG, "kv_length: bad sequence id");
  DeviceGuard g(kv->m->ctx->device);
  SM_TRY(kv_sync_host(kv));
  *len = kv->len_host[seq];
  return SM_OK;
}

SM_API int sm_prefill(sm_model* m, sm_kv* kv, int seq, const int* tokens, int T, float* last_logits,
                      int* next_token) {
  if (!m || !kv || !tokens) return fail(SM_ERR_INVALID_ARG, "prefill: null argument");
  if (!m->finalized) return fail(SM_ERR_STATE, "prefill: model not finalized");
  if (kv->m != m) return fail(SM_ERR_INVALID_ARG, "prefill: cache belongs to another model");
  if (seq < 0 || seq >= kv->max_seqs) return fail(SM_ERR_INVALID_ARG, "prefill: bad sequence id");
  if (T <= 0) return fail(SM_ERR_SHAPE, "prefill: need at least one token");
  DeviceGuard g(m->ctx->device);
  SM_TRY(kv_sync_host(kv));
  const int pos0 = kv->len_host[seq];
  // TransformerModel.cs:280-283: Sequence length + offset must not exceed block size
  if (pos0 + T > kv->max_tokens) return fail(SM_ERR_SHAPE, "prefill: Sequence length + offset exceeds block size");
  for (int i = 0; i < T; ++i)
    if (tokens[i] < 0 || tokens[i] >= m->cfg.vocab_size) return fail(SM_ERR_INVALID_ARG, "prefill: token id out of range");
  SM_TRY(work_reserve(m, T, 1, 1, kv->max_tokens));
  cudaStream_t st = m->ctx->stream;
  Work& w = m->work;
  std::vector<int> staging((size_t)4 * T);
  for (int i = 0; i < T; ++i) {
    staging[i] = tokens[i];
    staging[T + i] = seq;
    staging[2 * T + i] = pos0 + i;
    staging[3 * T + i] = pos0 + i + 1;
  }
  SM_CUDA_TRY(cudaMemcpyAsync(w.tok(), staging.data(), sizeof(int) * T, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(w.seq(), staging.data() + T, sizeof(int) * T, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(w.pos(), staging.data() + 2 * T, sizeof(int) * T, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(w.lens(), staging.data() + 3 * T, sizeof(int) * T, cudaMemcpyHostToDevice, st));
  int nl = 0;
  const PrefillSeg seg{seq, pos0, 0, T};
  SM_TRY(forward(m, kv, T, &seg, 1, nl));
  m->ctx->launches += nl;
  const int newlen = pos0 + T;
  SM_CUDA_TRY(cudaMemcpyAsync(kv->len_dev + seq, &newlen, sizeof(int), cudaMemcpyHostToDevice, st));
  if (last_logits)
    SM_CUDA_TRY(cudaMemcpyAsync(last_logits, w.logits, sizeof(float) * m->cfg.vocab_size, cudaMemcpyDeviceToHost, st));
  if (next_token) SM_CUDA_TRY(cudaMemcpyAsync(next_token, w.amax(), sizeof(int), cudaMemcpyDeviceToHost, st));
  SM_CUDA_TRY(cudaStreamSynchronize(st));
  kv->len_host[seq] = newlen;
  return SM_OK;
}

SM_API int sm_prefill_batch(sm_model* m, sm_kv* kv, const int* seq_ids, const int* tokens, const int* n_tokens,
                            int n, float* last_logits, int* next_tokens) {
  if (!m || !kv || !seq_ids || !tokens || !n_tokens) return fail(SM_ERR_INVALID_ARG, "prefill_batch: null argument");
  if (!m->finalized) return fail(SM_ERR_STATE, "prefill_batch: model not finalized");
  if (kv->m != m) return fail(SM_ERR_INVALID_ARG, "prefill_batch: cache belongs to another model");
  if (n <= 0 || n > kv->max_seqs) return fail(SM_ERR_SHAPE, "prefill_batch: prompt count out of range");
  DeviceGuard g(m->ctx->device);
  SM_TRY(kv_sync_host(kv));
  std::vector<PrefillSeg> segs(n);
  std::vector<char> seen(kv->max_seqs, 0);
  int rows = 0;
  for (int i = 0; i < n; ++i) {
    const int s = seq_ids[i], T = n_tokens[i];
    if (s < 0 || s >= kv->max_seqs) return fail(SM_ERR_INVALID_ARG, "prefill_batch: bad sequence id");
    if (seen[s]) return fail(SM_ERR_INVALID_ARG, "prefill_batch: a sequence appears twice");
    seen[s] = 1;
    if (T <= 0) return fail(SM_ERR_SHAPE, "prefill_batch: need at least one token per prompt");
    // TransformerModel.cs:280-283, per prompt
    if (kv->len_host[s] + T > kv->max_tokens)
      return fail(SM_ERR_SHAPE, "prefill_batch: Sequence length + offset exceeds block size");
    segs[i] = PrefillSeg{s, kv->len_host[s], rows, T};
    rows += T;
  }
  for (int r = 0; r < rows; ++r)
    if (tokens[r] < 0 || tokens[r] >= m->cfg.vocab_size)
      return fail(SM_ERR_INVALID_ARG, "prefill_batch: token id out of range");
  SM_TRY(work_reserve(m, rows, n, 1, kv->max_tokens));
  cudaStream_t st = m->ctx->stream;
  Work& w = m->work;
  std::vector<int> staging((size_t)4 * rows);
  for (const auto& sg : segs)
    for (int i = 0; i < sg.T; ++i) {
      const int r = sg.r0 + i;
      staging[r] = tokens[r];
      staging[rows + r] = sg.seq;
      staging[2 * rows + r] = sg.pos0 + i;
      staging[3 * rows + r] = sg.pos0 + i + 1;
    }
  SM_CUDA_TRY(cudaMemcpyAsync(w.tok(), staging.data(), sizeof(int) * rows, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(w.seq(), staging.data() + rows, sizeof(int) * rows, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(w.pos(), staging.data() + 2 * rows, sizeof(int) * rows, cudaMemcpyHostToDevice, st));
  SM_CUDA_TRY(cudaMemcpyAsync(w.lens(), staging.data() + 3 * rows, sizeof(int) * rows, cudaMemcpyHostToDevice, st));
  int nl = 0;
  SM_TRY(forward(m, kv, rows, segs.data(), n, nl));
  m->ctx->launches += nl;
  std::vector<int> newlen(n);
  for (int i = 0; i < n; ++i) {
    newlen[i] = segs[i].pos0 + segs[i].T;
    SM_CUDA_TRY(cudaMemcpyAsync(kv->len_dev + segs[i].seq, &newlen[i], sizeof(int), cudaMemcpyHostToDevice, st));
  }
  if (last_logits)
    SM_CUDA_TRY(cudaMemcpyAsync(last_logits, w.logits, sizeof(float) * (size_t)n * m->cfg.vocab_size,
                                cudaMemcpyDeviceToHost, st));
  if (next_tokens) SM_CUDA_TRY(cudaMemcpyAsync(next_tokens, w.amax(), sizeof(int) * n, cudaMemcpyDeviceToHost, st));
  SM_CUDA_TRY(cudaStreamSynchronize(st));
  for (int i = 0; i < n; ++i) kv->len_host[segs[i].seq] = newlen[i];
  return SM_OK;
}

SM_API int sm_decode(sm_model* m, sm_kv* kv, const int* seq_ids, const int* tokens, int n, float* logits,
                     int* next_tokens, int flags) {
  if (!m || !kv || !seq_ids || !tokens) return fail(SM_ERR_INVALID_ARG, "decode: null argument");
  if (!m->finalized) return fail(SM_ERR_STATE, "decode: model not finalized");
  if (kv->m != m) return fail(SM_ERR_INVALID_ARG, "decode: cache belongs to another model");
  if (n <= 0 || n > kv->max_seqs) return fail(SM_ERR_SHAPE, "decode: batch size out of range");
  DeviceGuard g(m->ctx->device);
  cudaStream_t st = m->ctx->stream;
  const bool host = flags == SM_PTR_HOST;
  if (host) {
    SM_TRY(kv_sync_host(kv));
    std::vector<char> seen(kv->max_seqs, 0);
    for (int i = 0; i < n; ++i) {
      const int s = seq_ids[i];
      if (s < 0 || s >= kv->max_seqs) return fail(SM_ERR_INVALID_ARG, "decode: bad sequence id");
      if (seen[s]) return fail(SM_ERR_INVALID_ARG, "decode: a sequence appears twice in one step");
      seen[s] = 1;
      if (kv->len_host[s] + 1 > kv->max_tokens) return fail(SM_ERR_SHAPE, "decode: context is full");
      if (tokens[i] < 0 || tokens[i] >= m->cfg.vocab_size) return fail(SM_ERR_INVALID_ARG, "decode: token id out of range");
    }
  }
  SM_TRY(work_reserve(m, n, n, n, kv->max_tokens));
  Work& w = m->work;
  // inputs -> work.tok / work.seq
  if (host) {
    if (kv->pinned_cap < 2 * n) {
      if (kv->pinned) cudaFreeHost(kv->pinned);
      SM_CUDA_TRY(cudaMallocHost((void**)&kv->pinned, sizeof(int) * 2 * n));
      kv->pinned_cap = 2 * n;
    }
    SM_CUDA_TRY(cudaStreamSynchronize(st));  // pinned staging reuse
    std::memcpy(kv->pinned, tokens, sizeof(int) * n);
    std::memcpy(kv->pinned + n, seq_ids, sizeof(int) * n);
    SM_CUDA_TRY(cudaMemcpyAsync(w.tok(), kv->pinned, sizeof(int) * n, cudaMemcpyHostToDevice, st));
    SM_CUDA_TRY(cudaMemcpyAsync(w.seq(), kv->pinned + n, sizeof(int) * n, cudaMemcpyHostToDevice, st));
  } else {
    SM_CUDA_TRY(cudaMemcpyAsync(w.tok(), tokens, sizeof(int) * n, cudaMemcpyDeviceToDevice, st));
    SM_CUDA_TRY(cudaMemcpyAsync(w.seq(), seq_ids, sizeof(int) * n, cudaMemcpyDeviceToDevice, st));
  }
  MegaArgs mega;
  const bool use_mega = n == 1 && mega_enabled(m) && mega_args(m, kv, mega) == SM_OK;
  auto body = [&](int& nl) -> int {
    if (use_mega) return launch_decode_mega(mega, st, &nl);
    decode_prep_kernel<<<ceil_div(n, 128), 128, 0, st>>>(w.seq(), w.pos(), w.lens(), kv->len_dev, n, kv->max_tokens,
                                                          m->ctx->dev_status);
    ++nl;
    SM_TRY(forward(m, kv, n, nullptr, 0, nl));
    decode_commit_kernel<<<ceil_div(n, 128), 128, 0, st>>>(w.seq(), kv->len_dev, n, kv->max_tokens);
    ++nl;
    SM_CUDA_TRY(cudaGetLastError());
    return SM_OK;
  };
  sm_kv::Graph& gr = kv->graphs[n];
  if (use_graphs() && gr.eager_runs > 0) {
    if (!gr.exec || gr.generation != w.generation) {
      if (gr.exec) cudaGraphExecDestroy(gr.exec);
      gr.exec = nullptr;
      // capture the step once; kernels read tok/seq/lengths from device buffers
      SM_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      int nl = 0;
      int rc = body(nl);
      cudaGraph_t graph = nullptr;
      cudaError_t e = cudaStreamEndCapture(st, &graph);
      if (rc != SM_OK) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
      }
      if (e != cudaSuccess) return fail(SM_ERR_CUDA, std::string("decode: graph capture failed: ") + cudaGetErrorString(e));
      e = cudaGraphInstantiate(&gr.exec, graph, 0);
      cudaGraphDestroy(graph);
      if (e != cudaSuccess) return fail(SM_ERR_CUDA, std::string("decode: graph instantiate failed: ") + cudaGetErrorString(e));
      gr.generation = w.generation;
      gr.launches = nl;
    }
    SM_CUDA_TRY(cudaGraphLaunch(gr.exec, st));
    m->ctx->launches += gr.launches;
  } else {
    // first step of a batch size runs eagerly (sets kernel attributes outside capture)
    int nl = 0;
    SM_TRY(body(nl));
    m->ctx->launches += nl;
    gr.eager_runs += 1;
  }
  const cudaMemcpyKind out_kind = host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
  if (logits)
    SM_CUDA_TRY(cudaMemcpyAsync(logits, w.logits, sizeof(float) * (size_t)n * m->cfg.vocab_size, out_kind, st));
  if (next_tokens) SM_CUDA_TRY(cudaMemcpyAsync(next_tokens, w.amax(), sizeof(int) * n, out_kind, st));
  if (use_mega && mega.trace) {
    // profiling: append this step's per-CTA phase timestamps to the trace file
    const int grid = mega_grid_size();
    std::vector<unsigned long long> t((size_t)grid * MEGA_TRACE_EVENTS);
    SM_CUDA_TRY(cudaMemcpyAsync(t.data(), mega.trace, t.size() * 8, cudaMemcpyDeviceToHost, st));
    SM_CUDA_TRY(cudaStreamSynchronize(st));
    if (FILE* f = std::fopen(std::getenv("SMALLMIND_MEGA_TRACE"), "ab")) {
      std::fwrite(t.data(), 8, t.size(), f);
      std::fclose(f);
    }
  }
  if (host) {
    SM_CUDA_TRY(cudaStreamSynchronize(st));
    for (int i = 0; i < n; ++i) kv->len_host[seq_ids[i]] += 1;
  } else {
    kv->host_stale = true;
  }
  return SM_OK;
}

}  // extern "C"
