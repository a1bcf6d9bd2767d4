// Allocation-free entry point for the batched decode attention.
//
// sm_attention_decode takes its working memory (scores, per-chunk maxima and
// partial sums) from the stream-ordered allocator on every call.  Some callers
// cannot let a library allocate device memory: a host that reserves its whole
// device budget up front and hands out fixed buffers (the engine's strict
// memory-budget mode), or code running where another framework's allocator
// owns the device and a second allocator is not allowed in.  This variant
// takes the same inputs and outputs but uses a fixed scratch array that lives
// in this library's device image instead.
//
//  * The single-launch cluster kernel, which needs no scratch at all, runs
//    whenever it takes the shape (head_dim 64, at most 8 q heads per kv head);
//    only the other shapes use the split-context kernels and the array below.
//  * The scratch is a file-scope static __device__ array of 16 MiB.  Every GPU
//    that loads the library holds it until the process exits.
//  * Host code cannot use the array's name as a device address (in host code
//    it names a host-side stand-in), so the first call on each device, with
//    that device current, looks up the real address with cudaGetSymbolAddress
//    and caches it.  Make that first call before any stream capture.
//  * Shapes the cluster kernel does not take and whose scratch would exceed
//    16 MiB are rejected with SM_ERR_SHAPE.
//  * The cached address belongs to the CUDA context current at the first call:
//    resetting or re-creating a device's primary context afterwards is not
//    supported by this entry point.
//  * All calls share the one array and it keeps the previous call's contents.
//    Nothing needs clearing: every scratch element a call reads is written
//    earlier in the same call.  Calls that overlap on the GPU (two streams,
//    two host threads) race on the array; serialise them.
//  * No cudaMalloc, cudaFree or other allocating call is made.
#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr size_t kNoAllocScratchFloats = kNoAllocScratchBytes / sizeof(float);

static __device__ __align__(256) float g_decode_attention_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on `device` (which must be current).
int scratch_address(int device, float** out) {
  if (device < 0 || device >= kMaxDevices) return sm::fail(SM_ERR_UNSUPPORTED, "attention_decode_noalloc: device id too large");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_decode_attention_scratch);
    if (e != cudaSuccess || !p)
      return sm::fail(SM_ERR_CUDA, std::string("attention_decode_noalloc: cudaGetSymbolAddress failed: ") +
                                       cudaGetErrorString(e));
    g_scratch_addr[device] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[device];
  return SM_OK;
}

}  // namespace

extern "C" SM_API int sm_attention_decode_noalloc(sm_ctx* ctx, const float* q, const float* k_cache,
                                                  const float* v_cache, float* out, const int* lens_dev, int B,
                                                  int max_ctx, int n_heads, int n_kv, int head_dim) {
  if (B <= 0 || max_ctx <= 0 || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv)
    return sm::fail(SM_ERR_SHAPE, "attention_decode_noalloc: bad shape");
  if (!ctx || !q || !k_cache || !v_cache || !out || !lens_dev)
    return sm::fail(SM_ERR_INVALID_ARG, "attention_decode_noalloc: null argument");
  int device = 0;
  cudaStream_t stream = nullptr;
  int64_t* launches = nullptr;
  SM_TRY(sm::ctx_view(ctx, &device, &stream, &launches));
  int prev = -1;
  SM_CUDA_TRY(cudaGetDevice(&prev));
  if (prev != device) SM_CUDA_TRY(cudaSetDevice(device));
  const int64_t head_stride = (int64_t)max_ctx * head_dim;
  int nl = 0;
  int rc = sm::launch_attention_decode_cluster(q, n_heads * head_dim, k_cache, v_cache, head_stride * n_kv, head_dim,
                                               head_stride, max_ctx, out, n_heads * head_dim, lens_dev, nullptr, B,
                                               n_heads, n_kv, head_dim, stream, &nl);
  if (rc != SM_ERR_UNSUPPORTED) {
    *launches += nl;
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    return rc;
  }
  nl = 0;
  float* scratch = nullptr;
  if (sm::attention_decode_scratch_floats(B, n_heads, max_ctx) > kNoAllocScratchFloats)
    rc = sm::fail(SM_ERR_SHAPE, "attention_decode_noalloc: B * n_heads * (max_ctx + 66 * ceil(max_ctx / 64)) "
                                "floats exceed the 16 MiB static scratch");
  else
    rc = scratch_address(device, &scratch);
  if (rc == SM_OK) {
    rc = sm::launch_attention_decode(q, n_heads * head_dim, k_cache, v_cache, head_stride * n_kv, head_dim,
                                     head_stride, max_ctx, out, n_heads * head_dim, lens_dev, nullptr, B, n_heads,
                                     n_kv, head_dim, scratch, kNoAllocScratchFloats, stream, &nl);
    *launches += nl;
  }
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  return rc;
}
