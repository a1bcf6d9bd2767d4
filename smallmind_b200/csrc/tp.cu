// Tensor-parallel decode plumbing: the NCCL calls, loaded at run time.
//
// A tensor-parallel group is one process per GPU.  Each rank holds a shard of
// every layer (its q / kv heads and its FFN units for the column-split Q|K|V and
// gate|up; the matching input columns of the row-split O and down projections)
// and, after each row-split projection, the ranks sum their partial outputs
// with one NCCL all-reduce before the residual add (MultiHeadAttention.cs:92-93
// _qkv / _proj, GatedMLP.cs:38-40 gate / up / down are the projections split).
//
// libnccl.so.2 is opened with dlopen on first use, so the library itself has no
// link-time dependency on NCCL: only callers that form a group need it (PyTorch
// ships the same NCCL build and has usually loaded it already).
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace sm {
namespace {

struct NcclApi {
  bool loaded = false;
  std::string error;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      api.error = std::string("libnccl.so.2 not loadable: ") + (e ? e : "?");
      return;
    }
    api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
    api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
    api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
    api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
    api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
    if (!api.get_unique_id || !api.comm_init_rank || !api.all_reduce || !api.comm_destroy || !api.error_string) {
      api.error = "libnccl.so.2 lacks an expected symbol";
      return;
    }
    api.loaded = true;
  });
  return api;
}

int nccl_fail(ncclResult_t r, const char* what) {
  return fail(SM_ERR_NCCL, std::string(what) + ": " + nccl().error_string(r));
}

}  // namespace

int tp_unique_id(void* out, size_t n) {
  if (!out || n < sizeof(ncclUniqueId)) return fail(SM_ERR_INVALID_ARG, "tp_unique_id: need a 128-byte buffer");
  NcclApi& api = nccl();
  if (!api.loaded) return fail(SM_ERR_NCCL, api.error);
  ncclUniqueId id;
  const ncclResult_t r = api.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(out, &id, sizeof(id));
  return SM_OK;
}

int tp_comm_create(int size, int rank, const void* id, size_t n, void** comm) {
  if (!id || n < sizeof(ncclUniqueId) || !comm) return fail(SM_ERR_INVALID_ARG, "tp_init: bad unique id");
  if (size < 1 || rank < 0 || rank >= size) return fail(SM_ERR_INVALID_ARG, "tp_init: rank outside [0, size)");
  NcclApi& api = nccl();
  if (!api.loaded) return fail(SM_ERR_NCCL, api.error);
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  const ncclResult_t r = api.comm_init_rank(&c, size, uid, rank);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
  *comm = c;
  return SM_OK;
}

void tp_comm_destroy(void* comm) {
  if (comm && nccl().loaded) nccl().comm_destroy((ncclComm_t)comm);
}

int tp_allreduce_sum(void* comm, float* buf, size_t n, cudaStream_t st) {
  NcclApi& api = nccl();
  if (!api.loaded) return fail(SM_ERR_NCCL, api.error);
  const ncclResult_t r = api.all_reduce(buf, buf, n, ncclFloat32, ncclSum, (ncclComm_t)comm, st);
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
  return SM_OK;
}

namespace {
__global__ void add_rows_kernel(float* __restrict__ x, const float* __restrict__ p, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] += p[i];
}
}  // namespace

int launch_add(float* x, const float* p, int64_t n, cudaStream_t st) {
  const int blocks = (int)std::min<int64_t>(1024, (n + 255) / 256);
  add_rows_kernel<<<blocks, 256, 0, st>>>(x, p, n);
  SM_CUDA_TRY(cudaGetLastError());
  return SM_OK;
}

}  // namespace sm
