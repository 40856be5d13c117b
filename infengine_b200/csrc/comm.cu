// Tensor-parallel exchange steps: allreduce of row-split partial sums and the
// cross-shard argmax merge, over NCCL (NVLink / NVSwitch within a B200 box).
//
// NCCL is resolved at run time (dlopen "libnccl.so.2", normally already loaded
// by the host process), so the library has no link-time NCCL dependency and
// single-GPU users never load it. The exchanges run on the caller's stream and
// can be recorded into CUDA graphs like the kernels around them.
#include <dlfcn.h>
#include <nccl.h>
#include <cstdio>
#include <cstring>
#include <mutex>
#include "ie_common.cuh"

struct ie_comm {
  ncclComm_t comm;
  int nranks;
  int rank;
};

namespace {

struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(h, "ncclAllReduce"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.get_unique_id && n.comm_init_rank && n.all_reduce && n.comm_destroy;
  });
  return n;
}

int from_nccl(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return IE_OK;
  const Nccl& n = nccl();
  std::fprintf(stderr, "infengine_b200: %s: %s\n", what, n.error_string ? n.error_string(r) : "NCCL error");
  return IE_ERR_LAUNCH;
}

__global__ void keys_to_ids_kernel(const unsigned long long* keys, int M, int* idx_out) {
  for (int m = threadIdx.x; m < M; m += blockDim.x) idx_out[m] = ie::argmax_key_index(keys[m]);
}

template <typename T>
__global__ void cast_kernel(const float* in, T* out, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = ie::DT<T>::from_f(in[i]);
}

// out[i] = round(out[i] + round(in[i])): the residual add of an allreduced
// fp32 projection (the reference rounds the projection, then adds, decode.cu:28).
template <typename T>
__global__ void add_kernel(const float* in, T* out, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = ie::DT<T>::from_f(ie::DT<T>::to_f(out[i]) + ie::round_to<T>(in[i]));
}

}  // namespace

extern "C" {

int ie_comm_unique_id(void* out) {
  const Nccl& n = nccl();
  if (!n.ok) return IE_ERR_UNSUPPORTED;
  if (!out) return IE_ERR_INVALID_ARG;
  ncclUniqueId id;
  int s = from_nccl(n.get_unique_id(&id), "ncclGetUniqueId");
  if (s == IE_OK) memcpy(out, &id, sizeof(id));
  return s;
}

int ie_comm_create(int nranks, int rank, const void* unique_id, ie_comm** out) {
  if (nranks <= 0 || rank < 0 || rank >= nranks || !unique_id || !out) return IE_ERR_INVALID_ARG;
  const Nccl& n = nccl();
  if (!n.ok) return IE_ERR_UNSUPPORTED;
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  ie_comm* c = new ie_comm{nullptr, nranks, rank};
  int s = from_nccl(n.comm_init_rank(&c->comm, nranks, id, rank), "ncclCommInitRank");
  if (s != IE_OK) {
    delete c;
    return s;
  }
  *out = c;
  return IE_OK;
}

int ie_comm_destroy(ie_comm* c) {
  if (!c) return IE_OK;
  int s = IE_OK;
  if (c->comm) s = from_nccl(nccl().comm_destroy(c->comm), "ncclCommDestroy");
  delete c;
  return s;
}

int ie_allreduce_sum_f32(ie_comm* c, float* buf, size_t count, void* stream) {
  if (!c || (!buf && count)) return IE_ERR_INVALID_ARG;
  if (count == 0) return IE_OK;
  return from_nccl(nccl().all_reduce(buf, buf, count, ncclFloat32, ncclSum, c->comm,
                                     reinterpret_cast<cudaStream_t>(stream)),
                   "ncclAllReduce(sum)");
}

int ie_argmax_allreduce(ie_comm* c, unsigned long long* keys, int M, int* idx_out, void* stream) {
  if (!c || !keys || M < 0) return IE_ERR_INVALID_ARG;
  if (M == 0) return IE_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int s = from_nccl(nccl().all_reduce(keys, keys, (size_t)M, ncclUint64, ncclMax, c->comm, st), "ncclAllReduce(max)");
  if (s != IE_OK || !idx_out) return s;
  keys_to_ids_kernel<<<1, 128, 0, st>>>(keys, M, idx_out);
  return cudaGetLastError() == cudaSuccess ? IE_OK : IE_ERR_LAUNCH;
}

int ie_cast_f32(ie_dtype dt, const float* in, void* out, size_t n, void* stream) {
  if ((dt != IE_DTYPE_F16 && dt != IE_DTYPE_BF16) || (n && (!in || !out))) return IE_ERR_INVALID_ARG;
  if (n == 0) return IE_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int blocks = (int)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
  if (dt == IE_DTYPE_BF16)
    cast_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(in, static_cast<__nv_bfloat16*>(out), n);
  else
    cast_kernel<__half><<<blocks, 256, 0, st>>>(in, static_cast<__half*>(out), n);
  return cudaGetLastError() == cudaSuccess ? IE_OK : IE_ERR_LAUNCH;
}

int ie_add_f32(ie_dtype dt, const float* in, void* out, size_t n, void* stream) {
  if ((dt != IE_DTYPE_F16 && dt != IE_DTYPE_BF16) || (n && (!in || !out))) return IE_ERR_INVALID_ARG;
  if (n == 0) return IE_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int blocks = (int)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
  if (dt == IE_DTYPE_BF16)
    add_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(in, static_cast<__nv_bfloat16*>(out), n);
  else
    add_kernel<__half><<<blocks, 256, 0, st>>>(in, static_cast<__half*>(out), n);
  return cudaGetLastError() == cudaSuccess ? IE_OK : IE_ERR_LAUNCH;
}

}  // extern "C"
