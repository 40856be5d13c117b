// Tensor-parallel row-split projection fused with its allreduce over NVLink
// peer memory (ie_gemm_allreduce: every CTA of the decode GEMV pushes its fp32
// partial rows, each value tagged with the call's epoch in one 64-bit word,
// into every rank's buffer; the CTA that completes a rank's grid waits for
// every rank's tagged words and sums them), and the CUDA IPC calls that map
// every rank's exchange buffer into every other rank's address space.
//
// The exchange buffers are ordinary device allocations of the caller (one per
// rank, ie_tp_exchange_bytes each, zeroed once). Each rank exports its buffer
// (ie_ipc_export: the IPC handle of the allocation that contains it plus the
// offset inside it), the caller distributes the handles, and each rank maps
// its peers' buffers (ie_ipc_import). Only plain loads and stores touch peer
// memory: no TMA, no multicast.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cstring>
#include <mutex>
#include "ie_common.cuh"
#include "skinny.cuh"

using namespace ie;

namespace {

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 3020, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(f);
  });
  return fn;
}

std::mutex g_import_mutex;
struct Import {
  void* ptr;
  void* base;
};
constexpr int kMaxImports = 256;
Import g_imports[kMaxImports];
int g_nimports = 0;

}  // namespace

extern "C" {

size_t ie_tp_exchange_bytes(int world, int max_rows, int max_cols) {
  if (world <= 0 || max_rows <= 0 || max_cols <= 0) return 0;
  return kTpInboxOffset + (size_t)2 * world * max_rows * max_cols * sizeof(unsigned long long);
}

int ie_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return IE_ERR_INVALID_ARG;
  auto range = address_range_fn();
  if (!range) return IE_ERR_UNSUPPORTED;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return IE_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return IE_ERR_UNSUPPORTED;
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (uint64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
  return IE_OK;
}

int ie_ipc_import(const void* handle, uint64_t offset, void** ptr_out) {
  if (!handle || !ptr_out) return IE_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  std::lock_guard<std::mutex> lock(g_import_mutex);
  // every mapping must be releasable: refuse a new one when the table is full
  if (g_nimports >= kMaxImports) return IE_ERR_UNSUPPORTED;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return IE_ERR_UNSUPPORTED;
  *ptr_out = static_cast<char*>(base) + offset;
  g_imports[g_nimports++] = Import{*ptr_out, base};
  return IE_OK;
}

int ie_ipc_release(void* ptr) {
  std::lock_guard<std::mutex> lock(g_import_mutex);
  for (int i = 0; i < g_nimports; ++i)
    if (g_imports[i].ptr == ptr) {
      const cudaError_t e = cudaIpcCloseMemHandle(g_imports[i].base);
      g_imports[i] = g_imports[--g_nimports];
      return e == cudaSuccess ? IE_OK : IE_ERR_LAUNCH;
    }
  return IE_ERR_INVALID_ARG;
}

static int gemm_allreduce(ie_dtype dt, int M, int N, int K, const void* X, int64_t ldx, const void* W, int64_t ldw,
                          void* Y, int64_t ldy, const ie_tp_exchange* ex, bool residual, void* stream) {
  if ((dt != IE_DTYPE_F16 && dt != IE_DTYPE_BF16) || M < 0 || N < 0 || K <= 0 || !ex) return IE_ERR_INVALID_ARG;
  if (ex->world < 1 || ex->world > kTpMaxWorld || ex->rank < 0 || ex->rank >= ex->world || !ex->sym)
    return IE_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return IE_OK;
  if (M > 16 || M > ex->max_rows || N > ex->max_cols) return IE_ERR_UNSUPPORTED;
  if (K % 8) return IE_ERR_ALIGNMENT;
  if (!X || !W || !Y || ldx < K || ldw < K || ldy < N) return IE_ERR_INVALID_ARG;
  if (!aligned16(X) || !aligned16(W) || (ldx % 8) || (ldw % 8)) return IE_ERR_ALIGNMENT;
  SkinnyParams p;
  p.X = X; p.ldx = ldx; p.M = M; p.N = N; p.K = K;
  p.W0 = W; p.ldw = ldw; p.Y = Y; p.ldy = ldy;
  p.tp_sym = ex->sym; p.tp_world = ex->world; p.tp_rank = ex->rank;
  p.tp_rows = ex->max_rows; p.tp_cols = ex->max_cols;
  p.residual = residual;
  return launch_skinny(dt, EPI_TP_ALLREDUCE, p, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess
             ? IE_OK
             : IE_ERR_LAUNCH;
}

int ie_gemm_allreduce(ie_dtype dt, int M, int N, int K, const void* X, int64_t ldx, const void* W, int64_t ldw,
                      void* Y, int64_t ldy, const ie_tp_exchange* ex, void* stream) {
  return gemm_allreduce(dt, M, N, K, X, ldx, W, ldw, Y, ldy, ex, false, stream);
}

int ie_gemm_allreduce_add(ie_dtype dt, int M, int N, int K, const void* X, int64_t ldx, const void* W, int64_t ldw,
                          void* Y, int64_t ldy, const ie_tp_exchange* ex, void* stream) {
  return gemm_allreduce(dt, M, N, K, X, ldx, W, ldw, Y, ldy, ex, true, stream);
}

}  // extern "C"
