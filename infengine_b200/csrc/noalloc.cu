// Allocation-free lm_head + greedy argmax (ie_lm_head_argmax_noalloc).
//
// ie_lm_head_argmax needs a few hundred bytes of device scratch (one packed
// argmax key per row and a completion counter), which its caller provides as
// a workspace. Some callers have no way to provide one: code written against
// the reference's fixed signatures (lm_head / sample_token_amax carry no
// workspace argument), processes whose device memory is entirely owned by a
// pool allocator so that a raw cudaMalloc may fail, and decode loops that
// must not call cudaMalloc / cudaFree because those calls can synchronize the
// device and stall the queued work. This entry point serves them from a
// fixed-size scratch array that the library declares itself.
//
// Limits and sharing rules (also stated in include/infengine_b200.h):
//  * at most kNoAllocMaxRows rows per call; larger M is rejected with
//    IE_ERR_UNSUPPORTED;
//  * the array is a file-scope __device__ variable: every GPU that loads this
//    library holds its 768 bytes until the process exits;
//  * every call uses the same array, so two calls whose kernels overlap on the
//    GPU (different streams or host threads on one device) race; serialize
//    them on one stream. Each call clears the array on its stream before its
//    kernel, so a call never depends on what an earlier call left there;
//  * the first call on each device looks up the array's device address with
//    cudaGetSymbolAddress while that device is current; make that first call
//    before any stream capture begins.
#include <mutex>
#include "ie_common.cuh"

namespace {

constexpr int kNoAllocMaxRows = 64;
// Same size as ie_lm_head_argmax_workspace_size(kNoAllocMaxRows): 64 keys +
// the counter, rounded up to 256 bytes.
constexpr size_t kScratchBytes = 768;
static_assert((kNoAllocMaxRows * 8 + 8 + 255) / 256 * 256 == kScratchBytes, "scratch size");

__device__ __align__(256) unsigned long long g_lm_head_scratch[kScratchBytes / 8];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_lm_head_scratch on the current device. In host code
// the symbol itself is only a host-side handle, so a kernel must never be
// given &g_lm_head_scratch directly.
int scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return IE_ERR_NO_DEVICE;
  if (dev < 0 || dev >= kMaxDevices) return IE_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_lm_head_scratch);
    if (e != cudaSuccess || p == nullptr) return IE_ERR_LAUNCH;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return IE_OK;
}

}  // namespace

extern "C" int ie_lm_head_argmax_noalloc(ie_dtype dt, int M, int K, int V, int64_t vocab_offset, const void* x,
                                         int64_t ldx, const void* W, void* logits, int64_t ld_logits, int* idx_out,
                                         unsigned long long* key_out, void* stream) {
  if (M > kNoAllocMaxRows) return IE_ERR_UNSUPPORTED;
  if (M <= 0 || V <= 0) return ie_lm_head_argmax(dt, M, K, V, vocab_offset, x, ldx, W, logits, ld_logits, idx_out,
                                                 key_out, nullptr, 0, stream);
  void* scratch = nullptr;
  int s = scratch_for_current_device(&scratch);
  if (s != IE_OK) return s;
  // keys and the completion counter must start at zero
  if (cudaMemsetAsync(scratch, 0, kScratchBytes, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
    return IE_ERR_LAUNCH;
  return ie_lm_head_argmax(dt, M, K, V, vocab_offset, x, ldx, W, logits, ld_logits, idx_out, key_out, scratch,
                           kScratchBytes, stream);
}
