// C++ drop-in for the reference's hot-path entry points (kernels/*.cuh).
// Each function keeps the reference's signature and forwards to the C-ABI of
// libinfengine_b200.so. The reference's functions return void and report
// failures by printf at best (kernels/attn.cu:290-292); these print the
// library status to stderr instead of dropping it.
//
// Stream: the reference launches everything on the legacy default stream and
// never sets a stream on its cuBLAS handle (manager.cpp:58-59). The handle's
// stream is honoured anyway: cublasGetStream_v2 is looked up in the running
// process (the caller created the handle, so libcublas is loaded), which keeps
// this library free of a link-time cuBLAS dependency and of cuBLAS math.
#include <dlfcn.h>
#include <cstdio>
#include "../../include/infengine_b200.h"
#include "../../include/kernels/ie_llama_config.h"
#include "../../include/kernels/multiply_by_weight.cuh"
#include "../../include/kernels/ffn.cuh"
#include "../../include/kernels/swiglu.cuh"
#include "../../include/kernels/lm_head.cuh"
#include "../../include/kernels/sampling.cuh"
#include "../../include/kernels/attn.cuh"

#define IE_DROPIN_EXPORT __attribute__((visibility("default")))

namespace {

void* stream_of(cublasHandle_t handle) {
  using GetStream = int (*)(cublasHandle_t, cudaStream_t*);
  static GetStream fn = reinterpret_cast<GetStream>(dlsym(RTLD_DEFAULT, "cublasGetStream_v2"));
  cudaStream_t s = nullptr;
  if (handle && fn && fn(handle, &s) != 0) s = nullptr;
  return reinterpret_cast<void*>(s);
}

void report(int status, const char* what) {
  if (status != IE_OK) std::fprintf(stderr, "infengine_b200 %s failed: %s (%d)\n", what, ie_status_string(status), status);
}

}  // namespace

IE_DROPIN_EXPORT void multiply_by_weight(cublasHandle_t handle, const int m, const int k, const int n,
                                         const half* d_in, const half* d_w, half* d_out) {
  report(ie_gemm(IE_DTYPE_F16, m, n, k, d_in, k, d_w, k, d_out, n, stream_of(handle)), "multiply_by_weight");
}

IE_DROPIN_EXPORT size_t ffn_workspace_size(int max_seq_len) {
  // The reference reserves G and U (ffn.cu:35-37); the fused kernel needs only
  // h, but returning the larger figure keeps callers' sizing valid both ways.
  const size_t ref = 2 * (size_t)max_seq_len * ie_llama::kFfnDim * sizeof(half);
  const size_t own = ie_ffn_workspace_size(max_seq_len, ie_llama::kFfnDim);
  return ref > own ? ref : own;
}

IE_DROPIN_EXPORT void ffn(cublasHandle_t handle, const int seq_len, half* d_in, half* d_out, half* d_wup,
                          half* d_wdown, half* d_wgate, void* workspace) {
  report(ie_ffn(IE_DTYPE_F16, seq_len, ie_llama::kHiddenSize, ie_llama::kFfnDim, d_in, d_wup, d_wdown, d_wgate,
                d_out, workspace, ie_ffn_workspace_size(seq_len, ie_llama::kFfnDim), stream_of(handle)),
         "ffn");
}

IE_DROPIN_EXPORT void swiglu(int seq_len, half* d_gate, half* d_up, half* d_output) {
  report(ie_swiglu(IE_DTYPE_F16, seq_len, ie_llama::kFfnDim, d_gate, d_up, d_output, nullptr), "swiglu");
}

IE_DROPIN_EXPORT void lm_head(cublasHandle_t handle, const int seq_len, half* d_input, half* d_weight,
                              half* d_output) {
  const half* last = d_input + (size_t)(seq_len - 1) * ie_llama::kHiddenSize;
  report(ie_gemm(IE_DTYPE_F16, 1, ie_llama::kVocabSize, ie_llama::kHiddenSize, last, ie_llama::kHiddenSize,
                 d_weight, ie_llama::kHiddenSize, d_output, ie_llama::kVocabSize, stream_of(handle)),
         "lm_head");
}

IE_DROPIN_EXPORT void sample_token_amax(const half* d_logits, int* d_output) {
  report(ie_argmax(IE_DTYPE_F16, 1, ie_llama::kVocabSize, d_logits, ie_llama::kVocabSize, d_output, nullptr),
         "sample_token_amax");
}

// ------------------------------------------------------------------ attention
namespace {

constexpr int64_t kCacheHeadStride = (int64_t)ie_llama::kMaxContextLength * ie_llama::kHeadDim;
constexpr int64_t kLayerCacheElems = 2 * ie_llama::kNumKvHeads * kCacheHeadStride;

// Q/K/V (+RoPE) into the workspace and the layer's cache rows, attention core,
// O projection. Workspace: Q [32][S][128] then the attention output [S][4096].
void attention_block(cublasHandle_t handle, const float* cos, const float* sin, int S, int pos0, const half* in,
                     const half* wq, const half* wk, const half* wv, const half* wo, half* out, void* workspace,
                     void* kv_cache, int layer_idx, const char* what) {
  void* st = stream_of(handle);
  half* q = static_cast<half*>(workspace);
  half* ao = q + (size_t)S * ie_llama::kHiddenSize;
  half* k_cache = static_cast<half*>(kv_cache) + (size_t)layer_idx * kLayerCacheElems;
  half* v_cache = k_cache + ie_llama::kNumKvHeads * kCacheHeadStride;
  int s = ie_qkv(IE_DTYPE_F16, S, ie_llama::kHiddenSize, ie_llama::kNumQHeads, ie_llama::kNumKvHeads,
                 ie_llama::kHeadDim, in, wq, wk, wv, q, k_cache, v_cache, kCacheHeadStride, pos0, cos, sin, st);
  if (s == IE_OK)
    s = ie_attention(IE_DTYPE_F16, S, pos0, ie_llama::kNumQHeads, ie_llama::kNumKvHeads, ie_llama::kHeadDim, q,
                     (int64_t)S * ie_llama::kHeadDim, k_cache, v_cache, kCacheHeadStride, ao, ie_llama::kHiddenSize,
                     st);
  if (s == IE_OK)
    s = ie_gemm(IE_DTYPE_F16, S, ie_llama::kHiddenSize, ie_llama::kHiddenSize, ao, ie_llama::kHiddenSize, wo,
                ie_llama::kHiddenSize, out, ie_llama::kHiddenSize, st);
  report(s, what);
}

}  // namespace

IE_DROPIN_EXPORT size_t attn_workspace_size(int max_seq_len) {
  return 2 * (size_t)max_seq_len * ie_llama::kHiddenSize * sizeof(half);
}

IE_DROPIN_EXPORT size_t kv_cache_size() {
  return (size_t)ie_llama::kNumLayers * kLayerCacheElems * sizeof(half);
}

IE_DROPIN_EXPORT void attn(cublasHandle_t handle, const float* d_rope_cos, const float* d_rope_sin, const int seq_len,
                           half* d_input, half* d_qproj, half* d_kproj, half* d_vproj, half* d_oproj, half* d_output,
                           void* workspace, void* kv_cache, const int layer_idx) {
  attention_block(handle, d_rope_cos, d_rope_sin, seq_len, 0, d_input, d_qproj, d_kproj, d_vproj, d_oproj, d_output,
                  workspace, kv_cache, layer_idx, "attn");
}

IE_DROPIN_EXPORT void decode_attn(cublasHandle_t handle, const float* d_rope_cos, const float* d_rope_sin,
                                  const int seq_len, half* d_input, half* d_qproj, half* d_kproj, half* d_vproj,
                                  half* d_oproj, half* d_output, void* workspace, void* kv_cache,
                                  const int layer_idx) {
  attention_block(handle, d_rope_cos, d_rope_sin, 1, seq_len - 1, d_input, d_qproj, d_kproj, d_vproj, d_oproj,
                  d_output, workspace, kv_cache, layer_idx, "decode_attn");
}
