// TEST INFRASTRUCTURE — extern "C" entry points into the reference's own
// hot-path code (Aryan470/infengine kernels/*.cu, compiled unchanged from the
// reference tree by oracle/Makefile into oracle/_ref/libinfengine_ref.so).
// Used by tests/ (GPU parity against the reference) and by bench.py's
// reference arm. Nothing here is part of the product.
//
// The reference launches on the legacy default stream and gives its cuBLAS
// handle no stream (manager.cpp:58-59); ref_set_stream lets the bench put both
// on one stream so CUDA events bracket them the same way as the product path.
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdio>
#include "kernels/ffn.cuh"
#include "kernels/swiglu.cuh"
#include "kernels/lm_head.cuh"
#include "kernels/sampling.cuh"
#include "kernels/multiply_by_weight.cuh"
#include "kernels/rope.cuh"
#include "kernels/rmsnorm.cuh"
#include "kernels/residual_add.cuh"
#include "kernels/emblookup.cuh"

// non-static helpers of kernels/attn.cu:12 and :265
void multiply_kqv_proj(cublasHandle_t handle, const half* d_W, const half* d_input, half* d_out, const int seq_len,
                       const int num_heads, bool is_kv_cache);
void multiply_preproj_Wo(cublasHandle_t handle, const int seq_len, const half* d_pre_proj, const half* d_W_o,
                         half* d_output);

#define REF_API extern "C" __attribute__((visibility("default")))

static cublasHandle_t g_handle = nullptr;

static cublasHandle_t handle() {
  if (!g_handle) {
    if (cublasCreate(&g_handle) != CUBLAS_STATUS_SUCCESS) {
      std::fprintf(stderr, "ref_shim: cublasCreate failed\n");
      g_handle = nullptr;
    }
  }
  return g_handle;
}

REF_API int ref_init(void) { return handle() ? 0 : -1; }

REF_API int ref_set_stream(void* stream) {
  return cublasSetStream(handle(), reinterpret_cast<cudaStream_t>(stream)) == CUBLAS_STATUS_SUCCESS ? 0 : -1;
}

REF_API void ref_multiply_by_weight(int m, int k, int n, const void* d_in, const void* d_w, void* d_out) {
  multiply_by_weight(handle(), m, k, n, (const half*)d_in, (const half*)d_w, (half*)d_out);
}

REF_API size_t ref_ffn_workspace_size(int max_seq_len) { return ffn_workspace_size(max_seq_len); }

REF_API void ref_ffn(int seq_len, void* d_in, void* d_out, void* d_wup, void* d_wdown, void* d_wgate,
                     void* workspace) {
  ffn(handle(), seq_len, (half*)d_in, (half*)d_out, (half*)d_wup, (half*)d_wdown, (half*)d_wgate, workspace);
}

REF_API void ref_swiglu(int seq_len, void* d_gate, void* d_up, void* d_output) {
  swiglu(seq_len, (half*)d_gate, (half*)d_up, (half*)d_output);
}

REF_API void ref_lm_head(int seq_len, void* d_input, void* d_weight, void* d_output) {
  lm_head(handle(), seq_len, (half*)d_input, (half*)d_weight, (half*)d_output);
}

REF_API void ref_sample_token_amax(const void* d_logits, int* d_output) {
  sample_token_amax((const half*)d_logits, d_output);
}

// Q/K/V projection exactly as decode_attn / attn issue it (kernels/attn.cu:345-347,
// :411-415): Q into q_out [heads][S][128], K/V into the cache rows starting at k_dst / v_dst.
REF_API void ref_qkv_proj(int seq_len, const void* d_input, const void* wq, const void* wk, const void* wv,
                          void* q_out, void* k_dst, void* v_dst, int n_q_heads, int n_kv_heads) {
  multiply_kqv_proj(handle(), (const half*)wq, (const half*)d_input, (half*)q_out, seq_len, n_q_heads, false);
  multiply_kqv_proj(handle(), (const half*)wk, (const half*)d_input, (half*)k_dst, seq_len, n_kv_heads, true);
  multiply_kqv_proj(handle(), (const half*)wv, (const half*)d_input, (half*)v_dst, seq_len, n_kv_heads, true);
}

REF_API void ref_apply_rope(int start_pos, int num_heads, int seq_len, const float* cos, const float* sin,
                            void* d_inout, int is_kv_cache) {
  apply_rope(start_pos, num_heads, seq_len, cos, sin, (half*)d_inout, (half*)d_inout, is_kv_cache != 0);
}

REF_API int ref_init_rope_buffer(float** cos, float** sin) {
  init_rope_buffer(cos, sin);
  return 0;
}

REF_API void ref_o_proj(int seq_len, const void* d_pre_proj, const void* w_o, void* d_out) {
  multiply_preproj_Wo(handle(), seq_len, (const half*)d_pre_proj, (const half*)w_o, (half*)d_out);
}

// The kernels a decode step runs between the projections (decode.cu:14-44).
REF_API void ref_rmsnorm(int seq_len, void* d_input, void* d_weight, void* d_output) {
  rmsnorm(seq_len, (half*)d_input, (half*)d_weight, (half*)d_output);
}

REF_API void ref_residual_add(int rows, int cols, void* d_x, void* d_delta) {
  residual_add(rows, cols, (half*)d_x, (half*)d_delta);
}

REF_API void ref_emblookup(int seq_len, int* d_tokens, void* d_table, void* d_output) {
  emblookup(seq_len, d_tokens, (half*)d_table, (half*)d_output);
}
