// Drop-in for the reference's kernels/attn.cuh:5-8 (kernels/attn.cu:295-439):
// the attention entry points, whose Q/K/V and O projections run on this
// library's kernels (fused QKV + RoPE, O GEMM) around its attention core.
#pragma once
#include <cuda_fp16.h>
#include <cublas_v2.h>

// Workspace bytes attn / decode_attn need for up to max_seq_len tokens
// (Q [32][S][128] and the attention output [S][4096]).
size_t attn_workspace_size(int max_seq_len);
// KV cache bytes: [layers][2][kv_heads][MAX_CONTEXT_LENGTH][head_dim] fp16,
// the reference's layout (kernels/attn.cu:304-307).
size_t kv_cache_size();
// Prefill: seq_len tokens of d_input [seq_len, 4096] at positions 0..seq_len-1.
void attn(cublasHandle_t handle, const float* d_rope_cos, const float* d_rope_sin, const int seq_len, half* d_input,
          half* d_qproj, half* d_kproj, half* d_vproj, half* d_oproj, half* d_output, void* workspace,
          void* kv_cache, const int layer_idx);
// Decode: one token d_input [1, 4096] at position seq_len-1.
void decode_attn(cublasHandle_t handle, const float* d_rope_cos, const float* d_rope_sin, const int seq_len,
                 half* d_input, half* d_qproj, half* d_kproj, half* d_vproj, half* d_oproj, half* d_output,
                 void* workspace, void* kv_cache, const int layer_idx);
