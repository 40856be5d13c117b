// Drop-in for the reference's kernels/ffn.cuh:5-6 (kernels/ffn.cu:35-64).
#pragma once
#include <cuda_fp16.h>
#include <cublas_v2.h>

// Bytes of workspace ffn() needs for up to max_seq_len tokens (never less
// than the reference reserves, so existing callers keep their sizing).
size_t ffn_workspace_size(int max_seq_len);
// out = W_down . (silu(W_gate . x) * (W_up . x)); note the weight order up, down, gate.
void ffn(cublasHandle_t handle, const int seq_len, half* d_in, half* d_out, half* d_wup, half* d_wdown,
         half* d_wgate, void* workspace);
