// Drop-in for the reference's kernels/lm_head.cuh:4 (kernels/lm_head.cu:5-20).
#pragma once
#include <cuda_fp16.h>
#include <cublas_v2.h>

// fp16 logits [1, VOCAB] of the last row (seq_len - 1) of d_input.
void lm_head(cublasHandle_t handle, const int seq_len, half* d_input, half* d_weight, half* d_output);
