// Drop-in for the reference's kernels/multiply_by_weight.cuh:3 (implemented
// there in kernels/ffn.cu:7-33 with cublasGemmEx). Same signature; the
// handle only supplies the stream (cublasGetStream), no cuBLAS math is used.
#pragma once
#include <cuda_fp16.h>
#include <cublas_v2.h>

// y[m, n] = x[m, k] . W[n, k]^T, fp16 in/out, fp32 accumulate.
void multiply_by_weight(cublasHandle_t handle, const int m, const int k, const int n, const half* d_in,
                        const half* d_w, half* d_out);
