// Drop-in for the reference's kernels/sampling.cuh:4 (kernels/sampling.cu:54-58).
#pragma once
#include <cuda_fp16.h>

// Greedy token id over VOCAB fp16 logits, with the reference's tie order.
void sample_token_amax(const half* d_logits, int* d_output);
