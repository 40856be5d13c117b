// Drop-in for the reference's kernels/swiglu.cuh:5 (kernels/swiglu.cu:8-31).
#pragma once
#include <cuda_fp16.h>

// out = silu(gate) * up over [seq_len, FFN_DIM]; out may alias gate.
void swiglu(int seq_len, half* d_gate, half* d_up, half* d_output);
