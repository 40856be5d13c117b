// Internal interface of norm.cu (RMSNorm, embedding, decode-step bookkeeping).
#pragma once
#include <cuda_runtime.h>

namespace ie {

// Programmatic dependent launch on (IE_PDL unset or not "0").
bool pdl_launch_enabled();

// history[step % slots][b] = tokens[b]; positions[b] += 1; *step += 1.
cudaError_t launch_advance(int B, const int* tokens, int* positions, int* history, int slots, int* step,
                           cudaStream_t st);

// Device status word of the embedding lookup (IE_ERR_INVALID_ARG for a token
// outside the vocabulary).
int read_norm_status(bool clear);

}  // namespace ie
