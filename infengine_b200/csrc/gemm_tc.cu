// Prefill-path GEMM (M > 16): tcgen05 / TMEM / TMA kernel.
#include "ie_common.cuh"
#include "gemm_tc.cuh"

namespace ie {

int launch_tc_gemm(ie_dtype, const TcGemmParams&, cudaStream_t) { return IE_ERR_UNSUPPORTED; }

}  // namespace ie
