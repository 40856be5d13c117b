// Parameters of the prefill-path (M > 16) tcgen05/TMEM GEMM; see gemm_tc.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "../../include/infengine_b200.h"

namespace ie {

enum TcEpilogue {
  TC_EPI_STORE = 0,   // D[m, n] = round(acc)
  TC_EPI_SWIGLU = 1,  // B = gate, B2 = up: D = round(silu(round(g)) * round(u))
  TC_EPI_ARGMAX = 2,  // logits (optional) + per-row packed-key argmax
  TC_EPI_QKV = 3,     // B/B2/B3 = Wq/Wk/Wv, head-major scatter + optional RoPE
  TC_EPI_STORE_F32 = 4,  // D (float) [m, n] = acc, unrounded (tensor-parallel partial sums)
};

// D[M, N] = A[M, K] . B[N, K]^T (A = activations, B = weights, both K-major).
struct TcGemmParams {
  const void* A = nullptr;
  int64_t lda = 0;
  const void* B = nullptr;
  const void* B2 = nullptr;
  const void* B3 = nullptr;
  int64_t ldb = 0;
  int M = 0, N = 0, K = 0;
  void* D = nullptr;
  int64_t ldd = 0;
  int epi = TC_EPI_STORE;
  // TC_EPI_STORE: D = round(D + round(acc)) (residual add after O / down)
  bool residual = false;
  // TC_EPI_ARGMAX
  int64_t vocab_offset = 0;
  unsigned long long* keys = nullptr;
  unsigned int* counter = nullptr;
  int* idx_out = nullptr;
  unsigned long long* key_out = nullptr;
  // TC_EPI_QKV
  int n_q_heads = 0, n_kv_heads = 0;
  void* q_out = nullptr;
  int64_t q_head_stride = 0;
  void* k_cache = nullptr;
  void* v_cache = nullptr;
  int64_t cache_head_stride = 0;
  int pos0 = 0;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  // batched rows of independent sequences (see SkinnyParams)
  const int* positions = nullptr;
  int64_t cache_batch_stride = 0;
  int cache_rows = 0;
  // split of the last wave's tiles along k (caller workspace, see
  // attach_split_workspace); null: whole tiles only
  unsigned int* split_flags = nullptr;
  float* split_ws = nullptr;
  long long split_slots = 0;  // partial tiles the workspace holds
};

// Returns an IE_* status.
int launch_tc_gemm(ie_dtype dt, const TcGemmParams& p, cudaStream_t st);

// Bytes of a tail-split workspace for this device (ie_split_workspace_size).
size_t split_workspace_bytes();
// Points q at a caller workspace (256-byte aligned; its flag words zeroed
// once when allocated). ws == NULL leaves q on whole tiles.
int attach_split_workspace(TcGemmParams& q, void* ws, size_t bytes);

// Device status word written by timed-out waits (IE_OK or IE_ERR_TIMEOUT).
int read_tc_status(bool clear);
// Sets this device's limit of the kernels' bounded waits (current device).
cudaError_t set_tc_wait_ns(unsigned long long ns);

}  // namespace ie
