// Parameters of the decode-path (M <= 16) kernels; see skinny.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "../../include/infengine_b200.h"

namespace ie {

enum SkinnyEpilogue {
  EPI_STORE = 0,   // Y[m, n] = round(acc)
  EPI_SWIGLU = 1,  // two matrices (gate = W0, up = W1): Y = round(silu(round(g)) * round(u))
  EPI_ARGMAX = 2,  // logits (optional store) + packed-key argmax per batch row
  EPI_QKV = 3,     // head-major scatter of Q / K-cache / V-cache rows, optional RoPE
  EPI_STORE_F32 = 4,  // Y (float) [m, n] = acc, unrounded (tensor-parallel partial sums)
  EPI_TP_ALLREDUCE = 5,  // partial rows pushed to every rank's inbox over NVLink; the last CTA
                         // sums all ranks' partials (rank order) into Y (dt)
};

// Layout of one rank's exchange buffer (ie_gemm_allreduce): a 256-byte
// header (call counter, CTA completion counter), then 2 x world inbox slots of
// tp_rows x tp_cols 64-bit words (fp32 value | call epoch << 32),
// double-buffered by call parity.
struct TpHeader {
  unsigned int epoch;
  unsigned int done;
};
constexpr size_t kTpInboxOffset = 1024;
constexpr int kTpMaxWorld = 8;

struct SkinnyParams {
  const void* X = nullptr;
  int64_t ldx = 0;
  int M = 0, N = 0, K = 0;
  const void* W0 = nullptr;
  const void* W1 = nullptr;
  const void* W2 = nullptr;
  int64_t ldw = 0;
  // set by launch_skinny: all weight / activation rows 32-byte aligned; tile count
  bool w_wide = false, x_wide = false;
  // set by launch_skinny: first weight batch requested before the
  // programmatic-launch wait (few activation rows)
  bool early_w = false;
  int tiles = 0;
  // set by launch_skinny: CTAs (one cluster) that split the K range of a tile
  int ksplit = 1;
  void* Y = nullptr;
  int64_t ldy = 0;
  // EPI_STORE / EPI_TP_ALLREDUCE: Y = round(Y + round(result)), the residual
  // add that follows the O and down projections
  bool residual = false;
  // EPI_ARGMAX
  int64_t vocab_offset = 0;
  unsigned long long* keys = nullptr;
  unsigned int* counter = nullptr;
  int* idx_out = nullptr;
  unsigned long long* key_out = nullptr;
  // EPI_QKV
  int n_q_heads = 0, n_kv_heads = 0;
  void* q_out = nullptr;
  int64_t q_head_stride = 0;
  void* k_cache = nullptr;
  void* v_cache = nullptr;
  int64_t cache_head_stride = 0;
  int pos0 = 0;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  // batched decode of independent sequences: row m at position positions[m]
  // of its own cache (offset m * cache_batch_stride); positions outside
  // [0, cache_rows) are skipped and reported through the device status
  const int* positions = nullptr;
  int64_t cache_batch_stride = 0;
  int cache_rows = 0;
  // EPI_TP_ALLREDUCE: device array [tp_world] of every rank's symmetric
  // buffer as mapped in this process (own buffer at tp_rank)
  void* const* tp_sym = nullptr;
  int tp_world = 0, tp_rank = 0, tp_rows = 0, tp_cols = 0;
};

cudaError_t launch_skinny(ie_dtype dt, int epi, const SkinnyParams& p, cudaStream_t st);
cudaError_t launch_swiglu(ie_dtype dt, int64_t n, const void* gate, const void* up, void* out, cudaStream_t st);
// Device status word of the decode kernels (IE_OK, IE_ERR_TIMEOUT from the
// tensor-parallel exchange, IE_ERR_INVALID_ARG from a batched QKV position).
int read_skinny_status(bool clear);
// Sets this device's limit of the kernels' bounded waits (current device).
cudaError_t set_skinny_wait_ns(unsigned long long ns);
cudaError_t launch_argmax(ie_dtype dt, int M, int V, const void* logits, int64_t ld, int* idx_out, cudaStream_t st);

}  // namespace ie
