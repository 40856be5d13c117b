// Internal interface of the attention kernels (attention.cu).
#pragma once

namespace ie {

// Device status word of the attention kernels: IE_ERR_TIMEOUT when a bounded
// wait for a cache copy gave up, IE_ERR_INVALID_ARG when a query row's
// position was outside its cache. Returns the word; clears it when asked.
int read_attn_status(bool clear);
// Sets this device's limit of the kernels' bounded waits (current device).
cudaError_t set_attn_wait_ns(unsigned long long ns);

// Causal prefill attention on tcgen05 (attention_tc.cu), head_dim 128; the
// arguments are ie_attention's after its checks. Returns an ie_status.
int launch_tc_attention(ie_dtype dt, int S, int pos0, int n_q_heads, int n_kv_heads, const void* q,
                        int64_t q_head_stride, const void* k_cache, const void* v_cache, int64_t cache_head_stride,
                        void* out, int64_t ld_out, void* stream);
// Status word of that kernel (IE_ERR_TIMEOUT when a bounded wait gave up).
int read_tca_status(bool clear);
// Sets this device's limit of the kernels' bounded waits (current device).
cudaError_t set_tca_wait_ns(unsigned long long ns);

}  // namespace ie
