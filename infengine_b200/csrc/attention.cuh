// Internal interface of the attention kernels (attention.cu).
#pragma once

namespace ie {

// Device status word of the attention kernels: IE_ERR_TIMEOUT when a bounded
// wait for a cache copy gave up, IE_ERR_INVALID_ARG when a query row's
// position was outside its cache. Returns the word; clears it when asked.
int read_attn_status(bool clear);

}  // namespace ie
