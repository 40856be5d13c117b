// Shared device helpers for the infengine_b200 kernels (sm_100a only).
#pragma once
#include <cstdlib>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include "../../include/infengine_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "infengine_b200 kernels are written for sm_100a only"
#endif

namespace ie {

// ---------------------------------------------------------------- dtypes
template <typename T> struct DT;
template <> struct DT<__half> {
  static constexpr ie_dtype id = IE_DTYPE_F16;
  __device__ static __forceinline__ float to_f(__half v) { return __half2float(v); }
  __device__ static __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct DT<__nv_bfloat16> {
  static constexpr ie_dtype id = IE_DTYPE_BF16;
  __device__ static __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ static __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// Round an fp32 value to the storage type and back (the value a reader of
// the stored tensor would see).
template <typename T>
__device__ __forceinline__ float round_to(float v) { return DT<T>::to_f(DT<T>::from_f(v)); }

// --------------------------------------------------------------- loads
// Weights are read exactly once per call: bypass L1 and mark the L2 lines
// evict-first so activations and partial results stay resident.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p, uint64_t policy) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "l"(policy));
  return r;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// Activations are re-read by every CTA: keep them in L1.
__device__ __forceinline__ uint4 ld_act_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// ----------------------------------------------------- argmax key packing
// A 64-bit key whose unsigned maximum is the reference's argmax winner.
// amax_kern (kernels/sampling.cu:28-51) gives thread t = id mod 1024 the ids
// t, t+1024, ... (strict '>' keeps the first, i.e. smallest, id of a class),
// and reduce_amax (:8-25) halves the thread range each level keeping the lower
// slot on ties, so the last level (delta=1) decides on bit 0 of t, the one
// before on bit 1, ...: among equal logits the class whose 10-bit reversed t
// is smallest wins, then the smallest id within the class.
// high word = order-preserving image of the (rounded) logit, +0 and -0 equal;
// low word  = ~(bitrev10(id mod 1024) << 21 | id / 1024). NaN maps to key 0.
__device__ __forceinline__ unsigned long long argmax_key(float v, long long id) {
  if (v != v) return 0ull;
  if (v == 0.0f) v = 0.0f;
  uint32_t b = __float_as_uint(v);
  uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  uint32_t r = __brev((uint32_t)(id & 1023)) >> 22, q = (uint32_t)(id >> 10);
  uint32_t tie = (r << 21) | q;
  return ((unsigned long long)ord << 32) | (unsigned long long)(~tie);
}

__device__ __forceinline__ int argmax_key_index(unsigned long long key) {
  uint32_t tie = ~(uint32_t)(key & 0xffffffffull);
  return (int)((tie & ((1u << 21) - 1u)) * 1024u + (__brev(tie >> 21) >> 22));
}

// ------------------------------------------------------------- waits
// Limit of a device-side wait on another party (a TMA copy, an MMA, a peer
// rank's data): 2 s unless ie_set_wait_limit_ns changes it. On expiry the
// kernel records IE_ERR_TIMEOUT and returns. Waits for work the kernel itself
// issued, when it leaves early (copies and MMAs in flight), keep the fixed
// kDrainWaitNs: they always end, and cutting them short would let a CTA exit
// with copies still landing in its shared memory.
constexpr unsigned long long kDefaultWaitNs = 2000000000ull;
constexpr unsigned long long kDrainWaitNs = 2000000000ull;
constexpr unsigned long long kMaxWaitNs = 60000000000ull;  // largest settable limit: 60 s

// ------------------------------------------------------- launch ordering
// Programmatic dependent launch (a kernel's CTAs may start while its
// predecessor drains) for the decode-path kernels: on for launches of at most
// pdl_max_rows() activation rows (IE_PDL_MAX_ROWS in the environment), off
// above. Measured on the decode engine (one B200): with PDL everywhere a
// batch-1 step takes 3.31 ms and a batch-8 step 4.59 ms; without PDL for the
// attention / the GEMVs / RMSNorm alone, batch 1 takes 3.45 / 3.38 / 3.30 ms
// and batch 8 4.37 / 4.21 / 4.17 ms. With the limit at 5 rows: batch 8 2046
// tok/s (1834 with PDL everywhere), the 5-row verify pass 3.84 ms (3.99 with
// the limit at 2), batch 1 unchanged. It changes no result. IE_PDL=0 turns it
// off everywhere.
constexpr int kPdlMaxRows = 5;
inline int pdl_max_rows() {
  static const int v = [] {
    const char* e = getenv("IE_PDL_MAX_ROWS");
    return e ? atoi(e) : kPdlMaxRows;
  }();
  return v;
}

// ------------------------------------------------------------- misc
__host__ __device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace ie
