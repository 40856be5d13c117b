// Attention core behind the drop-in attn / decode_attn entry points.
//
// Not a weight matmul: it exists so that the reference's attention entry
// points (kernels/attn.cuh:5-8), whose translation unit also holds the Q/K/V
// and O projections, can be served by this library. It reads Q written
// head-major by ie_qkv and the K/V cache rows, and writes the token-major
// [S, n_q_heads * 128] output the O projection consumes (the layout the
// reference produces with attn_permute, kernels/attn_permute.cu:15-32).
//
// Numerics follow the reference's chain (kernels/attn.cu:355-366,
// kernels/softmax.cu:55-160): a score is one fp32 dot product rounded to the
// storage type (the cuBLAS QK^T output), scaled by rsqrt(128) and rounded
// again; the row maximum is taken over those values; e = exp(t - max) is
// summed in fp32 and stored rounded; p = round(round(e) / sum); the output is
// one fp32 accumulation of p * V rounded once (the cuBLAS A.V output).
//
// One CTA per (KV head, query row) serves the n_q_heads / n_kv_heads query
// heads that share the KV head (grouped-query attention reads K and V once
// for all of them). Causal: query row s at position pos0 + s attends to
// positions 0 .. pos0 + s. Scores of a row live in shared memory (up to
// group * (pos0 + S) floats).
#include "ie_common.cuh"

namespace ie {
namespace {

constexpr int kAttnThreads = 256;
constexpr int kMaxGroup = 8;

template <typename T>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const T* __restrict__ q, int64_t q_head_stride,
                                                                  const T* __restrict__ kc,
                                                                  const T* __restrict__ vc, int64_t chs, int pos0,
                                                                  int group, T* __restrict__ out, int64_t ld_out) {
  extern __shared__ float sm[];
  const int hk = blockIdx.x, s = blockIdx.y;
  const int len = pos0 + s + 1;
  float* qs = sm;                      // [group][128]
  float* sc = sm + group * 128;        // [group][len]
  __shared__ float red[kAttnThreads / 32][kMaxGroup];
  __shared__ float stat[2][kMaxGroup];  // max, 1/sum
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  for (int i = tid; i < group * 128; i += kAttnThreads) {
    const int h = i >> 7, d = i & 127;
    qs[i] = DT<T>::to_f(q[(int64_t)(hk * group + h) * q_head_stride + (int64_t)s * 128 + d]);
  }
  __syncthreads();
  const float scale = rsqrtf(128.0f);
  const T* kh = kc + (int64_t)hk * chs;
  const T* vh = vc + (int64_t)hk * chs;

  // scores and per-thread maxima
  float mx[kMaxGroup];
#pragma unroll
  for (int h = 0; h < kMaxGroup; ++h) mx[h] = -INFINITY;
  for (int j = tid; j < len; j += kAttnThreads) {
    float acc[kMaxGroup];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) acc[h] = 0.f;
    const uint4* kr = reinterpret_cast<const uint4*>(kh + (int64_t)j * 128);
#pragma unroll 4
    for (int c = 0; c < 16; ++c) {
      const uint4 raw = kr[c];
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float kv = DT<T>::to_f(e[i]);
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h)
          if (h < group) acc[h] = fmaf(qs[h * 128 + c * 8 + i], kv, acc[h]);
      }
    }
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
      if (h < group) {
        const float t = round_to<T>(round_to<T>(acc[h]) * scale);
        sc[h * len + j] = t;
        mx[h] = fmaxf(mx[h], t);
      }
  }
  // row maxima
#pragma unroll
  for (int h = 0; h < kMaxGroup; ++h) {
    float v = mx[h];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[warp][h] = v;
  }
  __syncthreads();
  if (tid < group) {
    float v = -INFINITY;
    for (int w = 0; w < kAttnThreads / 32; ++w) v = fmaxf(v, red[w][tid]);
    stat[0][tid] = v;
  }
  __syncthreads();
  // exponentials (stored rounded) and their fp32 sum
  float sum[kMaxGroup];
#pragma unroll
  for (int h = 0; h < kMaxGroup; ++h) sum[h] = 0.f;
  for (int j = tid; j < len; j += kAttnThreads) {
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
      if (h < group) {
        const float e = expf(sc[h * len + j] - stat[0][h]);
        sum[h] += e;
        sc[h * len + j] = round_to<T>(e);
      }
  }
#pragma unroll
  for (int h = 0; h < kMaxGroup; ++h) {
    float v = sum[h];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp][h] = v;
  }
  __syncthreads();
  if (tid < group) {
    float v = 0.f;
    for (int w = 0; w < kAttnThreads / 32; ++w) v += red[w][tid];
    stat[1][tid] = 1.0f / v;
  }
  __syncthreads();
  for (int j = tid; j < len; j += kAttnThreads)
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
      if (h < group) sc[h * len + j] = round_to<T>(sc[h * len + j] * stat[1][h]);
  __syncthreads();

  // out[h][d] = sum_j p[h][j] * V[j][d]: two halves of the block take even /
  // odd j, 128 threads each cover d; halves are combined in a fixed order
  const int half = tid >> 7, d = tid & 127;
  float o[kMaxGroup];
#pragma unroll
  for (int h = 0; h < kMaxGroup; ++h) o[h] = 0.f;
  for (int j = half; j < len; j += 2) {
    const float v = DT<T>::to_f(vh[(int64_t)j * 128 + d]);
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
      if (h < group) o[h] = fmaf(sc[h * len + j], v, o[h]);
  }
  __syncthreads();
  float* comb = sm;  // reuse q area: [group][128] from the odd half
  if (half == 1)
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
      if (h < group) comb[h * 128 + d] = o[h];
  __syncthreads();
  if (half == 0) {
    T* orow = out + (int64_t)s * ld_out + (int64_t)hk * group * 128;
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
      if (h < group) orow[h * 128 + d] = DT<T>::from_f(o[h] + comb[h * 128 + d]);
  }
}

}  // namespace
}  // namespace ie

extern "C" int ie_attention(ie_dtype dt, int S, int pos0, int n_q_heads, int n_kv_heads, int head_dim, const void* q,
                            int64_t q_head_stride, const void* k_cache, const void* v_cache,
                            int64_t cache_head_stride, void* out, int64_t ld_out, void* stream) {
  using namespace ie;
  if ((dt != IE_DTYPE_F16 && dt != IE_DTYPE_BF16) || S < 0 || pos0 < 0 || n_kv_heads <= 0 || n_q_heads <= 0)
    return IE_ERR_INVALID_ARG;
  if (head_dim != 128 || n_q_heads % n_kv_heads || n_q_heads / n_kv_heads > kMaxGroup) return IE_ERR_UNSUPPORTED;
  if (S == 0) return IE_OK;
  if (!q || !k_cache || !v_cache || !out) return IE_ERR_INVALID_ARG;
  if (!aligned16(k_cache) || !aligned16(v_cache) || (cache_head_stride % 8)) return IE_ERR_ALIGNMENT;
  if (ld_out < (int64_t)n_q_heads * 128 || q_head_stride < (int64_t)S * 128) return IE_ERR_INVALID_ARG;
  if (cache_head_stride < (int64_t)(pos0 + S) * 128) return IE_ERR_INVALID_ARG;
  const int group = n_q_heads / n_kv_heads;
  const size_t smem = (size_t)group * (128 + (size_t)(pos0 + S)) * sizeof(float);
  if (smem > 200 * 1024) return IE_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid(n_kv_heads, S);
  cudaError_t e;
  if (dt == IE_DTYPE_F16) {
    auto k = attention_kernel<__half>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    k<<<grid, kAttnThreads, smem, st>>>(static_cast<const __half*>(q), q_head_stride,
                                        static_cast<const __half*>(k_cache), static_cast<const __half*>(v_cache),
                                        cache_head_stride, pos0, group, static_cast<__half*>(out), ld_out);
  } else {
    auto k = attention_kernel<__nv_bfloat16>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    k<<<grid, kAttnThreads, smem, st>>>(static_cast<const __nv_bfloat16*>(q), q_head_stride,
                                        static_cast<const __nv_bfloat16*>(k_cache),
                                        static_cast<const __nv_bfloat16*>(v_cache), cache_head_stride, pos0, group,
                                        static_cast<__nv_bfloat16*>(out), ld_out);
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? IE_OK : IE_ERR_LAUNCH;
}
