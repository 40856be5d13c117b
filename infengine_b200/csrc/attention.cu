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
#include <climits>
#include <cstdlib>
#include "ie_common.cuh"
#include "attention.cuh"

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

// ------------------------------------------------ split-KV decode attention
// Decode-time attention (a few query rows, each over its whole cache) spread
// over the GPU: one thread-block cluster of kFdCluster CTAs per (query row,
// KV head); CTA c of the cluster takes cache rows [c*len/8, (c+1)*len/8).
//  * Cache rows reach shared memory by untiled bulk copies
//    (cp.async.bulk, 64 rows = 16 KB each) through a 4-deep ring completed on
//    mbarriers, so a CTA keeps up to 64 KB of K/V in flight.
//  * The softmax keeps the reference's chain (scores rounded, scaled and
//    rounded; e = exp(t - max) summed in fp32 and stored rounded;
//    p = round(round(e) * (1/sum))): the row maximum and the sum are exact
//    cluster-wide values, exchanged through distributed shared memory in a
//    fixed rank order, so no rescaling of partial results is involved.
//  * p.V partials ([group][128] fp32 per CTA) are summed across the cluster in
//    rank order; each CTA rounds and stores 1/8 of the row's outputs.
// Results are deterministic. Every mbarrier wait is bounded (2 s): on expiry
// IE_ERR_TIMEOUT is recorded, no further copies are issued, the outstanding
// ones are waited for (bounded) before the CTA exits, and the cluster
// barriers are still passed by every CTA.
namespace ie {

__device__ int g_attn_status = 0;

namespace {

constexpr int kFdCluster = 8;
constexpr int kFdThreads = 256;
constexpr int kFdWarps = kFdThreads / 32;
constexpr int kFdRows = 64;
constexpr int kFdStages = 4;
constexpr int kFdRingBytes = kFdStages * kFdRows * 128 * 2;
constexpr unsigned long long kFdWaitNs = 2000000000ull;

struct FdParams {
  const void* q;
  int64_t q_head_stride;
  const void* kc;
  const void* vc;
  int64_t chs, cbs;
  int cache_rows;
  const int* positions;
  int pos0, rows_per_seq;
  void* out;
  int64_t ld_out;
  int cap;  // score slots per head in shared memory (>= ceil(cache_rows / 8))
};

__device__ __forceinline__ uint32_t fd_smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ bool fd_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long fd_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait; false when it gave up or another thread already did.
__device__ __forceinline__ bool fd_wait(uint32_t bar, uint32_t parity, volatile int* abort_s) {
  if (fd_try(bar, parity)) return true;
  const unsigned long long t0 = fd_now();
  while (!fd_try(bar, parity)) {
    if (*abort_s) return false;
    if (fd_now() - t0 > kFdWaitNs) {
      atomicExch(&g_attn_status, IE_ERR_TIMEOUT);
      *abort_s = 1;
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_cluster(const float* local, unsigned rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(fd_smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// Warp sum of G per-lane values, transposed on the way: at the level with
// offset 16 >> l the lanes with that bit set keep the upper half of their
// values. Lane l ends with the full sum of value l / (32 / G).
template <int G>
__device__ __forceinline__ float warp_sum_transposed(float (&s)[G], int lane) {
  float v[G];
#pragma unroll
  for (int i = 0; i < G; ++i) v[i] = s[i];
#pragma unroll
  for (int lvl = 0; (1 << lvl) < G; ++lvl) {
    const int off = 16 >> lvl, w = G >> lvl;
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < w / 2; ++i) {
      const float keep = upper ? v[i + w / 2] : v[i];
      const float send = upper ? v[i] : v[i + w / 2];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
#pragma unroll
  for (int off = 16 / G; off > 0; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
  return v[0];
}

template <typename T, int G>
__global__ void __cluster_dims__(kFdCluster, 1, 1) __launch_bounds__(kFdThreads)
    decode_attention_kernel(const FdParams p) {
  extern __shared__ __align__(128) unsigned char fd_smem[];
  __shared__ float qf[G][128];
  __shared__ float opart[G * 128];
  __shared__ float red[kFdWarps][G];
  __shared__ float cmax[G], csum[G], gmax[G], ginv[G];
  __shared__ __align__(8) unsigned long long bars[kFdStages];
  __shared__ int abort_s, fail_at;

  T* ring = reinterpret_cast<T*>(fd_smem);
  T* sc = reinterpret_cast<T*>(fd_smem + kFdRingBytes);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int hk = blockIdx.y, m = blockIdx.z;

  if (tid == 0) {
    for (int s = 0; s < kFdStages; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(fd_smem_u32(&bars[s])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_s = 0;
    fail_at = INT_MAX;
  }
  // q and the cache rows come from the previous kernel (programmatic launch)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __syncthreads();

  const int pos = p.positions ? p.positions[m] : p.pos0 + m;
  const bool bad = pos < 0 || pos >= p.cache_rows;
  if (bad && rank == 0 && tid == 0) atomicExch(&g_attn_status, IE_ERR_INVALID_ARG);
  const int len = bad ? 0 : pos + 1;
  const int j0 = (int)((int64_t)len * rank / kFdCluster);
  const int n = (int)((int64_t)len * (rank + 1) / kFdCluster) - j0;
  const int nk = (n + kFdRows - 1) / kFdRows, total = 2 * nk;
  const int64_t base = (int64_t)(m / p.rows_per_seq) * p.cbs + (int64_t)hk * p.chs;
  const T* kh = static_cast<const T*>(p.kc) + base;
  const T* vh = static_cast<const T*>(p.vc) + base;

  int issued = 0;  // thread 0 only
  auto issue = [&](int i) {
    const int slot = i % kFdStages, c = i < nk ? i : i - nk;
    const int r0 = j0 + c * kFdRows;
    const int rows = min(kFdRows, j0 + n - r0);
    const uint32_t bytes = (uint32_t)rows * 128u * sizeof(T);
    const T* src = (i < nk ? kh : vh) + (int64_t)r0 * 128;
    const uint32_t bar = fd_smem_u32(&bars[slot]);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     fd_smem_u32(ring + slot * kFdRows * 128)),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
    issued = i + 1;
  };
  if (tid == 0)
    for (int i = 0; i < min(kFdStages, total); ++i) issue(i);

  for (int i = tid; i < G * 128; i += kFdThreads) {
    const int h = i >> 7, d = i & 127;
    qf[h][d] = DT<T>::to_f(static_cast<const T*>(p.q)[(int64_t)(hk * G + h) * p.q_head_stride + (int64_t)m * 128 + d]);
  }
  __syncthreads();
  float qr[G][4];
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int d = 0; d < 4; ++d) qr[h][d] = qf[h][lane * 4 + d];

  auto wait_chunk = [&](int i) {
    if (!fd_wait(fd_smem_u32(&bars[i % kFdStages]), (uint32_t)((i / kFdStages) & 1), &abort_s))
      atomicMin(&fail_at, i);
  };
  auto next = [&](int i) {
    __syncthreads();  // every warp is done with slot i % kFdStages
    if (tid == 0 && !abort_s && i + kFdStages < total) issue(i + kFdStages);
  };

  // ---- scores: warp per cache row, lane per 4 dims
  const float scale = rsqrtf(128.0f);
  for (int i = 0; i < nk; ++i) {
    wait_chunk(i);
    const T* tile = ring + (i % kFdStages) * kFdRows * 128;
    const int r0 = i * kFdRows, rows = min(kFdRows, n - r0);
    for (int r = warp; r < rows; r += kFdWarps) {
      const uint2 raw = *reinterpret_cast<const uint2*>(tile + r * 128 + lane * 4);
      const T* e = reinterpret_cast<const T*>(&raw);
      float s[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float a = qr[h][0] * DT<T>::to_f(e[0]);
#pragma unroll
        for (int d = 1; d < 4; ++d) a = fmaf(qr[h][d], DT<T>::to_f(e[d]), a);
        s[h] = a;
      }
      const float v = warp_sum_transposed<G>(s, lane);
      if ((lane & (32 / G - 1)) == 0) {
        const int h = lane / (32 / G);
        sc[h * p.cap + r0 + r] = DT<T>::from_f(round_to<T>(round_to<T>(v) * scale));
      }
    }
    next(i);
  }

  // ---- softmax with cluster-wide max and sum
  float mx[G];
#pragma unroll
  for (int h = 0; h < G; ++h) mx[h] = -INFINITY;
  for (int j = tid; j < n; j += kFdThreads)
#pragma unroll
    for (int h = 0; h < G; ++h) mx[h] = fmaxf(mx[h], DT<T>::to_f(sc[h * p.cap + j]));
#pragma unroll
  for (int h = 0; h < G; ++h) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], off));
    if (lane == 0) red[warp][h] = mx[h];
  }
  __syncthreads();
  if (tid < G) {
    float v = -INFINITY;
    for (int w = 0; w < kFdWarps; ++w) v = fmaxf(v, red[w][tid]);
    cmax[tid] = v;
  }
  cluster_sync_all();
  if (tid < G) {
    float v = -INFINITY;
    for (unsigned r = 0; r < kFdCluster; ++r) v = fmaxf(v, ld_cluster(&cmax[tid], r));
    gmax[tid] = v;
  }
  __syncthreads();
  float sm[G];
#pragma unroll
  for (int h = 0; h < G; ++h) sm[h] = 0.f;
  for (int j = tid; j < n; j += kFdThreads)
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float e = expf(DT<T>::to_f(sc[h * p.cap + j]) - gmax[h]);
      sm[h] += e;
      sc[h * p.cap + j] = DT<T>::from_f(e);
    }
#pragma unroll
  for (int h = 0; h < G; ++h) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sm[h] += __shfl_xor_sync(0xffffffffu, sm[h], off);
  }
  __syncthreads();  // red is reused
  if (lane == 0)
#pragma unroll
    for (int h = 0; h < G; ++h) red[warp][h] = sm[h];
  __syncthreads();
  if (tid < G) {
    float v = 0.f;
    for (int w = 0; w < kFdWarps; ++w) v += red[w][tid];
    csum[tid] = v;
  }
  cluster_sync_all();
  if (tid < G) {
    float v = 0.f;
    for (unsigned r = 0; r < kFdCluster; ++r) v += ld_cluster(&csum[tid], r);
    ginv[tid] = 1.0f / v;
  }
  __syncthreads();
  for (int j = tid; j < n; j += kFdThreads)
#pragma unroll
    for (int h = 0; h < G; ++h) sc[h * p.cap + j] = DT<T>::from_f(DT<T>::to_f(sc[h * p.cap + j]) * ginv[h]);
  __syncthreads();

  // ---- p.V: warp per cache row, lane per 4 dims
  float acc[G][4];
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int d = 0; d < 4; ++d) acc[h][d] = 0.f;
  for (int i = nk; i < total; ++i) {
    wait_chunk(i);
    const T* tile = ring + (i % kFdStages) * kFdRows * 128;
    const int r0 = (i - nk) * kFdRows, rows = min(kFdRows, n - r0);
    for (int r = warp; r < rows; r += kFdWarps) {
      const uint2 raw = *reinterpret_cast<const uint2*>(tile + r * 128 + lane * 4);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float pw = DT<T>::to_f(sc[h * p.cap + r0 + r]);
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[h][d] = fmaf(pw, DT<T>::to_f(e[d]), acc[h][d]);
      }
    }
    next(i);
  }
  // copies a failed wait left in flight finish before the ring is reused
  if (tid == 0 && fail_at < issued) {
    for (int i = fail_at; i < issued; ++i) {
      const unsigned long long t0 = fd_now();
      while (!fd_try(fd_smem_u32(&bars[i % kFdStages]), (uint32_t)((i / kFdStages) & 1)) &&
             fd_now() - t0 < kFdWaitNs) {
      }
    }
  }
  __syncthreads();

  // ---- CTA partial (warps summed in order), then the cluster sum in rank order
  float* part = reinterpret_cast<float*>(fd_smem);  // [warps][G][128], over the drained ring
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int d = 0; d < 4; ++d) part[(warp * G + h) * 128 + lane * 4 + d] = acc[h][d];
  __syncthreads();
  for (int e = tid; e < G * 128; e += kFdThreads) {
    float s = 0.f;
    for (int w = 0; w < kFdWarps; ++w) s += part[w * G * 128 + e];
    opart[e] = s;
  }
  cluster_sync_all();
  constexpr int kPer = G * 128 / kFdCluster;
  if (tid < kPer) {
    const int e = (int)rank * kPer + tid;
    float s = 0.f;
    for (unsigned r = 0; r < kFdCluster; ++r) s += ld_cluster(&opart[e], r);
    const int h = e >> 7, d = e & 127;
    static_cast<T*>(p.out)[(int64_t)m * p.ld_out + (int64_t)(hk * G + h) * 128 + d] = DT<T>::from_f(s);
  }
  cluster_sync_all();  // remote reads of opart are done before any CTA exits
}

template <typename T, int G>
cudaError_t launch_decode_attention(const FdParams& p, int n_kv_heads, int R, cudaStream_t st) {
  auto kernel = decode_attention_kernel<T, G>;
  const size_t smem = kFdRingBytes + (size_t)G * p.cap * sizeof(T);
  static size_t configured[64] = {};  // per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kFdCluster, n_kv_heads, R);
  cfg.blockDim = dim3(kFdThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  const char* env = getenv("IE_PDL");
  cfg.numAttrs = (env && env[0] == '0') ? 0 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

}  // namespace

int read_attn_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_status, sizeof(int)) != cudaSuccess) return IE_ERR_LAUNCH;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_attn_status, &z, sizeof(int));
  }
  return v;
}

}  // namespace ie

extern "C" int ie_attention_decode(ie_dtype dt, int R, int rows_per_seq, int n_q_heads, int n_kv_heads,
                                   int head_dim, const void* q, int64_t q_head_stride, const void* k_cache,
                                   const void* v_cache, int64_t cache_head_stride, int64_t cache_batch_stride,
                                   int cache_rows, const int* positions, int pos0, void* out, int64_t ld_out,
                                   void* stream) {
  using namespace ie;
  if ((dt != IE_DTYPE_F16 && dt != IE_DTYPE_BF16) || R < 0 || rows_per_seq <= 0 || n_kv_heads <= 0 ||
      n_q_heads <= 0 || cache_rows <= 0 || pos0 < 0)
    return IE_ERR_INVALID_ARG;
  if (head_dim != 128 || n_q_heads % n_kv_heads) return IE_ERR_UNSUPPORTED;
  const int group = n_q_heads / n_kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8) return IE_ERR_UNSUPPORTED;
  if (R == 0) return IE_OK;
  if (!q || !k_cache || !v_cache || !out) return IE_ERR_INVALID_ARG;
  if (R % rows_per_seq || R > 65535 || n_kv_heads > 65535) return IE_ERR_INVALID_ARG;
  if (!aligned16(k_cache) || !aligned16(v_cache) || (cache_head_stride % 8) || (cache_batch_stride % 8))
    return IE_ERR_ALIGNMENT;
  if (ld_out < (int64_t)n_q_heads * 128 || q_head_stride < (int64_t)R * 128) return IE_ERR_INVALID_ARG;
  if (cache_head_stride < (int64_t)cache_rows * 128) return IE_ERR_INVALID_ARG;
  if (R / rows_per_seq > 1 && cache_batch_stride < (int64_t)n_kv_heads * cache_head_stride) return IE_ERR_INVALID_ARG;
  if (!positions && pos0 + R > cache_rows) return IE_ERR_INVALID_ARG;
  FdParams p;
  p.q = q;
  p.q_head_stride = q_head_stride;
  p.kc = k_cache;
  p.vc = v_cache;
  p.chs = cache_head_stride;
  p.cbs = cache_batch_stride;
  p.cache_rows = cache_rows;
  p.positions = positions;
  p.pos0 = pos0;
  p.rows_per_seq = rows_per_seq;
  p.out = out;
  p.ld_out = ld_out;
  p.cap = ((cache_rows + kFdCluster - 1) / kFdCluster + 7) / 8 * 8;
  if (kFdRingBytes + (size_t)group * p.cap * 2 > 200 * 1024) return IE_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
#define IE_FD(T)                                                                   \
  switch (group) {                                                                 \
    case 1: e = launch_decode_attention<T, 1>(p, n_kv_heads, R, st); break;        \
    case 2: e = launch_decode_attention<T, 2>(p, n_kv_heads, R, st); break;        \
    case 4: e = launch_decode_attention<T, 4>(p, n_kv_heads, R, st); break;        \
    default: e = launch_decode_attention<T, 8>(p, n_kv_heads, R, st); break;       \
  }
  if (dt == IE_DTYPE_F16) { IE_FD(__half) }
  else { IE_FD(__nv_bfloat16) }
#undef IE_FD
  return e == cudaSuccess ? IE_OK : IE_ERR_LAUNCH;
}
