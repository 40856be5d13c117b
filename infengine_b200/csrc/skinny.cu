// Decode-path kernels (M <= 16 activation rows): weight-streaming skinny GEMM
// with fused epilogues, standalone SwiGLU and the cluster argmax.
//
// Roofline: every kernel here is HBM-bound. One call reads each weight byte
// exactly once (N*K*2 bytes) plus M*K*2 activation bytes and writes M*N*2
// output bytes; that is the "algorithmic bytes" figure the bench divides by
// the measured duration.
//
// Skinny GEMM design (one CTA = 16 weight rows, 8 warps split K):
//  * each lane streams 16-byte chunks of two weight rows (g, g+8) with
//    L1-bypassing, L2-evict-first loads, four 32-element k-steps per batch so
//    every warp keeps 4-8 KB of weights in flight;
//  * the dot products run on the tensor cores through m16n8k16: the weight
//    tile is the A operand (16 rows) and the activation rows are the B
//    operand (n = 8 batch rows; two n-tiles for M <= 16). The 8 elements a
//    lane loads from one row are assigned to MMA k-slots so that A and B use
//    the same permutation of k, so no shuffles or shared-memory staging are
//    needed to build fragments;
//  * per-warp fp32 partials are summed across the 8 warps in shared memory in
//    a fixed order (deterministic results), then one warp runs the epilogue.
#include "ie_common.cuh"
#include "skinny.cuh"

namespace ie {

namespace {

template <typename T> struct Mma;
template <> struct Mma<__half> {
  __device__ static __forceinline__ void run(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};
template <> struct Mma<__nv_bfloat16> {
  __device__ static __forceinline__ void run(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kUnroll = 4;  // 32-element k-steps whose loads are issued together

template <int EPI> struct EpiTraits { static constexpr int nmat = 1; };
template <> struct EpiTraits<EPI_SWIGLU> { static constexpr int nmat = 2; };

// Weight row pointer of local row lr (0..15) of tile `tile`, matrix `mat`.
template <typename T, int EPI>
__device__ __forceinline__ const T* weight_row(const SkinnyParams& p, int tile, int lr, int mat,
                                               bool& valid, int& n_out) {
  if constexpr (EPI == EPI_QKV) {
    // 8 tiles per 128-wide head; rows lr and lr+8 are the RoPE pair (d, d+64).
    const int head = tile >> 3;
    const int d = ((tile & 7) << 3) + (lr & 7) + ((lr >> 3) << 6);
    n_out = head * 128 + d;
    valid = true;
    const T* base;
    int hl;
    if (head < p.n_q_heads) { base = static_cast<const T*>(p.W0); hl = head; }
    else if (head < p.n_q_heads + p.n_kv_heads) { base = static_cast<const T*>(p.W1); hl = head - p.n_q_heads; }
    else { base = static_cast<const T*>(p.W2); hl = head - p.n_q_heads - p.n_kv_heads; }
    return base + (int64_t)(hl * 128 + d) * p.ldw;
  } else {
    const int n = tile * 16 + lr;
    n_out = n;
    valid = n < p.N;
    const T* base = static_cast<const T*>(mat == 0 ? p.W0 : p.W1);
    return base + (int64_t)(valid ? n : 0) * p.ldw;
  }
}

template <typename T, int MT, int EPI>
__global__ void __launch_bounds__(kThreads) skinny_kernel(const SkinnyParams p) {
  constexpr int NMAT = EpiTraits<EPI>::nmat;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int tile = blockIdx.x;

  const T* wrow[NMAT][2];
  bool rvalid[2];
  int nidx[2];
#pragma unroll
  for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
    for (int r = 0; r < 2; ++r) wrow[mat][r] = weight_row<T, EPI>(p, tile, g + 8 * r, mat, rvalid[r], nidx[r]);

  const T* xrow[MT];
  bool xvalid[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int m = mt * 8 + g;
    xvalid[mt] = m < p.M;
    xrow[mt] = static_cast<const T*>(p.X) + (int64_t)(xvalid[mt] ? m : 0) * p.ldx;
  }

  const int nsteps = (p.K + 31) >> 5;
  const int s_begin = (warp * nsteps) / kWarps;
  const int s_end = ((warp + 1) * nsteps) / kWarps;

  float acc[NMAT][MT][4];
#pragma unroll
  for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mat][mt][i] = 0.f;

  const uint64_t pol = policy_evict_first();
  const uint4 zero = make_uint4(0, 0, 0, 0);

  for (int s = s_begin; s < s_end; s += kUnroll) {
    uint4 wv[kUnroll][NMAT][2];
    uint4 xv[kUnroll][MT];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int k = (s + u) * 32 + t * 8;
      const bool kv = (s + u < s_end) && (k < p.K);
#pragma unroll
      for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
        for (int r = 0; r < 2; ++r)
          wv[u][mat][r] = (kv && rvalid[r]) ? ld_stream_v4(wrow[mat][r] + k, pol) : zero;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) xv[u][mt] = (kv && xvalid[mt]) ? ld_act_v4(xrow[mt] + k) : zero;
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
#pragma unroll
      for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          // lane's 8 elements e0..e7 of rows g / g+8 / batch row g:
          //   MMA 0 k-slots (2t,2t+1) <- e0,e1 ; (2t+8,2t+9) <- e2,e3
          //   MMA 1 k-slots (2t,2t+1) <- e4,e5 ; (2t+8,2t+9) <- e6,e7
          Mma<T>::run(acc[mat][mt], wv[u][mat][0].x, wv[u][mat][1].x, wv[u][mat][0].y, wv[u][mat][1].y,
                      xv[u][mt].x, xv[u][mt].y);
          Mma<T>::run(acc[mat][mt], wv[u][mat][0].z, wv[u][mat][1].z, wv[u][mat][0].w, wv[u][mat][1].w,
                      xv[u][mt].z, xv[u][mt].w);
        }
  }

  // ---- cross-warp reduction (fixed order) ----
  constexpr int NR = NMAT * MT * 4;
  __shared__ float red[kWarps][NR][32];
#pragma unroll
  for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[warp][(mat * MT + mt) * 4 + i][lane] = acc[mat][mt][i];
  __syncthreads();
  if (warp != 0) return;
#pragma unroll
  for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) s += red[w][(mat * MT + mt) * 4 + i][lane];
        acc[mat][mt][i] = s;
      }

  // ---- epilogues. acc[.][mt][i]: row (g + 8*(i>>1)), batch m = mt*8 + 2t + (i&1)
  if constexpr (EPI == EPI_STORE) {
    T* Y = static_cast<T*>(p.Y);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = i >> 1, m = mt * 8 + 2 * t + (i & 1);
        if (rvalid[r] && m < p.M) Y[(int64_t)m * p.ldy + nidx[r]] = DT<T>::from_f(acc[0][mt][i]);
      }
  } else if constexpr (EPI == EPI_SWIGLU) {
    T* Y = static_cast<T*>(p.Y);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = i >> 1, m = mt * 8 + 2 * t + (i & 1);
        const float gv = round_to<T>(acc[0][mt][i]);
        const float uv = round_to<T>(acc[1][mt][i]);
        const float h = gv * (1.0f / (1.0f + expf(-gv))) * uv;
        if (rvalid[r] && m < p.M) Y[(int64_t)m * p.ldy + nidx[r]] = DT<T>::from_f(h);
      }
  } else if constexpr (EPI == EPI_ARGMAX) {
    T* Y = static_cast<T*>(p.Y);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      unsigned long long best[2] = {0ull, 0ull};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = i >> 1, m = mt * 8 + 2 * t + (i & 1);
        const T lv = DT<T>::from_f(acc[0][mt][i]);
        if (rvalid[r] && m < p.M) {
          if (Y) Y[(int64_t)m * p.ldy + nidx[r]] = lv;
          const unsigned long long key = argmax_key(DT<T>::to_f(lv), p.vocab_offset + nidx[r]);
          best[i & 1] = key > best[i & 1] ? key : best[i & 1];
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          const unsigned long long o = __shfl_xor_sync(0xffffffffu, best[j], off);
          best[j] = o > best[j] ? o : best[j];
        }
        const int m = mt * 8 + 2 * t + j;
        if (g == 0 && m < p.M && best[j] != 0ull) atomicMax(p.keys + m, best[j]);
      }
    }
    __threadfence();
    unsigned int last = 0;
    if (lane == 0) last = (atomicAdd(p.counter, 1u) == gridDim.x - 1) ? 1u : 0u;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence();
      for (int m = lane; m < p.M; m += 32) {
        const unsigned long long k = atomicExch(p.keys + m, 0ull);
        if (p.idx_out) p.idx_out[m] = argmax_key_index(k);
        if (p.key_out) p.key_out[m] = k;
      }
      if (lane == 0) atomicExch(p.counter, 0u);
    }
  } else if constexpr (EPI == EPI_QKV) {
    const int head = tile >> 3;
    const int d = ((tile & 7) << 3) + g;  // rows g -> d, g+8 -> d+64
    const bool rope = p.rope_cos != nullptr && head < p.n_q_heads + p.n_kv_heads;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int m = mt * 8 + 2 * t + j;
        if (m >= p.M) continue;
        float a = round_to<T>(acc[0][mt][j]);
        float b = round_to<T>(acc[0][mt][2 + j]);
        const int pos = p.pos0 + m;
        if (rope) {
          const float c = p.rope_cos[(int64_t)pos * 64 + d];
          const float s = p.rope_sin[(int64_t)pos * 64 + d];
          const float a2 = a * c - b * s;
          const float b2 = a * s + b * c;
          a = a2;
          b = b2;
        }
        T* dst;
        if (head < p.n_q_heads)
          dst = static_cast<T*>(p.q_out) + (int64_t)head * p.q_head_stride + (int64_t)m * 128;
        else if (head < p.n_q_heads + p.n_kv_heads)
          dst = static_cast<T*>(p.k_cache) + (int64_t)(head - p.n_q_heads) * p.cache_head_stride + (int64_t)pos * 128;
        else
          dst = static_cast<T*>(p.v_cache) + (int64_t)(head - p.n_q_heads - p.n_kv_heads) * p.cache_head_stride +
                (int64_t)pos * 128;
        dst[d] = DT<T>::from_f(a);
        dst[d + 64] = DT<T>::from_f(b);
      }
  }
}

// ------------------------------------------------------------------ SwiGLU
template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(const T* gate, const T* up, T* out, int64_t n) {
  const int64_t nvec = n >> 3;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec; v += (int64_t)gridDim.x * blockDim.x) {
    uint4 gv = *reinterpret_cast<const uint4*>(gate + v * 8);
    uint4 uv = *reinterpret_cast<const uint4*>(up + v * 8);
    const T* ge = reinterpret_cast<const T*>(&gv);
    const T* ue = reinterpret_cast<const T*>(&uv);
    uint4 ov;
    T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float gf = DT<T>::to_f(ge[i]);
      const float uf = DT<T>::to_f(ue[i]);
      oe[i] = DT<T>::from_f(gf * (1.0f / (1.0f + expf(-gf))) * uf);
    }
    *reinterpret_cast<uint4*>(out + v * 8) = ov;
  }
  // scalar tail (n % 8 elements)
  const int64_t tail0 = nvec * 8;
  if (blockIdx.x == 0)
    for (int64_t i = tail0 + threadIdx.x; i < n; i += blockDim.x) {
      const float gf = DT<T>::to_f(gate[i]);
      const float uf = DT<T>::to_f(up[i]);
      out[i] = DT<T>::from_f(gf * (1.0f / (1.0f + expf(-gf))) * uf);
    }
}

// ----------------------------------------------------- cluster argmax
// One cluster of kArgmaxCluster CTAs per logits row; each CTA scans a slice,
// the CTA winners meet in CTA 0's shared memory through DSMEM. No global
// scratch is needed.
constexpr int kArgmaxCluster = 8;
constexpr int kArgmaxThreads = 512;

__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}

template <typename T>
__global__ void __cluster_dims__(kArgmaxCluster, 1, 1) __launch_bounds__(kArgmaxThreads)
    argmax_kernel(const T* logits, int64_t ld, int V, int* idx_out) {
  __shared__ unsigned long long warp_best[kArgmaxThreads / 32];
  __shared__ unsigned long long cta_best;
  const int row = blockIdx.y;
  unsigned int rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const T* x = logits + (int64_t)row * ld;
  // slice boundaries in units of 8 elements (16-byte vectors)
  const int nvec = V >> 3;
  const int v0 = (int)(((int64_t)nvec * rank) / kArgmaxCluster);
  const int v1 = (int)(((int64_t)nvec * (rank + 1)) / kArgmaxCluster);
  unsigned long long best = 0ull;
  for (int v = v0 + threadIdx.x; v < v1; v += kArgmaxThreads) {
    const uint4 raw = ld_act_v4(x + (int64_t)v * 8);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) best = umax64(best, argmax_key(DT<T>::to_f(e[i]), (int64_t)v * 8 + i));
  }
  if (rank == kArgmaxCluster - 1)
    for (int i = nvec * 8 + threadIdx.x; i < V; i += kArgmaxThreads)
      best = umax64(best, argmax_key(DT<T>::to_f(x[i]), i));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, off));
  if ((threadIdx.x & 31) == 0) warp_best[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < kArgmaxThreads / 32; ++w) b = umax64(b, warp_best[w]);
    cta_best = b;
  }
  // cluster-wide barrier: every CTA's cta_best is written before CTA 0 reads
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (rank == 0 && threadIdx.x == 0) {
    const uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(&cta_best));
    unsigned long long b = 0ull;
    for (unsigned int r = 0; r < kArgmaxCluster; ++r) {
      uint32_t remote;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(r));
      unsigned long long v;
      asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(remote));
      b = umax64(b, v);
    }
    idx_out[row] = argmax_key_index(b);
  }
  // keep every CTA's shared memory alive until CTA 0 has read it
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

}  // namespace

// ------------------------------------------------------------------ launchers
template <typename T, int EPI>
static cudaError_t launch_skinny_t(const SkinnyParams& p, int tiles, cudaStream_t st) {
  if (p.M <= 8) skinny_kernel<T, 1, EPI><<<tiles, kThreads, 0, st>>>(p);
  else skinny_kernel<T, 2, EPI><<<tiles, kThreads, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_skinny(ie_dtype dt, int epi, const SkinnyParams& p, cudaStream_t st) {
  int tiles;
  if (epi == EPI_QKV) tiles = (p.n_q_heads + 2 * p.n_kv_heads) * 8;
  else tiles = ceil_div(p.N, 16);
  if (tiles <= 0) return cudaSuccess;
#define IE_SK(T)                                                         \
  switch (epi) {                                                         \
    case EPI_STORE: return launch_skinny_t<T, EPI_STORE>(p, tiles, st);  \
    case EPI_SWIGLU: return launch_skinny_t<T, EPI_SWIGLU>(p, tiles, st); \
    case EPI_ARGMAX: return launch_skinny_t<T, EPI_ARGMAX>(p, tiles, st); \
    case EPI_QKV: return launch_skinny_t<T, EPI_QKV>(p, tiles, st);      \
  }
  if (dt == IE_DTYPE_F16) { IE_SK(__half) }
  else { IE_SK(__nv_bfloat16) }
#undef IE_SK
  return cudaErrorInvalidValue;
}

cudaError_t launch_swiglu(ie_dtype dt, int64_t n, const void* gate, const void* up, void* out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int64_t nvec = (n >> 3) > 0 ? (n >> 3) : 1;
  const int blocks = (int)((nvec + 255) / 256 < 148 * 16 ? (nvec + 255) / 256 : 148 * 16);
  if (dt == IE_DTYPE_F16)
    swiglu_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(gate), static_cast<const __half*>(up),
                                                  static_cast<__half*>(out), n);
  else
    swiglu_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(gate),
                                                         static_cast<const __nv_bfloat16*>(up),
                                                         static_cast<__nv_bfloat16*>(out), n);
  return cudaGetLastError();
}

cudaError_t launch_argmax(ie_dtype dt, int M, int V, const void* logits, int64_t ld, int* idx_out, cudaStream_t st) {
  dim3 grid(kArgmaxCluster, M);
  if (dt == IE_DTYPE_F16)
    argmax_kernel<__half><<<grid, kArgmaxThreads, 0, st>>>(static_cast<const __half*>(logits), ld, V, idx_out);
  else
    argmax_kernel<__nv_bfloat16><<<grid, kArgmaxThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(logits), ld, V,
                                                                  idx_out);
  return cudaGetLastError();
}

}  // namespace ie
