// Attention core behind the drop-in attn / decode_attn entry points and the
// decode engine.
//
// Not a weight matmul: it exists so that the reference's attention entry
// points (kernels/attn.cuh:5-8), whose translation unit also holds the Q/K/V
// and O projections, can be served by this library. It reads Q written
// head-major by ie_qkv and the K/V cache rows, and writes the token-major
// [S, n_q_heads * 128] output the O projection consumes (the layout the
// reference produces with attn_permute, kernels/attn_permute.cu:15-32).
//
// The reference's chain (kernels/attn.cu:355-366, :423-431,
// kernels/softmax.cu:55-160): a score is one fp32 dot product rounded to the
// storage type (the cuBLAS QK^T output), scaled by rsqrt(128) and rounded
// again; e = exp(t - max) is summed in fp32 and stored rounded;
// p = round(round(e) * (1/sum)); out = round(p.V) (one fp32 accumulation).
// Two kernels:
//  * few query rows (decode, verify): split-KV over a thread-block cluster,
//    which keeps the chain exactly (exact row max and sum before any p);
//  * many query rows (prefill): a flash-attention kernel on the tensor cores
//    (mma.sync m16n8k16, fp32 accumulation) with the same roundings of s, t
//    and p, but the running-maximum form of the softmax: p is round(e) with
//    e taken against the running maximum, and the division by the sum comes
//    after the p.V accumulation. Its outputs differ from the chain by about a
//    rounding step of p.
#include <climits>
#include <cstring>
#include <cstdlib>
#include <type_traits>
#include "ie_common.cuh"
#include "attention.cuh"

// ------------------------------------------------ split-KV decode attention
// Decode-time attention (a few query rows, each over its whole cache) spread
// over the GPU: one thread-block cluster of C CTAs per (query row, KV head),
// C = 16 for at most 4 KV heads, else 8, whatever the number of rows (so a
// row's result does not depend on the batch); CTA c of the cluster takes
// cache rows [c*len/C, (c+1)*len/C). A CTA is 4 warps.
//  * Cache rows reach shared memory by untiled bulk copies
//    (cp.async.bulk, 64 rows = 16 KB each) through a ring of 2-6 slots
//    completed on mbarriers. Rows older than the launch's first query row are
//    requested before the kernel waits for its predecessor (programmatic
//    launch), so their latency overlaps the QKV projection's tail.
//  * Scores run on the tensor cores (m16n8k16: 16 cache rows x the group's
//    query heads, padded to 8): warp w takes rows 16w..16w+15 of a chunk, the
//    two 64-dimension halves in two accumulators added low + high, then
//    rounded, scaled and rounded; the row maximum is kept in registers.
//  * The softmax keeps the reference's chain (scores rounded, scaled and
//    rounded; e = exp(t - max) summed in fp32 and stored rounded;
//    p = round(round(e) * (1/sum))): the row maximum and the sum are exact
//    cluster-wide values. Each CTA pushes its maximum, its sum and its p.V
//    partial into every peer's shared memory (st.async, completing on the
//    peer's mbarrier), and sums what it receives in rank order.
//  * p.V runs on the tensor cores too: P (heads x 16 cache rows) is the A
//    operand, V the B operand, its pairs of rows packed by byte permutes from
//    8-byte shared-memory loads; warp w owns output dimensions 32w..32w+31
//    for the whole slice, so no cross-warp sum is needed. CTA r rounds and
//    stores the r-th 1/C of the row's outputs.
// Results are deterministic. Every mbarrier wait is bounded (2 s unless
// ie_set_wait_limit_ns says otherwise): on expiry IE_ERR_TIMEOUT is recorded,
// no further copies are issued, and before the CTA exits the outstanding
// copies and the peers' pushes into it are waited for (bounded).
namespace ie {

__device__ int g_attn_status = 0;
// limit of one bulk-copy or exchange wait (ie_set_wait_limit_ns)
__device__ unsigned long long g_attn_wait_ns = kDefaultWaitNs;

namespace {

constexpr int kFdThreads = 128;
constexpr int kFdWarps = kFdThreads / 32;
constexpr int kFdRows = 64;
constexpr int kFdStages = 6;  // deepest ring (the size limits are checked against it)
constexpr int kFdStageBytes = kFdRows * 128 * 2;
constexpr int kFdRingBytes = kFdStages * kFdStageBytes;

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
  int cap;     // score slots per head in shared memory (fd_score_cap)
  int stages;  // ring depth in 64-row chunks, 2 .. kFdStages (occupancy only; no effect on the results)
  int early;   // launched to overlap its predecessor: the older rows are requested before waiting for it
};

// Score slots per head: at least the longest slice rounded up to whole
// 16-row MMA steps (an 8-CTA slice of cache_rows rows); kept 16 above a
// multiple of 64 so that the heads' rows of P start in different banks.
__host__ __device__ constexpr int fd_score_cap(int cache_rows) {
  return ((cache_rows + 7) / 8 + 63) / 64 * 64 + 16;
}

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
// Phase 0 of an exchange barrier, which the peers' st.async complete. The
// pushed bytes are in this CTA's shared memory once the barrier has counted
// them, as with the bulk copies, so the default CTA-scope wait suffices (an
// acquire at cluster scope would add a fence to every poll).
__device__ __forceinline__ bool fd_try_cluster(uint32_t bar) { return fd_try(bar, 0u); }
__device__ __forceinline__ unsigned long long fd_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait; false when it gave up or another thread already did.
__device__ __forceinline__ bool fd_wait(uint32_t bar, uint32_t parity, volatile int* abort_s) {
  if (fd_try(bar, parity)) return true;
  const unsigned long long limit = g_attn_wait_ns;
  const unsigned long long t0 = fd_now();
  while (!fd_try(bar, parity)) {
    if (*abort_s) return false;
    if (fd_now() - t0 > limit) {
      atomicExch(&g_attn_status, IE_ERR_TIMEOUT);
      *abort_s = 1;
      return false;
    }
  }
  return true;
}
// Bounded wait for one exchange (single phase per launch).
__device__ __forceinline__ void fd_wait_exchange(uint32_t bar, volatile int* abort_s, unsigned long long limit) {
  if (fd_try_cluster(bar)) return;
  const unsigned long long t0 = fd_now();
  while (!fd_try_cluster(bar)) {
    if (fd_now() - t0 > limit) {
      atomicExch(&g_attn_status, IE_ERR_TIMEOUT);
      *abort_s = 1;
      return;
    }
  }
}
__device__ __forceinline__ uint32_t fd_peer(uint32_t local, unsigned rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  return remote;
}
// 4 bytes into a peer's shared memory, counted on the peer's mbarrier
__device__ __forceinline__ void fd_push(uint32_t raddr, float v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
               "r"(__float_as_uint(v)), "r"(rbar)
               : "memory");
}
__device__ __forceinline__ void fd_push4(uint32_t raddr, float a, float b, float c, float d, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   raddr),
               "r"(__float_as_uint(a)), "r"(__float_as_uint(b)), "r"(__float_as_uint(c)), "r"(__float_as_uint(d)),
               "r"(rbar)
               : "memory");
}

// m16n8k16 tensor-core product, fp32 accumulation (A and B of the same type).
template <typename T>
__device__ __forceinline__ void fd_mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <typename T, int G, int C>
__global__ void __launch_bounds__(kFdThreads) decode_attention_kernel(const FdParams p) {
  constexpr int kPer = G * 128 / C;  // outputs each CTA of the cluster reduces and stores
  static_assert(kPer % 8 == 0 && kPer <= kFdThreads, "output slice per CTA");
  extern __shared__ __align__(128) unsigned char fd_smem[];
  __shared__ __align__(16) float xout[C * kPer];  // [source rank][kPer] p.V partials pushed by the cluster
  __shared__ float xmax[C][G], xsum[C][G];         // [source rank][head] maxima and sums pushed by the cluster
  __shared__ float wred[kFdWarps][G];
  __shared__ float gmax[G], ginv[G];
  __shared__ __align__(8) unsigned long long bars[kFdStages];
  __shared__ __align__(8) unsigned long long xbar[3];  // maxima, sums, partials
  __shared__ int abort_s, fail_at;

  T* ring = reinterpret_cast<T*>(fd_smem);
  const int S = p.stages;
  T* sc = reinterpret_cast<T*>(fd_smem + S * kFdStageBytes);  // [G][cap]: scores, then e, then p
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int fg = lane >> 2, ft = lane & 3;
  unsigned rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int hk = blockIdx.y, m = blockIdx.z;

  // The cache rows before the first query row of this row's sequence were
  // written by earlier launches; the preceding kernel (the QKV projection)
  // writes only rows from there on, and q. So the copies of the older rows
  // are issued before waiting for that kernel, the rest after it.
  const int pos = p.positions ? p.positions[m] : p.pos0 + m;
  const int m_first = m - m % p.rows_per_seq;
  const int first_new = p.positions ? p.positions[m_first] : p.pos0 + m_first;
  const bool bad = pos < 0 || pos >= p.cache_rows;
  if (bad && rank == 0 && tid == 0) atomicExch(&g_attn_status, IE_ERR_INVALID_ARG);
  const int len = bad ? 0 : pos + 1;
  const int j0 = (int)((int64_t)len * rank / C);
  const int n = (int)((int64_t)len * (rank + 1) / C) - j0;
  const int nk = (n + kFdRows - 1) / kFdRows, total = 2 * nk;
  const int64_t base = (int64_t)(m / p.rows_per_seq) * p.cbs + (int64_t)hk * p.chs;
  const T* kh = static_cast<const T*>(p.kc) + base;
  const T* vh = static_cast<const T*>(p.vc) + base;

  int issued = 0;  // thread 0 only
  auto chunk_of = [&](int i, int& r0, int& rows) {
    const int c = i < nk ? i : i - nk;
    r0 = j0 + c * kFdRows;
    rows = min(kFdRows, j0 + n - r0);
  };
  // expect the whole chunk on its slot's barrier
  auto arm = [&](int i) {
    int r0, rows;
    chunk_of(i, r0, rows);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fd_smem_u32(&bars[i % S])),
                 "r"((uint32_t)rows * 128u * (uint32_t)sizeof(T))
                 : "memory");
    issued = i + 1;
  };
  // copy cache rows [lo, hi) (absolute) of chunk i into its slot
  auto copy = [&](int i, int lo, int hi) {
    int r0, rows;
    chunk_of(i, r0, rows);
    lo = max(lo, r0);
    hi = min(hi, r0 + rows);
    if (hi <= lo) return;
    const int slot = i % S;
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     fd_smem_u32(ring + (slot * kFdRows + (lo - r0)) * 128)),
                 "l"((i < nk ? kh : vh) + (int64_t)lo * 128), "r"((uint32_t)(hi - lo) * 128u * (uint32_t)sizeof(T)),
                 "r"(fd_smem_u32(&bars[slot]))
                 : "memory");
  };
  auto issue = [&](int i) {
    arm(i);
    copy(i, 0, INT_MAX);
  };

  // B fragments of q for the score MMAs, from global memory: lane (g, t)
  // holds, for each half hf and 32-dimension k-step ks, the 8 dimensions
  // 64 hf + 32 ks + 8t .. +7 of head g (zero for g >= G) as one 16-byte load,
  // in the order the A fragments use (MMA j takes elements 4j .. 4j+3 of a
  // lane's 8-dimension load). Without a predecessor to overlap, q is read
  // before the cache copies fill the memory system; otherwise after the wait
  // (the predecessor writes it).
  uint4 qf[2][2];
  auto load_q = [&] {
    const uint4* qv = reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) +
                                                     (int64_t)(hk * G + (fg < G ? fg : 0)) * p.q_head_stride +
                                                     (int64_t)m * 128);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) qf[hf][ks] = fg < G ? qv[8 * hf + 4 * ks + ft] : make_uint4(0u, 0u, 0u, 0u);
  };
  if (!p.early) load_q();

  const int first = min(S, total);
  if (tid == 0) {
    for (int s = 0; s < S; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(fd_smem_u32(&bars[s])) : "memory");
    // each exchange completes when all C peers' bytes have landed
    const uint32_t xbytes[3] = {C * G * 4u, C * G * 4u, C * kPer * 4u};
    for (int k = 0; k < 3; ++k) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(fd_smem_u32(&xbar[k])) : "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fd_smem_u32(&xbar[k])),
                   "r"(xbytes[k])
                   : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_s = 0;
    fail_at = INT_MAX;
    for (int i = 0; i < first; ++i) {
      arm(i);
      if (p.early) copy(i, 0, first_new);
    }
  }
  __syncwarp();
  // every peer's exchange barriers are initialised before the first push:
  // arrive now (the init fence above orders the initialisation), wait right
  // before pushing
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (p.early) load_q();
  if (tid == 0)
    for (int i = 0; i < first; ++i) copy(i, p.early ? first_new : 0, INT_MAX);
  __syncthreads();  // abort_s, fail_at

  auto wait_chunk = [&](int i) {
    if (!fd_wait(fd_smem_u32(&bars[i % S]), (uint32_t)((i / S) & 1), &abort_s))
      atomicMin(&fail_at, i);
  };
  // a slot that takes another chunk is refilled once every warp is done
  // with it; the last S chunks free nothing, so warps run on through them
  // without a barrier (the condition is the same for the whole CTA)
  auto next = [&](int i) {
    if (i + S >= total) return;
    __syncthreads();
    if (tid == 0 && !abort_s) issue(i + S);
  };

  // ---- scores: S[row][head] = K[row] . q[head] over the low and the high
  // 64 dimensions (4 MMAs each), added low + high, then rounded, scaled by
  // rsqrt(128) and rounded; lane (g, t) gets rows g, g + 8 of its warp's tile
  // and heads 2t, 2t + 1
  const float scale = rsqrtf(128.0f);
  float mx[2] = {-INFINITY, -INFINITY};
  for (int i = 0; i < nk; ++i) {
    wait_chunk(i);
    const T* tile = ring + (i % S) * kFdRows * 128;
    const int r0 = i * kFdRows, rows = min(kFdRows, n - r0);
    if (16 * warp < rows) {
      float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const T* ra = tile + (16 * warp + fg) * 128 + 64 * hf + 8 * ft;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const uint4 wa = *reinterpret_cast<const uint4*>(ra + 32 * ks);            // row g
          const uint4 wb = *reinterpret_cast<const uint4*>(ra + 8 * 128 + 32 * ks);  // row g + 8
          fd_mma<T>(c[hf], wa.x, wb.x, wa.y, wb.y, qf[hf][ks].x, qf[hf][ks].y);
          fd_mma<T>(c[hf], wa.z, wb.z, wa.w, wb.w, qf[hf][ks].z, qf[hf][ks].w);
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int row = 16 * warp + fg + 8 * (k >> 1), h = 2 * ft + (k & 1);
        if (h < G && row < rows) {
          const float s = round_to<T>(round_to<T>(c[0][k] + c[1][k]) * scale);
          sc[h * p.cap + r0 + row] = DT<T>::from_f(s);
          mx[k & 1] = fmaxf(mx[k & 1], s);
        }
      }
    }
    next(i);
  }

  // ---- softmax with cluster-wide max and sum
#pragma unroll
  for (int e = 0; e < 2; ++e) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], off));
    if (fg == 0 && 2 * ft + e < G) wred[warp][2 * ft + e] = mx[e];
  }
  __syncthreads();
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (tid < C * G) {  // this CTA's maximum of head h to rank r
    const int h = tid % G, r = tid / G;
    float v = wred[0][h];
#pragma unroll
    for (int w = 1; w < kFdWarps; ++w) v = fmaxf(v, wred[w][h]);
    fd_push(fd_peer(fd_smem_u32(&xmax[rank][h]), r), v, fd_peer(fd_smem_u32(&xbar[0]), r));
  }
  const unsigned long long xlimit = g_attn_wait_ns;
  fd_wait_exchange(fd_smem_u32(&xbar[0]), &abort_s, xlimit);
  if (tid < G) {
    float v = xmax[0][tid];
#pragma unroll
    for (int r = 1; r < C; ++r) v = fmaxf(v, xmax[r][tid]);
    gmax[tid] = v;
  }
  __syncthreads();
  // e = exp(t - max), stored rounded, in blocks of 8 slots per thread (head
  // h, slots 8b .. 8b+7); slots from n up to the next 16-row step get 0. A
  // thread adds its slots in order, then its blocks in order.
  const int n16 = (n + 15) & ~15, nb = n16 / 8;
  float sm[G];
#pragma unroll
  for (int h = 0; h < G; ++h) sm[h] = 0.f;
  for (int v = tid; v < G * nb; v += kFdThreads) {
    const int h = v / nb, j = (v - h * nb) * 8;
    uint4* blk = reinterpret_cast<uint4*>(sc + h * p.cap + j);
    uint4 raw = *blk;
    T* x = reinterpret_cast<T*>(&raw);
    const float g = gmax[h];
    float s8 = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float e = j + k < n ? expf(DT<T>::to_f(x[k]) - g) : 0.f;
      s8 += e;
      x[k] = DT<T>::from_f(e);
    }
    *blk = raw;
#pragma unroll
    for (int hh = 0; hh < G; ++hh)
      if (hh == h) sm[hh] += s8;
  }
#pragma unroll
  for (int h = 0; h < G; ++h) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sm[h] += __shfl_xor_sync(0xffffffffu, sm[h], off);
  }
  if (lane == 0)
#pragma unroll
    for (int h = 0; h < G; ++h) wred[warp][h] = sm[h];
  __syncthreads();
  if (tid < C * G) {  // this CTA's sum of head h (warps in order) to rank r
    const int h = tid % G, r = tid / G;
    float v = wred[0][h];
#pragma unroll
    for (int w = 1; w < kFdWarps; ++w) v += wred[w][h];
    fd_push(fd_peer(fd_smem_u32(&xsum[rank][h]), r), v, fd_peer(fd_smem_u32(&xbar[1]), r));
  }
  fd_wait_exchange(fd_smem_u32(&xbar[1]), &abort_s, xlimit);
  if (tid < G) {
    float v = xsum[0][tid];
#pragma unroll
    for (int r = 1; r < C; ++r) v += xsum[r][tid];
    ginv[tid] = 1.0f / v;
  }
  __syncthreads();
  // p = round(round(e) / sum) (the zero slots stay zero)
  for (int v = tid; v < G * nb; v += kFdThreads) {
    const int h = v / nb, j = (v - h * nb) * 8;
    uint4* blk = reinterpret_cast<uint4*>(sc + h * p.cap + j);
    uint4 raw = *blk;
    T* x = reinterpret_cast<T*>(&raw);
    const float iv = ginv[h];
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = DT<T>::from_f(DT<T>::to_f(x[k]) * iv);
    *blk = raw;
  }
  __syncthreads();

  // ---- p.V on the tensor cores: out[head][dim] += P[head][row] V[row][dim]
  // per 16-row step. A = P (rows g of lane (g, t) = head g, zero from G on),
  // B = V: lane (g, t) loads dimensions 32w + 4g .. +3 of rows 2t, 2t+1,
  // 2t+8, 2t+9 and packs the row pairs of each dimension; the MMA of
  // dimension offset d (0..3) then holds, in its column n, dimension
  // 32w + 4n + d.
  float acc[4][4];
#pragma unroll
  for (int d = 0; d < 4; ++d)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[d][e] = 0.f;
  // one 16-row step; rows past the slice hold stale data and are read as
  // zero (their p is zero too)
  auto pv_step = [&](const T* tile, int r0, int k0, int rows, bool full) {
    const int kr = k0 + 2 * ft;
    uint32_t a0 = 0u, a2 = 0u;
    if (fg < G) {
      const T* pr = sc + fg * p.cap + r0 + kr;
      a0 = *reinterpret_cast<const uint32_t*>(pr);
      a2 = *reinterpret_cast<const uint32_t*>(pr + 8);
    }
    const T* vr = tile + kr * 128 + 32 * warp + 4 * fg;
    const uint2 z = make_uint2(0u, 0u);
    const uint2 va = full || kr < rows ? *reinterpret_cast<const uint2*>(vr) : z;
    const uint2 vb = full || kr + 1 < rows ? *reinterpret_cast<const uint2*>(vr + 128) : z;
    const uint2 vc = full || kr + 8 < rows ? *reinterpret_cast<const uint2*>(vr + 8 * 128) : z;
    const uint2 vd = full || kr + 9 < rows ? *reinterpret_cast<const uint2*>(vr + 9 * 128) : z;
    fd_mma<T>(acc[0], a0, 0u, a2, 0u, __byte_perm(va.x, vb.x, 0x5410), __byte_perm(vc.x, vd.x, 0x5410));
    fd_mma<T>(acc[1], a0, 0u, a2, 0u, __byte_perm(va.x, vb.x, 0x7632), __byte_perm(vc.x, vd.x, 0x7632));
    fd_mma<T>(acc[2], a0, 0u, a2, 0u, __byte_perm(va.y, vb.y, 0x5410), __byte_perm(vc.y, vd.y, 0x5410));
    fd_mma<T>(acc[3], a0, 0u, a2, 0u, __byte_perm(va.y, vb.y, 0x7632), __byte_perm(vc.y, vd.y, 0x7632));
  };
  for (int i = nk; i < total; ++i) {
    wait_chunk(i);
    const T* tile = ring + (i % S) * kFdRows * 128;
    const int r0 = (i - nk) * kFdRows, rows = min(kFdRows, n - r0);
    if (rows == kFdRows) {
#pragma unroll
      for (int k0 = 0; k0 < kFdRows; k0 += 16) pv_step(tile, r0, k0, rows, true);
    } else {
      for (int k0 = 0; k0 < rows; k0 += 16) pv_step(tile, r0, k0, rows, false);
    }
    next(i);
  }
  // copies a failed wait left in flight finish before the CTA exits
  if (tid == 0 && fail_at < issued) {
    for (int i = fail_at; i < issued; ++i) {
      const unsigned long long t0 = fd_now();
      while (!fd_try(fd_smem_u32(&bars[i % S]), (uint32_t)((i / S) & 1)) &&
             fd_now() - t0 < kDrainWaitNs) {
      }
    }
  }

  // ---- the cluster sum of the p.V partials: lane (g, t) of warp w holds head
  // g, dimensions 32w + 8t .. +7 (acc[d][0] is dimension 8t + d, acc[d][1]
  // dimension 8t + 4 + d); they go to the CTA that stores them
  if (fg < G) {
    const int e = fg * 128 + 32 * warp + 8 * ft;
    const unsigned owner = (unsigned)(e / kPer);
    const uint32_t raddr = fd_peer(fd_smem_u32(&xout[rank * kPer + (e - (int)owner * kPer)]), owner);
    const uint32_t rbar = fd_peer(fd_smem_u32(&xbar[2]), owner);
    fd_push4(raddr, acc[0][0], acc[1][0], acc[2][0], acc[3][0], rbar);
    fd_push4(raddr + 16, acc[0][1], acc[1][1], acc[2][1], acc[3][1], rbar);
  }
  fd_wait_exchange(fd_smem_u32(&xbar[2]), &abort_s, xlimit);
  if (tid < kPer) {
    float s = xout[tid];
#pragma unroll
    for (int r = 1; r < C; ++r) s += xout[r * kPer + tid];
    const int e = (int)rank * kPer + tid;
    const int h = e >> 7, d = e & 127;
    static_cast<T*>(p.out)[(int64_t)m * p.ld_out + (int64_t)(hk * G + h) * 128 + d] = DT<T>::from_f(s);
  }
  // after a timeout, late pushes from the peers land before this CTA exits
  if (abort_s)
    for (int k = 0; k < 3; ++k) fd_wait_exchange(fd_smem_u32(&xbar[k]), &abort_s, kDrainWaitNs);
}

template <typename T, int G, int C>
cudaError_t launch_decode_attention(const FdParams& p, int n_kv_heads, int R, cudaStream_t st) {
  auto kernel = decode_attention_kernel<T, G, C>;
  const size_t smem = (size_t)p.stages * kFdStageBytes + (size_t)G * p.cap * sizeof(T);
  static size_t configured[64] = {};  // per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess && C > 8) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, n_kv_heads, R);
  cfg.blockDim = dim3(kFdThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  const char* env = getenv("IE_PDL");
  cfg.numAttrs = ((env && env[0] == '0') || R > pdl_max_rows()) ? 1 : 2;
  FdParams pl = p;
  pl.early = cfg.numAttrs == 2;
  return cudaLaunchKernelEx(&cfg, kernel, pl);
}

// Ring depth of a launch: the full 6 stages while the grid fits twice per SM,
// else the deepest ring that lets every CTA be resident at once (the ring is
// most of a CTA's shared memory), at least 2. Only residency depends on it:
// which MMA adds which cache row, and so every result bit, comes from the
// 64-row chunks. IE_FD_STAGES=2..6 in the environment fixes it (for
// measurements).
int fd_stages(int ctas, int group, int cap, int cluster) {
  static const int forced = [] {
    const char* e = getenv("IE_FD_STAGES");
    const int v = e ? atoi(e) : 0;
    return (v >= 2 && v <= kFdStages) ? v : 0;
  }();
  if (forced) return forced;
  static const int sms = [] {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
  }();
  const int per_sm = (ctas + sms - 1) / sms;
  if (per_sm <= 2) return kFdStages;
  // static shared memory (exchange buffers, barriers) and the 1 KB the
  // runtime keeps per CTA, against the 228 KB of a B200 SM
  const size_t fixed = (size_t)group * 128 * 4 + (size_t)2 * cluster * group * 4 + 512 + 1024;
  for (int s = kFdStages; s > 2; --s)
    if ((size_t)per_sm * ((size_t)s * kFdStageBytes + (size_t)group * cap * 2 + fixed) <= 228u * 1024u) return s;
  return 2;
}

// Cluster size from the KV head count alone: 16 CTAs per (row, KV head) for
// at most 4 KV heads (the tensor-parallel shards of an 8-head model), else 8.
// The key slices and the order in which their partial sums meet follow from
// the cluster size, so it must not depend on how many rows share a launch: a
// row then gets the same bits alone, in a batch, or inside a verify block.
// IE_FD_CLUSTER=8|16 in the environment forces one (for measurements).
int fd_cluster_size(int n_kv_heads) {
  static const int forced = [] {
    const char* e = getenv("IE_FD_CLUSTER");
    return e ? atoi(e) : 0;
  }();
  if (forced == 8 || forced == 16) return forced;
  return n_kv_heads <= 4 ? 16 : 8;
}

}  // namespace

cudaError_t set_attn_wait_ns(unsigned long long ns) {
  return cudaMemcpyToSymbol(g_attn_wait_ns, &ns, sizeof(ns));
}

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
  if (!aligned16(k_cache) || !aligned16(v_cache) || (cache_head_stride % 8) || (cache_batch_stride % 8) ||
      !aligned16(q) || (q_head_stride % 8))
    return IE_ERR_ALIGNMENT;
  if (ld_out < (int64_t)n_q_heads * 128 || q_head_stride < (int64_t)R * 128) return IE_ERR_INVALID_ARG;
  if (cache_head_stride < (int64_t)cache_rows * 128) return IE_ERR_INVALID_ARG;
  if (R / rows_per_seq > 1 && cache_batch_stride < (int64_t)n_kv_heads * cache_head_stride) return IE_ERR_INVALID_ARG;
  if (!positions && (int64_t)pos0 + R > cache_rows) return IE_ERR_INVALID_ARG;
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
  const int C = fd_cluster_size(n_kv_heads);
  // score slots per head: the 8-CTA slice bound serves both cluster sizes
  p.cap = fd_score_cap(cache_rows);
  if (kFdRingBytes + (size_t)group * p.cap * 2 > 200 * 1024) return IE_ERR_UNSUPPORTED;
  p.stages = fd_stages(C * n_kv_heads * R, group, p.cap, C);
  p.early = 0;  // set by the launcher
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
#define IE_FD(T, CL)                                                                   \
  switch (group) {                                                                     \
    case 1: e = launch_decode_attention<T, 1, CL>(p, n_kv_heads, R, st); break;        \
    case 2: e = launch_decode_attention<T, 2, CL>(p, n_kv_heads, R, st); break;        \
    case 4: e = launch_decode_attention<T, 4, CL>(p, n_kv_heads, R, st); break;        \
    default: e = launch_decode_attention<T, 8, CL>(p, n_kv_heads, R, st); break;       \
  }
  if (dt == IE_DTYPE_F16) {
    if (C == 16) { IE_FD(__half, 16) } else { IE_FD(__half, 8) }
  } else {
    if (C == 16) { IE_FD(__nv_bfloat16, 16) } else { IE_FD(__nv_bfloat16, 8) }
  }
#undef IE_FD
  return e == cudaSuccess ? IE_OK : IE_ERR_LAUNCH;
}

// ------------------------------------------------------ prefill attention
// Causal flash attention for many query rows of one sequence. CTA = 4 warps =
// 64 query rows of one query head; each warp owns 16 rows and walks the key
// blocks of 64 positions up to its causal limit:
//   S = Q.K^T (m16n8k16, fp32) -> t = round(round(s) * rsqrt(128)) -> mask
//   -> running max m, e = exp(t - m), p = round(e) -> O = O * exp(m_old - m)
//   + p.V (m16n8k16) ; l = l * exp(m_old - m) + sum(e)
// and writes round(O / l). Q, K and V tiles reach shared memory with 16-byte
// cp.async copies into an XOR-swizzled layout (chunk c of row r at c ^ (r & 7))
// so the ldmatrix fragment loads are conflict-free; K/V blocks are double
// buffered. Query blocks are issued heaviest first (the causal work grows
// with the block index). GQA: the K/V rows of head h / group.
namespace ie {
namespace {

constexpr int kPaRows = 64, kPaKeys = 64, kPaThreads = 128;
constexpr int kPaTile = 64 * 128 * 2;                  // one 64 x 128 tile, bytes
constexpr int kPaSmem = kPaTile * 5;                   // Q + 2 x (K, V)

struct PaParams {
  const void* q;
  int64_t q_head_stride;
  const void* kc;
  const void* vc;
  int64_t chs;
  int cache_rows, pos0, S, group;
  void* out;
  int64_t ld_out;
};

__device__ __forceinline__ uint32_t pa_swz(int r, int c) {  // byte offset of 16-B chunk c of tile row r
  return (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4));
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr));
}
template <typename T>
__device__ __forceinline__ void pa_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  T a = DT<T>::from_f(lo), b = DT<T>::from_f(hi);
  return (uint32_t)(*reinterpret_cast<uint16_t*>(&a)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&b)) << 16);
}

// 64 rows x 128 dims starting at `src` (row stride 128 elements) into a
// swizzled tile; rows >= valid_rows are zero-filled.
template <typename T>
__device__ __forceinline__ void load_tile(uint32_t dst, const T* src, int valid_rows) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = threadIdx.x + i * kPaThreads;  // 0 .. 1023
    const int r = idx >> 4, c = idx & 15;
    const bool v = r < valid_rows;
    cp16(dst + pa_swz(r, c), src + (int64_t)(v ? r : 0) * 128 + c * 8, v);
  }
}

template <typename T>
__global__ void __launch_bounds__(kPaThreads) prefill_attention_kernel(const PaParams p) {
  extern __shared__ __align__(128) unsigned char pa_smem[];
  const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(pa_smem));
  // Q, then (K, V) of buffer 0, then (K, V) of buffer 1
  const uint32_t sQ = sbase;
  auto sK = [&](int b) { return sbase + (uint32_t)(1 + 2 * b) * kPaTile; };
  auto sV = [&](int b) { return sbase + (uint32_t)(2 + 2 * b) * kPaTile; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int qb = gridDim.x - 1 - blockIdx.x, h = blockIdx.y, hk = h / p.group;
  const int row0 = qb * kPaRows;
  const int last_q = min(row0 + kPaRows, p.S) - 1;        // last real query row of the block
  const int nkb = (p.pos0 + last_q) / kPaKeys + 1;         // key blocks the block needs
  const T* qh = static_cast<const T*>(p.q) + (int64_t)h * p.q_head_stride + (int64_t)row0 * 128;
  const T* kh = static_cast<const T*>(p.kc) + (int64_t)hk * p.chs;
  const T* vh = static_cast<const T*>(p.vc) + (int64_t)hk * p.chs;

  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  load_tile<T>(sQ, qh, p.S - row0);
  load_tile<T>(sK(0), kh, p.cache_rows);
  load_tile<T>(sV(0), vh, p.cache_rows);
  asm volatile("cp.async.commit_group;" ::: "memory");

  const float scale = rsqrtf(128.0f);
  const int qr0 = p.pos0 + row0 + warp * 16 + g;  // absolute positions of this lane's rows g and g+8
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
  uint32_t qf[8][4];

  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      const int r = (kb + 1) * kPaKeys;
      load_tile<T>(sK(buf ^ 1), kh + (int64_t)r * 128, p.cache_rows - r);
      load_tile<T>(sV(buf ^ 1), vh + (int64_t)r * 128, p.cache_rows - r);
      asm volatile("cp.async.commit_group;" ::: "memory");
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int r = warp * 16 + (lane & 15), c = ks * 2 + (lane >> 4);
        ldsm_x4(sQ + pa_swz(r, c), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
      }
    }
    // ---- S = Q K^T for 64 keys (8 n-tiles)
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks)
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3), c = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(sK(buf) + pa_swz(r, c), b0, b1, b2, b3);
        pa_mma<T>(s[2 * np], qf[ks], b0, b1);
        pa_mma<T>(s[2 * np + 1], qf[ks], b2, b3);
      }
    // ---- scores, mask, running max
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = kb * kPaKeys + nt * 8 + 2 * t4 + (j & 1);
        const int qpos = qr0 + ((j >> 1) << 3);
        const float v = key <= qpos ? round_to<T>(round_to<T>(s[nt][j]) * scale) : -INFINITY;
        s[nt][j] = v;
        mx[j >> 1] = fmaxf(mx[j >> 1], v);
      }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mn = fmaxf(m[r], mx[r]);
      corr[r] = expf(m[r] - mn);  // 0 on the first block (m = -inf, mn finite)
      m[r] = mn;
      l[r] *= corr[r];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    // ---- p = round(exp(t - m)); O += P V
    uint32_t pf[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float e[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        e[j] = expf(s[nt][j] - m[j >> 1]);
        l[j >> 1] += e[j];
      }
      const int kk = nt >> 1, hi = nt & 1;
      pf[kk][hi * 2 + 0] = pack2<T>(e[0], e[1]);
      pf[kk][hi * 2 + 1] = pack2<T>(e[2], e[3]);
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), c = dp * 2 + (lane >> 4);
        ldsm_x4_t(sV(buf) + pa_swz(r, c), b0, b1, b2, b3);
        pa_mma<T>(o[2 * dp], pf[kk], b0, b1);
        pa_mma<T>(o[2 * dp + 1], pf[kk], b2, b3);
      }
    __syncthreads();  // the buffer is refilled two blocks later
  }
  // ---- normalise and store
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
  }
  const float inv[2] = {1.0f / l[0], 1.0f / l[1]};
  T* out = static_cast<T*>(p.out);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = row0 + warp * 16 + g + 8 * r;
    if (row >= p.S) continue;
    T* orow = out + (int64_t)row * p.ld_out + (int64_t)h * 128;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const uint32_t v = pack2<T>(o[nt][2 * r] * inv[r], o[nt][2 * r + 1] * inv[r]);
      *reinterpret_cast<uint32_t*>(orow + nt * 8 + 2 * t4) = v;
    }
  }
}

// The tcgen05 kernel unless IE_PREFILL_ATTN=mma selects the mma.sync one.
bool use_tc_prefill() {
  static const bool tc = [] {
    const char* e = getenv("IE_PREFILL_ATTN");
    return !(e && std::strcmp(e, "mma") == 0);
  }();
  return tc;
}

template <typename T>
cudaError_t launch_prefill_attention(const PaParams& p, int n_q_heads, cudaStream_t st) {
  auto kernel = prefill_attention_kernel<T>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPaSmem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.S + kPaRows - 1) / kPaRows, n_q_heads);
  cfg.blockDim = dim3(kPaThreads);
  cfg.dynamicSmemBytes = kPaSmem;
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
}  // namespace ie

extern "C" int ie_attention(ie_dtype dt, int S, int pos0, int n_q_heads, int n_kv_heads, int head_dim, const void* q,
                            int64_t q_head_stride, const void* k_cache, const void* v_cache,
                            int64_t cache_head_stride, void* out, int64_t ld_out, void* stream) {
  using namespace ie;
  if ((dt != IE_DTYPE_F16 && dt != IE_DTYPE_BF16) || S < 0 || pos0 < 0 || n_kv_heads <= 0 || n_q_heads <= 0)
    return IE_ERR_INVALID_ARG;
  if (head_dim != 128 || n_q_heads % n_kv_heads) return IE_ERR_UNSUPPORTED;
  if (S == 0) return IE_OK;
  if (!q || !k_cache || !v_cache || !out) return IE_ERR_INVALID_ARG;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out) || (cache_head_stride % 8) ||
      (q_head_stride % 8) || (ld_out % 8))
    return IE_ERR_ALIGNMENT;
  if (ld_out < (int64_t)n_q_heads * 128 || q_head_stride < (int64_t)S * 128) return IE_ERR_INVALID_ARG;
  if ((int64_t)pos0 + S > INT_MAX) return IE_ERR_INVALID_ARG;
  if (cache_head_stride < ((int64_t)pos0 + S) * 128) return IE_ERR_INVALID_ARG;
  if (S <= 16)  // few rows: the split-KV kernel (exact chain)
    return ie_attention_decode(dt, S, S, n_q_heads, n_kv_heads, head_dim, q, q_head_stride, k_cache, v_cache,
                               cache_head_stride, 0, pos0 + S, nullptr, pos0, out, ld_out, stream);
  if ((int64_t)S > 65535LL * kPaRows || n_q_heads > 65535) return IE_ERR_UNSUPPORTED;
  if (use_tc_prefill())
    return launch_tc_attention(dt, S, pos0, n_q_heads, n_kv_heads, q, q_head_stride, k_cache, v_cache,
                               cache_head_stride, out, ld_out, stream);
  PaParams p;
  p.q = q;
  p.q_head_stride = q_head_stride;
  p.kc = k_cache;
  p.vc = v_cache;
  p.chs = cache_head_stride;
  const int64_t rows = cache_head_stride / 128;
  p.cache_rows = rows > INT_MAX ? INT_MAX : (int)rows;
  p.pos0 = pos0;
  p.S = S;
  p.group = n_q_heads / n_kv_heads;
  p.out = out;
  p.ld_out = ld_out;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const cudaError_t e = dt == IE_DTYPE_F16 ? launch_prefill_attention<__half>(p, n_q_heads, st)
                                           : launch_prefill_attention<__nv_bfloat16>(p, n_q_heads, st);
  return e == cudaSuccess ? IE_OK : IE_ERR_LAUNCH;
}
