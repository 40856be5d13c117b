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
//    L1-bypassing, L2-evict-first loads, two 32-element k-steps per batch,
//    and issues its next batch before computing on the current one, so every
//    warp keeps 2-4 KB of weights in flight at all times;
//  * the dot products run on the tensor cores through m16n8k16: the weight
//    tile is the A operand (16 rows) and the activation rows are the B
//    operand (n = 8 batch rows; two n-tiles for M <= 16). The 8 elements a
//    lane loads from one row are assigned to MMA k-slots so that A and B use
//    the same permutation of k, so no shuffles or shared-memory staging are
//    needed to build fragments;
//  * per-warp fp32 partials are summed across the 8 warps in shared memory in
//    a fixed order (deterministic results), then one warp runs the epilogue;
//  * when the tiles alone would leave most SMs idle (the column-split shards
//    of tensor parallelism: QKV of 4+1+1 heads is 48 tiles at 8 GPUs), the
//    K range of a tile is split over a thread-block cluster of 2 or 4 CTAs
//    (ksplit). Each CTA reduces its warps as above, writes its partial tile
//    into the leading CTA's shared memory through DSMEM, and after one
//    cluster barrier the leader adds the partials in rank order and runs the
//    epilogue. No global scratch and no spin-waits; still deterministic.
#include "ie_common.cuh"
#include "skinny.cuh"
#include <cstdlib>

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
// Build-time shape of the weight stream (one configuration is compiled in).
// Chosen by an A/B on one B200 over the full decode step (129 launches, 15 GB):
// 16-byte loads, 2 k-steps per batch, register double-buffering gave 2.79 ms;
// 16 B x 4 without double-buffering 2.81 ms; 32-byte (v8) loads 2.90-3.43 ms;
// persistent grids 3.18-3.36 ms.
#ifndef IE_SK_LOADW
#define IE_SK_LOADW 16   // bytes each lane loads per weight row per k-step (16 or 32)
#endif
#ifndef IE_SK_UNROLL
#define IE_SK_UNROLL 2   // k-steps whose loads are issued together
#endif
#ifndef IE_SK_PIPE
#define IE_SK_PIPE 1     // 1: next batch's loads issued before this batch's MMAs
#endif
#ifndef IE_SK_PERSIST
#define IE_SK_PERSIST 0  // 1: resident CTAs walk the tiles with a grid stride
#endif
#ifndef IE_SK_MINBLOCKS
#define IE_SK_MINBLOCKS 1  // __launch_bounds__ minimum resident CTAs per SM (register cap)
#endif
#ifndef IE_SK_MINBLOCKS_MT1
#define IE_SK_MINBLOCKS_MT1 IE_SK_MINBLOCKS  // the same for M <= 8 (one n-tile of activation rows)
#endif
#ifndef IE_SK_EARLY_W_MAX_M
// Launches with at most this many activation rows request their first weight
// batch before waiting for the previous kernel (SkinnyParams::early_w).
// Measured on the decode engine: +3 % at 1 row, -18 % at 8 rows.
#define IE_SK_EARLY_W_MAX_M 2
#endif
constexpr int kWords = IE_SK_LOADW / 4;  // 32-bit words per lane per row per k-step
constexpr int kStep = kWords * 2 * 4;    // k elements per step (4 lanes share a row)
#ifndef IE_SK_UNROLL_ONE
// k-steps per batch for one weight matrix and at most 8 activation rows: the
// registers these variants leave free (88 of 128 at 2 CTAs per SM) hold a
// batch twice as deep, which doubles the weight bytes in flight per warp.
#define IE_SK_UNROLL_ONE 4
#endif
// k-steps whose loads are issued together, per variant
template <int NMAT, int MT>
struct Unroll { static constexpr int value = (NMAT == 1 && MT == 1) ? IE_SK_UNROLL_ONE : IE_SK_UNROLL; };
// The fused QKV at up to 8 rows is the one launch whose grid exceeds two CTAs
// per SM (384 CTAs for Llama-3.1-8B on one GPU, 296 slots): it keeps 2-step
// batches (80 registers) so that 3 CTAs per SM hold the whole grid at once.
// Measured per launch: 10.5 -> 9.0 us at 1 row, 13.5 -> 10.1 us at 8 rows.
template <int EPI, int MT>
struct QkvOneWave { static constexpr bool value = EPI == EPI_QKV && MT == 1; };
constexpr int kMaxKSplit = 4;  // CTAs of one tile's cluster (K split)

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

// Device status word of the decode kernels: IE_ERR_TIMEOUT when a bounded wait
// for another rank's rows gave up, IE_ERR_INVALID_ARG when a batched QKV row
// carried a position outside its cache.
__device__ int g_skinny_status = 0;
// limit of the wait for other ranks' rows (ie_set_wait_limit_ns)
__device__ unsigned long long g_skinny_wait_ns = kDefaultWaitNs;

// Epilogues, run by warp 0 on the fully reduced tile.
// acc[.][mt][i]: weight row g + 8*(i>>1) of the tile, batch row m = mt*8 + 2t + (i&1).
template <typename T, int MT, int EPI>
__device__ __forceinline__ void epilogue(const SkinnyParams& p, int tile, int g, int t, int lane,
                                         const bool (&rvalid)[2], const int (&nidx)[2],
                                         float (&acc)[EpiTraits<EPI>::nmat][MT][4]) {
  if constexpr (EPI == EPI_TP_ALLREDUCE) {
    // Each partial value travels with the call's epoch in one 64-bit word
    // (single-copy atomic), pushed straight into this rank's slot of every
    // rank's inbox (NVLink stores for peers). The CTA then reads back, from
    // its own inbox, the same tile rows of every rank (waiting, bounded, for
    // words still carrying an older epoch) and writes their rank-ordered sum.
    // A value has arrived exactly when its epoch matches: no fence, no flag.
    // Every rank's CTA j waits only for the other ranks' CTA j, so the whole
    // grid must be resident (checked at launch).
    const unsigned int e =
        *reinterpret_cast<const volatile unsigned int*>(&static_cast<const TpHeader*>(p.tp_sym[p.tp_rank])->epoch) + 1u;
    const int parity = (int)(e & 1u);
    const size_t slot = (size_t)p.tp_rows * p.tp_cols;
    const size_t base = (size_t)parity * p.tp_world * slot;
    for (int peer = 0; peer < p.tp_world; ++peer) {
      unsigned long long* box = reinterpret_cast<unsigned long long*>(static_cast<char*>(p.tp_sym[peer]) +
                                                                       kTpInboxOffset) +
                                base + (size_t)p.tp_rank * slot;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = i >> 1, m = mt * 8 + 2 * t + (i & 1);
          if (rvalid[r] && m < p.M) {
            const unsigned long long word =
                ((unsigned long long)e << 32) | (unsigned long long)__float_as_uint(acc[0][mt][i]);
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(box + (size_t)m * p.tp_cols + nidx[r]),
                         "l"(word)
                         : "memory");
          }
        }
    }
    const unsigned long long* inbox = reinterpret_cast<const unsigned long long*>(
                                          static_cast<const char*>(p.tp_sym[p.tp_rank]) + kTpInboxOffset) +
                                      base;
    T* Y = static_cast<T*>(p.Y);
    const unsigned long long limit = g_skinny_wait_ns;
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    bool gave_up = false;
    // A lane's words are polled in passes, two values (batch rows m, m+1 of
    // one output column) at a time: each pass issues the loads of every word
    // of the pair still missing, from all ranks, back to back and only then
    // checks them, so a pass costs about one memory round trip whatever the
    // number of ranks (polling rank after rank cost one round trip per rank).
#pragma unroll 1
    for (int grp = 0; grp < 2 * MT && !gave_up; ++grp) {
      const int mt = grp >> 1, r = grp & 1;
      const unsigned long long* w[2];
      unsigned int missing[2];
      float part[2][kTpMaxWorld];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int m = mt * 8 + 2 * t + j;
        const bool valid = rvalid[r] && m < p.M;
        w[j] = inbox + (size_t)(valid ? m : 0) * p.tp_cols + nidx[r];
        missing[j] = valid ? (1u << p.tp_world) - 1u : 0u;
      }
      while ((missing[0] | missing[1]) != 0u) {
        unsigned long long got[2][kTpMaxWorld];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int q = 0; q < kTpMaxWorld; ++q)
            if ((missing[j] >> q) & 1u)
              asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(got[j][q]) : "l"(w[j] + (size_t)q * slot)
                           : "memory");
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int q = 0; q < kTpMaxWorld; ++q)
            if (((missing[j] >> q) & 1u) && (unsigned int)(got[j][q] >> 32) == e) {
              part[j][q] = __uint_as_float((unsigned int)(got[j][q] & 0xffffffffull));
              missing[j] &= ~(1u << q);
            }
        if ((missing[0] | missing[1]) == 0u) break;
        unsigned long long now;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
        if (now - t0 > limit) {
          atomicExch(&g_skinny_status, IE_ERR_TIMEOUT);
          gave_up = true;
          break;
        }
      }
      if (gave_up) break;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int m = mt * 8 + 2 * t + j;
        if (!rvalid[r] || m >= p.M) continue;
        float sum = 0.f;  // rank order, as always
#pragma unroll
        for (int q = 0; q < kTpMaxWorld; ++q)
          if (q < p.tp_world) sum += part[j][q];
        T* y = Y + (int64_t)m * p.ldy + nidx[r];
        *y = DT<T>::from_f(p.residual ? DT<T>::to_f(*y) + round_to<T>(sum) : sum);
      }
    }
  } else if constexpr (EPI == EPI_STORE_F32) {
    float* Y = static_cast<float*>(p.Y);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = i >> 1, m = mt * 8 + 2 * t + (i & 1);
        if (rvalid[r] && m < p.M) Y[(int64_t)m * p.ldy + nidx[r]] = acc[0][mt][i];
      }
  } else if constexpr (EPI == EPI_STORE) {
    T* Y = static_cast<T*>(p.Y);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = i >> 1, m = mt * 8 + 2 * t + (i & 1);
        if (rvalid[r] && m < p.M) {
          T* y = Y + (int64_t)m * p.ldy + nidx[r];
          *y = DT<T>::from_f(p.residual ? DT<T>::to_f(*y) + round_to<T>(acc[0][mt][i]) : acc[0][mt][i]);
        }
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
    if (lane == 0) last = (atomicAdd(p.counter, 1u) == p.tiles - 1) ? 1u : 0u;
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
        const int pos = p.positions ? p.positions[m] : p.pos0 + m;
        if (p.positions && (pos < 0 || pos >= p.cache_rows)) {
          atomicExch(&g_skinny_status, IE_ERR_INVALID_ARG);
          continue;
        }
        const int64_t cb = p.positions ? (int64_t)m * p.cache_batch_stride : 0;
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
          dst = static_cast<T*>(p.k_cache) + cb + (int64_t)(head - p.n_q_heads) * p.cache_head_stride +
                (int64_t)pos * 128;
        else
          dst = static_cast<T*>(p.v_cache) + cb + (int64_t)(head - p.n_q_heads - p.n_kv_heads) * p.cache_head_stride +
                (int64_t)pos * 128;
        dst[d] = DT<T>::from_f(a);
        dst[d + 64] = DT<T>::from_f(b);
      }
  }
}

// Call bookkeeping of EPI_TP_ALLREDUCE: the CTA that completes the grid
// (every CTA has read this call's epoch and finished its rows by then)
// advances the epoch and re-arms the completion counter for the next call.
// The inbox slots alternate with the call parity, so a fast rank's next call
// never overwrites words a slow rank has not read yet: a rank finishes call
// e+1 only after every rank wrote its call-e+1 words, which each rank does
// only after finishing call e.
template <typename T>
__device__ void tp_finish(const SkinnyParams& p) {
  TpHeader* own = static_cast<TpHeader*>(p.tp_sym[p.tp_rank]);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&own->done, 1u) == (unsigned)p.tiles - 1u) {
      own->done = 0u;
      *reinterpret_cast<volatile unsigned int*>(&own->epoch) += 1u;
    }
  }
}

// One k-step chunk of a row for one lane: kLoadBytes (16 or 32) bytes = E
// 32-bit words, starting at element k; zero past K (K % 8 == 0, so a 32-byte
// chunk is full, half-full or empty). `wide` (row 32-byte aligned) allows
// one 256-bit load; otherwise 128-bit loads.
template <int E>
__device__ __forceinline__ void ld_chunk(const void* row, int k, int K, bool valid, bool wide, bool stream,
                                         uint64_t pol, uint32_t (&r)[E]) {
  const char* a = static_cast<const char*>(row) + (int64_t)k * 2;
  if constexpr (E == 8) {
    if (valid && k + 16 <= K && wide) {
      if (stream)
        asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8], %9;"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                     : "l"(a), "l"(pol));
      else
        asm volatile("ld.global.nc.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                     : "l"(a));
      return;
    }
  }
#pragma unroll
  for (int h = 0; h < E / 4; ++h) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (valid && k + 8 * (h + 1) <= K) v = stream ? ld_stream_v4(a + 16 * h, pol) : ld_act_v4(a + 16 * h);
    r[4 * h] = v.x; r[4 * h + 1] = v.y; r[4 * h + 2] = v.z; r[4 * h + 3] = v.w;
  }
}

// Registers of one load batch: UNR k-steps of two rows per weight matrix
// and of the activation row(s).
template <int NMAT, int MT, int UNR>
struct Batch {
  uint32_t w[UNR][NMAT][2][kWords];
  uint32_t x[UNR][MT][kWords];
};

// Grid = one CTA per 16-row tile (IE_SK_PERSIST = 0) or a persistent grid of
// resident CTAs that walk the tiles with a grid stride. Inside a CTA the 8
// warps split the K range of the tile; with IE_SK_PIPE each warp issues the
// loads of its next batch before the MMAs of the current one, so it always
// has loads in flight.
template <typename T, int MT, int EPI>
// (3 CTAs per SM for the one-wave QKV; 2 are kept for the deeper one-matrix
// batches and for the exchange kernel, whose whole grid must be resident)
__global__ void __launch_bounds__(kThreads, QkvOneWave<EPI, MT>::value ? 3 : ((MT == 1 && EpiTraits<EPI>::nmat == 1 && IE_SK_UNROLL_ONE > IE_SK_UNROLL) ||
                                             EPI == EPI_TP_ALLREDUCE)
                                                ? 2
                                                : (MT == 1 ? IE_SK_MINBLOCKS_MT1 : IE_SK_MINBLOCKS))
    skinny_kernel(const SkinnyParams p) {
  constexpr int NMAT = EpiTraits<EPI>::nmat;
  constexpr int NR = NMAT * MT * 4;
  constexpr int kUnroll = QkvOneWave<EPI, MT>::value ? IE_SK_UNROLL : Unroll<NMAT, MT>::value;
  __shared__ float red[kWarps][NR][32];
  __shared__ float xred[kMaxKSplit][NR][32];  // cluster split: partial tile of every CTA (in the leader)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  const T* xrow[MT];
  bool xvalid[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int m = mt * 8 + g;
    xvalid[mt] = m < p.M;
    xrow[mt] = static_cast<const T*>(p.X) + (int64_t)(xvalid[mt] ? m : 0) * p.ldx;
  }
  const int nsteps = (p.K + kStep - 1) / kStep;
  // cluster split: this CTA's share of the k-steps, then the warps' shares
  unsigned int krank = 0;
  if (p.ksplit > 1) asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(krank));
  const int c_begin = ((int)krank * nsteps) / p.ksplit;
  const int c_steps = (((int)krank + 1) * nsteps) / p.ksplit - c_begin;
  const int s_begin = c_begin + (warp * c_steps) / kWarps;
  const int s_end = c_begin + ((warp + 1) * c_steps) / kWarps;
  const uint64_t pol = policy_evict_first();

  // Programmatic dependent launch: activations (X) come from the previous
  // kernel and the outputs may be buffers it still reads, so neither is
  // touched before this wait; the next kernel may be scheduled from here.
  // With early_w the first weight batch is requested before the wait
  // (weights are never written by the kernels this one can overlap with).
  const bool early = !IE_SK_PERSIST && IE_SK_PIPE && p.early_w;
  if (!early) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  }

#if IE_SK_PERSIST
  for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x) {
#else
  {
    const int tile = p.ksplit > 1 ? (int)blockIdx.x / p.ksplit : (int)blockIdx.x;
#endif
    const T* wrow[NMAT][2];
    bool rvalid[2];
    int nidx[2];
#pragma unroll
    for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
      for (int r = 0; r < 2; ++r) wrow[mat][r] = weight_row<T, EPI>(p, tile, g + 8 * r, mat, rvalid[r], nidx[r]);

    float acc[NMAT][MT][4];
#pragma unroll
    for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mat][mt][i] = 0.f;

    auto load_w = [&](Batch<NMAT, MT, kUnroll>& b, int s) {
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int k = (s + u) * kStep + t * (kWords * 2);
        const bool kv = s + u < s_end;
#pragma unroll
        for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
          for (int r = 0; r < 2; ++r)
            ld_chunk<kWords>(wrow[mat][r], k, p.K, kv && rvalid[r], p.w_wide, true, pol, b.w[u][mat][r]);
      }
    };
    auto load_x = [&](Batch<NMAT, MT, kUnroll>& b, int s) {
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int k = (s + u) * kStep + t * (kWords * 2);
        const bool kv = s + u < s_end;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) ld_chunk<kWords>(xrow[mt], k, p.K, kv && xvalid[mt], p.x_wide, false, pol, b.x[u][mt]);
      }
    };
    auto load = [&](Batch<NMAT, MT, kUnroll>& b, int s) {
      load_w(b, s);
      load_x(b, s);
    };
    auto compute = [&](const Batch<NMAT, MT, kUnroll>& b) {
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
#pragma unroll
        for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < kWords / 2; ++j) {
              // lane's chunk e0.. of rows g / g+8 / batch row g: MMA j takes
              // k-slots (2t,2t+1) <- e[4j],e[4j+1] and (2t+8,2t+9) <- e[4j+2],e[4j+3]
              Mma<T>::run(acc[mat][mt], b.w[u][mat][0][2 * j], b.w[u][mat][1][2 * j], b.w[u][mat][0][2 * j + 1],
                          b.w[u][mat][1][2 * j + 1], b.x[u][mt][2 * j], b.x[u][mt][2 * j + 1]);
            }
    };

#if IE_SK_PIPE
    {
      Batch<NMAT, MT, kUnroll> b0, b1;
      int s = s_begin;
      if (s < s_end) load_w(b0, s);
      if (early) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
      }
      if (s < s_end) load_x(b0, s);
      while (s < s_end) {
        if (s + kUnroll < s_end) load(b1, s + kUnroll);
        compute(b0);
        s += kUnroll;
        if (s >= s_end) break;
        if (s + kUnroll < s_end) load(b0, s + kUnroll);
        compute(b1);
        s += kUnroll;
      }
    }
#else
    for (int s = s_begin; s < s_end; s += kUnroll) {
      Batch<NMAT, MT, kUnroll> b;
      load(b, s);
      compute(b);
    }
#endif

    // ---- cross-warp reduction (fixed order) ----
#pragma unroll
    for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[warp][(mat * MT + mt) * 4 + i][lane] = acc[mat][mt][i];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float sum = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) sum += red[w][(mat * MT + mt) * 4 + i][lane];
            acc[mat][mt][i] = sum;
          }
    }
    if (p.ksplit > 1) {
      // every CTA of the cluster hands its partial tile to the leader (rank 0)
      if (warp == 0) {
        const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(&xred[krank][0][lane]));
        uint32_t remote;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(base), "r"(0));
#pragma unroll
        for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote + (uint32_t)(((mat * MT + mt) * 4 + i) * 32 * 4)),
                           "f"(acc[mat][mt][i])
                           : "memory");
      }
      asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
      if (krank == 0 && warp == 0) {
#pragma unroll
        for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float sum = xred[0][(mat * MT + mt) * 4 + i][lane];
              for (int r = 1; r < p.ksplit; ++r) sum += xred[r][(mat * MT + mt) * 4 + i][lane];
              acc[mat][mt][i] = sum;
            }
      }
    }
    if (warp == 0 && krank == 0) epilogue<T, MT, EPI>(p, tile, g, t, lane, rvalid, nidx, acc);
    if constexpr (EPI == EPI_TP_ALLREDUCE) {
      if (krank == 0) tp_finish<T>(p);
    }
#if IE_SK_PERSIST
    __syncthreads();  // red is reused by the next tile
#endif
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
// Launches with programmatic stream serialization, so the kernel may start
// while its predecessor drains (see the griddepcontrol notes in the kernel).
// IE_PDL=0 in the environment turns it off (plain stream ordering).
static bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("IE_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename K, typename... Args>
static cudaError_t launch_pdl(K kernel, dim3 grid, dim3 block, cudaStream_t st, int cluster, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl && pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

static bool rows_wide(const void* base, int64_t ld) {
  return (reinterpret_cast<uintptr_t>(base) & 31u) == 0 && (ld % 16) == 0;
}

// Persistent grids: as many CTAs as fit on the device at once.
template <typename K>
static int resident_ctas(K kernel) {
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0);
  return (sms > 0 ? sms : 148) * (per_sm > 0 ? per_sm : 1);
}

// K split over a cluster (SkinnyParams::ksplit): doubled (up to 4) while
// the grid still fits twice per SM and every CTA keeps >= 1024 elements of K.
// Depends only on the tile count and K, never on M, so a row gets the same
// bits alone and in a batch. IE_SK_KSPLIT=1, 2 or 4 in the environment fixes
// the split instead (where K allows 512 elements per CTA).
static int ksplit_for(int tiles, int K) {
  static const int forced = [] {
    const char* e = getenv("IE_SK_KSPLIT");
    const int v = e ? atoi(e) : 0;
    return (v == 1 || v == 2 || v == 4) ? v : 0;
  }();
  if (IE_SK_PERSIST) return 1;
  if (forced) {
    int s = forced;
    while (s > 1 && K / s < 512) s /= 2;
    return s;
  }
  static const int slots = [] {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return 2 * (sms > 0 ? sms : 148);
  }();
  int s = 1;
  while (s < kMaxKSplit && (int64_t)tiles * s * 2 <= slots && K / (s * 2) >= 1024) s *= 2;
  return s;
}

template <typename T, int MT, int EPI>
static cudaError_t launch_variant(const SkinnyParams& p, cudaStream_t st) {
  auto kernel = skinny_kernel<T, MT, EPI>;
  int grid = p.tiles * p.ksplit;
  if constexpr (EPI == EPI_TP_ALLREDUCE) {
    // every CTA waits for the same tile of the other ranks: all must fit at once
    static const int resident = resident_ctas(kernel);
    if (grid > resident) return cudaErrorCooperativeLaunchTooLarge;
  }
#if IE_SK_PERSIST
  static const int resident = resident_ctas(kernel);
  grid = p.tiles < resident ? p.tiles : resident;
#endif
  return launch_pdl(kernel, dim3(grid), dim3(kThreads), st, p.ksplit, p.M <= pdl_max_rows(), p);
}

template <typename T, int EPI>
static cudaError_t launch_skinny_t(const SkinnyParams& p0, int tiles, cudaStream_t st) {
  SkinnyParams p = p0;
  constexpr int nmat = EpiTraits<EPI>::nmat;
  p.tiles = tiles;
  p.w_wide = rows_wide(p.W0, p.ldw) && (nmat < 2 || rows_wide(p.W1, p.ldw)) &&
             (EPI != EPI_QKV || p.n_kv_heads == 0 || (rows_wide(p.W1, p.ldw) && rows_wide(p.W2, p.ldw)));
  p.x_wide = rows_wide(p.X, p.ldx);
  p.early_w = p.M <= IE_SK_EARLY_W_MAX_M;
  p.ksplit = ksplit_for(tiles, p.K);
  if (p.M <= 8) return launch_variant<T, 1, EPI>(p, st);
  return launch_variant<T, 2, EPI>(p, st);
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
    case EPI_STORE_F32: return launch_skinny_t<T, EPI_STORE_F32>(p, tiles, st); \
    case EPI_TP_ALLREDUCE: return launch_skinny_t<T, EPI_TP_ALLREDUCE>(p, tiles, st); \
  }
  if (dt == IE_DTYPE_F16) { IE_SK(__half) }
  else { IE_SK(__nv_bfloat16) }
#undef IE_SK
  return cudaErrorInvalidValue;
}

cudaError_t set_skinny_wait_ns(unsigned long long ns) {
  return cudaMemcpyToSymbol(g_skinny_wait_ns, &ns, sizeof(ns));
}

int read_skinny_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_skinny_status, sizeof(int)) != cudaSuccess) return IE_ERR_LAUNCH;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_skinny_status, &z, sizeof(int));
  }
  return v;
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
