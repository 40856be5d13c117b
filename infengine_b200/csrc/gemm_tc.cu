// Prefill-path GEMM (M > 16): D[M,N] = A[M,K] . B[N,K]^T on the sm_100a
// tensor cores (tcgen05.mma kind::f16, fp32 accumulation in TMEM), fed by TMA.
//
// Roofline: at M = 2048 every projection of the hot path is compute-bound
// (arithmetic intensity 1000+ FLOP/byte); the bound is the dense bf16
// tensor-core peak. Algorithmic FLOPs per launch = 2*M*N*K.
//
// Design (one persistent CTA per SM, 192 threads, ~194 KB shared memory):
//   warp 0, one lane  — TMA producer: per 64-wide k-block it loads the
//                       128x64 activation tile and two 128x64 weight tiles
//                       (128-byte swizzle) into a 4-stage ring;
//   warp 1, one lane  — MMA issuer: four tcgen05.mma (M=128, N=256, K=16)
//                       per k-block into one of two TMEM accumulators
//                       (2 x 256 fp32 columns = all 512 TMEM columns), and
//                       tcgen05.commit to release ring stages / publish
//                       finished accumulators;
//   warps 2..5        — epilogue: tcgen05.ld of the accumulator (thread =
//                       output row), the fused epilogue, global stores; the
//                       double-buffered accumulator lets the epilogue of one
//                       tile overlap the main loop of the next.
// The two 128-row weight tiles of a stage are independent TMA loads, which is
// what lets the fused epilogues pair rows from different matrices:
//   SWIGLU — gate rows [n0,n0+128) next to up rows [n0,n0+128);
//   QKV    — two heads per tile, each taken from Wq, Wk or Wv;
//   ARGMAX — 256 consecutive vocabulary rows.
// No TMA multicast and no clusters: every load reads this GPU's own memory.
//
// Tail split (a separate instantiation, SPLIT = true, used when the caller
// passes a workspace). With W tiles on G persistent CTAs the last wave holds
// R = W mod G tiles and leaves G - R SMs idle (O and down at M = 2048: 256
// tiles, 108 in the second wave of 148). The SPLIT kernel runs the first
// W - R tiles whole, exactly as above, then splits each of the R tail tiles
// into s ranges of k-blocks, numbered split-major (unit j * R + r is range j
// of tail tile r), so that in every round all CTAs stream the same k-slices
// of the operands (L2 sharing stays as in the whole-tile waves). Ranges
// 0 .. s-2 store their fp32 partial tile in the workspace and count it on a
// per-(tile, warp quarter) flag; range s-1 waits (bounded) for its flag,
// adds the partials in range order, then its own accumulator, and runs the
// fused epilogue on the sum. A unit only waits for units with a lower index,
// which no CTA reaches after a higher one, so the waits cannot form a cycle.
// The summation order is fixed: results are deterministic (their last bits
// differ from the whole-tile kernel's). The host picks s per shape from a
// wave count plus the fix-up reads (plan_split), for the shapes where the
// split measured faster (see launch_tc_gemm).
//
// Every mbarrier wait is bounded by the global timer; a wait that gives up
// records IE_ERR_TIMEOUT in a device status word (ie_device_status()), makes
// every role leave its loop, drains the copies and MMAs the CTA issued and
// frees its TMEM before the CTA exits.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include "ie_common.cuh"
#include "gemm_tc.cuh"
#include "tc_ptx.cuh"

namespace ie {

__device__ int g_tc_status = 0;
// limit of one mbarrier wait (ie_set_wait_limit_ns)
__device__ unsigned long long g_tc_wait_ns = kDefaultWaitNs;

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_TILE = BM * BK * 2;     // 16 KB
constexpr int B_HALF = 128 * BK * 2;    // 16 KB
constexpr int STAGE_BYTES = A_TILE + 2 * B_HALF;
constexpr int TILE_BYTES = STAGES * STAGE_BYTES;  // 192 KB
constexpr int SMEM_BYTES = TILE_BYTES + 1024 + 256;
constexpr int THREADS = 192;
constexpr int kMaxSplit = 4;  // k-ranges per split tile (the fix-up holds s - 1 partial chunks)
constexpr uint32_t TMEM_COLS = 512;

struct TcArgs {
  CUtensorMap tmA;
  CUtensorMap tmB[3];
  TcGemmParams p;
  int nm, nn, nk;
  int heads;  // QKV: n_q_heads + 2 * n_kv_heads
  // tail split (SPLIT kernel): whole tiles [0, split_F * gridDim.x), then
  // split_R tiles in split_s k-ranges each
  int split_s, split_F, split_R;
};

// One unit of a CTA's work: tile `tile`, k-blocks [k0, k1); j = -1 for a
// whole tile, else k-range j of tail tile r.
struct Unit {
  int tile, k0, k1, j, r;
};
// The q-th unit of this CTA (false when it has no more).
template <bool SPLIT>
__device__ __forceinline__ bool unit_at(const TcArgs& a, int q, Unit& u) {
  const int v = (int)blockIdx.x + q * (int)gridDim.x;
  if constexpr (!SPLIT) {
    if (v >= a.nm * a.nn) return false;
    u.tile = v; u.k0 = 0; u.k1 = a.nk; u.j = -1; u.r = 0;
    return true;
  } else {
    const int whole = a.split_F * (int)gridDim.x;
    if (v < whole) {
      u.tile = v; u.k0 = 0; u.k1 = a.nk; u.j = -1; u.r = 0;
      return true;
    }
    const int w = v - whole;
    if (w >= a.split_R * a.split_s) return false;
    u.j = w / a.split_R;
    u.r = w - u.j * a.split_R;
    u.tile = whole + u.r;
    u.k0 = u.j * a.nk / a.split_s;
    u.k1 = (u.j + 1) * a.nk / a.split_s;
    return true;
  }
}

// ------------------------------------------------------------ PTX helpers
using namespace tc;
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  return tc::mbar_wait(bar, parity, abort_flag, &g_tc_status, &g_tc_wait_ns);
}
template <typename T>
__device__ __forceinline__ uint32_t idesc_f16() {
  return tc::idesc_f16<T>(BM, BN);
}
// Lane 0 waits (bounded) until *f reaches target, with acquire ordering at
// GPU scope; the warp then continues together. False on timeout or abort.
__device__ __forceinline__ bool wait_count(const unsigned int* f, unsigned int target, volatile int* abort_flag,
                                           int lane) {
  int ok = 1;
  if (lane == 0) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (v < target) {
      const unsigned long long limit = g_tc_wait_ns;
      const unsigned long long t0 = globaltimer();
      while (true) {
        if (*abort_flag) { ok = 0; break; }
        __nanosleep(64);
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        if (v >= target) break;
        if (globaltimer() - t0 > limit) {
          atomicExch(&g_tc_status, IE_ERR_TIMEOUT);
          *abort_flag = 1;
          ok = 0;
          break;
        }
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}
// 32 entries of a RoPE table row (position pos, dimensions 32c .. 32c+31) as
// 16-byte vectors (tables are 16-byte aligned, rows 256 bytes).
__device__ __forceinline__ void load_rope32(const float* cos_t, const float* sin_t, int pos, int c, float (&cs)[32],
                                            float (&sn)[32]) {
  const float4* cp = reinterpret_cast<const float4*>(cos_t + (int64_t)pos * 64 + c * 32);
  const float4* sp = reinterpret_cast<const float4*>(sin_t + (int64_t)pos * 64 + c * 32);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 a4 = __ldg(cp + j), b4 = __ldg(sp + j);
    cs[4 * j] = a4.x; cs[4 * j + 1] = a4.y; cs[4 * j + 2] = a4.z; cs[4 * j + 3] = a4.w;
    sn[4 * j] = b4.x; sn[4 * j + 1] = b4.y; sn[4 * j + 2] = b4.z; sn[4 * j + 3] = b4.w;
  }
}

// Partial tile in the workspace (128 x 256 fp32 = 128 KB), laid out as
// [32-column chunk c][float4 group i of the chunk][row][4]: the 32 rows of an
// epilogue warp then read or write 512 contiguous bytes per access. Accessed
// through L2 only (other SMs write and read it).
__device__ __forceinline__ void store32_part(float* slot, int row, int c, const float (&v)[32]) {
  float4* q = reinterpret_cast<float4*>(slot) + (size_t)c * 8 * BM + row;
#pragma unroll
  for (int i = 0; i < 8; ++i) __stcg(q + i * BM, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
}
__device__ __forceinline__ void load32_part(const float* slot, int row, int c, float (&v)[32]) {
  const float4* q = reinterpret_cast<const float4*>(slot) + (size_t)c * 8 * BM + row;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 x = __ldcg(q + i * BM);
    v[4 * i] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
  }
}

// Store 32 consecutive values of one output row (columns col0.. col0+31,
// those < ncols), 16-byte vectors when the whole chunk is in range.
// With `add`, the stored value is round(old + round(v)) (residual add).
template <typename T>
__device__ __forceinline__ void store_row32(T* dst, int col0, int ncols, const float (&v)[32], bool add = false) {
  if (col0 + 32 <= ncols) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 pk, old;
      if (add) old = *reinterpret_cast<const uint4*>(dst + col0 + j * 8);
      const T* o = reinterpret_cast<const T*>(&old);
      T* e = reinterpret_cast<T*>(&pk);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        e[i] = DT<T>::from_f(add ? DT<T>::to_f(o[i]) + round_to<T>(v[j * 8 + i]) : v[j * 8 + i]);
      *reinterpret_cast<uint4*>(dst + col0 + j * 8) = pk;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < ncols)
        dst[col0 + i] = DT<T>::from_f(add ? DT<T>::to_f(dst[col0 + i]) + round_to<T>(v[i]) : v[i]);
  }
}

// 32 fp32 values of one output row (tensor-parallel partial sums).
__device__ __forceinline__ void store_row32_f32(float* dst, int col0, int ncols, const float (&v)[32]) {
  if (col0 + 32 <= ncols) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float4*>(dst + col0 + j * 4) = make_float4(v[j * 4], v[j * 4 + 1], v[j * 4 + 2], v[j * 4 + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < ncols) dst[col0 + i] = v[i];
  }
}

// Which weight map / row feeds B half h of column block nb.
template <int EPI>
__device__ __forceinline__ void b_source(const TcArgs& a, int nb, int h, int& map, int& row) {
  if constexpr (EPI == TC_EPI_SWIGLU) {
    map = h;
    row = nb * 128;
  } else if constexpr (EPI == TC_EPI_QKV) {
    int head = 2 * nb + h;
    if (head >= a.heads) head = 2 * nb;  // odd head count: reload, result unused
    if (head < a.p.n_q_heads) { map = 0; row = head * 128; }
    else if (head < a.p.n_q_heads + a.p.n_kv_heads) { map = 1; row = (head - a.p.n_q_heads) * 128; }
    else { map = 2; row = (head - a.p.n_q_heads - a.p.n_kv_heads) * 128; }
  } else {
    map = 0;
    row = nb * BN + h * 128;
    // a half that lies wholly past the last weight row (N within 128 of the
    // last tile's start) reloads the first half: those columns are not stored
    if (row >= a.p.N) row = nb * BN;
  }
}

template <typename T, int EPI, bool SPLIT>
__global__ void __launch_bounds__(THREADS, 1) tc_gemm_kernel(const __grid_constant__ TcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TILE_BYTES);
  // bars: full[0..S), empty[S..2S), acc_full[2S..2S+2), acc_empty[2S+2..2S+4), drain[2S+4]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* issued_p = reinterpret_cast<int*>(tmem_holder + 2);
  int* consumed_p = reinterpret_cast<int*>(tmem_holder + 3);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const TcGemmParams& p = args.p;
  const int num_tiles = args.nm * args.nn;
  (void)num_tiles;

  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  auto accf_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + a); };
  auto acce_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + 2 + a); };
  const uint32_t drain_bar = smem_u32(bars + 2 * STAGES + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(accf_bar(a), 1);
      mbar_init(acce_bar(a), 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *issued_p = 0;
    *consumed_p = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&args.tmA)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_holder;

  // Activations come from the previous kernel in the stream; outputs may be
  // buffers it still reads.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      Unit u;
      for (int q = 0; !*abort_flag && unit_at<SPLIT>(args, q, u); ++q) {
        const int mb = u.tile % args.nm, nb = u.tile / args.nm;
        for (int kb = u.k0; kb < u.k1; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag)) break;
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          mbar_expect_tx(full_bar(stage), STAGE_BYTES);
          tma_load_2d(sa, &args.tmA, full_bar(stage), kb * BK, mb * BM);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            int map, row;
            b_source<EPI>(args, nb, h, map, row);
            tma_load_2d(sa + A_TILE + h * B_HALF, &args.tmB[map], full_bar(stage), kb * BK, row);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      *issued_p = issued;
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_f16<T>();
      int stage = 0, consumed = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool issued_any = false;
      Unit u;
      for (int q = 0; !*abort_flag && unit_at<SPLIT>(args, q, u); ++q) {
        if (!mbar_wait(acce_bar(acc), acc_phase ^ 1, abort_flag)) break;
        fence_after();
        const uint32_t d_tmem = tmem + acc * BN;
        bool ok = true;
        for (int kb = u.k0; kb < u.k1; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag)) { ok = false; break; }
          fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint64_t adesc = sw128_desc(sa), bdesc = sw128_desc(sa + A_TILE);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb != u.k0 || k != 0) ? 1u : 0u);
          mma_commit(empty_bar(stage));
          issued_any = true;
          ++consumed;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(accf_bar(acc));
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      *consumed_p = consumed;
      if (*abort_flag && issued_any) {
        // let every MMA this thread issued finish before TMEM is released
        mma_commit(drain_bar);
        const unsigned long long t0 = globaltimer();
        while (!mbar_try(drain_bar, 0) && globaltimer() - t0 < kDrainWaitNs) {
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------- epilogue warps
    const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
    const int row = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    Unit u;
    for (int q = 0; !*abort_flag && unit_at<SPLIT>(args, q, u); ++q) {
      const int mb = u.tile % args.nm, nb = u.tile / args.nm;
      const int m = mb * BM + row;
      const bool mvalid = m < p.M;
      // QKV: this row's position and the first half of its RoPE table rows
      // (shared by the tile's two heads) are fetched while the MMAs run
      int qpos = 0;
      bool qrow_ok = mvalid;
      float rcos[32], rsin[32];
      if constexpr (EPI == TC_EPI_QKV) {
        qpos = p.pos0 + m;
        if (p.positions && mvalid) {
          qpos = p.positions[m];
          if (qpos < 0 || qpos >= p.cache_rows) {
            atomicExch(&g_tc_status, IE_ERR_INVALID_ARG);
            qrow_ok = false;
            qpos = 0;
          }
        }
        if (p.rope_cos && qrow_ok) load_rope32(p.rope_cos, p.rope_sin, qpos, 0, rcos, rsin);
      }
      if (!mbar_wait(accf_bar(acc), acc_phase, abort_flag)) break;
      fence_after();
      const uint32_t tbase = tmem + acc * BN + ((uint32_t)(quad * 32) << 16);
      float v[32];
      // tail split: ranges 0 .. s-2 hand their partial sums to range s-1
      bool producer = false;
      const float* parts = nullptr;  // range s-1: the tile's first partial
      unsigned int* flag = nullptr;
      if constexpr (SPLIT) {
        if (u.j >= 0) {
          flag = p.split_flags + u.r * 4 + quad;
          if (u.j < args.split_s - 1) {
            producer = true;
          } else {
            if (!wait_count(flag, (unsigned)(args.split_s - 1), abort_flag, lane)) break;
            parts = p.split_ws + (size_t)u.r * (args.split_s - 1) * BM * BN;
          }
        }
      }
      // 32 accumulator columns from col: with partials, sum = p_0 + ... +
      // p_{s-2} + own, in that order
      auto acc_ld = [&](int col, float (&x)[32]) {
        tmem_ld32(tbase + col, x);
        if constexpr (SPLIT) {
          if (parts) {
            // all partials of the chunk requested together (s <= kMaxSplit),
            // then added in range order
            const int np = args.split_s - 1;
            float p0[32], p1[32], p2[32];
            load32_part(parts, row, col >> 5, p0);
            if (np > 1) load32_part(parts + (size_t)BM * BN, row, col >> 5, p1);
            if (np > 2) load32_part(parts + (size_t)2 * BM * BN, row, col >> 5, p2);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              float sum = p0[i];
              if (np > 1) sum += p1[i];
              if (np > 2) sum += p2[i];
              x[i] = sum + x[i];
            }
          }
        }
      };
      if (producer) {
        float* slot = p.split_ws + (size_t)(u.r * (args.split_s - 1) + u.j) * BM * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(tbase + c * 32, v);
          store32_part(slot, row, c, v);
        }
        __syncwarp();
        if (lane == 0) {
          __threadfence();
          atomicAdd(flag, 1u);
        }
      } else if constexpr (EPI == TC_EPI_STORE_F32) {
        float* drow = static_cast<float*>(p.D) + (int64_t)m * p.ldd;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          acc_ld(c * 32, v);
          if (mvalid) store_row32_f32(drow, nb * BN + c * 32, p.N, v);
        }
      } else if constexpr (EPI == TC_EPI_STORE) {
        T* drow = static_cast<T*>(p.D) + (int64_t)m * p.ldd;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          acc_ld(c * 32, v);
          if (mvalid) store_row32<T>(drow, nb * BN + c * 32, p.N, v, p.residual);
        }
      } else if constexpr (EPI == TC_EPI_SWIGLU) {
        T* drow = static_cast<T*>(p.D) + (int64_t)m * p.ldd;
        float uu[32];
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          acc_ld(c * 32, v);
          acc_ld(128 + c * 32, uu);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float gv = round_to<T>(v[i]), uv = round_to<T>(uu[i]);
            v[i] = gv * (1.0f / (1.0f + expf(-gv))) * uv;
          }
          if (mvalid) store_row32<T>(drow, nb * 128 + c * 32, p.N, v);
        }
      } else if constexpr (EPI == TC_EPI_QKV) {
        // the tile's two heads (the second absent for an odd head count)
        T* dsth[2] = {nullptr, nullptr};
        bool ropeh[2] = {false, false};
        const int64_t cb = p.positions ? (int64_t)m * p.cache_batch_stride : 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int head = 2 * nb + h;
          if (head >= args.heads) continue;
          if (head < p.n_q_heads) {
            dsth[h] = static_cast<T*>(p.q_out) + (int64_t)head * p.q_head_stride + (int64_t)m * 128;
            ropeh[h] = p.rope_cos != nullptr;
          } else if (head < p.n_q_heads + p.n_kv_heads) {
            dsth[h] = static_cast<T*>(p.k_cache) + cb + (int64_t)(head - p.n_q_heads) * p.cache_head_stride +
                      (int64_t)qpos * 128;
            ropeh[h] = p.rope_cos != nullptr;
          } else {
            dsth[h] = static_cast<T*>(p.v_cache) + cb +
                      (int64_t)(head - p.n_q_heads - p.n_kv_heads) * p.cache_head_stride + (int64_t)qpos * 128;
          }
        }
        float b[32];
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          // this row's 32 table entries of dimension chunk c (chunk 0 was
          // fetched before the accumulator wait), for both heads
          if (c == 1 && p.rope_cos && qrow_ok) load_rope32(p.rope_cos, p.rope_sin, qpos, 1, rcos, rsin);
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            if (!dsth[h]) break;
            acc_ld(h * 128 + c * 32, v);       // d in [32c, 32c+32)
            acc_ld(h * 128 + 64 + c * 32, b);  // d + 64
            const bool rope = ropeh[h] && qrow_ok;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              float x0 = round_to<T>(v[i]), x1 = round_to<T>(b[i]);
              if (rope) {
                const float y0 = x0 * rcos[i] - x1 * rsin[i];
                const float y1 = x0 * rsin[i] + x1 * rcos[i];
                x0 = y0;
                x1 = y1;
              }
              v[i] = x0;
              b[i] = x1;
            }
            if (qrow_ok) {
              store_row32<T>(dsth[h], c * 32, 128, v);
              store_row32<T>(dsth[h], 64 + c * 32, 128, b);
            }
          }
        }
      } else if constexpr (EPI == TC_EPI_ARGMAX) {
        T* drow = p.D ? static_cast<T*>(p.D) + (int64_t)m * p.ldd : nullptr;
        unsigned long long best = 0ull;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          acc_ld(c * 32, v);
          const int col0 = nb * BN + c * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v[i] = round_to<T>(v[i]);
            if (col0 + i < p.N) {
              const unsigned long long k = argmax_key(v[i], p.vocab_offset + col0 + i);
              best = k > best ? k : best;
            }
          }
          if (mvalid && drow) store_row32<T>(drow, col0, p.N, v);
        }
        if (mvalid && best) atomicMax(p.keys + m, best);
      }
      if constexpr (SPLIT) {
        if (parts) {  // partials read: lower the flag for the next call
          __syncwarp();
          if (lane == 0) *flag = 0u;
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar(acc));
      if constexpr (EPI == TC_EPI_ARGMAX) {
        // each epilogue warp counts its own part of the tile after its
        // atomics; the warp that brings the count to 4 * tiles finalizes
        if (lane == 0 && !producer) {
          __threadfence();
          if (atomicAdd(p.counter, 1u) == 4u * (unsigned)num_tiles - 1u) {
            __threadfence();
            for (int r = 0; r < p.M; ++r) {
              const unsigned long long k = atomicExch(p.keys + r, 0ull);
              if (p.idx_out) p.idx_out[r] = argmax_key_index(k);
              if (p.key_out) p.key_out[r] = k;
            }
            atomicExch(p.counter, 0u);
          }
        }
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  // ---------------------------------------------------------- teardown
  fence_before();
  __syncthreads();
  fence_after();
  if (*abort_flag && threadIdx.x == 0) {
    // wait for TMA copies that were issued but never consumed
    const int issued = *issued_p, consumed = *consumed_p;
    for (int i = consumed; i < issued; ++i) {
      const unsigned long long t0 = globaltimer();
      while (!mbar_try(full_bar(i % STAGES), (uint32_t)((i / STAGES) & 1)) && globaltimer() - t0 < kDrainWaitNs / 4) {
      }
    }
  }
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

// --------------------------------------------------------------- host side
// 2-D K-major tensor map: rows x K elements, row stride ld elements, box of
// 64 x box_rows elements, 128-byte swizzle, zero fill outside the tensor.
bool make_map(CUtensorMap* map, ie_dtype dt, const void* base, int rows, int K, int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapDataType t = dt == IE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, t, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <typename T, int EPI, bool SPLIT>
int launch_t(TcArgs& a, cudaStream_t st) {
  static bool configured = false;
  auto kernel = tc_gemm_kernel<T, EPI, SPLIT>;
  if (!configured) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
      return IE_ERR_LAUNCH;
    configured = true;
  }
  const int tiles = a.nm * a.nn;
  cudaLaunchConfig_t cfg = {};
  // the split plan assumes one persistent CTA per SM
  cfg.gridDim = dim3(SPLIT ? sm_count() : (tiles < sm_count() ? tiles : sm_count()));
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, a);
  if (e != cudaSuccess) {
    std::fprintf(stderr, "infengine_b200: tcgen05 GEMM launch failed: %s\n", cudaGetErrorString(e));
    return IE_ERR_LAUNCH;
  }
  return IE_OK;
}

template <typename T, bool SPLIT>
int dispatch(TcArgs& a, int epi, cudaStream_t st) {
  switch (epi) {
    case TC_EPI_STORE: return launch_t<T, TC_EPI_STORE, SPLIT>(a, st);
    case TC_EPI_SWIGLU: return launch_t<T, TC_EPI_SWIGLU, SPLIT>(a, st);
    case TC_EPI_QKV: return launch_t<T, TC_EPI_QKV, SPLIT>(a, st);
    case TC_EPI_ARGMAX: return launch_t<T, TC_EPI_ARGMAX, SPLIT>(a, st);
    case TC_EPI_STORE_F32: return launch_t<T, TC_EPI_STORE_F32, SPLIT>(a, st);
  }
  return IE_ERR_UNSUPPORTED;
}

// Split of the last wave's tiles (SPLIT kernel): s k-ranges for each of the
// R = W mod G tail tiles, or s = 1 (whole-tile kernel). In tile-times of
// the tail, whole tiles cost 1; s ranges in ceil(R s / G) rounds cost
// rounds / s, plus the hand-off at the end of the kernel: the partial stores
// and the last range's chunk-by-chunk reads of the others' partials, each
// chunk one L2 round trip (~3-4 us in all on B200, against ~0.43 us of MMAs
// per k-block, hence 8 / nk tile-times). Ranges keep at least 4 k-blocks so
// the 4-stage ring fills; the workspace bounds R (s - 1). IE_TC_SPLIT_MAX in
// the environment lowers the largest s (1 turns the split off).
int split_max() {
  static const int v = [] {
    const char* e = getenv("IE_TC_SPLIT_MAX");
    const int x = e ? atoi(e) : kMaxSplit;
    return x < 1 ? 1 : (x > kMaxSplit ? kMaxSplit : x);
  }();
  return v;
}
struct SplitPlan {
  int s = 1, F = 0, R = 0;
};
SplitPlan plan_split(int tiles, int nk, int G, long long slots_cap) {
  SplitPlan best;
  if (tiles <= 0 || G <= 0) return best;
  const int F = tiles / G, R = tiles - F * G;
  if (R == 0) return best;
  double best_cost = 1.0;
  for (int s = 2; s <= split_max(); ++s) {
    if (nk / s < 4) break;
    if ((long long)R * (s - 1) > slots_cap) break;
    const int rounds = (R * s + G - 1) / G;
    const double cost = (double)rounds / s + 8.0 / nk;
    if (cost < best_cost - 0.02) {
      best_cost = cost;
      best.s = s;
    }
  }
  if (best.s > 1) {
    best.F = F;
    best.R = R;
  }
  return best;
}

}  // namespace

int launch_tc_gemm(ie_dtype dt, const TcGemmParams& p, cudaStream_t st) {
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return IE_OK;
  TcArgs a;
  memset(&a, 0, sizeof(a));
  a.p = p;
  a.nm = ceil_div(p.M, BM);
  a.nk = ceil_div(p.K, BK);
  if (!make_map(&a.tmA, dt, p.A, p.M, p.K, p.lda, BM)) return IE_ERR_UNSUPPORTED;
  switch (p.epi) {
    case TC_EPI_STORE:
    case TC_EPI_STORE_F32:
    case TC_EPI_ARGMAX:
      a.nn = ceil_div(p.N, BN);
      if (!make_map(&a.tmB[0], dt, p.B, p.N, p.K, p.ldb, 128)) return IE_ERR_UNSUPPORTED;
      break;
    case TC_EPI_SWIGLU:
      a.nn = ceil_div(p.N, 128);
      if (!make_map(&a.tmB[0], dt, p.B, p.N, p.K, p.ldb, 128) || !make_map(&a.tmB[1], dt, p.B2, p.N, p.K, p.ldb, 128))
        return IE_ERR_UNSUPPORTED;
      break;
    case TC_EPI_QKV:
      a.heads = p.n_q_heads + 2 * p.n_kv_heads;
      a.nn = ceil_div(a.heads, 2);
      if (!make_map(&a.tmB[0], dt, p.B, p.n_q_heads * 128, p.K, p.ldb, 128)) return IE_ERR_UNSUPPORTED;
      if (p.n_kv_heads > 0) {
        if (!make_map(&a.tmB[1], dt, p.B2, p.n_kv_heads * 128, p.K, p.ldb, 128) ||
            !make_map(&a.tmB[2], dt, p.B3, p.n_kv_heads * 128, p.K, p.ldb, 128))
          return IE_ERR_UNSUPPORTED;
      } else {
        a.tmB[1] = a.tmB[2] = a.tmB[0];
      }
      break;
    default:
      return IE_ERR_UNSUPPORTED;
  }
  a.split_s = 1;
  // Where the split pays, measured on B200 (per-layer times over 32 layers'
  // weights): plain-store GEMMs whose tiles fill less than one wave (M = 128:
  // O 29.6 -> 22.2 us, down 91.1 -> 40.7 us) or whose K is long enough to
  // amortise the hand-off (down at M = 2048: about -5 %). It did not pay for
  // the QKV and SwiGLU epilogues (QKV at M = 2048: 91 -> 98 us) nor for
  // K = 4096 over more than one wave (O at M = 2048: 55 -> 68 us).
  const bool split_shape = p.epi != TC_EPI_QKV && p.epi != TC_EPI_SWIGLU &&
                           (a.nm * a.nn < sm_count() || a.nk >= 128);
  if (split_shape && p.split_ws && p.split_flags && p.split_slots > 0) {
    const SplitPlan sp = plan_split(a.nm * a.nn, a.nk, sm_count(), p.split_slots);
    a.split_s = sp.s;
    a.split_F = sp.F;
    a.split_R = sp.R;
  }
  if (a.split_s > 1)
    return dt == IE_DTYPE_BF16 ? dispatch<__nv_bfloat16, true>(a, p.epi, st) : dispatch<__half, true>(a, p.epi, st);
  return dt == IE_DTYPE_BF16 ? dispatch<__nv_bfloat16, false>(a, p.epi, st) : dispatch<__half, false>(a, p.epi, st);
}

// Workspace of the tail split: per-(tile, warp quarter) flags for up to one
// wave of tail tiles, then the partial tiles (128 x 256 fp32 each), room for
// three waves of them.
size_t split_flags_bytes() { return ((size_t)sm_count() * 4 * sizeof(unsigned int) + 255) / 256 * 256; }
size_t split_workspace_bytes() { return split_flags_bytes() + (size_t)3 * sm_count() * BM * BN * sizeof(float); }

int attach_split_workspace(TcGemmParams& q, void* ws, size_t bytes) {
  if (!ws) return IE_OK;  // no workspace: whole tiles
  if (reinterpret_cast<uintptr_t>(ws) & 255u) return IE_ERR_ALIGNMENT;
  const size_t fb = split_flags_bytes();
  if (bytes < fb + (size_t)BM * BN * sizeof(float)) return IE_ERR_WORKSPACE;
  q.split_flags = static_cast<unsigned int*>(ws);
  q.split_ws = reinterpret_cast<float*>(static_cast<char*>(ws) + fb);
  q.split_slots = (long long)((bytes - fb) / ((size_t)BM * BN * sizeof(float)));
  return IE_OK;
}

cudaError_t set_tc_wait_ns(unsigned long long ns) {
  return cudaMemcpyToSymbol(g_tc_wait_ns, &ns, sizeof(ns));
}

int read_tc_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int)) != cudaSuccess) return IE_ERR_LAUNCH;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_tc_status, &z, sizeof(int));
  }
  return v;
}

}  // namespace ie
