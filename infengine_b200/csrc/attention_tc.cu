// Prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA = 128 query rows of one query head (GQA: the K/V rows of head
// h / group); key blocks of 128 positions up to the causal limit. Two passes
// over the key blocks, so that the softmax uses the exact row maximum the
// reference uses (kernels/softmax.cu:55-103) and never rescales an
// accumulator:
//   pass 1: S = Q K^T (tcgen05.mma 128x128x128, fp32 in TMEM) -> the row
//           maximum of the raw scores over the causal keys; rounding and the
//           positive scale are monotone, so max t = round(round(max s) * scale)
//           for t = round(round(s) * rsqrt(128));
//   pass 2: S again -> t -> e = exp(t - m) (fp32, summed into l), p = round(e)
//           -> O += P V;
//   out = round(O / l).
// exp is 2^(t*log2(e) - m*log2(e)) on the special-function unit (ex2.approx,
// relative error about 2^-22, plus one fp32 rounding of the exponent), where
// the reference calls expf; the reference also rounds p after the division
// by the sum, while here the division follows the P.V accumulation. Outputs
// therefore differ from the chain by about a rounding step of p (tests bound
// it). Deterministic: no atomics, fixed summation order.
//
// Operands. The A operands live in tensor memory, so shared memory only holds
// K and V (its bandwidth, shared by the TMA writes and the tensor cores'
// operand reads, is what limits this kernel): Q is copied once into TMEM
// columns [384, 448) (row = lane, two 16-bit values per 32-bit column, the
// lower-indexed one in the low half), and each P block is written by the
// softmax into the S buffer it was computed from — key half k of the row
// into the first 32 columns of the 64 it read, so the two warps that share a
// row never touch each other's columns. K is the K-major B operand of Q K^T,
// V the MN-major B operand of P V straight from its TMA tile (no transpose).
// TMEM: S0 [0,128), S1 [128,256), O [256,384), Q [384,448).
//
// Warp roles (320 threads): warp 0 = TMA producer (the K / V tiles in the
// order the MMAs use them, through a 6-stage ring), warp 1 = MMA issuer (one
// elected thread), warps 2-9 = softmax and epilogue: TMEM lane = query row,
// warp w reads lane quarter w & 3 and key half (w - 2) >> 2 of each block, so
// each scheduler holds two of them; the halves of a row meet once, in shared
// memory, for the row maximum and for the sum. An S buffer is released by
// the softmax warps in pass 1 (after they loaded it) and by the commit of the
// P.V that read its P in pass 2. Every mbarrier wait is bounded (2 s): on
// expiry IE_ERR_TIMEOUT is recorded, every role leaves its loop, the MMAs and
// copies in flight are drained and the TMEM is freed before the CTA exits.
#include <cstdio>
#include <cstring>
#include "ie_common.cuh"
#include "attention.cuh"
#include "tc_ptx.cuh"

namespace ie {

__device__ int g_tca_status = 0;
// limit of one mbarrier wait (ie_set_wait_limit_ns)
__device__ unsigned long long g_tca_wait_ns = kDefaultWaitNs;

namespace {

using namespace tc;

constexpr int kBM = 128, kBN = 128, kD = 128;
constexpr int kStages = 6;
constexpr int kTile = kBN * kD * 2;          // one K or V tile: two 64-column boxes, 32 KB
constexpr int kHalf = kTile / 2;             // 16 KB
constexpr int kSoftThreads = 256;            // 8 softmax / epilogue warps
constexpr int kThreads = 64 + kSoftThreads;  // + TMA warp + MMA warp
constexpr int kSBufs = 2;                    // S (then P) buffers in TMEM
constexpr int kOCol = kSBufs * kBN;          // O accumulator columns [256, 384)
constexpr int kQCol = kOCol + kD;            // Q (A operand of Q K^T), 64 columns
constexpr uint32_t kTmemCols = 512;
// smem: K/V ring | cross-half row exchange | barriers
constexpr int kOffRed = kStages * kTile;
constexpr int kOffBars = kOffRed + 2 * kBM * 4;
constexpr int kSmem = kOffBars + 256 + 1024;  // + alignment slack
static_assert(kSmem <= 227 * 1024, "shared memory per CTA");

struct TcaArgs {
  CUtensorMap tmK, tmV;  // 3-D (dim, row, head), boxes 64 x 128 x 1, 128-byte swizzle
  const void* q;         // [heads][S][128]
  int64_t q_head_stride;
  int S, pos0, group;
  float scale;
  void* out;
  int64_t ld_out;
};

__device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  return tc::mbar_wait(bar, parity, abort_flag, &g_tca_status, &g_tca_wait_ns);
}

// two fp32 values rounded to T (to nearest even) and packed, lo in bits 0-15
template <typename T>
__device__ __forceinline__ uint32_t pack2_rn(float lo, float hi) {
  uint32_t r;
  if constexpr (DT<T>::id == IE_DTYPE_BF16)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
template <typename T>
__device__ __forceinline__ float lo_f(uint32_t r) {
  if constexpr (DT<T>::id == IE_DTYPE_BF16) return __uint_as_float(r << 16);
  else return __half2float(__ushort_as_half((unsigned short)(r & 0xFFFFu)));
}
template <typename T>
__device__ __forceinline__ float hi_f(uint32_t r) {
  if constexpr (DT<T>::id == IE_DTYPE_BF16) return __uint_as_float(r & 0xFFFF0000u);
  else return __half2float(__ushort_as_half((unsigned short)(r >> 16)));
}
__device__ __forceinline__ float ex2(float x) {  // 2^x (MUFU; 2^-inf = 0)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 64 consecutive fp32 columns of this warp's 32 TMEM lanes (load and wait in
// one statement, so no use of the values can be scheduled before the wait).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]),
        "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]),
        "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]),
        "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]),
        "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes from registers;
// waits until the stores are done.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// D (TMEM) (+)= A (TMEM, K-major) . B (shared memory descriptor)
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                       uint32_t accum) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) tc_attention_kernel(const __grid_constant__ TcaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  // bars: full[kStages] empty[kStages] q_full s_full[2] s_rel_sm[2] s_rel_mma[2]
  // p_full[2] o_full drain
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* issued_p = reinterpret_cast<int*>(tmem_holder + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (query heads, query blocks): the hardware starts CTAs in linear
  // order, so the heaviest (causal) query blocks go first
  const int qb = gridDim.y - 1 - blockIdx.y;
  const int h = blockIdx.x, hk = h / a.group;
  const int q0 = qb * kBM;
  const int last_pos = a.pos0 + min(q0 + kBM, a.S) - 1;
  const int nkb = last_pos / kBN + 1;  // key blocks this query block needs
  const int n_tiles = 3 * nkb;         // pass 1: K; pass 2: K, V per block

  constexpr int kB = 2 * kStages;  // barriers after the ring's full / empty pairs
  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + kStages + s); };
  const uint32_t q_full = smem_u32(bars + kB);
  auto s_full = [&](int b) { return smem_u32(bars + kB + 1 + b); };
  auto s_rel_sm = [&](int b) { return smem_u32(bars + kB + 3 + b); };   // pass 1: softmax read S
  auto s_rel_mma = [&](int b) { return smem_u32(bars + kB + 5 + b); };  // pass 2: P.V read P
  auto p_full = [&](int b) { return smem_u32(bars + kB + 7 + b); };
  const uint32_t o_full = smem_u32(bars + kB + 9), drain_bar = smem_u32(bars + kB + 10);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(q_full, kSoftThreads / 32);
    for (int b = 0; b < kSBufs; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(s_rel_sm(b), kSoftThreads / 32);
      mbar_init(s_rel_mma(b), 1);
      mbar_init(p_full(b), kSoftThreads / 32);
    }
    mbar_init(o_full, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *issued_p = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_holder;

  // Q and the cache rows come from the previous kernel (programmatic launch)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // Tile t, in the order the MMAs consume them (so the ring's lookahead is
  // kStages tiles of that order): pass 1 K_0 .. K_{n-1}; pass 2 K_0, then
  // K_{j+1}, V_j for j = 0 .. n-2, then V_{n-1} (the next block's scores are
  // computed before the current block's P.V).
  auto tile_kind = [&](int t, int& kb, bool& is_v) {
    const int u = t - nkb;
    if (u < 0) {
      kb = t;
      is_v = false;
    } else if (u == 0) {
      kb = 0;
      is_v = false;
    } else if (u == 2 * nkb - 1) {
      kb = nkb - 1;
      is_v = true;
    } else {
      is_v = (u & 1) == 0;
      kb = is_v ? u / 2 - 1 : (u + 1) / 2;
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int issued = 0;
      for (int t = 0; t < n_tiles && !*abort_flag; ++t) {
        const int s = t % kStages;
        if (!wait(empty_bar(s), (uint32_t)(((t / kStages) & 1) ^ 1), abort_flag)) break;
        int kb;
        bool is_v;
        tile_kind(t, kb, is_v);
        const uint32_t dst = smem_u32(smem + s * kTile);
        const CUtensorMap* map = is_v ? &a.tmV : &a.tmK;
        mbar_expect_tx(full_bar(s), kTile);
        tma_load_3d(dst, map, full_bar(s), 0, kb * kBN, hk);
        tma_load_3d(dst + kHalf, map, full_bar(s), 64, kb * kBN, hk);
        issued = t + 1;
      }
      *issued_p = issued;
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t id_qk = idesc_f16<T>(kBM, kBN, 0), id_pv = idesc_f16<T>(kBM, kD, 1);
      bool ok = wait(q_full, 0, abort_flag);
      fence_after();
      int sidx = 0;
      bool issued_any = false;
      // S = Q . K_kb^T into S buffer sidx & 1 (tile t). The buffer's previous
      // use (sidx - 2) was released by the softmax (pass 1) or by a P.V.
      auto qk = [&](int t) -> bool {
        const int b = sidx & 1, prev = sidx - 2;
        if (prev >= 0) {
          bool w;
          if (prev < nkb) {
            w = wait(s_rel_sm(b), (uint32_t)((prev >> 1) & 1), abort_flag);
          } else {
            const int first = nkb + ((b - nkb) & 1);  // first pass-2 use of buffer b
            w = wait(s_rel_mma(b), (uint32_t)(((prev - first) >> 1) & 1), abort_flag);
          }
          if (!w) return false;
        }
        const int s = t % kStages;
        if (!wait(full_bar(s), (uint32_t)((t / kStages) & 1), abort_flag)) return false;
        fence_after();
        const uint32_t sk = smem_u32(smem + s * kTile);
#pragma unroll
        for (int k = 0; k < kD / 16; ++k)
          mma_ts(tmem + b * kBN, tmem + kQCol + 8 * k, sw128_desc(sk + (uint32_t)(k >> 2) * kHalf) + 2 * (k & 3),
                 id_qk, k != 0 ? 1u : 0u);
        mma_commit(empty_bar(s));
        mma_commit(s_full(b));
        issued_any = true;
        ++sidx;
        return true;
      };
      // O += P_kb . V_kb (tile t); P_kb sits in the S buffer of pass-2 block kb
      auto pv = [&](int t, int kb) -> bool {
        if (!wait(p_full(kb & 1), (uint32_t)((kb >> 1) & 1), abort_flag)) return false;
        const int s = t % kStages;
        if (!wait(full_bar(s), (uint32_t)((t / kStages) & 1), abort_flag)) return false;
        fence_after();
        const int b = (nkb + kb) & 1;
        const uint32_t sv = smem_u32(smem + s * kTile);
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k)
          mma_ts(tmem + kOCol, tmem + b * kBN + 64 * (k >> 2) + 8 * (k & 3),
                 sw128_desc_mn(sv + (uint32_t)k * 16 * 128, kHalf), id_pv, (kb | k) != 0 ? 1u : 0u);
        mma_commit(empty_bar(s));
        mma_commit(s_rel_mma(b));
        issued_any = true;
        return true;
      };
      for (int t = 0; ok && t < n_tiles; ++t) {  // the producer's order
        int kb;
        bool is_v;
        tile_kind(t, kb, is_v);
        ok = is_v ? pv(t, kb) : qk(t);
      }
      if (ok) mma_commit(o_full);
      if (*abort_flag && issued_any) {
        // every MMA this thread issued finishes before TMEM is released
        mma_commit(drain_bar);
        const unsigned long long t0 = globaltimer();
        while (!mbar_try(drain_bar, 0) && globaltimer() - t0 < kDrainWaitNs) {
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------- softmax and epilogue
    // warps 2..9: TMEM lane quarter warp & 3 (rows 32*quad ..), key / output
    // column half (warp - 2) >> 2 of each 128-column block
    const int quad = warp & 3, half = (warp - 2) >> 2;
    const int row = quad * 32 + lane;
    const int qpos = a.pos0 + q0 + row;
    const uint32_t tlane = (uint32_t)(quad * 32) << 16;
    float* red = reinterpret_cast<float*>(smem + kOffRed);  // [2][128] cross-half exchange
    // Q row (this half's 64 dimensions) into TMEM; rows past S are zero
    {
      uint32_t w[32];
      if (q0 + row < a.S) {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(a.q) + (int64_t)h * a.q_head_stride +
                                                          (int64_t)(q0 + row) * kD + half * 64);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 x = __ldg(src + j);
          w[4 * j] = x.x;
          w[4 * j + 1] = x.y;
          w[4 * j + 2] = x.z;
          w[4 * j + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = 0u;
      }
      tmem_st32(tmem + tlane + kQCol + half * 32, w);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full);
    }
    int sidx = 0;
    bool ok = true;
    // pass 1: the row maximum of the raw scores over the causal keys. Rounding
    // and the positive scale are monotone, so max t = round(round(max s) * scale).
    float mr = -INFINITY;
    for (int kb = 0; ok && kb < nkb; ++kb) {
      const int b = sidx & 1;
      if (!wait(s_full(b), (uint32_t)((sidx >> 1) & 1), abort_flag)) { ok = false; break; }
      fence_after();
      float v[64];
      tmem_ld64(tmem + tlane + b * kBN + half * 64, v);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_rel_sm(b));
      ++sidx;
      const int lim = qpos - (kb * kBN + half * 64);  // keys i <= lim are visible
      if (lim >= 63) {
#pragma unroll
        for (int w = 32; w >= 1; w >>= 1)
#pragma unroll
          for (int i = 0; i < w; ++i) v[i] = fmaxf(v[i], v[i + w]);
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = i <= lim ? v[i] : -INFINITY;
#pragma unroll
        for (int w = 32; w >= 1; w >>= 1)
#pragma unroll
          for (int i = 0; i < w; ++i) v[i] = fmaxf(v[i], v[i + w]);
      }
      mr = fmaxf(mr, v[0]);
    }
    // the two halves of a row meet in shared memory (named barrier of the
    // softmax warps; a role that gave up still arrives, so nothing waits on it)
    red[half * kBM + row] = mr;
    asm volatile("bar.sync 1, %0;" ::"n"(kSoftThreads) : "memory");
    mr = fmaxf(mr, red[(half ^ 1) * kBM + row]);
    ok = ok && !*abort_flag;
    const float m = round_to<T>(round_to<T>(mr) * a.scale);
    // e = exp(t - m) = 2^(t * log2(e) - m * log2(e)), t = round(round(s) * scale)
    constexpr float kLog2e = 1.4426950408889634f;
    const float mb = -m * kLog2e;
    float l0 = 0.f, l1 = 0.f;
    // pass 2: p = round(e) into the first 32 columns of this half's 64
    for (int kb = 0; ok && kb < nkb; ++kb) {
      const int b = sidx & 1;
      if (!wait(s_full(b), (uint32_t)((sidx >> 1) & 1), abort_flag)) { ok = false; break; }
      fence_after();
      float v[64];
      tmem_ld64(tmem + tlane + b * kBN + half * 64, v);
      ++sidx;
      const int lim = qpos - (kb * kBN + half * 64);
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const uint32_t r = pack2_rn<T>(v[i], v[i + 1]);
        const uint32_t t = pack2_rn<T>(lo_f<T>(r) * a.scale, hi_f<T>(r) * a.scale);
        float e0 = ex2(fmaf(lo_f<T>(t), kLog2e, mb)), e1 = ex2(fmaf(hi_f<T>(t), kLog2e, mb));
        if (lim < 63) {  // the diagonal block: keys past the row's position get 0
          e0 = i <= lim ? e0 : 0.f;
          e1 = i + 1 <= lim ? e1 : 0.f;
        }
        l0 += e0;
        l1 += e1;
        pk[i >> 1] = pack2_rn<T>(e0, e1);
      }
      tmem_st32(tmem + tlane + b * kBN + half * 64, pk);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full(kb & 1));
    }
    // epilogue: out = round(O / l), each half stores its 64 output columns
    asm volatile("bar.sync 1, %0;" ::"n"(kSoftThreads) : "memory");
    red[half * kBM + row] = l0 + l1;
    asm volatile("bar.sync 1, %0;" ::"n"(kSoftThreads) : "memory");
    const float l = red[row] + red[kBM + row];
    if (ok && wait(o_full, 0, abort_flag)) {
      fence_after();
      const float inv = 1.0f / l;
      float v[64];
      tmem_ld64(tmem + tlane + kOCol + half * 64, v);
      if (q0 + row < a.S) {
        T* orow = static_cast<T*>(a.out) + (int64_t)(q0 + row) * a.ld_out + (int64_t)h * kD + half * 64;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 o;
          o.x = pack2_rn<T>(v[8 * j] * inv, v[8 * j + 1] * inv);
          o.y = pack2_rn<T>(v[8 * j + 2] * inv, v[8 * j + 3] * inv);
          o.z = pack2_rn<T>(v[8 * j + 4] * inv, v[8 * j + 5] * inv);
          o.w = pack2_rn<T>(v[8 * j + 6] * inv, v[8 * j + 7] * inv);
          *reinterpret_cast<uint4*>(orow + 8 * j) = o;
        }
      }
    }
  }

  // ---------------------------------------------------------- teardown
  fence_before();
  __syncthreads();
  fence_after();
  if (*abort_flag && threadIdx.x == 0) {
    // copies still in flight land before the CTA exits: the last kStages
    // tiles (an earlier tile's stage was reused, so it had landed)
    const int issued = *issued_p;
    for (int t = max(0, issued - kStages); t < issued; ++t) {
      const unsigned long long t0 = globaltimer();
      while (!mbar_try(full_bar(t % kStages), (uint32_t)((t / kStages) & 1)) && globaltimer() - t0 < kDrainWaitNs / 4) {
      }
    }
  }
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// 3-D tensor map over [heads][rows][128] (row stride 256 bytes, head stride
// head_stride elements), boxes of 64 x 128 x 1, 128-byte swizzle, zero fill.
bool make_map3(CUtensorMap* map, ie_dtype dt, const void* base, int rows, int heads, int64_t head_stride) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)rows, (cuuint64_t)heads};
  cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)head_stride * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMapDataType t = dt == IE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return fn(map, t, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <typename T>
int launch(const TcaArgs& a, int n_q_heads, cudaStream_t st) {
  auto kernel = tc_attention_kernel<T>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return IE_ERR_LAUNCH;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
      return IE_ERR_LAUNCH;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_q_heads, (a.S + kBM - 1) / kBM);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  const char* env = getenv("IE_PDL");
  cfg.numAttrs = (env && env[0] == '0') ? 0 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, a);
  if (e != cudaSuccess) {
    std::fprintf(stderr, "infengine_b200: tcgen05 attention launch failed: %s\n", cudaGetErrorString(e));
    return IE_ERR_LAUNCH;
  }
  return IE_OK;
}

}  // namespace

int launch_tc_attention(ie_dtype dt, int S, int pos0, int n_q_heads, int n_kv_heads, const void* q,
                        int64_t q_head_stride, const void* k_cache, const void* v_cache, int64_t cache_head_stride,
                        void* out, int64_t ld_out, void* stream) {
  TcaArgs a;
  memset(&a, 0, sizeof(a));
  const int64_t rows = cache_head_stride / kD;
  if (rows > 0x7fffffff || S <= 0) return IE_ERR_UNSUPPORTED;
  if ((S + kBM - 1) / kBM > 65535) return IE_ERR_UNSUPPORTED;
  if (!make_map3(&a.tmK, dt, k_cache, (int)rows, n_kv_heads, cache_head_stride) ||
      !make_map3(&a.tmV, dt, v_cache, (int)rows, n_kv_heads, cache_head_stride))
    return IE_ERR_UNSUPPORTED;
  a.q = q;
  a.q_head_stride = q_head_stride;
  a.S = S;
  a.pos0 = pos0;
  a.group = n_q_heads / n_kv_heads;
  a.scale = 1.0f / sqrtf(128.0f);
  a.out = out;
  a.ld_out = ld_out;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dt == IE_DTYPE_F16 ? launch<__half>(a, n_q_heads, st) : launch<__nv_bfloat16>(a, n_q_heads, st);
}

cudaError_t set_tca_wait_ns(unsigned long long ns) {
  return cudaMemcpyToSymbol(g_tca_wait_ns, &ns, sizeof(ns));
}

int read_tca_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tca_status, sizeof(int)) != cudaSuccess) return IE_ERR_LAUNCH;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_tca_status, &z, sizeof(int));
  }
  return v;
}

}  // namespace ie
