// RMSNorm, embedding lookup and the per-step bookkeeping of the decode engine.
//
// These are not weight matmuls; they are the glue a complete decode step
// needs between the projections (decode.cu:14-44): the engine runs them on
// the device so that a step replays as one CUDA graph with no host work.
//
// RMSNorm keeps the reference's arithmetic bit for bit (kernels/rmsnorm.cu:
// 29-62, launched with 1024 threads): virtual thread t of 1024 sums x[i]^2
// over i = t, t+1024, ... in increasing i; the 1024 partial sums are combined
// by the halving tree s[t] += s[t + d], d = 512 .. 1; then
// out = round(round(x * rsqrt(sum / H + eps)) * w). Here one 256-thread CTA
// per row holds four virtual threads per thread and runs the same tree (the
// first two levels in registers, the next three in shared memory, the last
// five as shuffles), so its sums are identical to the reference's.
// (Fusing this into the prologue of the consuming projection was measured
// slower: every CTA of every wave then re-reads the row through an L2 that is
// saturated by the weight stream.)
#include "ie_common.cuh"
#include "norm.cuh"

namespace ie {

__device__ int g_norm_status = 0;

namespace {

constexpr int kNormThreads = 256;
constexpr int kVirtual = 1024;  // the reference's block size

constexpr int kNormMaxChunks = 8;  // 16-byte chunks per thread: H <= 256 * 8 * 8

// One CTA per row. The weight chunks are requested before waiting for the
// previous kernel (they are never written by it); the row is read once with
// 16-byte loads, kept in registers for the output and staged in shared memory
// for the sums, which then follow the reference's per-virtual-thread order.
template <typename T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const T* x, int64_t ldx, const T* __restrict__ w,
                                                               T* out, int64_t ldo, int H, float eps) {
  extern __shared__ __align__(16) unsigned char norm_smem[];
  __shared__ float s[kNormThreads];
  T* xs = reinterpret_cast<T*>(norm_smem);
  const int row = blockIdx.x, t = threadIdx.x, nv = H / 8;
  uint4 wv[kNormMaxChunks], xv[kNormMaxChunks];
#pragma unroll
  for (int k = 0; k < kNormMaxChunks; ++k) {
    const int c = t + k * kNormThreads;
    if (c < nv) wv[k] = ld_act_v4(w + 8 * c);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const T* xr = x + (int64_t)row * ldx;
#pragma unroll
  for (int k = 0; k < kNormMaxChunks; ++k) {
    const int c = t + k * kNormThreads;
    if (c < nv) {
      xv[k] = ld_act_v4(xr + 8 * c);
      *reinterpret_cast<uint4*>(xs + 8 * c) = xv[k];
    }
  }
  __syncthreads();
  float v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float a = 0.f;
    for (int i = t + k * kNormThreads; i < H; i += kVirtual) {
      const float d = DT<T>::to_f(xs[i]);
      a += d * d;
    }
    v[k] = a;  // virtual thread t + 256 k
  }
  v[0] += v[2];  // d = 512: t += t + 512
  v[1] += v[3];  //          t + 256 += t + 768
  v[0] += v[1];  // d = 256
  s[t] = v[0];
  __syncthreads();
  if (t < 128) s[t] += s[t + 128];
  __syncthreads();
  if (t < 64) s[t] += s[t + 64];
  __syncthreads();
  if (t < 32) {
    float a = s[t] + s[t + 32];
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) a += __shfl_down_sync(0xffffffffu, a, d);
    if (t == 0) s[0] = a;
  }
  __syncthreads();
  const float scale = rsqrtf(s[0] / (float)H + eps);
  T* orow = out + (int64_t)row * ldo;
#pragma unroll
  for (int k = 0; k < kNormMaxChunks; ++k) {
    const int c = t + k * kNormThreads;
    if (c < nv) {
      const T* xe = reinterpret_cast<const T*>(&xv[k]);
      const T* we = reinterpret_cast<const T*>(&wv[k]);
      uint4 ov;
      T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
      for (int i = 0; i < 8; ++i) oe[i] = DT<T>::from_f(round_to<T>(DT<T>::to_f(xe[i]) * scale) * DT<T>::to_f(we[i]));
      *reinterpret_cast<uint4*>(orow + 8 * c) = ov;
    }
  }
}

// out[m] = table[tokens[m]]; a token outside [0, vocab) gives a zero row and
// IE_ERR_INVALID_ARG in the status word.
template <typename T>
__global__ void __launch_bounds__(256) embed_kernel(const int* tokens, const T* __restrict__ table, int vocab, int H,
                                                    T* out, int64_t ldo) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int m = blockIdx.x;
  const int tok = tokens[m];
  const bool ok = tok >= 0 && tok < vocab;
  if (!ok && threadIdx.x == 0) atomicExch(&g_norm_status, IE_ERR_INVALID_ARG);
  const uint4* src = reinterpret_cast<const uint4*>(table + (int64_t)(ok ? tok : 0) * H);
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)m * ldo);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = ok ? src[i] : make_uint4(0, 0, 0, 0);
}

// End of a decode step: history[step][b] = tokens[b]; positions[b] += 1;
// step += 1 (history has `slots` rows and wraps).
__global__ void advance_kernel(int B, const int* tokens, int* positions, int* history, int slots, int* step) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int s = *step;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    history[(int64_t)(s % slots) * B + b] = tokens[b];
    positions[b] += 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) *step = s + 1;
}

template <typename K, typename... Args>
cudaError_t launch(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  // grid.x is the row count of RMSNorm and the embedding (1 for the step's
  // bookkeeping kernel)
  cfg.numAttrs = (pdl_launch_enabled() && (int)grid.x <= pdl_max_rows()) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

bool pdl_launch_enabled() {
  static const bool on = [] {
    const char* e = getenv("IE_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

cudaError_t launch_advance(int B, const int* tokens, int* positions, int* history, int slots, int* step,
                           cudaStream_t st) {
  return launch(advance_kernel, dim3(1), dim3(256), 0, st, B, tokens, positions, history, slots, step);
}

int read_norm_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_norm_status, sizeof(int)) != cudaSuccess) return IE_ERR_LAUNCH;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_norm_status, &z, sizeof(int));
  }
  return v;
}

}  // namespace ie

using namespace ie;

extern "C" int ie_rmsnorm(ie_dtype dt, int M, int H, const void* x, int64_t ldx, const void* w, void* out,
                          int64_t ldo, float eps, void* stream) {
  if ((dt != IE_DTYPE_F16 && dt != IE_DTYPE_BF16) || M < 0 || H <= 0) return IE_ERR_INVALID_ARG;
  if (M == 0) return IE_OK;
  if (!x || !w || !out || ldx < H || ldo < H) return IE_ERR_INVALID_ARG;
  if (H % 8 || ldx % 8 || ldo % 8 || !aligned16(x) || !aligned16(w) || !aligned16(out)) return IE_ERR_ALIGNMENT;
  if (H > kNormThreads * kNormMaxChunks * 8) return IE_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)H * 2;
  cudaError_t e;
  if (dt == IE_DTYPE_F16)
    e = launch(rmsnorm_kernel<__half>, dim3(M), dim3(kNormThreads), smem, st, static_cast<const __half*>(x), ldx,
               static_cast<const __half*>(w), static_cast<__half*>(out), ldo, H, eps);
  else
    e = launch(rmsnorm_kernel<__nv_bfloat16>, dim3(M), dim3(kNormThreads), smem, st,
               static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(w),
               static_cast<__nv_bfloat16*>(out), ldo, H, eps);
  return e == cudaSuccess ? IE_OK : IE_ERR_LAUNCH;
}

extern "C" int ie_embed(ie_dtype dt, int M, int H, int vocab, const int* tokens, const void* table, void* out,
                        int64_t ldo, void* stream) {
  if ((dt != IE_DTYPE_F16 && dt != IE_DTYPE_BF16) || M < 0 || H <= 0 || vocab <= 0) return IE_ERR_INVALID_ARG;
  if (M == 0) return IE_OK;
  if (!tokens || !table || !out || ldo < H) return IE_ERR_INVALID_ARG;
  if (H % 8 || ldo % 8 || !aligned16(table) || !aligned16(out)) return IE_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dt == IE_DTYPE_F16)
    e = launch(embed_kernel<__half>, dim3(M), dim3(256), 0, st, tokens, static_cast<const __half*>(table), vocab, H,
               static_cast<__half*>(out), ldo);
  else
    e = launch(embed_kernel<__nv_bfloat16>, dim3(M), dim3(256), 0, st, tokens,
               static_cast<const __nv_bfloat16*>(table), vocab, H, static_cast<__nv_bfloat16*>(out), ldo);
  return e == cudaSuccess ? IE_OK : IE_ERR_LAUNCH;
}
