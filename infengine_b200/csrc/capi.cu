// extern "C" entry points of libinfengine_b200.so: argument validation and
// dispatch to the decode (skinny) or prefill (tcgen05) kernels.
#include <cstdio>
#include "ie_common.cuh"
#include "skinny.cuh"
#include "gemm_tc.cuh"
#include "attention.cuh"
#include "norm.cuh"

using namespace ie;

namespace {

constexpr int kSkinnyMaxM = 16;

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int from_cuda(cudaError_t e) {
  if (e == cudaSuccess) return IE_OK;
  std::fprintf(stderr, "infengine_b200: CUDA error %d (%s)\n", (int)e, cudaGetErrorString(e));
  return IE_ERR_LAUNCH;
}

inline bool valid_dtype(ie_dtype dt) { return dt == IE_DTYPE_F16 || dt == IE_DTYPE_BF16; }

// Matrix operand checks shared by every projection: 16-byte aligned base and
// a leading dimension that keeps every row 16-byte aligned.
inline int check_matrix(const void* p, int64_t ld, int cols) {
  if (!p) return IE_ERR_INVALID_ARG;
  if (ld < cols) return IE_ERR_INVALID_ARG;
  if (!aligned16(p) || (ld % 8) != 0) return IE_ERR_ALIGNMENT;
  return IE_OK;
}

inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

extern "C" {

const char* ie_status_string(int status) {
  switch (status) {
    case IE_OK: return "ok";
    case IE_ERR_INVALID_ARG: return "invalid argument";
    case IE_ERR_ALIGNMENT: return "misaligned pointer or leading dimension";
    case IE_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case IE_ERR_LAUNCH: return "CUDA launch error";
    case IE_ERR_TIMEOUT: return "device-side wait timed out";
    case IE_ERR_NO_DEVICE: return "no usable sm_100 device";
    case IE_ERR_WORKSPACE: return "workspace missing or too small";
  }
  return "unknown status";
}

const char* ie_version(void) { return "0.1.0"; }

int ie_device_status(int clear) {
  if (cudaDeviceSynchronize() != cudaSuccess) return IE_ERR_LAUNCH;
  const int a = read_tc_status(clear != 0);
  const int b = read_skinny_status(clear != 0);
  const int c = read_attn_status(clear != 0);
  const int d = read_norm_status(clear != 0);
  const int e = read_tca_status(clear != 0);
  return a != IE_OK ? a : (b != IE_OK ? b : (c != IE_OK ? c : (d != IE_OK ? d : e)));
}

int ie_set_wait_limit_ns(unsigned long long ns) {
  if (ns > kMaxWaitNs) return IE_ERR_INVALID_ARG;
  const unsigned long long v = ns ? ns : kDefaultWaitNs;
  const cudaError_t e[4] = {set_tc_wait_ns(v), set_skinny_wait_ns(v), set_attn_wait_ns(v), set_tca_wait_ns(v)};
  for (const cudaError_t x : e)
    if (x != cudaSuccess) return IE_ERR_LAUNCH;
  return IE_OK;
}

static int gemm_store(ie_dtype dt, int M, int N, int K, const void* X, int64_t ldx, const void* W, int64_t ldw,
                      void* Y, int64_t ldy, bool residual, void* ws, size_t ws_bytes, void* stream) {
  if (!valid_dtype(dt) || M < 0 || N < 0 || K <= 0) return IE_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return IE_OK;
  if (K % 8) return IE_ERR_ALIGNMENT;
  int s;
  if ((s = check_matrix(X, ldx, K)) || (s = check_matrix(W, ldw, K))) return s;
  if (!Y || ldy < N) return IE_ERR_INVALID_ARG;
  if (M <= kSkinnyMaxM) {
    SkinnyParams p;
    p.X = X; p.ldx = ldx; p.M = M; p.N = N; p.K = K;
    p.W0 = W; p.ldw = ldw; p.Y = Y; p.ldy = ldy;
    p.residual = residual;
    return from_cuda(launch_skinny(dt, EPI_STORE, p, as_stream(stream)));
  }
  if ((s = check_matrix(Y, ldy, N))) return s;
  TcGemmParams q;
  q.A = X; q.lda = ldx; q.B = W; q.ldb = ldw; q.M = M; q.N = N; q.K = K;
  q.D = Y; q.ldd = ldy; q.epi = TC_EPI_STORE;
  q.residual = residual;
  if ((s = attach_split_workspace(q, ws, ws_bytes))) return s;
  return launch_tc_gemm(dt, q, as_stream(stream));
}

int ie_gemm(ie_dtype dt, int M, int N, int K, const void* X, int64_t ldx, const void* W, int64_t ldw, void* Y,
            int64_t ldy, void* stream) {
  return gemm_store(dt, M, N, K, X, ldx, W, ldw, Y, ldy, false, nullptr, 0, stream);
}

int ie_gemm_add(ie_dtype dt, int M, int N, int K, const void* X, int64_t ldx, const void* W, int64_t ldw, void* Y,
                int64_t ldy, void* stream) {
  return gemm_store(dt, M, N, K, X, ldx, W, ldw, Y, ldy, true, nullptr, 0, stream);
}

size_t ie_split_workspace_size(void) { return split_workspace_bytes(); }

int ie_gemm_ws(ie_dtype dt, int M, int N, int K, const void* X, int64_t ldx, const void* W, int64_t ldw, void* Y,
               int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
  return gemm_store(dt, M, N, K, X, ldx, W, ldw, Y, ldy, false, workspace, workspace_bytes, stream);
}

int ie_gemm_add_ws(ie_dtype dt, int M, int N, int K, const void* X, int64_t ldx, const void* W, int64_t ldw, void* Y,
                   int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
  return gemm_store(dt, M, N, K, X, ldx, W, ldw, Y, ldy, true, workspace, workspace_bytes, stream);
}

int ie_gemm_f32out(ie_dtype dt, int M, int N, int K, const void* X, int64_t ldx, const void* W, int64_t ldw, float* Y,
                   int64_t ldy, void* stream) {
  if (!valid_dtype(dt) || M < 0 || N < 0 || K <= 0) return IE_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return IE_OK;
  if (K % 8) return IE_ERR_ALIGNMENT;
  int s;
  if ((s = check_matrix(X, ldx, K)) || (s = check_matrix(W, ldw, K))) return s;
  if (!Y || ldy < N) return IE_ERR_INVALID_ARG;
  if (M <= kSkinnyMaxM) {
    SkinnyParams p;
    p.X = X; p.ldx = ldx; p.M = M; p.N = N; p.K = K;
    p.W0 = W; p.ldw = ldw; p.Y = Y; p.ldy = ldy;
    return from_cuda(launch_skinny(dt, EPI_STORE_F32, p, as_stream(stream)));
  }
  if (!aligned16(Y) || (ldy % 4) != 0) return IE_ERR_ALIGNMENT;
  TcGemmParams q;
  q.A = X; q.lda = ldx; q.B = W; q.ldb = ldw; q.M = M; q.N = N; q.K = K;
  q.D = Y; q.ldd = ldy; q.epi = TC_EPI_STORE_F32;
  return launch_tc_gemm(dt, q, as_stream(stream));
}

int ie_swiglu(ie_dtype dt, int M, int F, const void* gate, const void* up, void* out, void* stream) {
  if (!valid_dtype(dt) || M < 0 || F < 0) return IE_ERR_INVALID_ARG;
  if ((int64_t)M * F == 0) return IE_OK;
  if (!gate || !up || !out) return IE_ERR_INVALID_ARG;
  if (!aligned16(gate) || !aligned16(up) || !aligned16(out)) return IE_ERR_ALIGNMENT;
  return from_cuda(launch_swiglu(dt, (int64_t)M * F, gate, up, out, as_stream(stream)));
}

size_t ie_ffn_workspace_size(int M, int F) {
  if (M <= 0 || F <= 0) return 0;
  return round_up((size_t)M * (size_t)F * 2u, 256);
}

int ie_ffn(ie_dtype dt, int M, int H, int F, const void* x, const void* W_up, const void* W_down, const void* W_gate,
           void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!valid_dtype(dt) || M < 0 || H <= 0 || F <= 0) return IE_ERR_INVALID_ARG;
  if (M == 0) return IE_OK;
  if ((H % 8) || (F % 8)) return IE_ERR_ALIGNMENT;
  int s;
  if ((s = check_matrix(x, H, H)) || (s = check_matrix(W_up, H, H)) || (s = check_matrix(W_gate, H, H)) ||
      (s = check_matrix(W_down, F, F)) || (s = check_matrix(out, H, H)))
    return s;
  if (!workspace || workspace_bytes < ie_ffn_workspace_size(M, F)) return IE_ERR_WORKSPACE;
  if (!aligned16(workspace)) return IE_ERR_ALIGNMENT;
  if ((s = ie_ffn_gate_up(dt, M, H, F, x, W_gate, W_up, workspace, F, stream))) return s;
  return ie_gemm(dt, M, H, F, workspace, F, W_down, F, out, H, stream);
}

static int ffn_gate_up(ie_dtype dt, int M, int H, int F, const void* x, const void* W_gate, const void* W_up,
                       void* h, int64_t ldh, void* ws, size_t ws_bytes, void* stream) {
  if (!valid_dtype(dt) || M < 0 || H <= 0 || F <= 0) return IE_ERR_INVALID_ARG;
  if (M == 0) return IE_OK;
  if ((H % 8) || (F % 8)) return IE_ERR_ALIGNMENT;
  int s;
  if ((s = check_matrix(x, H, H)) || (s = check_matrix(W_up, H, H)) || (s = check_matrix(W_gate, H, H)) ||
      (s = check_matrix(h, ldh, F)))
    return s;
  cudaStream_t st = as_stream(stream);
  if (M <= kSkinnyMaxM) {
    SkinnyParams p;
    p.X = x; p.ldx = H; p.M = M; p.N = F; p.K = H;
    p.W0 = W_gate; p.W1 = W_up; p.ldw = H; p.Y = h; p.ldy = ldh;
    return from_cuda(launch_skinny(dt, EPI_SWIGLU, p, st));
  }
  TcGemmParams q;
  q.A = x; q.lda = H; q.B = W_gate; q.B2 = W_up; q.ldb = H; q.M = M; q.N = F; q.K = H;
  q.D = h; q.ldd = ldh; q.epi = TC_EPI_SWIGLU;
  if ((s = attach_split_workspace(q, ws, ws_bytes))) return s;
  return launch_tc_gemm(dt, q, st);
}

int ie_ffn_gate_up(ie_dtype dt, int M, int H, int F, const void* x, const void* W_gate, const void* W_up, void* h,
                   int64_t ldh, void* stream) {
  return ffn_gate_up(dt, M, H, F, x, W_gate, W_up, h, ldh, nullptr, 0, stream);
}

int ie_ffn_gate_up_ws(ie_dtype dt, int M, int H, int F, const void* x, const void* W_gate, const void* W_up, void* h,
                      int64_t ldh, void* workspace, size_t workspace_bytes, void* stream) {
  return ffn_gate_up(dt, M, H, F, x, W_gate, W_up, h, ldh, workspace, workspace_bytes, stream);
}

namespace {

int qkv_common(ie_dtype dt, int M, int H, int n_q_heads, int n_kv_heads, int head_dim, const void* x, const void* Wq,
               const void* Wk, const void* Wv, void* q_out, void* k_cache, void* v_cache, int64_t cache_head_stride,
               int pos0, const int* positions, int64_t cache_batch_stride, int cache_rows, const float* rope_cos,
               const float* rope_sin, void* ws, size_t ws_bytes, void* stream) {
  if (!valid_dtype(dt) || M < 0 || H <= 0 || n_q_heads <= 0 || n_kv_heads < 0 || pos0 < 0) return IE_ERR_INVALID_ARG;
  if (head_dim != 128) return IE_ERR_UNSUPPORTED;
  if (M == 0) return IE_OK;
  if (H % 8) return IE_ERR_ALIGNMENT;
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return IE_ERR_INVALID_ARG;
  if (rope_cos && (!aligned16(rope_cos) || !aligned16(rope_sin))) return IE_ERR_ALIGNMENT;
  int s;
  if ((s = check_matrix(x, H, H)) || (s = check_matrix(Wq, H, H))) return s;
  if (n_kv_heads > 0) {
    if ((s = check_matrix(Wk, H, H)) || (s = check_matrix(Wv, H, H))) return s;
    if (!k_cache || !v_cache) return IE_ERR_INVALID_ARG;
    const int64_t rows_needed = positions ? (int64_t)cache_rows : (int64_t)(pos0 + M);
    if (cache_head_stride < rows_needed * head_dim) return IE_ERR_INVALID_ARG;
    if (positions && cache_batch_stride < (int64_t)n_kv_heads * cache_head_stride) return IE_ERR_INVALID_ARG;
  }
  if (!q_out) return IE_ERR_INVALID_ARG;
  cudaStream_t st = as_stream(stream);
  if (M <= kSkinnyMaxM) {
    SkinnyParams p;
    p.X = x; p.ldx = H; p.M = M; p.K = H; p.N = (n_q_heads + 2 * n_kv_heads) * head_dim;
    p.W0 = Wq; p.W1 = Wk; p.W2 = Wv; p.ldw = H;
    p.n_q_heads = n_q_heads; p.n_kv_heads = n_kv_heads;
    p.q_out = q_out; p.q_head_stride = (int64_t)M * head_dim;
    p.k_cache = k_cache; p.v_cache = v_cache; p.cache_head_stride = cache_head_stride; p.pos0 = pos0;
    p.rope_cos = rope_cos; p.rope_sin = rope_sin;
    p.positions = positions; p.cache_batch_stride = cache_batch_stride; p.cache_rows = cache_rows;
    return from_cuda(launch_skinny(dt, EPI_QKV, p, st));
  }
  TcGemmParams q;
  q.A = x; q.lda = H; q.M = M; q.K = H; q.N = (n_q_heads + 2 * n_kv_heads) * head_dim;
  q.B = Wq; q.B2 = Wk; q.B3 = Wv; q.ldb = H; q.epi = TC_EPI_QKV;
  q.n_q_heads = n_q_heads; q.n_kv_heads = n_kv_heads;
  q.q_out = q_out; q.q_head_stride = (int64_t)M * head_dim;
  q.k_cache = k_cache; q.v_cache = v_cache; q.cache_head_stride = cache_head_stride; q.pos0 = pos0;
  q.rope_cos = rope_cos; q.rope_sin = rope_sin;
  q.positions = positions; q.cache_batch_stride = cache_batch_stride; q.cache_rows = cache_rows;
  if ((s = attach_split_workspace(q, ws, ws_bytes))) return s;
  return launch_tc_gemm(dt, q, st);
}

}  // namespace

int ie_qkv(ie_dtype dt, int M, int H, int n_q_heads, int n_kv_heads, int head_dim, const void* x, const void* Wq,
           const void* Wk, const void* Wv, void* q_out, void* k_cache, void* v_cache, int64_t cache_head_stride,
           int pos0, const float* rope_cos, const float* rope_sin, void* stream) {
  return qkv_common(dt, M, H, n_q_heads, n_kv_heads, head_dim, x, Wq, Wk, Wv, q_out, k_cache, v_cache,
                    cache_head_stride, pos0, nullptr, 0, 0, rope_cos, rope_sin, nullptr, 0, stream);
}

int ie_qkv_ws(ie_dtype dt, int M, int H, int n_q_heads, int n_kv_heads, int head_dim, const void* x, const void* Wq,
              const void* Wk, const void* Wv, void* q_out, void* k_cache, void* v_cache, int64_t cache_head_stride,
              int pos0, const float* rope_cos, const float* rope_sin, void* workspace, size_t workspace_bytes,
              void* stream) {
  return qkv_common(dt, M, H, n_q_heads, n_kv_heads, head_dim, x, Wq, Wk, Wv, q_out, k_cache, v_cache,
                    cache_head_stride, pos0, nullptr, 0, 0, rope_cos, rope_sin, workspace, workspace_bytes, stream);
}

int ie_qkv_batched(ie_dtype dt, int B, int H, int n_q_heads, int n_kv_heads, int head_dim, const void* x,
                   const void* Wq, const void* Wk, const void* Wv, void* q_out, void* k_cache, void* v_cache,
                   int64_t cache_head_stride, int64_t cache_batch_stride, int cache_rows, const int* positions,
                   const float* rope_cos, const float* rope_sin, void* stream) {
  if (!positions || cache_rows <= 0) return IE_ERR_INVALID_ARG;
  return qkv_common(dt, B, H, n_q_heads, n_kv_heads, head_dim, x, Wq, Wk, Wv, q_out, k_cache, v_cache,
                    cache_head_stride, 0, positions, cache_batch_stride, cache_rows, rope_cos, rope_sin, nullptr, 0,
                    stream);
}

size_t ie_lm_head_argmax_workspace_size(int M) {
  if (M <= 0) return 0;
  return round_up((size_t)M * 8u + 8u, 256);
}

int ie_lm_head_argmax(ie_dtype dt, int M, int K, int V, int64_t vocab_offset, const void* x, int64_t ldx,
                      const void* W, void* logits, int64_t ld_logits, int* idx_out, unsigned long long* key_out,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (!valid_dtype(dt) || M < 0 || K <= 0 || V < 0 || vocab_offset < 0) return IE_ERR_INVALID_ARG;
  if (vocab_offset + (int64_t)V >= (int64_t(1) << 31)) return IE_ERR_UNSUPPORTED;
  if (M == 0 || V == 0) return IE_OK;
  if (M > kSkinnyMaxM * 4) return IE_ERR_UNSUPPORTED;
  if (K % 8) return IE_ERR_ALIGNMENT;
  int s;
  if ((s = check_matrix(x, ldx, K)) || (s = check_matrix(W, K, K))) return s;
  if (logits && ld_logits < V) return IE_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < ie_lm_head_argmax_workspace_size(M)) return IE_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 7u) != 0) return IE_ERR_ALIGNMENT;
  cudaStream_t st = as_stream(stream);
  unsigned long long* keys = static_cast<unsigned long long*>(workspace);
  unsigned int* counter = reinterpret_cast<unsigned int*>(keys + M);
  if (M <= kSkinnyMaxM) {
    SkinnyParams p;
    p.X = x; p.ldx = ldx; p.M = M; p.N = V; p.K = K; p.W0 = W; p.ldw = K;
    p.Y = logits; p.ldy = ld_logits; p.vocab_offset = vocab_offset;
    p.keys = keys; p.counter = counter; p.idx_out = idx_out; p.key_out = key_out;
    return from_cuda(launch_skinny(dt, EPI_ARGMAX, p, st));
  }
  TcGemmParams q;
  q.A = x; q.lda = ldx; q.B = W; q.ldb = K; q.M = M; q.N = V; q.K = K;
  q.D = logits; q.ldd = ld_logits; q.epi = TC_EPI_ARGMAX; q.vocab_offset = vocab_offset;
  q.keys = keys; q.counter = counter; q.idx_out = idx_out; q.key_out = key_out;
  return launch_tc_gemm(dt, q, st);
}

int ie_argmax(ie_dtype dt, int M, int V, const void* logits, int64_t ld, int* idx_out, void* stream) {
  if (!valid_dtype(dt) || M < 0 || V < 0 || ld < V) return IE_ERR_INVALID_ARG;
  if (M == 0) return IE_OK;
  if (V == 0 || !logits || !idx_out) return IE_ERR_INVALID_ARG;
  if (M > 65535) return IE_ERR_UNSUPPORTED;
  if (!aligned16(logits) || (ld % 8) != 0) return IE_ERR_ALIGNMENT;
  return from_cuda(launch_argmax(dt, M, V, logits, ld, idx_out, as_stream(stream)));
}

}  // extern "C"
