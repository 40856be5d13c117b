// TEST INFRASTRUCTURE — drives the reference's own decode loop.
//
// Links the reference's prefill() / decode_step() (prefill.cu:11-48,
// decode.cu:11-49) and its non-hot-path kernels (embedding lookup, RMSNorm,
// residual add, RoPE tables) with either
//   * the reference's own hot-path kernels (libref_model_ref.so), or
//   * infengine_b200's drop-in library (libref_model_ie.so),
// as oracle/Makefile builds them, so the two can be run on identical
// random-init Llama-3.1-8B weights and compared token by token.
//
// Weights: every tensor of ModelWeights gets seeded N(0, 0.02) values drawn by
// a counter-based generator on the device, rounded to bf16 and stored as fp16
// (what model_weights.cu:61-78 does with a bf16 checkpoint); RMSNorm weights
// are 1 (the Hugging Face initialisation). The request flow follows
// manager.cpp:31-86: buffers sized for the context, one cuBLAS handle with no
// stream set, prefill, then decode_step in a loop.
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <vector>
#include "config.h"
#include "decode.cuh"
#include "prefill.cuh"
#include "kernels/attn.cuh"
#include "kernels/ffn.cuh"
#include "kernels/model_weights.cuh"
#include "kernels/rope.cuh"

#define REF_API extern "C" __attribute__((visibility("default")))
using namespace InfEngineConfig;

namespace {

__device__ __forceinline__ uint32_t mix32(uint64_t x) {
  x ^= x >> 33;
  x *= 0xff51afd7ed558ccdull;
  x ^= x >> 33;
  x *= 0xc4ceb9fe1a85ec53ull;
  x ^= x >> 33;
  return (uint32_t)x;
}

// N(0, std) from two counter-hashed uniforms (Box-Muller), rounded to bf16,
// stored as fp16.
__global__ void fill_normal(half* p, size_t n, uint64_t seed, float stddev) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t a = mix32(seed * 0x9e3779b97f4a7c15ull + 2 * i), b = mix32(seed * 0x9e3779b97f4a7c15ull + 2 * i + 1);
    const float u1 = ((a >> 8) + 1) * (1.0f / 16777217.0f), u2 = (b >> 8) * (1.0f / 16777216.0f);
    const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    p[i] = __float2half(__bfloat162float(__float2bfloat16(z * stddev)));
  }
}

__global__ void fill_const(half* p, size_t n, float v) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    p[i] = __float2half(v);
}

ModelWeights g_w{};
std::vector<void*> g_allocs;
uint64_t g_seed_counter = 0;

half* tensor(size_t n, uint64_t seed, float stddev, bool ones = false) {
  half* p = nullptr;
  if (cudaMalloc(&p, n * sizeof(half)) != cudaSuccess) return nullptr;
  g_allocs.push_back(p);
  if (ones) fill_const<<<1184, 256>>>(p, n, 1.0f);
  else fill_normal<<<1184, 256>>>(p, n, seed * 1000003ull + (++g_seed_counter), stddev);
  return p;
}

}  // namespace

REF_API int model_init(unsigned long long seed) {
  g_seed_counter = 0;
  const size_t H = HIDDEN_SIZE, F = FFN_DIM, D = HEAD_DIM;
  g_w.emb_lookup = tensor((size_t)VOCAB_SIZE * H, seed, 0.02f);
  for (int l = 0; l < NUM_LAYERS; ++l) {
    Layer& L = g_w.layers[l];
    L.input_layernorm = tensor(H, seed, 0, true);
    L.transformer.w_q = tensor(NUM_Q_HEADS * D * H, seed, 0.02f);
    L.transformer.w_k = tensor(NUM_KV_HEADS * D * H, seed, 0.02f);
    L.transformer.w_v = tensor(NUM_KV_HEADS * D * H, seed, 0.02f);
    L.transformer.w_o = tensor(H * H, seed, 0.02f);
    L.post_attention_layernorm = tensor(H, seed, 0, true);
    L.ffn_block.w_gate = tensor(F * H, seed, 0.02f);
    L.ffn_block.w_up = tensor(F * H, seed, 0.02f);
    L.ffn_block.w_down = tensor(H * F, seed, 0.02f);
  }
  g_w.final_norm = tensor(H, seed, 0, true);
  g_w.lm_head = tensor((size_t)VOCAB_SIZE * H, seed, 0.02f);
  init_rope_buffer(&g_w.rope.cos, &g_w.rope.sin);
  g_allocs.push_back(g_w.rope.cos);
  g_allocs.push_back(g_w.rope.sin);
  return cudaDeviceSynchronize() == cudaSuccess ? 0 : -1;
}

REF_API void model_free() {
  for (void* p : g_allocs) cudaFree(p);
  g_allocs.clear();
  g_w = ModelWeights{};
}

// Device pointers of the current weights, for running another engine on the
// same model: out[0..4] = embedding, final norm, lm_head, rope cos, rope sin;
// then per layer input_layernorm, w_q, w_k, w_v, w_o, post_attention_layernorm,
// w_gate, w_up, w_down. n: capacity of out. Returns the count written.
REF_API int model_weight_ptrs(void** out, int n) {
  const int need = 5 + 9 * NUM_LAYERS;
  if (n < need) return -1;
  out[0] = g_w.emb_lookup; out[1] = g_w.final_norm; out[2] = g_w.lm_head;
  out[3] = g_w.rope.cos; out[4] = g_w.rope.sin;
  for (int l = 0; l < NUM_LAYERS; ++l) {
    const Layer& L = g_w.layers[l];
    void** o = out + 5 + 9 * l;
    o[0] = L.input_layernorm; o[1] = L.transformer.w_q; o[2] = L.transformer.w_k; o[3] = L.transformer.w_v;
    o[4] = L.transformer.w_o; o[5] = L.post_attention_layernorm; o[6] = L.ffn_block.w_gate;
    o[7] = L.ffn_block.w_up; o[8] = L.ffn_block.w_down;
  }
  return need;
}

// Prefill the prompt, then n_new - 1 decode steps (n_new tokens in total).
// forced (nullable, n_new entries): the token appended after step i is
// forced[i] instead of the model's own pick (teacher forcing); out_tokens[i]
// is always the model's pick. out_margin[i] (nullable): top-1 minus top-2
// logit of step i (fp16 logits read back).
REF_API int model_generate_ex(const int* prompt, int n_prompt, int n_new, const int* forced, int* out_tokens,
                              float* out_margin, float* out_top, double* prefill_ms, double* decode_ms);

REF_API int model_generate(const int* prompt, int n_prompt, int n_new, const int* forced, int* out_tokens,
                           float* out_margin) {
  return model_generate_ex(prompt, n_prompt, n_new, forced, out_tokens, out_margin, nullptr, nullptr, nullptr);
}

// As model_generate; prefill_ms / decode_ms (nullable) receive the host wall
// time of the prefill call and of the n_new - 1 decode_step calls (each of
// which ends in the reference's blocking copy of the token, decode.cu:47).
// With out_margin set the margin read-backs fall inside the decode time.
REF_API int model_generate_timed(const int* prompt, int n_prompt, int n_new, const int* forced, int* out_tokens,
                                 float* out_margin, double* prefill_ms, double* decode_ms) {
  return model_generate_ex(prompt, n_prompt, n_new, forced, out_tokens, out_margin, nullptr, prefill_ms, decode_ms);
}

// As model_generate_timed; out_top (nullable, n_new entries) receives the
// largest fp16 logit of each step, so a margin can be expressed in units of
// the fp16 spacing at the top logit.
REF_API int model_generate_ex(const int* prompt, int n_prompt, int n_new, const int* forced, int* out_tokens,
                              float* out_margin, float* out_top, double* prefill_ms, double* decode_ms) {
  int* tokenid_buff;
  half *data_buffer, *aux_buffer, *attn_buffer, *output_distr;
  int* output_token;
  const size_t row = (size_t)MAX_CONTEXT_LENGTH * HIDDEN_SIZE * sizeof(half);
  if (cudaMalloc(&tokenid_buff, MAX_CONTEXT_LENGTH * sizeof(int)) || cudaMalloc(&data_buffer, row) ||
      cudaMalloc(&aux_buffer, row) || cudaMalloc(&attn_buffer, row) ||
      cudaMalloc(&output_distr, VOCAB_SIZE * sizeof(half)) || cudaMalloc(&output_token, sizeof(int)))
    return -1;
  cublasHandle_t handle;
  cublasCreate(&handle);
  const int max_seq_len = n_prompt + n_new + 1;
  void *workspace, *kv_cache;
  cudaMalloc(&workspace, std::max(attn_workspace_size(max_seq_len), ffn_workspace_size(max_seq_len)));
  cudaMalloc(&kv_cache, kv_cache_size());
  cudaMemset(kv_cache, 0, kv_cache_size());
  std::vector<half> logits(VOCAB_SIZE);
  float top = 0.f;
  auto margin = [&]() {
    cudaMemcpy(logits.data(), output_distr, VOCAB_SIZE * sizeof(half), cudaMemcpyDeviceToHost);
    float a = -INFINITY, b = -INFINITY;
    for (int i = 0; i < VOCAB_SIZE; ++i) {
      const float v = __half2float(logits[i]);
      if (v > a) { b = a; a = v; } else if (v > b) b = v;
    }
    top = a;
    return a - b;
  };
  int seq_len = n_prompt;
  cudaDeviceSynchronize();
  const auto t0 = std::chrono::steady_clock::now();
  cudaMemcpy(tokenid_buff, prompt, n_prompt * sizeof(int), cudaMemcpyHostToDevice);
  int tok = prefill(handle, g_w, seq_len, tokenid_buff, data_buffer, aux_buffer, attn_buffer, output_distr,
                    output_token, workspace, kv_cache);
  const auto t1 = std::chrono::steady_clock::now();
  for (int i = 0; i < n_new; ++i) {
    out_tokens[i] = tok;
    if (out_margin || out_top) {
      const float m = margin();
      if (out_margin) out_margin[i] = m;
      if (out_top) out_top[i] = top;
    }
    if (i + 1 == n_new) break;
    const int next = forced ? forced[i] : tok;
    cudaMemcpy(tokenid_buff + seq_len, &next, sizeof(int), cudaMemcpyHostToDevice);
    ++seq_len;
    tok = decode_step(handle, g_w, seq_len, tokenid_buff, data_buffer, aux_buffer, attn_buffer, output_distr,
                      output_token, workspace, kv_cache);
  }
  const cudaError_t e = cudaDeviceSynchronize();
  const auto t2 = std::chrono::steady_clock::now();
  if (prefill_ms) *prefill_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
  if (decode_ms) *decode_ms = std::chrono::duration<double, std::milli>(t2 - t1).count();
  cudaFree(workspace); cudaFree(kv_cache); cudaFree(data_buffer); cudaFree(aux_buffer); cudaFree(attn_buffer);
  cudaFree(output_distr); cudaFree(output_token); cudaFree(tokenid_buff);
  cublasDestroy(handle);
  return e == cudaSuccess ? 0 : -1;
}
