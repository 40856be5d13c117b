// Llama decode engine: the reference's request flow (manager.cpp:31-86 with
// prefill.cu:11-48 and decode.cu:11-49) run on this library's kernels, with
// the step kept on the device.
//
//  * One engine holds max_batch sequences, each with its own KV cache
//    ([layer][K|V][seq][kv head][max_ctx][128]), position and next input token.
//  * Prefill appends a chunk of tokens to one sequence (tensor-core GEMMs for
//    chunks of more than 16 tokens) and leaves the greedy next token on the
//    device.
//  * A decode step advances every sequence by one token: embedding, per layer
//    RMSNorm -> fused QKV+RoPE+cache write at each sequence's device-resident
//    position -> split-KV attention -> O projection with the residual add ->
//    RMSNorm -> gate/up+SwiGLU -> down projection with the residual add, then
//    the final RMSNorm, lm_head with the fused argmax (ids written straight
//    into the next step's input), and a bookkeeping kernel that appends the
//    ids to a device history and advances the positions. Nothing in the step
//    depends on host values, so it is captured once as a CUDA graph and
//    replayed; n steps cost n graph launches and one copy of the ids at the
//    end (the reference: about 612 launches and one blocking copy per token,
//    decode.cu:47).
//  * Verify runs M rows of one sequence (draft tokens) through the model at
//    its current position and returns the greedy id after each row.
//  * Tensor parallel (ie_engine_create_tp): every rank holds its shards; the
//    O and down projections are reduced over the ranks with the residual add
//    fused (NVLink exchange kernel for decode rows, NCCL otherwise) and the
//    vocabulary-split lm_head is merged with a max over packed argmax keys.
//    The collectives are captured in the same decode graph.
//
// Numerics are the library's kernels' (one rounding per projection as the
// reference's cuBLAS calls, RMSNorm and residual add as the reference's
// kernels); the engine adds no arithmetic of its own.
#include <cstring>
#include <new>
#include <vector>
#include "ie_common.cuh"
#include "norm.cuh"

namespace {

constexpr int kHistorySlots = 4096;

struct Engine {
  ie_dtype dt;
  ie_llama_desc d;
  std::vector<ie_llama_layer_weights> layers;
  int B, ctx, max_rows;
  size_t esz;
  cudaStream_t st = nullptr;
  bool own_stream = false;
  // activations (rows = max(max_prefill, max_batch))
  void *x = nullptr, *a = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr;
  void* kv = nullptr;  // [L][2][B][nkv][ctx][128]
  int64_t chs = 0, cbs = 0, layer_elems = 0;
  int *tok_in = nullptr, *positions = nullptr, *history = nullptr, *step = nullptr, *chunk = nullptr,
      *ids = nullptr;
  void* lm_ws = nullptr;
  size_t lm_ws_bytes = 0;
  // tail-split workspace of the prefill projections (chunks of > 16 rows)
  void* split_ws = nullptr;
  size_t split_ws_bytes = 0;
  std::vector<int> pos_host;
  long long step_host = 0;
  // pinned staging of ie_engine_step's tokens in [0, B) and ids out [B, 2B)
  int* h_tok = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  // tensor parallelism (world == 1: single GPU)
  int world = 1, rank = 0;
  ie_comm* comm = nullptr;
  bool has_ex = false;
  ie_tp_exchange ex{};
  int lm_rows = 0;
  int64_t lm_offset = 0;
  float* part = nullptr;               // fp32 [max_rows][H] partial sums (NCCL reduction)
  unsigned long long* keys = nullptr;  // packed argmax keys [max(B, 16)]

  void* kcache(int l, int seq) const {
    return static_cast<char*>(kv) + ((size_t)l * layer_elems + (size_t)seq * cbs) * esz;
  }
  void* vcache(int l, int seq) const {
    return static_cast<char*>(kv) + ((size_t)l * layer_elems + (size_t)B * cbs + (size_t)seq * cbs) * esz;
  }
  void* row(void* base, int64_t r, int64_t width) const { return static_cast<char*>(base) + r * width * esz; }
};

int check(cudaError_t e) { return e == cudaSuccess ? IE_OK : IE_ERR_LAUNCH; }

#define IE_TRY(expr)             \
  do {                           \
    const int s_ = (expr);       \
    if (s_ != IE_OK) return s_;  \
  } while (0)

// x += round(X . W^T) for the O and down projections: one kernel on one GPU;
// with tensor parallelism X and W are the rank's input columns and the
// partial products are summed over the ranks before the rounding, by the
// NVLink exchange kernel (decode rows) or NCCL (longer chunks).
int proj_add(Engine& E, int M, int K, const void* X, const void* W) {
  const int H = E.d.hidden;
  if (E.world == 1) return ie_gemm_add_ws(E.dt, M, H, K, X, K, W, K, E.x, H, E.split_ws, E.split_ws_bytes, E.st);
  if (E.has_ex && M <= 16 && M <= E.ex.max_rows)
    return ie_gemm_allreduce_add(E.dt, M, H, K, X, K, W, K, E.x, H, &E.ex, E.st);
  IE_TRY(ie_gemm_f32out(E.dt, M, H, K, X, K, W, K, E.part, H, E.st));
  IE_TRY(ie_allreduce_sum_f32(E.comm, E.part, (size_t)M * H, E.st));
  return ie_add_f32(E.dt, E.part, E.x, (size_t)M * H, E.st);
}

// One transformer layer over M rows of the residual stream x. seq >= 0: the M
// rows are consecutive tokens of sequence seq from position pos0 (prefill /
// verify); seq < 0: row b is the next token of sequence b at its device
// position (decode step, M = B).
int layer_forward(Engine& E, int l, int M, int seq, int pos0) {
  const ie_llama_desc& d = E.d;
  const ie_llama_layer_weights& w = E.layers[l];
  const int H = d.hidden, F = d.ffn_dim, nq = d.n_q_heads, nkv = d.n_kv_heads, hd = d.head_dim;
  void* st = E.st;
  IE_TRY(ie_rmsnorm(E.dt, M, H, E.x, H, w.attn_norm, E.a, H, d.rms_eps, st));
  if (seq < 0) {
    IE_TRY(ie_qkv_batched(E.dt, M, H, nq, nkv, hd, E.a, w.wq, w.wk, w.wv, E.q, E.kcache(l, 0), E.vcache(l, 0), E.chs,
                          E.cbs, E.ctx, E.positions, d.rope_cos, d.rope_sin, st));
    IE_TRY(ie_attention_decode(E.dt, M, 1, nq, nkv, hd, E.q, (int64_t)M * hd, E.kcache(l, 0), E.vcache(l, 0), E.chs,
                               E.cbs, E.ctx, E.positions, 0, E.attn, (int64_t)nq * hd, st));
  } else {
    IE_TRY(ie_qkv_ws(E.dt, M, H, nq, nkv, hd, E.a, w.wq, w.wk, w.wv, E.q, E.kcache(l, seq), E.vcache(l, seq), E.chs,
                     pos0, d.rope_cos, d.rope_sin, E.split_ws, E.split_ws_bytes, st));
    if (M <= 16)
      IE_TRY(ie_attention_decode(E.dt, M, M, nq, nkv, hd, E.q, (int64_t)M * hd, E.kcache(l, seq), E.vcache(l, seq),
                                 E.chs, E.cbs, E.ctx, nullptr, pos0, E.attn, (int64_t)nq * hd, st));
    else
      IE_TRY(ie_attention(E.dt, M, pos0, nq, nkv, hd, E.q, (int64_t)M * hd, E.kcache(l, seq), E.vcache(l, seq), E.chs,
                          E.attn, (int64_t)nq * hd, st));
  }
  IE_TRY(proj_add(E, M, nq * hd, E.attn, w.wo));
  IE_TRY(ie_rmsnorm(E.dt, M, H, E.x, H, w.ffn_norm, E.a, H, d.rms_eps, st));
  IE_TRY(ie_ffn_gate_up_ws(E.dt, M, H, F, E.a, w.w_gate, w.w_up, E.h, F, E.split_ws, E.split_ws_bytes, st));
  IE_TRY(proj_add(E, M, F, E.h, w.w_down));
  return IE_OK;
}

// Final norm + lm_head/argmax of `rows` rows starting at row r0 into ids_out.
int head_forward(Engine& E, int r0, int rows, int* ids_out) {
  const ie_llama_desc& d = E.d;
  const int H = d.hidden;
  IE_TRY(ie_rmsnorm(E.dt, rows, H, E.row(E.x, r0, H), H, d.final_norm, E.a, H, d.rms_eps, E.st));
  if (E.world == 1)
    return ie_lm_head_argmax(E.dt, rows, H, d.vocab, 0, E.a, H, d.lm_head, nullptr, 0, ids_out, nullptr, E.lm_ws,
                             E.lm_ws_bytes, E.st);
  // vocabulary shard: local winners as packed keys, then the max over ranks
  IE_TRY(ie_lm_head_argmax(E.dt, rows, H, E.lm_rows, E.lm_offset, E.a, H, d.lm_head, nullptr, 0, nullptr, E.keys,
                           E.lm_ws, E.lm_ws_bytes, E.st));
  return ie_argmax_allreduce(E.comm, E.keys, rows, ids_out, E.st);
}

int decode_step(Engine& E) {
  const ie_llama_desc& d = E.d;
  IE_TRY(ie_embed(E.dt, E.B, d.hidden, d.vocab, E.tok_in, d.embedding, E.x, d.hidden, E.st));
  for (int l = 0; l < d.n_layers; ++l) IE_TRY(layer_forward(E, l, E.B, -1, 0));
  IE_TRY(head_forward(E, 0, E.B, E.tok_in));
  return check(ie::launch_advance(E.B, E.tok_in, E.positions, E.history, kHistorySlots, E.step, E.st));
}

int capture(Engine& E) {
  if (E.exec) return IE_OK;
  if (cudaStreamBeginCapture(E.st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return IE_ERR_LAUNCH;
  const int s = decode_step(E);
  cudaGraph_t g = nullptr;
  const cudaError_t e = cudaStreamEndCapture(E.st, &g);
  if (s != IE_OK || e != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    return s != IE_OK ? s : IE_ERR_LAUNCH;
  }
  if (cudaGraphInstantiate(&E.exec, g, 0) != cudaSuccess) {
    cudaGraphDestroy(g);
    E.exec = nullptr;
    return IE_ERR_LAUNCH;
  }
  E.graph = g;
  return IE_OK;
}

void release(Engine* E) {
  if (E->exec) cudaGraphExecDestroy(E->exec);
  if (E->graph) cudaGraphDestroy(E->graph);
  void* bufs[] = {E->x,       E->a,     E->q,    E->attn,  E->h,     E->kv,    E->tok_in, E->positions,
                  E->history, E->step,  E->chunk, E->ids,  E->lm_ws, E->part, E->keys, E->split_ws};
  for (void* p : bufs)
    if (p) cudaFree(p);
  if (E->h_tok) cudaFreeHost(E->h_tok);
  if (E->own_stream && E->st) cudaStreamDestroy(E->st);
  delete E;
}

bool valid_desc(const ie_llama_desc* d) {
  if (!d || d->n_layers <= 0 || d->hidden <= 0 || d->n_q_heads <= 0 || d->n_kv_heads <= 0 || d->ffn_dim <= 0 ||
      d->vocab <= 0 || !d->embedding || !d->layers || !d->final_norm || !d->lm_head || !d->rope_cos || !d->rope_sin)
    return false;
  if (d->head_dim != 128 || d->n_q_heads % d->n_kv_heads || d->hidden % 8 || d->ffn_dim % 8) return false;
  for (int l = 0; l < d->n_layers; ++l) {
    const ie_llama_layer_weights& w = d->layers[l];
    if (!w.attn_norm || !w.wq || !w.wk || !w.wv || !w.wo || !w.ffn_norm || !w.w_gate || !w.w_up || !w.w_down)
      return false;
  }
  return true;
}

}  // namespace

struct ie_engine {
  Engine* e;
};

extern "C" {

int ie_engine_create(ie_dtype dt, const ie_llama_desc* desc, int max_batch, int max_ctx, int max_prefill,
                     void* stream, ie_engine** out) {
  return ie_engine_create_tp(dt, desc, max_batch, max_ctx, max_prefill, stream, nullptr, out);
}

int ie_engine_create_tp(ie_dtype dt, const ie_llama_desc* desc, int max_batch, int max_ctx, int max_prefill,
                        void* stream, const ie_engine_tp* tp, ie_engine** out) {
  if (!out) return IE_ERR_INVALID_ARG;
  *out = nullptr;
  if ((dt != IE_DTYPE_F16 && dt != IE_DTYPE_BF16) || !valid_desc(desc)) return IE_ERR_INVALID_ARG;
  if (max_batch <= 0 || max_batch > 64 || max_ctx <= 0 || max_prefill < 0) return IE_ERR_INVALID_ARG;
  if (tp && tp->world > 1) {
    if (tp->rank < 0 || tp->rank >= tp->world || !tp->comm || tp->lm_rows <= 0 || tp->lm_offset < 0 ||
        tp->lm_offset + tp->lm_rows > desc->vocab)
      return IE_ERR_INVALID_ARG;
    if (tp->exchange && (tp->exchange->world != tp->world || tp->exchange->rank != tp->rank)) return IE_ERR_INVALID_ARG;
  }
  Engine* E = new (std::nothrow) Engine();
  if (!E) return IE_ERR_INVALID_ARG;
  if (tp && tp->world > 1) {
    E->world = tp->world;
    E->rank = tp->rank;
    E->comm = tp->comm;
    E->has_ex = tp->exchange != nullptr;
    if (tp->exchange) E->ex = *tp->exchange;
    E->lm_rows = tp->lm_rows;
    E->lm_offset = tp->lm_offset;
  }
  E->dt = dt;
  E->d = *desc;
  E->layers.assign(desc->layers, desc->layers + desc->n_layers);
  E->d.layers = E->layers.data();
  E->B = max_batch;
  E->ctx = max_ctx;
  E->max_rows = max_prefill > max_batch ? max_prefill : max_batch;
  E->esz = 2;
  E->pos_host.assign(max_batch, 0);
  const ie_llama_desc& d = E->d;
  const size_t R = E->max_rows, H = d.hidden, qd = (size_t)d.n_q_heads * d.head_dim;
  E->chs = (int64_t)max_ctx * d.head_dim;
  E->cbs = (int64_t)d.n_kv_heads * E->chs;
  E->layer_elems = 2 * (int64_t)max_batch * E->cbs;
  E->lm_ws_bytes = ie_lm_head_argmax_workspace_size(max_batch > 16 ? max_batch : 16);
  bool ok = true;
  if (stream) {
    E->st = static_cast<cudaStream_t>(stream);
  } else {
    ok = cudaStreamCreateWithFlags(&E->st, cudaStreamNonBlocking) == cudaSuccess;
    E->own_stream = ok;
  }
  auto alloc = [&](void** p, size_t bytes) {
    if (ok) ok = cudaMalloc(p, bytes) == cudaSuccess;
  };
  alloc(&E->x, R * H * 2);
  alloc(&E->a, R * H * 2);
  alloc(&E->q, R * qd * 2);
  alloc(&E->attn, R * qd * 2);
  alloc(&E->h, R * d.ffn_dim * 2);
  alloc(&E->kv, (size_t)d.n_layers * E->layer_elems * 2);
  alloc(reinterpret_cast<void**>(&E->tok_in), max_batch * sizeof(int));
  alloc(reinterpret_cast<void**>(&E->positions), max_batch * sizeof(int));
  alloc(reinterpret_cast<void**>(&E->history), (size_t)kHistorySlots * max_batch * sizeof(int));
  alloc(reinterpret_cast<void**>(&E->step), sizeof(int));
  alloc(reinterpret_cast<void**>(&E->chunk), R * sizeof(int));
  alloc(reinterpret_cast<void**>(&E->ids), R * sizeof(int));
  alloc(&E->lm_ws, E->lm_ws_bytes);
  if (ok) ok = cudaMallocHost(reinterpret_cast<void**>(&E->h_tok), 2 * max_batch * sizeof(int)) == cudaSuccess;
  if (E->max_rows > 16) {  // prefill chunks run the tensor-core kernels
    E->split_ws_bytes = ie_split_workspace_size();
    alloc(&E->split_ws, E->split_ws_bytes);
  }
  if (E->world > 1) {
    alloc(reinterpret_cast<void**>(&E->part), R * H * sizeof(float));
    alloc(reinterpret_cast<void**>(&E->keys), (size_t)(max_batch > 16 ? max_batch : 16) * sizeof(unsigned long long));
  }
  if (ok) {
    ok = cudaMemsetAsync(E->kv, 0, (size_t)d.n_layers * E->layer_elems * 2, E->st) == cudaSuccess &&
         cudaMemsetAsync(E->tok_in, 0, max_batch * sizeof(int), E->st) == cudaSuccess &&
         cudaMemsetAsync(E->positions, 0, max_batch * sizeof(int), E->st) == cudaSuccess &&
         cudaMemsetAsync(E->step, 0, sizeof(int), E->st) == cudaSuccess &&
         cudaMemsetAsync(E->lm_ws, 0, E->lm_ws_bytes, E->st) == cudaSuccess &&
         (!E->split_ws || cudaMemsetAsync(E->split_ws, 0, E->split_ws_bytes, E->st) == cudaSuccess) &&
         cudaStreamSynchronize(E->st) == cudaSuccess;
  }
  if (!ok) {
    cudaGetLastError();
    release(E);
    return IE_ERR_WORKSPACE;
  }
  *out = new (std::nothrow) ie_engine{E};
  if (!*out) {
    release(E);
    return IE_ERR_INVALID_ARG;
  }
  return IE_OK;
}

int ie_engine_destroy(ie_engine* eng) {
  if (!eng) return IE_OK;
  if (eng->e->st) cudaStreamSynchronize(eng->e->st);
  release(eng->e);
  delete eng;
  return IE_OK;
}

int ie_engine_prefill(ie_engine* eng, int seq, const int* tokens, int n, int* next_token) {
  if (!eng || !tokens || n <= 0) return IE_ERR_INVALID_ARG;
  Engine& E = *eng->e;
  if (seq < 0 || seq >= E.B) return IE_ERR_INVALID_ARG;
  const int pos0 = E.pos_host[seq];
  if (n > E.max_rows || (int64_t)pos0 + n > E.ctx) return IE_ERR_UNSUPPORTED;
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= E.d.vocab) return IE_ERR_INVALID_ARG;
  IE_TRY(check(cudaMemcpyAsync(E.chunk, tokens, n * sizeof(int), cudaMemcpyHostToDevice, E.st)));
  IE_TRY(ie_embed(E.dt, n, E.d.hidden, E.d.vocab, E.chunk, E.d.embedding, E.x, E.d.hidden, E.st));
  for (int l = 0; l < E.d.n_layers; ++l) IE_TRY(layer_forward(E, l, n, seq, pos0));
  IE_TRY(head_forward(E, n - 1, 1, E.tok_in + seq));
  const int pos = pos0 + n;
  IE_TRY(check(cudaMemcpyAsync(E.positions + seq, &pos, sizeof(int), cudaMemcpyHostToDevice, E.st)));
  if (next_token)
    IE_TRY(check(cudaMemcpyAsync(next_token, E.tok_in + seq, sizeof(int), cudaMemcpyDeviceToHost, E.st)));
  IE_TRY(check(cudaStreamSynchronize(E.st)));
  E.pos_host[seq] = pos;
  return IE_OK;
}

int ie_engine_decode(ie_engine* eng, int n_steps, int* out_tokens) {
  if (!eng || n_steps < 0) return IE_ERR_INVALID_ARG;
  Engine& E = *eng->e;
  if (n_steps == 0) return IE_OK;
  for (int b = 0; b < E.B; ++b)
    if ((int64_t)E.pos_host[b] + n_steps > E.ctx) return IE_ERR_UNSUPPORTED;
  IE_TRY(capture(E));
  int done = 0;
  while (done < n_steps) {
    const int first = (int)(E.step_host % kHistorySlots);
    int n = n_steps - done;
    if (n > kHistorySlots - first) n = kHistorySlots - first;
    for (int i = 0; i < n; ++i) IE_TRY(check(cudaGraphLaunch(E.exec, E.st)));
    if (out_tokens)
      IE_TRY(check(cudaMemcpyAsync(out_tokens + (size_t)done * E.B, E.history + (size_t)first * E.B,
                                   (size_t)n * E.B * sizeof(int), cudaMemcpyDeviceToHost, E.st)));
    IE_TRY(check(cudaStreamSynchronize(E.st)));
    E.step_host += n;
    done += n;
  }
  for (int b = 0; b < E.B; ++b) E.pos_host[b] += n_steps;
  return IE_OK;
}

int ie_engine_verify(ie_engine* eng, int seq, const int* tokens, int M, int* out_ids) {
  if (!eng || !tokens || !out_ids || M <= 0) return IE_ERR_INVALID_ARG;
  Engine& E = *eng->e;
  if (seq < 0 || seq >= E.B || M > 16 || M > E.max_rows) return IE_ERR_INVALID_ARG;
  const int pos0 = E.pos_host[seq];
  if ((int64_t)pos0 + M > E.ctx) return IE_ERR_UNSUPPORTED;
  for (int i = 0; i < M; ++i)
    if (tokens[i] < 0 || tokens[i] >= E.d.vocab) return IE_ERR_INVALID_ARG;
  IE_TRY(check(cudaMemcpyAsync(E.chunk, tokens, M * sizeof(int), cudaMemcpyHostToDevice, E.st)));
  IE_TRY(ie_embed(E.dt, M, E.d.hidden, E.d.vocab, E.chunk, E.d.embedding, E.x, E.d.hidden, E.st));
  for (int l = 0; l < E.d.n_layers; ++l) IE_TRY(layer_forward(E, l, M, seq, pos0));
  IE_TRY(head_forward(E, 0, M, E.ids));
  IE_TRY(check(cudaMemcpyAsync(out_ids, E.ids, M * sizeof(int), cudaMemcpyDeviceToHost, E.st)));
  return check(cudaStreamSynchronize(E.st));
}

int ie_engine_step(ie_engine* eng, const int* tokens_in, int* tokens_out) {
  if (!eng || !tokens_in || !tokens_out) return IE_ERR_INVALID_ARG;
  Engine& E = *eng->e;
  for (int b = 0; b < E.B; ++b) {
    if (tokens_in[b] < 0 || tokens_in[b] >= E.d.vocab) return IE_ERR_INVALID_ARG;
    if (E.pos_host[b] + 1 > E.ctx) return IE_ERR_UNSUPPORTED;
  }
  IE_TRY(capture(E));
  // the copies go through pinned staging, so both are plain DMA transfers
  std::memcpy(E.h_tok, tokens_in, E.B * sizeof(int));
  IE_TRY(check(cudaMemcpyAsync(E.tok_in, E.h_tok, E.B * sizeof(int), cudaMemcpyHostToDevice, E.st)));
  IE_TRY(check(cudaGraphLaunch(E.exec, E.st)));
  IE_TRY(check(cudaMemcpyAsync(E.h_tok + E.B, E.tok_in, E.B * sizeof(int), cudaMemcpyDeviceToHost, E.st)));
  IE_TRY(check(cudaStreamSynchronize(E.st)));
  std::memcpy(tokens_out, E.h_tok + E.B, E.B * sizeof(int));
  E.step_host += 1;
  for (int b = 0; b < E.B; ++b) E.pos_host[b] += 1;
  return IE_OK;
}

int ie_engine_set_position(ie_engine* eng, int seq, int pos, int next_token) {
  if (!eng) return IE_ERR_INVALID_ARG;
  Engine& E = *eng->e;
  if (seq < 0 || seq >= E.B || pos < 0 || pos > E.ctx || next_token < 0 || next_token >= E.d.vocab)
    return IE_ERR_INVALID_ARG;
  IE_TRY(check(cudaMemcpyAsync(E.positions + seq, &pos, sizeof(int), cudaMemcpyHostToDevice, E.st)));
  IE_TRY(check(cudaMemcpyAsync(E.tok_in + seq, &next_token, sizeof(int), cudaMemcpyHostToDevice, E.st)));
  IE_TRY(check(cudaStreamSynchronize(E.st)));
  E.pos_host[seq] = pos;
  return IE_OK;
}

int ie_engine_position(const ie_engine* eng, int seq) {
  if (!eng || seq < 0 || seq >= eng->e->B) return IE_ERR_INVALID_ARG;
  return eng->e->pos_host[seq];
}

void* ie_engine_stream(const ie_engine* eng) { return eng ? static_cast<void*>(eng->e->st) : nullptr; }

}  // extern "C"
