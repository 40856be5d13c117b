/*
 * infengine_b200 — C-ABI of the B200 (sm_100a) weight-matmul hot path.
 *
 * Every entry point:
 *   - takes plain device pointers, element counts and a cudaStream_t passed as
 *     `void*` (NULL = the legacy default stream, which is what the reference
 *     launches on);
 *   - allocates nothing: scratch is a caller-owned `workspace` sized by the
 *     matching *_workspace_size() function;
 *   - returns IE_OK (0) or a negative IE_ERR_* status; no C++ exception crosses
 *     this boundary;
 *   - validates shapes, pointer alignment (16 bytes for every matrix, leading
 *     dimensions a multiple of 8 elements) before launching anything.
 *
 * Layouts follow the reference: row-major, weights are HF nn.Linear [out, in]
 * ("W[N,K]"), and a projection computes Y[M,N] = X[M,K] . W[N,K]^T with fp32
 * accumulation and one rounding to the storage type at the end.
 *
 * The reference interface each function replaces is cited as
 * path:line inside the Aryan470/infengine tree.
 */
#ifndef INFENGINE_B200_H
#define INFENGINE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- status codes ---------------------------------------------------- */
#define IE_OK                 0
#define IE_ERR_INVALID_ARG   -1 /* null pointer, non-positive or inconsistent size */
#define IE_ERR_ALIGNMENT     -2 /* pointer not 16-byte aligned or ld % 8 != 0     */
#define IE_ERR_UNSUPPORTED   -3 /* shape / dtype combination has no kernel         */
#define IE_ERR_LAUNCH        -4 /* CUDA reported an error at launch                 */
#define IE_ERR_TIMEOUT       -5 /* a bounded device-side wait gave up               */
#define IE_ERR_NO_DEVICE     -6 /* no CUDA device / not an sm_100 device            */
#define IE_ERR_WORKSPACE     -7 /* workspace pointer null or smaller than required  */

/* ---- element types ---------------------------------------------------- */
typedef enum ie_dtype {
  IE_DTYPE_F16 = 0,  /* the reference's storage type (its kernel headers take half*) */
  IE_DTYPE_BF16 = 1  /* the BASELINE configs' storage type                        */
} ie_dtype;

/* Human-readable text of a status code (static storage). */
const char* ie_status_string(int status);

/* Library version, "major.minor.patch". */
const char* ie_version(void);

/* Device-side status of the current device: IE_OK, or IE_ERR_TIMEOUT when a
 * bounded wait inside a tensor-core kernel gave up (the kernel then drained
 * its own copies, freed its tensor memory and returned without finishing).
 * IE_ERR_INVALID_ARG when a batched QKV row carried a position outside its
 * cache (the row was skipped). Synchronizes the device. clear != 0 resets the
 * words to IE_OK. */
int ie_device_status(int clear);

/* Limit, in nanoseconds, of every bounded device-side wait on another party
 * (a TMA copy or MMA inside the tensor-core kernels, a bulk copy inside the
 * decode attention, another rank's rows inside ie_gemm_allreduce). On expiry
 * the kernel records IE_ERR_TIMEOUT (see ie_device_status) and returns.
 * ns = 0 restores the default of 2 s; at most 60 s (IE_ERR_INVALID_ARG
 * above). Applies to the current device, to kernels that start after the
 * call, and to graphs captured before it (the kernels read the limit when
 * they run). A kernel that gives up still waits, for up to 2 s, for the copies
 * and MMAs it issued itself before it exits. The reference has no
 * counterpart (its kernels do not wait on one another). */
int ie_set_wait_limit_ns(unsigned long long ns);

/* ---- a1 / a5: projection GEMM --------------------------------------------
 * Replaces multiply_by_weight (kernels/ffn.cu:7-33, declared in
 * kernels/multiply_by_weight.cuh:3) and the O projection
 * multiply_preproj_Wo (kernels/attn.cu:265-293).
 *   Y[M,N] = X[M,K] . W[N,K]^T ; X row stride ldx, W row stride ldw, Y row stride ldy.
 * M <= 16 runs the decode kernel (weights streamed once with 128-bit loads and
 * warp-level tensor-core dot products); larger M runs the tcgen05/TMEM GEMM.
 */
int ie_gemm(ie_dtype dt, int M, int N, int K,
            const void* X, int64_t ldx,
            const void* W, int64_t ldw,
            void* Y, int64_t ldy,
            void* stream);

/* Same product followed by the residual add of the decode / prefill loop
 * (decode.cu:28,38 with kernels/residual_add.cu:10-20): Y = round(Y +
 * round(X . W^T)), in place on the residual stream Y. No single counterpart in
 * the reference (there: the projection, then residual_add). */
int ie_gemm_add(ie_dtype dt, int M, int N, int K,
                const void* X, int64_t ldx,
                const void* W, int64_t ldw,
                void* Y, int64_t ldy,
                void* stream);

/* Same projection with unrounded fp32 output Y[M,N] (row stride ldy floats,
 * 16-byte aligned): the partial sums of a row-split (tensor-parallel) O or
 * down projection, to be summed across ranks before the one rounding. */
int ie_gemm_f32out(ie_dtype dt, int M, int N, int K,
                   const void* X, int64_t ldx,
                   const void* W, int64_t ldw,
                   float* Y, int64_t ldy,
                   void* stream);

/* ---- a3: SwiGLU ------------------------------------------------------------
 * Replaces swiglu (kernels/swiglu.cu:8-31, kernels/swiglu.cuh:5):
 *   out[i] = g * (1 / (1 + expf(-g))) * u in fp32, rounded to dt.
 * gate/up/out are [M, F] contiguous; out may alias gate or up.
 */
int ie_swiglu(ie_dtype dt, int M, int F,
              const void* gate, const void* up, void* out, void* stream);

/* ---- a2: FFN block -----------------------------------------------------------
 * Replaces ffn / ffn_workspace_size (kernels/ffn.cu:35-64, kernels/ffn.cuh:5-6):
 *   out = W_down . (silu(W_gate . x) * (W_up . x)).
 * Argument order of the weights mirrors ffn(): up, down, gate.
 * Gate and up are rounded to dt before SwiGLU and the SwiGLU product is
 * rounded to dt before the down projection, as in the reference, but the
 * gate/up pair is computed by one kernel whose epilogue applies SwiGLU, so
 * only h[M,F] (not G and U) is written.
 * x: [M,H], W_gate/W_up: [F,H], W_down: [H,F], out: [M,H].
 */
size_t ie_ffn_workspace_size(int M, int F);
int ie_ffn(ie_dtype dt, int M, int H, int F,
           const void* x, const void* W_up, const void* W_down, const void* W_gate,
           void* out, void* workspace, size_t workspace_bytes, void* stream);

/* First half of ie_ffn on its own: h[M,F] (row stride ldh) =
 * round(silu(round(x.W_gate^T)) * round(x.W_up^T)) — the gate/up GEMMs of
 * kernels/ffn.cu:53-54 with swiglu (kernels/swiglu.cu:8-31) as their
 * epilogue. With F a column shard of the FFN width this is the
 * tensor-parallel gate/up step; the down projection of the shard is ie_gemm. */
int ie_ffn_gate_up(ie_dtype dt, int M, int H, int F,
                   const void* x, const void* W_gate, const void* W_up,
                   void* h, int64_t ldh, void* stream);

/* ---- a4: fused Q/K/V projection ------------------------------------------
 * Replaces the three multiply_kqv_proj calls (kernels/attn.cu:12-39, called at
 * :345-347 and :413-415) and, when rope_cos/rope_sin are non-NULL, the two
 * apply_rope calls that follow them (kernels/rope.cu:20-66).
 * One launch computes all n_q_heads + 2*n_kv_heads heads of x[M,H] and writes
 * them head-major like the reference:
 *   q_out  [n_q_heads][M][head_dim]                      (row m at token m)
 *   k_cache[n_kv_heads][.][head_dim], row (pos0 + m), head stride cache_head_stride elements
 *   v_cache same layout as k_cache.
 * Wq: [n_q_heads*head_dim, H], Wk/Wv: [n_kv_heads*head_dim, H].
 * RoPE (rotate-half, pairs (d, d+head_dim/2), table rows = position,
 * table [*, head_dim/2] fp32, 16-byte aligned) is applied to Q and K at
 * position pos0 + m.
 * head_dim must be 128 (the Llama-3.1 value, config.h:16).
 */
int ie_qkv(ie_dtype dt, int M, int H, int n_q_heads, int n_kv_heads, int head_dim,
           const void* x, const void* Wq, const void* Wk, const void* Wv,
           void* q_out, void* k_cache, void* v_cache,
           int64_t cache_head_stride, int pos0,
           const float* rope_cos, const float* rope_sin,
           void* stream);

/* ---- prefill projections with a split of the last wave ------------------
 * ie_gemm, ie_gemm_add, ie_ffn_gate_up and ie_qkv with a caller-owned
 * workspace. For M > 16 the tensor-core kernel runs one persistent CTA per
 * SM; when the tiles leave SMs idle in the last wave it can run the full
 * waves whole and split each tail tile's k-loop into up to 4 ranges spread
 * over all SMs; the last range of a tile adds the others' fp32 partial sums,
 * kept in the workspace, in range order and applies the fused epilogue. It
 * does so for the plain projections (ie_gemm_ws, ie_gemm_add_ws) whose tiles
 * fill less than one wave (short prefill chunks: at M = 128 the O projection
 * takes 22 us instead of 30, down 41 instead of 91) or whose K is at least
 * 8192 (down); ie_qkv_ws and ie_ffn_gate_up_ws accept the workspace but run
 * whole tiles (measured: no gain). The split is chosen per shape and is
 * deterministic; results may differ from the workspace-free call in their
 * last bits (another fp32 summation order).
 * workspace: ie_split_workspace_size() bytes (smaller ones allow fewer
 * splits), 256-byte aligned, zero-filled once when allocated; every call that
 * completes leaves its flag words zeroed again (after IE_ERR_TIMEOUT in
 * ie_device_status, zero it again). NULL runs whole tiles. Calls sharing a
 * workspace must not overlap on the GPU (one stream, or ordered streams).
 * The split assumes that all SMs are available to the launch; with fewer, a
 * tile's last range can wait until its bounded wait expires (IE_ERR_TIMEOUT).
 * M <= 16 ignores the workspace. The reference has no counterpart (cuBLAS
 * chooses its own split inside multiply_by_weight, kernels/ffn.cu:14). */
size_t ie_split_workspace_size(void);
int ie_gemm_ws(ie_dtype dt, int M, int N, int K,
               const void* X, int64_t ldx,
               const void* W, int64_t ldw,
               void* Y, int64_t ldy,
               void* workspace, size_t workspace_bytes, void* stream);
int ie_gemm_add_ws(ie_dtype dt, int M, int N, int K,
                   const void* X, int64_t ldx,
                   const void* W, int64_t ldw,
                   void* Y, int64_t ldy,
                   void* workspace, size_t workspace_bytes, void* stream);
int ie_ffn_gate_up_ws(ie_dtype dt, int M, int H, int F,
                      const void* x, const void* W_gate, const void* W_up,
                      void* h, int64_t ldh,
                      void* workspace, size_t workspace_bytes, void* stream);
int ie_qkv_ws(ie_dtype dt, int M, int H, int n_q_heads, int n_kv_heads, int head_dim,
              const void* x, const void* Wq, const void* Wk, const void* Wv,
              void* q_out, void* k_cache, void* v_cache,
              int64_t cache_head_stride, int pos0,
              const float* rope_cos, const float* rope_sin,
              void* workspace, size_t workspace_bytes, void* stream);

/* Batched decode of B independent sequences (BASELINE config 5 at batch 8):
 * row b of x is a token of sequence b at position positions[b] (device array
 * [B]); its K/V rows go to sequence b's cache, which starts cache_batch_stride
 * elements after sequence b-1's ([B][n_kv_heads][cache_rows][128] with the
 * usual head stride). Q is written [n_q_heads][B][128]. A position outside
 * [0, cache_rows) leaves that row unwritten and sets IE_ERR_INVALID_ARG in
 * ie_device_status. No counterpart in the reference (batch 1 only). */
int ie_qkv_batched(ie_dtype dt, int B, int H, int n_q_heads, int n_kv_heads, int head_dim,
                   const void* x, const void* Wq, const void* Wk, const void* Wv,
                   void* q_out, void* k_cache, void* v_cache,
                   int64_t cache_head_stride, int64_t cache_batch_stride, int cache_rows,
                   const int* positions, const float* rope_cos, const float* rope_sin,
                   void* stream);

/* ---- attention core behind the drop-in attn / decode_attn ---------------
 * Replaces the score / softmax / value steps of attn and decode_attn
 * (kernels/attn.cu:355-366 and :423-431, kernels/softmax.cu:55-160,
 * kernels/attn_permute.cu:15-32). Causal grouped-query attention of S query
 * rows at positions pos0 .. pos0+S-1 over cache rows 0 .. pos0+S-1:
 *   q      [n_q_heads][S][128] (head stride q_head_stride), as ie_qkv writes it;
 *   caches [n_kv_heads][.][128] (head stride cache_head_stride);
 *   out    [S][n_q_heads*128] (row stride ld_out), the input of the O projection.
 * Scores are rounded to dt, scaled by rsqrt(128) and rounded, softmaxed with
 * the reference's roundings. Limits: head_dim 128; n_q_heads a multiple of
 * n_kv_heads; pos0 + S <= INT_MAX and within cache_head_stride / 128 rows.
 * S <= 16 runs the decode kernel below, so its limits apply (group
 * n_q_heads / n_kv_heads in {1, 2, 4, 8}, (pos0 + S) * group <= ~270k, q
 * 16-byte aligned with q_head_stride a multiple of 8).
 * Longer chunks run the tensor-core kernel, which streams scores and needs
 * only ceil(S / 128) <= 65535 and n_q_heads <= 65535. A limit that is not met
 * returns IE_ERR_UNSUPPORTED (or IE_ERR_INVALID_ARG for a too-small cache). */
int ie_attention(ie_dtype dt, int S, int pos0, int n_q_heads, int n_kv_heads, int head_dim,
                 const void* q, int64_t q_head_stride,
                 const void* k_cache, const void* v_cache, int64_t cache_head_stride,
                 void* out, int64_t ld_out, void* stream);

/* Decode-time attention (same chain as ie_attention) for R query rows that
 * each read their whole cache, split over the GPU: every (row, KV head) is
 * served by a cluster of 8 CTAs (16 for at most 4 KV heads), each over an
 * equal share of the cache rows, merged through distributed shared memory. Row m belongs to sequence
 * m / rows_per_seq (cache at + that * cache_batch_stride elements) and sits at
 * position positions[m] (device array, R entries; read when the kernel runs,
 * so a captured graph follows it) or, when positions is NULL, pos0 + m; it
 * attends cache rows 0 .. its position. q [n_q_heads][R][128] (head stride
 * q_head_stride), out [R][n_q_heads*128] (row stride ld_out). A position
 * outside [0, cache_rows) writes zeros and sets IE_ERR_INVALID_ARG in
 * ie_device_status. n_q_heads / n_kv_heads in {1, 2, 4, 8}; cache_rows *
 * group <= ~270k. q, k_cache and v_cache 16-byte aligned, q_head_stride and
 * the cache strides multiples of 8 (IE_ERR_ALIGNMENT otherwise). The reference has no batched or device-positioned form of
 * this (decode_attn, kernels/attn.cu:390-439, serves one row). */
int ie_attention_decode(ie_dtype dt, int R, int rows_per_seq, int n_q_heads, int n_kv_heads, int head_dim,
                        const void* q, int64_t q_head_stride,
                        const void* k_cache, const void* v_cache, int64_t cache_head_stride,
                        int64_t cache_batch_stride, int cache_rows, const int* positions, int pos0,
                        void* out, int64_t ld_out, void* stream);

/* ---- a6 + a7: lm_head with fused greedy argmax --------------------------
 * Replaces lm_head (kernels/lm_head.cu:5-20) followed by sample_token_amax
 * (kernels/sampling.cu:54-58), for M rows at once.
 * Computes logits[m, v] = round_dt(x[m,:] . W[v,:]) for the V rows of W (a
 * vocab shard starting at global id vocab_offset) and picks per row m the
 * index the reference's argmax would pick: the largest rounded logit; among
 * equal logits the id whose (id mod 1024), bit-reversed over 10 bits, is
 * smallest, then the smallest id (the order produced by amax_kern's strided
 * scan over 1024 threads and reduce_amax's halving tree,
 * kernels/sampling.cu:8-51).
 * Outputs (each may be NULL): logits [M, ld_logits], idx_out [M] (global id),
 * key_out [M] packed 64-bit keys; the max of keys across vocab shards is the
 * key of the global winner (ie_argmax_key_index() recovers the id).
 * workspace: ie_lm_head_argmax_workspace_size(M) bytes, zeroed once by the
 * caller when allocated; every call that completes leaves it zeroed again.
 * A call whose device-side wait timed out (IE_ERR_TIMEOUT in
 * ie_device_status) may leave keys and the completion counter set: the
 * caller must zero the workspace again before its next use.
 */
size_t ie_lm_head_argmax_workspace_size(int M);
int ie_lm_head_argmax(ie_dtype dt, int M, int K, int V, int64_t vocab_offset,
                      const void* x, int64_t ldx, const void* W,
                      void* logits, int64_t ld_logits,
                      int* idx_out, unsigned long long* key_out,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ---- allocation-free lm_head + argmax ---------------------------------------
 * No counterpart in the reference. Same computation and outputs as
 * ie_lm_head_argmax, for callers that cannot hand the library a workspace:
 * code written against the reference's signatures (lm_head and
 * sample_token_amax take none), processes whose device memory belongs to a
 * pool allocator, and decode loops that must not call cudaMalloc/cudaFree
 * because those can synchronize the device.
 * It allocates nothing: its scratch (one key per row + a counter) is a fixed
 * 768-byte array declared by the library in device memory, held by every GPU
 * that loads the library until the process exits.
 *   - M is at most 64; larger M returns IE_ERR_UNSUPPORTED.
 *   - All calls share that array: calls whose kernels overlap on the GPU
 *     (other streams or host threads on the same device) race. Each call
 *     clears the array on its stream before launching.
 *   - The first call on a device looks up the array's device address with
 *     that device current; make that first call before any stream capture
 *     begins.
 */
int ie_lm_head_argmax_noalloc(ie_dtype dt, int M, int K, int V, int64_t vocab_offset,
                              const void* x, int64_t ldx, const void* W,
                              void* logits, int64_t ld_logits,
                              int* idx_out, unsigned long long* key_out, void* stream);

/* ---- a7: argmax over stored logits ----------------------------------------
 * Replaces sample_token_amax (kernels/sampling.cu:54-58, sampling.cuh:4) for
 * M rows of V logits (row stride ld). Same tie rule as above. Needs no
 * workspace: one thread-block cluster reduces each row through distributed
 * shared memory.
 */
int ie_argmax(ie_dtype dt, int M, int V, const void* logits, int64_t ld,
              int* idx_out, void* stream);

/* ---- e1: tensor-parallel exchange steps -------------------------------------
 * No counterpart in the reference (single GPU only). Megatron-style split of
 * the path: Q/K/V by heads and gate/up by FFN rows (ie_qkv / ie_ffn_gate_up
 * on the shard), O and down by their input columns (ie_gemm_f32out on the
 * shard, then ie_allreduce_sum_f32, then ie_cast_f32), lm_head by vocabulary
 * rows (ie_lm_head_argmax with vocab_offset and key_out, then
 * ie_argmax_allreduce). The exchanges use NCCL, loaded at run time from the
 * process ("libnccl.so.2"); IE_ERR_UNSUPPORTED when it cannot be found.
 * The communicator is created once per rank from a 128-byte unique id that
 * rank 0 makes with ie_comm_unique_id and the caller distributes. */
typedef struct ie_comm ie_comm;
int ie_comm_unique_id(void* out_128_bytes);
int ie_comm_create(int nranks, int rank, const void* unique_id, ie_comm** out);
int ie_comm_destroy(ie_comm* comm);
/* In-place sum over ranks of count floats. */
int ie_allreduce_sum_f32(ie_comm* comm, float* buf, size_t count, void* stream);
/* In-place max over ranks of M packed argmax keys; idx_out (nullable) [M]
 * receives the winning global vocabulary ids. */
int ie_argmax_allreduce(ie_comm* comm, unsigned long long* keys, int M, int* idx_out, void* stream);
/* out[i] = round_dt(in[i]) for n values. */
int ie_cast_f32(ie_dtype dt, const float* in, void* out, size_t n, void* stream);
/* out[i] = round_dt(out[i] + round_dt(in[i])): a reduced row-split projection
 * added to the residual stream (decode.cu:28,38). */
int ie_add_f32(ie_dtype dt, const float* in, void* out, size_t n, void* stream);

/* Row-split projection fused with its allreduce (decode, M <= 16): every
 * rank runs this on its column shard of X and W; each CTA pushes its fp32
 * partial rows, every value tagged with the call's epoch in one 64-bit word,
 * into every rank's exchange buffer over NVLink as soon as they are computed;
 * the CTA that completes a rank's grid waits (bounded; IE_ERR_TIMEOUT in
 * ie_device_status) until every rank's words of this call have arrived and
 * writes
 *   Y[M,N] = round_dt(sum over ranks, in rank order, of the partials).
 * One kernel per projection replaces ie_gemm_f32out + ie_allreduce_sum_f32 +
 * ie_cast_f32. All ranks must make the same sequence of calls.
 * The exchange: one device buffer per rank of ie_tp_exchange_bytes(world,
 * max_rows, max_cols) bytes, zeroed once, exported with ie_ipc_export and
 * mapped by every other rank with ie_ipc_import; sym is a DEVICE array of
 * world pointers (this process's mapping of every rank's buffer). */
typedef struct ie_tp_exchange {
  int world, rank;
  void* const* sym;
  int max_rows, max_cols;
} ie_tp_exchange;
size_t ie_tp_exchange_bytes(int world, int max_rows, int max_cols);
int ie_ipc_export(const void* dev_ptr, void* handle_out_64_bytes, uint64_t* offset_out);
int ie_ipc_import(const void* handle_64_bytes, uint64_t offset, void** dev_ptr_out);
int ie_ipc_release(void* dev_ptr);
int ie_gemm_allreduce(ie_dtype dt, int M, int N, int K,
                      const void* X, int64_t ldx, const void* W, int64_t ldw,
                      void* Y, int64_t ldy, const ie_tp_exchange* ex, void* stream);
/* The same with the residual add fused: Y = round(Y + round(sum over ranks)). */
int ie_gemm_allreduce_add(ie_dtype dt, int M, int N, int K,
                          const void* X, int64_t ldx, const void* W, int64_t ldw,
                          void* Y, int64_t ldy, const ie_tp_exchange* ex, void* stream);

/* ---- glue of a complete decode step -----------------------------------------
 * RMSNorm with the reference's arithmetic (kernels/rmsnorm.cu:29-62: the same
 * 1024-way partial sums and halving tree, rsqrt(sum / H + eps), out =
 * round(round(x * scale) * w)); out may alias x. */
int ie_rmsnorm(ie_dtype dt, int M, int H, const void* x, int64_t ldx, const void* w,
               void* out, int64_t ldo, float eps, void* stream);
/* Embedding rows (kernels/emblookup.cu:12-27): out[m] = table[tokens[m]],
 * tokens a device array [M]; a token outside [0, vocab) gives a zero row and
 * IE_ERR_INVALID_ARG in ie_device_status. H % 8 == 0. */
int ie_embed(ie_dtype dt, int M, int H, int vocab, const int* tokens, const void* table,
             void* out, int64_t ldo, void* stream);

/* ---- decode engine ------------------------------------------------------------
 * The reference's request flow (manager.cpp:31-86: prefill, then greedy
 * decode_step in a loop, prefill.cu:11-48, decode.cu:11-49) on this library's
 * kernels. Weights are the caller's device pointers, laid out like the
 * reference's ModelWeights (kernels/model_weights.cuh:7-34), in dt. The
 * engine owns its activations, the KV caches of max_batch sequences
 * (max_ctx positions each) and a CUDA graph of one decode step: a step runs
 * every sequence one token forward with positions and tokens kept on the
 * device, so n steps are n graph launches and one copy of the ids. */
typedef struct ie_llama_layer_weights {
  const void* attn_norm;                 /* [H]                         input_layernorm   */
  const void *wq, *wk, *wv;              /* [nq*128, H], [nkv*128, H] x2 transformer.w_q.. */
  const void* wo;                        /* [H, nq*128]                 transformer.w_o   */
  const void* ffn_norm;                  /* [H]                   post_attention_layernorm */
  const void *w_gate, *w_up;             /* [F, H]                      ffn_block         */
  const void* w_down;                    /* [H, F]                                        */
} ie_llama_layer_weights;
typedef struct ie_llama_desc {
  int n_layers, hidden, n_q_heads, n_kv_heads, head_dim, ffn_dim, vocab;
  float rms_eps;
  const void* embedding;                 /* [vocab, H]                                    */
  const ie_llama_layer_weights* layers;  /* host array [n_layers] (copied at create)      */
  const void* final_norm;                /* [H]                                           */
  const void* lm_head;                   /* [vocab, H]                                    */
  const float *rope_cos, *rope_sin;      /* device [>= max_ctx][head_dim/2], 16-B aligned */
} ie_llama_desc;
typedef struct ie_engine ie_engine;
/* stream NULL: the engine makes its own non-blocking stream. max_prefill is
 * the longest chunk ie_engine_prefill accepts. */
int ie_engine_create(ie_dtype dt, const ie_llama_desc* desc, int max_batch, int max_ctx, int max_prefill,
                     void* stream, ie_engine** out);
/* Tensor-parallel engine, one per rank (Megatron split, as ShardPlan in the
 * Python package describes): desc holds this rank's shards, so n_q_heads,
 * n_kv_heads and ffn_dim are the local counts, wq/wk/wv/w_gate/w_up are the
 * rank's rows, wo/w_down the rank's input columns; embedding and norms are
 * full copies and vocab is the full vocabulary. lm_head holds lm_rows rows
 * starting at global id lm_offset. O and down are reduced over the ranks
 * (the NVLink exchange for decode rows when `exchange` is given, else NCCL)
 * with the residual add fused; greedy ids are merged with a max over packed
 * argmax keys (NCCL). Every rank must make the same calls in the same order. */
typedef struct ie_engine_tp {
  int world, rank;
  ie_comm* comm;                    /* required */
  const ie_tp_exchange* exchange;   /* nullable */
  int lm_rows;
  int64_t lm_offset;
} ie_engine_tp;
int ie_engine_create_tp(ie_dtype dt, const ie_llama_desc* desc, int max_batch, int max_ctx, int max_prefill,
                        void* stream, const ie_engine_tp* tp, ie_engine** out);
int ie_engine_destroy(ie_engine* eng);
/* Append n tokens (host array) to sequence seq from its current position;
 * the greedy next token becomes the sequence's next input (and *next_token,
 * when non-NULL). Blocks until done. */
int ie_engine_prefill(ie_engine* eng, int seq, const int* tokens, int n, int* next_token);
/* n_steps greedy steps of all max_batch sequences; out_tokens (host,
 * nullable) receives [n_steps][max_batch] ids. Blocks until done. */
int ie_engine_decode(ie_engine* eng, int n_steps, int* out_tokens);
/* Speculative verify: M <= 16 tokens (host) of sequence seq at positions
 * pos .. pos+M-1 (pos = its current position) in one pass; out_ids[m] is the
 * greedy id after row m. The cache rows are written; the position is not
 * moved (ie_engine_set_position accepts a prefix). */
int ie_engine_verify(ie_engine* eng, int seq, const int* tokens, int M, int* out_ids);
/* One greedy step of all max_batch sequences with host tokens: tokens_in
 * [max_batch] (host) become the sequences' next inputs, tokens_out
 * [max_batch] (host) receive the step's ids; the reference's decode_step
 * contract (decode.cu:11-49: the token comes from and returns to the host).
 * Blocks until done. */
int ie_engine_step(ie_engine* eng, const int* tokens_in, int* tokens_out);
int ie_engine_set_position(ie_engine* eng, int seq, int pos, int next_token);
int ie_engine_position(const ie_engine* eng, int seq);
void* ie_engine_stream(const ie_engine* eng);

/* ---- safetensors weight loading ---------------------------------------------
 * Replaces ModelWeights::from_safetensors (kernels/model_weights.cu:80-154)
 * without a JSON library. ie_st_* read a file's header (host only, no GPU
 * needed); ie_llama_load puts one rank's weights of a Hugging Face Llama
 * checkpoint (model.embed_tokens / model.layers.N.{input_layernorm,
 * self_attn.{q,k,v,o}_proj, post_attention_layernorm, mlp.{gate,up,down}_proj}
 * / model.norm / lm_head, tied embeddings accepted) into one device slab in
 * dt, sharded for rank `rank` of `world` as ie_engine_create_tp expects, plus
 * the RoPE tables for max_ctx positions. The desc it returns is ready for
 * ie_engine_create / ie_engine_create_tp (with ie_llama_model_shard giving
 * lm_rows and lm_offset) and lives as long as the model. */
#define IE_ST_OTHER 0
#define IE_ST_BF16  1
#define IE_ST_F16   2
#define IE_ST_F32   3
typedef struct ie_safetensors ie_safetensors;
int ie_st_open(const char* path, ie_safetensors** out);
int ie_st_close(ie_safetensors* f);
int ie_st_count(const ie_safetensors* f);
const char* ie_st_name(const ie_safetensors* f, int i);
/* shape: room for 8 dimensions */
int ie_st_info(const ie_safetensors* f, const char* name, int* dtype, int* ndim, int64_t* shape, uint64_t* nbytes);
typedef struct ie_llama_model ie_llama_model;
int ie_llama_load(const char* const* paths, int n_paths, ie_dtype dt, int world, int rank, int max_ctx,
                  float rms_eps, void* stream, ie_llama_model** out);
const ie_llama_desc* ie_llama_model_desc(const ie_llama_model* m);
int ie_llama_model_shard(const ie_llama_model* m, int* lm_rows, int64_t* lm_offset);
int ie_llama_model_free(ie_llama_model* m);

/* Global vocabulary id held in a packed argmax key. */
static inline int ie_argmax_key_index(unsigned long long key) {
  unsigned int tie = ~(unsigned int)(key & 0xffffffffull);
  unsigned int rr = tie >> 21, q = tie & ((1u << 21) - 1u), r = 0u, b;
  for (b = 0; b < 10u; ++b) r |= ((rr >> b) & 1u) << (9u - b); /* undo the 10-bit reversal */
  return (int)(q * 1024u + r);
}

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* INFENGINE_B200_H */
