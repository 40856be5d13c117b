"""infengine_b200 — B200 (sm_100a) weight-matmul hot path of infengine.

Python mirror of the reference's kernel entry points (kernels/*.cuh of
Aryan470/infengine) over the C-ABI in include/infengine_b200.h. The names and
argument meanings follow the reference:

    multiply_by_weight(m, k, n, d_in, d_w, d_out)      kernels/multiply_by_weight.cuh:3
    ffn(seq_len, d_in, d_out, d_wup, d_wdown, d_wgate,
        workspace)                                       kernels/ffn.cuh:6
    ffn_workspace_size(max_seq_len)                      kernels/ffn.cuh:5
    swiglu(seq_len, d_gate, d_up, d_output)              kernels/swiglu.cuh:5
    lm_head(seq_len, d_input, d_weight, d_output)        kernels/lm_head.cuh:4
    sample_token_amax(d_logits, d_output)                kernels/sampling.cuh:4

Device buffers are torch CUDA tensors (torch is only the allocator and the
stream provider here). The reference takes a cublasHandle_t whose only role
on this path is the stream; these functions take `stream=` instead (default:
torch's current stream). Failures raise IEError carrying the library status,
where the reference would silently continue.

There is no CPU path: every call goes to libinfengine_b200.so and raises if
the library or a CUDA device is missing.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libinfengine_b200.so"
DROPIN_PATH = _PKG / "libinfengine_dropin.so"

# Llama-3.1-8B constants (reference config.h:5-26)
MAX_CONTEXT_LENGTH = 8192
VOCAB_SIZE = 128256
NUM_LAYERS = 32
HIDDEN_SIZE = 4096
NUM_Q_HEADS = 32
NUM_KV_HEADS = 8
HEAD_DIM = 128
FFN_DIM = 14336

IE_DTYPE_F16 = 0
IE_DTYPE_BF16 = 1

STATUS = {
    0: "ok", -1: "invalid argument", -2: "misaligned pointer or leading dimension",
    -3: "unsupported shape or dtype", -4: "CUDA launch error", -5: "device-side wait timed out",
    -6: "no usable sm_100 device", -7: "workspace missing or too small",
}

EXPORTED_SYMBOLS = (
    "ie_status_string", "ie_version", "ie_gemm", "ie_swiglu", "ie_ffn_workspace_size", "ie_ffn", "ie_ffn_gate_up",
    "ie_qkv", "ie_lm_head_argmax_workspace_size", "ie_lm_head_argmax", "ie_argmax", "ie_device_status",
    "ie_lm_head_argmax_noalloc", "ie_attention", "ie_gemm_f32out", "ie_comm_unique_id", "ie_comm_create",
    "ie_comm_destroy", "ie_allreduce_sum_f32", "ie_argmax_allreduce", "ie_cast_f32", "ie_tp_exchange_bytes",
    "ie_ipc_export", "ie_ipc_import", "ie_ipc_release", "ie_gemm_allreduce", "ie_qkv_batched",
    "ie_attention_decode", "ie_gemm_add", "ie_gemm_allreduce_add", "ie_rmsnorm", "ie_embed", "ie_engine_create",
    "ie_engine_destroy", "ie_engine_prefill", "ie_engine_decode", "ie_engine_verify", "ie_engine_set_position",
    "ie_engine_position", "ie_engine_stream", "ie_engine_step", "ie_engine_create_tp", "ie_add_f32",
    "ie_set_wait_limit_ns", "ie_split_workspace_size", "ie_gemm_ws", "ie_gemm_add_ws", "ie_ffn_gate_up_ws",
    "ie_qkv_ws",
    "ie_st_open", "ie_st_close", "ie_st_count", "ie_st_name", "ie_st_info", "ie_llama_load", "ie_llama_model_desc",
    "ie_llama_model_shard", "ie_llama_model_free",
)


class IEError(RuntimeError):
    def __init__(self, status: int, what: str):
        super().__init__(f"{what}: {STATUS.get(status, 'unknown')} ({status})")
        self.status = status


_lib_handle = None


def lib() -> ctypes.CDLL:
    """Load libinfengine_b200.so (raises if it was not built)."""
    global _lib_handle
    if _lib_handle is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m infengine_b200.build`")
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
        L.ie_status_string.restype = ctypes.c_char_p
        L.ie_status_string.argtypes = [i32]
        L.ie_version.restype = ctypes.c_char_p
        L.ie_device_status.argtypes = [i32]
        L.ie_device_status.restype = i32
        L.ie_set_wait_limit_ns.argtypes = [ctypes.c_ulonglong]
        L.ie_set_wait_limit_ns.restype = i32
        L.ie_split_workspace_size.restype = sz
        L.ie_split_workspace_size.argtypes = []
        L.ie_gemm_ws.argtypes = [i32, i32, i32, i32, vp, i64, vp, i64, vp, i64, vp, sz, vp]
        L.ie_gemm_add_ws.argtypes = [i32, i32, i32, i32, vp, i64, vp, i64, vp, i64, vp, sz, vp]
        L.ie_ffn_gate_up_ws.argtypes = [i32, i32, i32, i32, vp, vp, vp, vp, i64, vp, sz, vp]
        L.ie_qkv_ws.argtypes = [i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, i64, i32, vp, vp, vp, sz,
                                vp]
        L.ie_gemm.argtypes = [i32, i32, i32, i32, vp, i64, vp, i64, vp, i64, vp]
        L.ie_gemm_add.argtypes = [i32, i32, i32, i32, vp, i64, vp, i64, vp, i64, vp]
        L.ie_gemm_add.restype = i32
        L.ie_swiglu.argtypes = [i32, i32, i32, vp, vp, vp, vp]
        L.ie_ffn_workspace_size.restype = sz
        L.ie_ffn_workspace_size.argtypes = [i32, i32]
        L.ie_ffn.argtypes = [i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, sz, vp]
        L.ie_ffn_gate_up.argtypes = [i32, i32, i32, i32, vp, vp, vp, vp, i64, vp]
        L.ie_ffn_gate_up.restype = i32
        L.ie_qkv.argtypes = [i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, i64, i32, vp, vp, vp]
        L.ie_qkv_batched.argtypes = [i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, i64, i64, i32, vp, vp,
                                     vp, vp]
        L.ie_qkv_batched.restype = i32
        L.ie_lm_head_argmax_workspace_size.restype = sz
        L.ie_lm_head_argmax_workspace_size.argtypes = [i32]
        L.ie_lm_head_argmax.argtypes = [i32, i32, i32, i32, i64, vp, i64, vp, vp, i64, vp, vp, vp, sz, vp]
        L.ie_argmax.argtypes = [i32, i32, i32, vp, i64, vp, vp]
        L.ie_attention.argtypes = [i32, i32, i32, i32, i32, i32, vp, i64, vp, vp, i64, vp, i64, vp]
        L.ie_attention.restype = i32
        L.ie_attention_decode.argtypes = [i32, i32, i32, i32, i32, i32, vp, i64, vp, vp, i64, i64, i32, vp, i32, vp,
                                          i64, vp]
        L.ie_attention_decode.restype = i32
        L.ie_lm_head_argmax_noalloc.argtypes = [i32, i32, i32, i32, i64, vp, i64, vp, vp, i64, vp, vp, vp]
        L.ie_lm_head_argmax_noalloc.restype = i32
        for name in ("ie_gemm", "ie_swiglu", "ie_ffn", "ie_qkv", "ie_lm_head_argmax", "ie_argmax"):
            getattr(L, name).restype = i32
        _lib_handle = L
    return _lib_handle


# ------------------------------------------------------------------ helpers
def _torch():
    import torch
    return torch


def _dt(t) -> int:
    torch = _torch()
    if t.dtype == torch.float16:
        return IE_DTYPE_F16
    if t.dtype == torch.bfloat16:
        return IE_DTYPE_BF16
    raise TypeError(f"unsupported dtype {t.dtype} (float16 or bfloat16)")


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("infengine_b200 operates on CUDA tensors only")
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        return ctypes.c_void_p(_torch().cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return ctypes.c_void_p(stream)
    return ctypes.c_void_p(stream.cuda_stream)


def _check(status: int, what: str) -> None:
    if status != 0:
        raise IEError(status, what)


# -------------------------------------------------------------- C-ABI mirror
def gemm_add(x, w, y, stream=None, workspace=None):
    """y[M,N] = round(y + round(x[M,K] . w[N,K]^T)) in place (ie_gemm_add):
    a projection with the residual add fused. workspace (split_workspace()):
    ie_gemm_add_ws, the prefill kernel splits its last wave."""
    M, K = x.shape
    N = w.shape[0]
    if workspace is not None:
        _check(lib().ie_gemm_add_ws(_dt(x), M, N, K, _ptr(x), x.stride(0), _ptr(w), w.stride(0), _ptr(y),
                                    y.stride(0), _ptr(workspace), _nbytes(workspace), _stream(stream)),
               "ie_gemm_add_ws")
        return
    _check(lib().ie_gemm_add(_dt(x), M, N, K, _ptr(x), x.stride(0), _ptr(w), w.stride(0), _ptr(y), y.stride(0),
                             _stream(stream)), "ie_gemm_add")


def _nbytes(t) -> int:
    return t.numel() * t.element_size()


def split_workspace_bytes() -> int:
    """ie_split_workspace_size: bytes of the prefill tail-split workspace."""
    return int(lib().ie_split_workspace_size())


def split_workspace(device="cuda"):
    """A zeroed tail-split workspace for the *_ws entry points (256-byte
    aligned, as torch's allocator returns)."""
    import torch
    return torch.zeros(split_workspace_bytes(), dtype=torch.uint8, device=device)


def gemm(x, w, y, M=None, N=None, K=None, ldx=None, ldw=None, ldy=None, stream=None, workspace=None):
    """y[M,N] = x[M,K] . w[N,K]^T (ie_gemm; ie_gemm_ws with a workspace)."""
    M = x.shape[0] if M is None else M
    K = x.shape[-1] if K is None else K
    N = w.shape[0] if N is None else N
    ldx = x.stride(0) if ldx is None else ldx
    ldw = w.stride(0) if ldw is None else ldw
    ldy = y.stride(0) if ldy is None else ldy
    if workspace is not None:
        _check(lib().ie_gemm_ws(_dt(x), M, N, K, _ptr(x), ldx, _ptr(w), ldw, _ptr(y), ldy, _ptr(workspace),
                                _nbytes(workspace), _stream(stream)), "ie_gemm_ws")
        return
    _check(lib().ie_gemm(_dt(x), M, N, K, _ptr(x), ldx, _ptr(w), ldw, _ptr(y), ldy, _stream(stream)), "ie_gemm")


def ffn_fused(x, w_up, w_down, w_gate, out, workspace, stream=None):
    M, H = x.shape
    F = w_up.shape[0]
    _check(lib().ie_ffn(_dt(x), M, H, F, _ptr(x), _ptr(w_up), _ptr(w_down), _ptr(w_gate), _ptr(out),
                        _ptr(workspace), workspace.numel() * workspace.element_size(), _stream(stream)), "ie_ffn")


def ffn_gate_up(x, w_gate, w_up, h, stream=None, workspace=None):
    """h = silu(x.Wg^T) * (x.Wu^T) with the reference's roundings
    (ie_ffn_gate_up; ie_ffn_gate_up_ws with a workspace)."""
    M, H = x.shape
    F = w_gate.shape[0]
    if workspace is not None:
        _check(lib().ie_ffn_gate_up_ws(_dt(x), M, H, F, _ptr(x), _ptr(w_gate), _ptr(w_up), _ptr(h), h.stride(0),
                                       _ptr(workspace), _nbytes(workspace), _stream(stream)), "ie_ffn_gate_up_ws")
        return
    _check(lib().ie_ffn_gate_up(_dt(x), M, H, F, _ptr(x), _ptr(w_gate), _ptr(w_up), _ptr(h), h.stride(0),
                                _stream(stream)), "ie_ffn_gate_up")


def ffn_workspace_bytes(M: int, F: int = FFN_DIM) -> int:
    return int(lib().ie_ffn_workspace_size(M, F))


def qkv(x, wq, wk, wv, q_out, k_cache, v_cache, cache_head_stride, pos0=0, rope_cos=None, rope_sin=None,
        n_q_heads=NUM_Q_HEADS, n_kv_heads=NUM_KV_HEADS, head_dim=HEAD_DIM, stream=None, workspace=None):
    M, H = x.shape
    if workspace is not None:
        _check(lib().ie_qkv_ws(_dt(x), M, H, n_q_heads, n_kv_heads, head_dim, _ptr(x), _ptr(wq), _ptr(wk), _ptr(wv),
                               _ptr(q_out), _ptr(k_cache), _ptr(v_cache), cache_head_stride, pos0, _ptr(rope_cos),
                               _ptr(rope_sin), _ptr(workspace), _nbytes(workspace), _stream(stream)), "ie_qkv_ws")
        return
    _check(lib().ie_qkv(_dt(x), M, H, n_q_heads, n_kv_heads, head_dim, _ptr(x), _ptr(wq), _ptr(wk), _ptr(wv),
                        _ptr(q_out), _ptr(k_cache), _ptr(v_cache), cache_head_stride, pos0, _ptr(rope_cos),
                        _ptr(rope_sin), _stream(stream)), "ie_qkv")


def attention(q, k_cache, v_cache, out, pos0, n_kv_heads=NUM_KV_HEADS, stream=None):
    """ie_attention: causal GQA over the cache; q [nq, S, 128] head-major,
    caches [nkv, ctx, 128], out [S, nq*128]."""
    nq, S, D = q.shape
    _check(lib().ie_attention(_dt(q), S, pos0, nq, n_kv_heads, D, _ptr(q), q.stride(0), _ptr(k_cache), _ptr(v_cache),
                              k_cache.stride(0), _ptr(out), out.stride(0), _stream(stream)), "ie_attention")


def attention_decode(q, k_cache, v_cache, out, positions=None, pos0=0, rows_per_seq=None, stream=None):
    """ie_attention_decode: q [nq, R, 128] head-major; caches [nkv, rows, 128]
    (one sequence) or [B, nkv, rows, 128] (row m belongs to sequence
    m // rows_per_seq); positions: device int32 [R] or None (row m at pos0 + m);
    out [R, nq*128]."""
    nq, R, D = q.shape
    if k_cache.dim() == 4:
        B, nkv, rows = k_cache.shape[:3]
        cbs, chs = k_cache.stride(0), k_cache.stride(1)
    else:
        B, (nkv, rows) = 1, k_cache.shape[:2]
        cbs, chs = 0, k_cache.stride(0)
    rps = rows_per_seq if rows_per_seq is not None else max(R // B, 1)
    _check(lib().ie_attention_decode(_dt(q), R, rps, nq, nkv, D, _ptr(q), q.stride(0), _ptr(k_cache), _ptr(v_cache),
                                     chs, cbs, rows, _ptr(positions), pos0, _ptr(out), out.stride(0),
                                     _stream(stream)), "ie_attention_decode")


def qkv_batched(x, wq, wk, wv, q_out, k_cache, v_cache, positions, rope_cos=None, rope_sin=None,
                n_q_heads=NUM_Q_HEADS, n_kv_heads=NUM_KV_HEADS, head_dim=HEAD_DIM, stream=None):
    """ie_qkv_batched: row b of x is sequence b's token at positions[b];
    caches are [B, n_kv_heads, rows, 128]."""
    B, H = x.shape
    _check(lib().ie_qkv_batched(_dt(x), B, H, n_q_heads, n_kv_heads, head_dim, _ptr(x), _ptr(wq), _ptr(wk), _ptr(wv),
                                _ptr(q_out), _ptr(k_cache), _ptr(v_cache), k_cache.stride(1), k_cache.stride(0),
                                k_cache.shape[2], _ptr(positions), _ptr(rope_cos), _ptr(rope_sin), _stream(stream)),
           "ie_qkv_batched")


def lm_head_workspace_bytes(M: int) -> int:
    return int(lib().ie_lm_head_argmax_workspace_size(M))


def lm_head_argmax(x, w, workspace, logits=None, idx_out=None, key_out=None, vocab_offset=0, stream=None):
    M, K = x.shape
    V = w.shape[0]
    ld_logits = logits.stride(0) if logits is not None else 0
    _check(lib().ie_lm_head_argmax(_dt(x), M, K, V, vocab_offset, _ptr(x), x.stride(0), _ptr(w), _ptr(logits),
                                   ld_logits, _ptr(idx_out), _ptr(key_out), _ptr(workspace),
                                   workspace.numel() * workspace.element_size(), _stream(stream)),
           "ie_lm_head_argmax")


def lm_head_argmax_noalloc(x, w, logits=None, idx_out=None, key_out=None, vocab_offset=0, stream=None):
    """ie_lm_head_argmax_noalloc: lm_head + greedy id without a caller workspace
    (at most 64 rows; calls overlapping on the GPU race on the library's
    fixed scratch)."""
    M, K = x.shape
    V = w.shape[0]
    ld_logits = logits.stride(0) if logits is not None else 0
    _check(lib().ie_lm_head_argmax_noalloc(_dt(x), M, K, V, vocab_offset, _ptr(x), x.stride(0), _ptr(w),
                                           _ptr(logits), ld_logits, _ptr(idx_out), _ptr(key_out), _stream(stream)),
           "ie_lm_head_argmax_noalloc")


def argmax(logits, idx_out, stream=None):
    M, V = logits.shape
    _check(lib().ie_argmax(_dt(logits), M, V, _ptr(logits), logits.stride(0), _ptr(idx_out), _stream(stream)),
           "ie_argmax")


def device_status(clear: bool = True) -> int:
    """ie_device_status: IE_OK or IE_ERR_TIMEOUT from a bounded device wait."""
    return int(lib().ie_device_status(1 if clear else 0))


def set_wait_limit_ns(ns: int = 0) -> None:
    """ie_set_wait_limit_ns: limit of the kernels' bounded device-side waits
    on the current device (0 restores the default of 2 s)."""
    _check(lib().ie_set_wait_limit_ns(int(ns)), "ie_set_wait_limit_ns")


def key_index(key: int) -> int:
    """Global vocabulary id held in a packed argmax key (ie_argmax_key_index)."""
    tie = (~key) & 0xFFFFFFFF
    rr = tie >> 21
    r = sum(((rr >> b) & 1) << (9 - b) for b in range(10))  # undo the 10-bit reversal
    return (tie & ((1 << 21) - 1)) * 1024 + r


# ------------------------------------------------- reference-named mirror
def multiply_by_weight(m, k, n, d_in, d_w, d_out, stream=None):
    """kernels/multiply_by_weight.cuh:3 — d_out[m,n] = d_in[m,k] . d_w[n,k]^T."""
    _check(lib().ie_gemm(_dt(d_in), m, n, k, _ptr(d_in), k, _ptr(d_w), k, _ptr(d_out), n, _stream(stream)),
           "multiply_by_weight")


def ffn_workspace_size(max_seq_len: int) -> int:
    """kernels/ffn.cuh:5 — never less than the reference's 2*S*FFN_DIM*2 bytes."""
    return max(2 * max_seq_len * FFN_DIM * 2, ffn_workspace_bytes(max_seq_len, FFN_DIM))


def ffn(seq_len, d_in, d_out, d_wup, d_wdown, d_wgate, workspace, stream=None):
    """kernels/ffn.cuh:6 — weight order up, down, gate as in the reference."""
    H, F = d_wup.shape[1], d_wup.shape[0]
    _check(lib().ie_ffn(_dt(d_in), seq_len, H, F, _ptr(d_in), _ptr(d_wup), _ptr(d_wdown), _ptr(d_wgate),
                        _ptr(d_out), _ptr(workspace), workspace.numel() * workspace.element_size(),
                        _stream(stream)), "ffn")


def swiglu(seq_len, d_gate, d_up, d_output, stream=None):
    """kernels/swiglu.cuh:5 — d_output may alias d_gate."""
    F = d_gate.numel() // max(seq_len, 1)
    _check(lib().ie_swiglu(_dt(d_gate), seq_len, F, _ptr(d_gate), _ptr(d_up), _ptr(d_output), _stream(stream)),
           "swiglu")


def lm_head(seq_len, d_input, d_weight, d_output, stream=None):
    """kernels/lm_head.cuh:4 — logits of row seq_len-1 of d_input."""
    K = d_weight.shape[1]
    V = d_weight.shape[0]
    last = d_input.reshape(-1, K)[seq_len - 1:seq_len]
    _check(lib().ie_gemm(_dt(d_input), 1, V, K, _ptr(last), K, _ptr(d_weight), K, _ptr(d_output), V,
                         _stream(stream)), "lm_head")


def sample_token_amax(d_logits, d_output, stream=None):
    """kernels/sampling.cuh:4 — greedy id with the reference's tie order."""
    V = d_logits.numel()
    _check(lib().ie_argmax(_dt(d_logits), 1, V, _ptr(d_logits), V, _ptr(d_output), _stream(stream)),
           "sample_token_amax")
