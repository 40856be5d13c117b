"""Python mirror of the decode engine (ie_engine_* in include/infengine_b200.h).

The engine is the reference's request flow (manager.cpp:31-86: prefill, then
greedy decode steps) on this library's kernels, with each decode step kept on
the device and replayed as one CUDA graph. Weights stay the caller's: device
tensors (or raw device pointers) laid out like the reference's ModelWeights
(kernels/model_weights.cuh:7-34).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import IE_DTYPE_BF16, IE_DTYPE_F16, _check, lib

_vp = ctypes.c_void_p


class LayerWeights(ctypes.Structure):
    _fields_ = [("attn_norm", _vp), ("wq", _vp), ("wk", _vp), ("wv", _vp), ("wo", _vp), ("ffn_norm", _vp),
                ("w_gate", _vp), ("w_up", _vp), ("w_down", _vp)]


class LlamaDesc(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("hidden", ctypes.c_int), ("n_q_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn_dim", ctypes.c_int),
                ("vocab", ctypes.c_int), ("rms_eps", ctypes.c_float), ("embedding", _vp),
                ("layers", ctypes.POINTER(LayerWeights)), ("final_norm", _vp), ("lm_head", _vp),
                ("rope_cos", _vp), ("rope_sin", _vp)]


class EngineTP(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int), ("comm", _vp), ("exchange", _vp),
                ("lm_rows", ctypes.c_int), ("lm_offset", ctypes.c_int64)]


_bound = False


def _bind():
    global _bound
    if _bound:
        return
    L = lib()
    i32, vp = ctypes.c_int, ctypes.c_void_p
    L.ie_engine_create.argtypes = [i32, ctypes.POINTER(LlamaDesc), i32, i32, i32, vp, ctypes.POINTER(vp)]
    L.ie_engine_create_tp.argtypes = [i32, ctypes.POINTER(LlamaDesc), i32, i32, i32, vp, ctypes.POINTER(EngineTP),
                                      ctypes.POINTER(vp)]
    L.ie_engine_step.argtypes = [vp, vp, vp]
    L.ie_engine_destroy.argtypes = [vp]
    L.ie_engine_prefill.argtypes = [vp, i32, vp, i32, vp]
    L.ie_engine_decode.argtypes = [vp, i32, vp]
    L.ie_engine_verify.argtypes = [vp, i32, vp, i32, vp]
    L.ie_engine_set_position.argtypes = [vp, i32, i32, i32]
    L.ie_engine_position.argtypes = [vp, i32]
    L.ie_engine_stream.argtypes = [vp]
    L.ie_engine_stream.restype = vp
    L.ie_rmsnorm.argtypes = [i32, i32, i32, vp, ctypes.c_int64, vp, vp, ctypes.c_int64, ctypes.c_float, vp]
    L.ie_embed.argtypes = [i32, i32, i32, i32, vp, vp, vp, ctypes.c_int64, vp]
    _bound = True


def _addr(t) -> int:
    return t if isinstance(t, int) else t.data_ptr()


class LlamaEngine:
    """Greedy decoding of up to max_batch sequences.

    weights: dict with "embedding", "final_norm", "lm_head", "rope_cos",
    "rope_sin" and "layers" (a list of dicts with attn_norm, wq, wk, wv, wo,
    ffn_norm, w_gate, w_up, w_down); values are CUDA tensors or device
    addresses. dims: n_layers, hidden, n_q_heads, n_kv_heads, head_dim,
    ffn_dim, vocab, rms_eps.
    """

    def __init__(self, weights: dict, dims: dict, dtype: str = "bf16", max_batch: int = 1, max_ctx: int = 4096,
                 max_prefill: int = 2048, tp: dict | None = None):
        """tp (tensor parallel, one engine per rank): dict with world, rank,
        comm (infengine_b200.tp.Comm), exchange (tp.P2PExchange or None),
        lm_rows and lm_offset; weights then hold this rank's shards and dims
        the local head / FFN counts (vocab stays the full vocabulary)."""
        _bind()
        self.B = max_batch
        self._layers = (LayerWeights * dims["n_layers"])()
        for i, w in enumerate(weights["layers"]):
            self._layers[i] = LayerWeights(*[_addr(w[k]) for k, _ in LayerWeights._fields_])
        self.desc = LlamaDesc(dims["n_layers"], dims["hidden"], dims["n_q_heads"], dims["n_kv_heads"],
                              dims["head_dim"], dims["ffn_dim"], dims["vocab"], dims.get("rms_eps", 1e-5),
                              _addr(weights["embedding"]), self._layers, _addr(weights["final_norm"]),
                              _addr(weights["lm_head"]), _addr(weights["rope_cos"]), _addr(weights["rope_sin"]))
        self._keep = weights  # the engine reads these buffers
        h = ctypes.c_void_p()
        dt = IE_DTYPE_BF16 if dtype == "bf16" else IE_DTYPE_F16
        if tp is None:
            _check(lib().ie_engine_create(dt, ctypes.byref(self.desc), max_batch, max_ctx, max_prefill, None,
                                          ctypes.byref(h)), "ie_engine_create")
        else:
            ex = tp.get("exchange")
            self._tp = EngineTP(tp["world"], tp["rank"], tp["comm"].handle,
                                ctypes.addressof(ex.desc) if ex is not None else None, tp["lm_rows"], tp["lm_offset"])
            self._tp_keep = (tp["comm"], ex)
            _check(lib().ie_engine_create_tp(dt, ctypes.byref(self.desc), max_batch, max_ctx, max_prefill, None,
                                             ctypes.byref(self._tp), ctypes.byref(h)), "ie_engine_create_tp")
        self.h = h

    def prefill(self, seq: int, tokens) -> int:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = ctypes.c_int()
        _check(lib().ie_engine_prefill(self.h, seq, t.ctypes.data_as(_vp), len(t), ctypes.byref(nxt)),
               "ie_engine_prefill")
        return int(nxt.value)

    def decode(self, n_steps: int) -> np.ndarray:
        """[n_steps, max_batch] greedy ids (row i: the ids produced by step i)."""
        out = np.zeros((n_steps, self.B), np.int32)
        _check(lib().ie_engine_decode(self.h, n_steps, out.ctypes.data_as(_vp)), "ie_engine_decode")
        return out

    def step(self, tokens_in) -> np.ndarray:
        """One greedy step with host tokens in and out (ie_engine_step)."""
        t = np.ascontiguousarray(tokens_in, dtype=np.int32)
        out = np.zeros(self.B, np.int32)
        _check(lib().ie_engine_step(self.h, t.ctypes.data_as(_vp), out.ctypes.data_as(_vp)), "ie_engine_step")
        return out

    def verify(self, seq: int, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(len(t), np.int32)
        _check(lib().ie_engine_verify(self.h, seq, t.ctypes.data_as(_vp), len(t), out.ctypes.data_as(_vp)),
               "ie_engine_verify")
        return out

    def set_position(self, seq: int, pos: int, next_token: int):
        _check(lib().ie_engine_set_position(self.h, seq, pos, next_token), "ie_engine_set_position")

    def position(self, seq: int) -> int:
        return int(lib().ie_engine_position(self.h, seq))

    @property
    def stream(self) -> int:
        return int(lib().ie_engine_stream(self.h) or 0)

    def close(self):
        if self.h:
            lib().ie_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


def rmsnorm(x, w, out, eps: float = 1e-5, stream=None):
    """ie_rmsnorm: the reference's RMSNorm (kernels/rmsnorm.cu:29-62)."""
    from . import _dt, _ptr, _stream
    _bind()
    M, H = x.shape
    _check(lib().ie_rmsnorm(_dt(x), M, H, _ptr(x), x.stride(0), _ptr(w), _ptr(out), out.stride(0), eps,
                            _stream(stream)), "ie_rmsnorm")


def embed(tokens, table, out, stream=None):
    """ie_embed: out[m] = table[tokens[m]] (tokens: device int32)."""
    from . import _dt, _ptr, _stream
    _bind()
    M = tokens.shape[0]
    V, H = table.shape
    _check(lib().ie_embed(_dt(table), M, H, V, _ptr(tokens), _ptr(table), _ptr(out), out.stride(0),
                          _stream(stream)), "ie_embed")
