"""Python mirror of the safetensors loader (ie_st_*, ie_llama_load in
include/infengine_b200.h): reads a Hugging Face Llama checkpoint into one
device slab per rank, sharded for tensor parallelism, and hands the engine
its weight descriptor (the reference's ModelWeights::from_safetensors,
kernels/model_weights.cu:80-154)."""
from __future__ import annotations

import ctypes

from . import IE_DTYPE_BF16, IE_DTYPE_F16, _check, lib

ST_DTYPES = {0: "other", 1: "bf16", 2: "f16", 3: "f32"}
_bound = False


def _bind():
    global _bound
    if _bound:
        return
    from .engine import LlamaDesc
    L = lib()
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    L.ie_st_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
    L.ie_st_close.argtypes = [vp]
    L.ie_st_count.argtypes = [vp]
    L.ie_st_name.argtypes = [vp, i32]
    L.ie_st_name.restype = ctypes.c_char_p
    L.ie_st_info.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(i32), ctypes.POINTER(i32),
                             ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_uint64)]
    L.ie_llama_load.argtypes = [ctypes.POINTER(ctypes.c_char_p), i32, i32, i32, i32, i32, ctypes.c_float, vp,
                                ctypes.POINTER(vp)]
    L.ie_llama_model_desc.argtypes = [vp]
    L.ie_llama_model_desc.restype = ctypes.POINTER(LlamaDesc)
    L.ie_llama_model_shard.argtypes = [vp, ctypes.POINTER(i32), ctypes.POINTER(ctypes.c_int64)]
    L.ie_llama_model_free.argtypes = [vp]
    _bound = True


class SafeTensors:
    """Header of one .safetensors file (host only)."""

    def __init__(self, path: str):
        _bind()
        self.h = ctypes.c_void_p()
        _check(lib().ie_st_open(str(path).encode(), ctypes.byref(self.h)), "ie_st_open")

    def names(self) -> list[str]:
        L = lib()
        return [L.ie_st_name(self.h, i).decode() for i in range(L.ie_st_count(self.h))]

    def info(self, name: str) -> dict:
        dt, nd, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_uint64()
        shape = (ctypes.c_int64 * 8)()
        _check(lib().ie_st_info(self.h, name.encode(), ctypes.byref(dt), ctypes.byref(nd), shape, ctypes.byref(nb)),
               "ie_st_info")
        return {"dtype": ST_DTYPES.get(dt.value, "other"), "shape": tuple(shape[i] for i in range(nd.value)),
                "nbytes": nb.value}

    def close(self):
        if self.h:
            lib().ie_st_close(self.h)
            self.h = ctypes.c_void_p()


class LlamaModel:
    """One rank's weights on the device (ie_llama_load)."""

    def __init__(self, paths, dtype: str = "bf16", world: int = 1, rank: int = 0, max_ctx: int = 8192,
                 rms_eps: float = 1e-5):
        _bind()
        arr = (ctypes.c_char_p * len(paths))(*[str(p).encode() for p in paths])
        self.h = ctypes.c_void_p()
        dt = IE_DTYPE_BF16 if dtype == "bf16" else IE_DTYPE_F16
        _check(lib().ie_llama_load(arr, len(paths), dt, world, rank, max_ctx, rms_eps, None, ctypes.byref(self.h)),
               "ie_llama_load")
        self.desc = lib().ie_llama_model_desc(self.h).contents
        rows, off = ctypes.c_int(), ctypes.c_int64()
        lib().ie_llama_model_shard(self.h, ctypes.byref(rows), ctypes.byref(off))
        self.lm_rows, self.lm_offset = rows.value, off.value
        self.world, self.rank, self.dtype = world, rank, dtype

    def dims(self) -> dict:
        d = self.desc
        return dict(n_layers=d.n_layers, hidden=d.hidden, n_q_heads=d.n_q_heads, n_kv_heads=d.n_kv_heads,
                    head_dim=d.head_dim, ffn_dim=d.ffn_dim, vocab=d.vocab, rms_eps=d.rms_eps)

    def weights(self) -> dict:
        """Device addresses in the layout LlamaEngine takes."""
        d = self.desc
        names = ["attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "w_gate", "w_up", "w_down"]
        layers = [{n: getattr(d.layers[l], n) for n in names} for l in range(d.n_layers)]
        return dict(embedding=d.embedding, final_norm=d.final_norm, lm_head=d.lm_head, rope_cos=d.rope_cos,
                    rope_sin=d.rope_sin, layers=layers)

    def engine(self, max_batch: int = 1, max_ctx: int = 4096, max_prefill: int = 2048, comm=None, exchange=None):
        from .engine import LlamaEngine
        tp = None
        if self.world > 1:
            tp = dict(world=self.world, rank=self.rank, comm=comm, exchange=exchange, lm_rows=self.lm_rows,
                      lm_offset=self.lm_offset)
        e = LlamaEngine(self.weights(), self.dims(), dtype=self.dtype, max_batch=max_batch, max_ctx=max_ctx,
                        max_prefill=max_prefill, tp=tp)
        e._model = self  # the engine reads the slab
        return e

    def close(self):
        if self.h:
            lib().ie_llama_model_free(self.h)
            self.h = ctypes.c_void_p()


def write_safetensors(path, tensors: dict, dtype: str = "bf16", metadata: dict | None = None):
    """Write float32 numpy arrays (values representable in dtype) as a
    .safetensors file: 8-byte little-endian header length, JSON header, data."""
    import json
    import struct

    import numpy as np
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = metadata
    for name, a in tensors.items():
        a = np.ascontiguousarray(a, dtype=np.float32)
        if dtype == "bf16":
            raw = (a.view(np.uint32) >> 16).astype(np.uint16).tobytes()
            code = "BF16"
        elif dtype == "f16":
            raw = a.astype(np.float16).tobytes()
            code = "F16"
        else:
            raw = a.tobytes()
            code = "F32"
        header[name] = {"dtype": code, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def hf_names(weights: dict) -> dict:
    """Map a LlamaOracle-style weight dict to Hugging Face tensor names."""
    out = {"model.embed_tokens.weight": weights["embedding"], "model.norm.weight": weights["final_norm"],
           "lm_head.weight": weights["lm_head"]}
    sub = {"attn_norm": "input_layernorm.weight", "ffn_norm": "post_attention_layernorm.weight",
           "wq": "self_attn.q_proj.weight", "wk": "self_attn.k_proj.weight", "wv": "self_attn.v_proj.weight",
           "wo": "self_attn.o_proj.weight", "w_gate": "mlp.gate_proj.weight", "w_up": "mlp.up_proj.weight",
           "w_down": "mlp.down_proj.weight"}
    for l, lw in enumerate(weights["layers"]):
        for k, v in lw.items():
            out[f"model.layers.{l}.{sub[k]}"] = v
    return out
