"""Loader for the reference's own hot-path code built for sm_100a
(oracle/_ref/libinfengine_ref.so, see oracle/Makefile). Test infrastructure."""
from __future__ import annotations

import ctypes
from pathlib import Path

REF_LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libinfengine_ref.so"
_ref = None


def ref():
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise RuntimeError(f"{REF_LIB} missing: run `make -C oracle` where the reference tree exists")
        L = ctypes.CDLL(str(REF_LIB))
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        L.ref_init.restype = i32
        L.ref_set_stream.argtypes = [vp]
        L.ref_multiply_by_weight.argtypes = [i32, i32, i32, vp, vp, vp]
        L.ref_ffn_workspace_size.restype = ctypes.c_size_t
        L.ref_ffn_workspace_size.argtypes = [i32]
        L.ref_ffn.argtypes = [i32, vp, vp, vp, vp, vp, vp]
        L.ref_swiglu.argtypes = [i32, vp, vp, vp]
        L.ref_lm_head.argtypes = [i32, vp, vp, vp]
        L.ref_sample_token_amax.argtypes = [vp, vp]
        L.ref_qkv_proj.argtypes = [i32, vp, vp, vp, vp, vp, vp, vp, i32, i32]
        L.ref_apply_rope.argtypes = [i32, i32, i32, vp, vp, vp, i32]
        L.ref_o_proj.argtypes = [i32, vp, vp, vp]
        assert L.ref_init() == 0
        _ref = L
    return _ref


def p(t):
    return ctypes.c_void_p(t.data_ptr())
