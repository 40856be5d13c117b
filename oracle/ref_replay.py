"""TEST INFRASTRUCTURE — the reference's decode loop, replayed teacher-forced.

Runs the reference's own prefill + decode_step loop (prefill.cu, decode.cu and
its kernels with cuBLAS, built unchanged by oracle/Makefile into
oracle/_ref/libref_model_ref.so) on its seeded random-init fp16 model, feeding
it a given id sequence, and saves the ids it picks, its top-2 logit margins
and its top logits. bench.py's parity checker runs it in a second process
with another cuBLAS environment (CUBLAS_WORKSPACE_CONFIG), so that cuBLAS
chooses other kernels and split-K reductions: the ids that change then are
the reference's own noise floor, the near-ties that any change of fp32
summation order can flip.

    python oracle/ref_replay.py <seed> <prompt.npy> <forced_ids.npy> <out.npz>
"""
from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "_ref" / "libref_model_ref.so"


def replay(seed: int, prompt: np.ndarray, forced: np.ndarray) -> dict:
    R = ctypes.CDLL(str(LIB))
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    R.model_init.argtypes = [ctypes.c_ulonglong]
    R.model_generate_ex.argtypes = [vp, i32, i32, vp, vp, vp, vp, vp, vp]
    if R.model_init(seed) != 0:
        raise RuntimeError("model_init failed")
    prompt = np.ascontiguousarray(prompt, dtype=np.int32)
    forced = np.ascontiguousarray(forced, dtype=np.int32)
    n = len(forced)
    ids, margin, top = np.zeros(n, np.int32), np.zeros(n, np.float32), np.zeros(n, np.float32)
    rc = R.model_generate_ex(prompt.ctypes.data_as(vp), len(prompt), n, forced.ctypes.data_as(vp),
                             ids.ctypes.data_as(vp), margin.ctypes.data_as(vp), top.ctypes.data_as(vp), None, None)
    R.model_free()
    if rc != 0:
        raise RuntimeError("model_generate_ex failed")
    return {"ids": ids, "margin": margin, "top": top}


if __name__ == "__main__":
    if len(sys.argv) != 5:
        sys.exit(__doc__)
    res = replay(int(sys.argv[1]), np.load(sys.argv[2]), np.load(sys.argv[3]))
    np.savez(sys.argv[4], **res)
