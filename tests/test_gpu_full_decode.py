"""GPU, BASELINE config 5 (2048-token prompt, 64 steps): the reference's own decode loop
(prefill.cu / decode.cu, built from its sources) on random-init
Llama-3.1-8B weights, linked once with the reference's hot-path kernels
(cuBLAS) and once with infengine_b200's drop-in library. Both builds get the
same seeded weights and prompt.

Greedy ids are compared with teacher forcing: the drop-in build is fed the
reference build's tokens, so every step is scored on the same context. A
step may disagree only at a near-tie: where the reference's own top-2 logit
margin is at most a few fp16 spacings of its top logit, the size of the
rounding differences that cuBLAS's summation order and ours leave in the
hidden state after 32 layers. The free-running sequences are reported too.
"""
import ctypes
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parent.parent / "oracle" / "_ref"
N_PROMPT, N_NEW, SEED = 2048, 64, 1234
# a miss is allowed only at a near-tie: the reference's top-2 margin at most
# this many fp16 spacings of its top logit (logits ~ N(0, 1.3), top ~ 5.5,
# where one spacing is 0.0039)
NEAR_TIE_ULPS = 8
MIN_AGREEMENT = 0.9  # a guard against wholesale failure; the near-tie bar is the contract


def _load(name):
    L = ctypes.CDLL(str(REF / name))
    L.model_init.argtypes = [ctypes.c_ulonglong]
    vp = ctypes.c_void_p
    L.model_generate_ex.argtypes = [vp, ctypes.c_int, ctypes.c_int, vp, vp, vp, vp, vp, vp]
    return L


def _generate(L, prompt, forced=None):
    """ids, top-2 margins and top logits of N_NEW greedy steps."""
    vp = ctypes.c_void_p
    out = np.zeros(N_NEW, np.int32)
    margin = np.zeros(N_NEW, np.float32)
    top = np.zeros(N_NEW, np.float32)
    fp = forced.ctypes.data_as(vp) if forced is not None else None
    rc = L.model_generate_ex(prompt.ctypes.data_as(vp), N_PROMPT, N_NEW, fp, out.ctypes.data_as(vp),
                             margin.ctypes.data_as(vp), top.ctypes.data_as(vp), None, None)
    assert rc == 0
    return out, margin, top


def fp16_spacing(x):
    return 2.0 ** (np.floor(np.log2(np.maximum(np.abs(x), 2.0 ** -14))) - 10)


def test_full_decode_dropin_matches_reference(cuda):
    rng = np.random.default_rng(SEED)
    prompt = rng.integers(0, 128256, size=N_PROMPT).astype(np.int32)
    ref, ie = _load("libref_model_ref.so"), _load("libref_model_ie.so")
    assert ref.model_init(SEED) == 0
    toks_ref, m_ref, top_ref = _generate(ref, prompt)
    ref.model_free()
    assert ie.model_init(SEED) == 0
    toks_tf, _, _ = _generate(ie, prompt, forced=toks_ref)  # teacher-forced on the reference's tokens
    toks_free, _, _ = _generate(ie, prompt)
    ie.model_free()
    agree = toks_tf == toks_ref
    ulps = m_ref / fp16_spacing(top_ref)
    first_div = int(np.argmin(toks_free == toks_ref)) if not np.all(toks_free == toks_ref) else N_NEW
    print(f"teacher-forced agreement {agree.sum()}/{N_NEW}; free-running identical for {first_div} steps; "
          f"reference margins at disagreements (fp16 spacings of the top logit) {ulps[~agree].tolist()}")
    assert np.all(ulps[~agree] <= NEAR_TIE_ULPS), (toks_ref, toks_tf, m_ref, top_ref)
    assert agree.mean() >= MIN_AGREEMENT
