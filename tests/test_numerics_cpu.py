"""CPU: the arithmetic identities the tcgen05 prefill attention relies on,
checked on the storage types' exact rounding (numpy), without a device.

Pass 1 of that kernel keeps only the maximum of the raw fp32 scores s of a
row and forms the softmax maximum as round(round(max s) * scale); the
reference's chain (kernels/softmax.cu:55-103 after the cuBLAS scores,
kernels/attn.cu:355-366) takes max over round(round(s) * scale). The two are
equal because rounding to nearest and multiplication by a positive float are
both monotone non-decreasing.
"""
import math

import numpy as np
import pytest

from conftest import oracle

SCALE = np.float32(1.0 / math.sqrt(128.0))


def _t(s, dt):
    """t = round(round(s) * scale) in fp32 arithmetic, as both compute it."""
    return oracle.round_dt(oracle.round_dt(s, dt) * SCALE, dt)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_rounded_max_equals_max_of_rounded(dt):
    rng = np.random.default_rng(5)
    for trial in range(400):
        n = int(rng.integers(1, 300))
        spread = 10.0 ** rng.uniform(-3, 2.5)   # scores from tiny to near the f16 range
        s = (rng.standard_normal(n) * spread).astype(np.float32)
        if trial % 7 == 0:                       # ties and near-ties around one value
            s[: n // 2] = s[0] + rng.integers(-2, 3, n // 2).astype(np.float32) * np.float32(1e-3) * spread
        want = _t(s, dt).max()
        got = _t(np.array([s.max()], np.float32), dt)[0]
        assert got == want, (dt, trial, float(got), float(want))


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_masked_keys_do_not_change_the_maximum(dt):
    """Causal masking to -inf before the maximum (pass 1) and zero weights
    after the exponent (pass 2) leave the visible keys' maximum unchanged."""
    rng = np.random.default_rng(6)
    s = (rng.standard_normal(256) * 8).astype(np.float32)
    for lim in (0, 1, 63, 64, 127, 200, 255):
        visible = s[: lim + 1]
        masked = np.where(np.arange(256) <= lim, s, -np.inf).astype(np.float32)
        assert _t(np.array([masked.max()], np.float32), dt)[0] == _t(visible, dt).max()


def test_exp2_with_folded_log2e_matches_exp():
    """e = 2^(t*log2(e) - m*log2(e)), with the product and the sum rounded
    once to fp32 (one fused multiply-add), stays within a few parts in 10^6
    of exp(t - m) over the range the softmax uses (t <= m, down to the point
    where e no longer survives rounding to the storage types): the error is
    the fp32 rounding of an exponent of up to ~115 (5.5e-6 at worst over 20
    seeds; near e = 1 it is far smaller)."""
    log2e = np.float32(1.4426950408889634)
    rng = np.random.default_rng(7)
    m = np.float32(rng.uniform(-20, 60))
    t = (m - rng.uniform(0, 80, 20000)).astype(np.float32)
    mb = np.float32(-m * log2e)
    arg = (t.astype(np.float64) * np.float64(log2e) + np.float64(mb)).astype(np.float32)  # one rounding (FMA)
    e = np.exp2(arg.astype(np.float64))
    ref = np.exp(t.astype(np.float64) - np.float64(m))
    keep = ref > 1e-30
    rel = np.abs(e[keep] - ref[keep]) / ref[keep]
    assert rel.max() < 8e-6, rel.max()
    # rounded to bf16, the probabilities agree except at rounding boundaries
    pe, pr = oracle.round_dt(e[keep].astype(np.float32), "bf16"), oracle.round_dt(ref[keep].astype(np.float32), "bf16")
    assert (pe == pr).mean() > 0.99
