"""GPU: the attention core behind the drop-in attn / decode_attn (ie_attention)
against the oracle's restatement of the reference's chain."""
import numpy as np
import pytest

from conftest import from_dev, oracle, to_dev, torch_dtype, ulp

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("S,pos0,nq,nkv", [(1, 0, 32, 8), (1, 300, 32, 8), (37, 0, 32, 8), (16, 50, 8, 2),
                                           (5, 2043, 4, 1)])
def test_attention_core(ie, cuda, dt, S, pos0, nq, nkv):
    ctx = 2048 + 64
    rng = np.random.default_rng(S * 1000 + pos0 + nq)
    q = oracle.round_dt(rng.standard_normal((nq, S, 128), dtype=np.float32), dt)
    k = np.zeros((nkv, ctx, 128), np.float32)
    v = np.zeros((nkv, ctx, 128), np.float32)
    k[:, :pos0 + S] = oracle.round_dt(rng.standard_normal((nkv, pos0 + S, 128), dtype=np.float32), dt)
    v[:, :pos0 + S] = oracle.round_dt(rng.standard_normal((nkv, pos0 + S, 128), dtype=np.float32), dt)
    out = cuda.full((S, nq * 128), float("nan"), dtype=torch_dtype(dt), device="cuda")
    ie.attention(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), out, pos0, n_kv_heads=nkv)
    got = from_dev(out)
    want = oracle.attention(q, k, v, pos0, dt)
    assert not np.isnan(got).any()
    # a rounding flip of one probability moves an output by about one p-ulp
    # times |V|; bound: two output rounding steps plus 2 % of the output scale
    err = np.abs(got - want)
    assert np.all(err <= 2 * ulp(want, dt) + 0.02 * np.abs(want).max()), err.max()
    assert oracle.normwise_rel_err(got, want) < (5e-3 if dt == "f16" else 2e-2)
