"""CPU: pin the oracle against the reference's own golden vectors.

The fixtures were produced by the reference's generator functions
(tests/golden/make_golden.py); their inputs come from torch.manual_seed(42)
and are regenerated here, checked by SHA-256 before use.
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from conftest import oracle

GOLD = Path(__file__).resolve().parent / "golden"
REF = json.loads((GOLD / "reference_golden.json").read_text())


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def swiglu_inputs():
    """Inputs of save_swiglu_data (scripts/generate_test_data.py:113-118)."""
    import torch
    torch.manual_seed(42)
    gate = torch.randn(128, 14336, dtype=torch.float16)
    up = torch.randn(128, 14336, dtype=torch.float16)
    return gate.numpy(), up.numpy()


def amax_input():
    """Input of save_sampling_amax_data (scripts/generate_test_data.py:163-166)."""
    import torch
    torch.manual_seed(42)
    return torch.randn(128256, dtype=torch.float16).numpy()


def test_swiglu_inputs_regenerate_bit_identically():
    g, u = swiglu_inputs()
    assert _sha(g) == REF["swiglu"]["gate_sha256"]
    assert _sha(u) == REF["swiglu"]["up_sha256"]


def test_oracle_swiglu_matches_reference_golden():
    g, u = swiglu_inputs()
    out = oracle.swiglu(g.astype(np.float32), u.astype(np.float32), "f16")
    sample = np.load(GOLD / "swiglu_out_sample.npy").astype(np.float32)
    mine = out.ravel()[:: REF["swiglu"]["sample_stride"]]
    # thresholds of the reference's tests/test_swiglu.cu:33-36
    r = oracle.compare(mine, sample, atol=2e-5)
    assert r["max_abs_err"] < 1e-3
    assert r["pct_within_tol"] > 99.0
    # the restatement is in fact (nearly) bit-identical to torch's CPU silu
    assert np.mean(mine == sample) > 0.999


def test_oracle_argmax_matches_reference_golden():
    x = amax_input()
    assert _sha(x) == REF["sampling_amax"]["input_sha256"]
    want = REF["sampling_amax"]["argmax"]
    assert oracle.argmax_reference(x.astype(np.float32)) == want
    assert oracle.argmax_reference_fast(x.astype(np.float32)) == want


def test_oracle_rope_tables_match_reference_golden():
    gold = np.load(GOLD / "rope_tables_128.npz")
    cos, sin = oracle.rope_tables(128)
    # tests/test_rope.cu compares the reference's tables to these within 1e-3
    assert np.abs(cos - gold["cos"]).max() < 1e-3
    assert np.abs(sin - gold["sin"]).max() < 1e-3


@pytest.mark.parametrize("seed", range(6))
def test_argmax_fast_equals_exact_restatement_on_ties(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1024, 6000))
    # few distinct values -> many ties across residues and quotients
    v = rng.integers(-3, 4, size=n).astype(np.float32)
    assert oracle.argmax_reference_fast(v) == oracle.argmax_reference(v)


def test_argmax_tie_rule_is_not_lowest_index():
    # max at 5 (residue 5 = 0b0000000101) and 1024 (residue 0): the reference picks 1024
    v = np.zeros(4096, dtype=np.float32)
    v[5] = v[1024] = 3.0
    assert oracle.argmax_reference(v) == 1024
    assert int(np.argmax(v)) == 5


def test_argmax_key_order_equals_reference_rule():
    rng = np.random.default_rng(7)
    for _ in range(20):
        n = int(rng.integers(1024, 5000))
        v = oracle.round_dt(rng.integers(-2, 3, size=n) * 0.5, "f16")
        v[rng.integers(0, n)] = -0.0  # signed zero ties with +0
        keys = [oracle.argmax_key(float(x), i) for i, x in enumerate(v)]
        assert oracle.key_index(max(keys)) == oracle.argmax_reference(v)


def test_bf16_rounding_matches_torch():
    import torch
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(100000) * 10 ** rng.uniform(-8, 8, 100000)).astype(np.float32)
    x[:4] = [0.0, -0.0, np.inf, -np.inf]
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(oracle.round_dt(x, "bf16"), ref)


def test_oracle_gemm_is_fp32_golden_rounded():
    d = oracle.seeded_inputs(0, {"x": (3, 64), "w": (40, 64)}, "bf16")
    y = oracle.multiply_by_weight(d["x"], d["w"], "bf16")
    g = oracle.gemm_fp32(d["x"], d["w"])
    assert np.array_equal(y, oracle.round_dt(g, "bf16"))


def test_argmax_tie_rule_follows_reversed_thread_bits():
    # residues 2 (reversed 0b0100000000) and 512 (reversed 0b0000000001):
    # the reduction tree's last level prefers bit 0 clear, so 512 beats 2
    v = np.zeros(8192, dtype=np.float32)
    v[3074] = v[512] = 1.0
    assert oracle.argmax_reference(v) == 512
    assert oracle.argmax_reference_fast(v) == 512
