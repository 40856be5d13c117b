"""CPU: the bench's bookkeeping that turns measurements into the JSON line
(no GPU; the timed legs themselves run in the -m gpu suite and on the box)."""
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


@pytest.mark.parametrize("x,want", [(1.0, 2.0 ** -10), (5.0390625, 2.0 ** -8), (-5.0, 2.0 ** -8),
                                    (0.75, 2.0 ** -11), (1024.0, 1.0), (0.0, 2.0 ** -24), (3e-6, 2.0 ** -24)])
def test_fp16_spacing(x, want):
    """One fp16 unit in the last place at |x| (subnormal spacing below 2^-14):
    the unit in which the parity leg reports the reference's top-2 margins."""
    assert bench.fp16_spacing(x) == want


def test_margin_in_ulps_matches_a_recorded_miss():
    """A miss the parity leg recorded: top logit 5.0390625, margin 0.01953125
    = 5 spacings of 2^-8."""
    assert 0.01953125 / bench.fp16_spacing(5.0390625) == 5.0


def test_versus_reference_ratios():
    """Speed-ups are reference time / our time per config; missing or zero
    times give None instead of a number."""
    ours = {"c1_gemv_4096x4096": {"us": 6.0},
            "c2_ffn_decode": {"m1": {"us": 40.0}, "m4": {"us": 50.0}, "m8": {"us": 0.0}},
            "c4_lm_head_argmax": {"b1": {"us": 150.0}, "b8": {"us": 180.0}, "b64": {"us": 200.0}},
            "c3_prefill_m2048": {"o_4096x4096": {"us": 50.0}}}
    ref = {"c1_gemv_4096x4096": {"us": 15.0},
           "c2_ffn_decode": {"m1": {"us": 60.0}, "m4": {"us": None}, "m8": {"us": 70.0}},
           "c4_lm_head_argmax": {"b1": {"us": 180.0}, "b8": {"us": 360.0}, "b64": {"us": 1000.0}},
           "c3_prefill_m2048": {"o_4096x4096": {"path_us": 45.0, "gemm_us": 40.0}}}
    vs = bench.versus_reference(ours, ref)
    assert vs["c1_gemv_4096x4096"] == 2.5
    assert vs["c2_ffn_decode"] == {"m1": 1.5, "m4": None, "m8": None}
    assert vs["c4_lm_head_argmax"] == {"b1": 1.2, "b8": 2.0, "b64": 5.0}
    assert vs["c3_prefill_m2048"]["o_4096x4096"] == {"vs_path": 0.9, "vs_gemm_only": 0.8}


def test_weight_bytes_of_the_roofline():
    """The decode roofline's algorithmic bytes: 32 layers of Llama-3.1-8B
    projections plus the lm_head in bf16 (15.01 GB a token), and one gate/up +
    SwiGLU launch at one row (234.9 MB)."""
    per_layer = (32 + 2 * 8) * 128 * 4096 + 4096 * 4096 + 3 * 14336 * 4096
    assert bench.WEIGHT_BYTES == 2 * (32 * per_layer + 128256 * 4096)
    assert round(bench.WEIGHT_BYTES / 1e9, 2) == 15.01
    assert bench.GATE_UP_BYTES == 234917888


def test_cli_lists_the_cases_without_a_gpu():
    """`bench.py --help` parses on a machine without a GPU (the driver's
    contract flags are there)."""
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    for flag in ("--gpus", "--steps", "--warmup", "--impl", "--case", "--parity-steps"):
        assert flag in r.stdout
