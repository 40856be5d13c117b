"""Shared test helpers.

Markers:
  gpu  — needs a CUDA device (a B200); everything else runs on the CPU.

The CUDA side is always reached through the C-ABI library
(infengine_b200/libinfengine_b200.so); the oracle (oracle/ie_oracle.py) is the
checker.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

import ie_oracle as oracle  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        have_gpu = False
    if have_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


# ----------------------------------------------------------- conversions
def torch_dtype(dt: str):
    import torch
    return {"f16": torch.float16, "bf16": torch.bfloat16}[dt]


def to_dev(a: np.ndarray, dt: str):
    """numpy float32 (values representable in dt) -> torch CUDA tensor of dt."""
    import torch
    bits = oracle.to_bits(np.ascontiguousarray(a, dtype=np.float32), dt)
    t = torch.from_numpy(bits.view(np.int16).copy())
    return t.view(torch_dtype(dt)).cuda()


def from_dev(t) -> np.ndarray:
    """torch tensor (f16/bf16/f32) -> numpy float32."""
    import torch
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return oracle.bf16_bits_to_f32(t.view(torch.int16).numpy().view(np.uint16))
    return t.float().numpy()


def ulp(x: np.ndarray, dt: str) -> np.ndarray:
    """Spacing of dt at |x| (the size of one rounding step)."""
    x = np.abs(np.asarray(x, dtype=np.float32))
    mant = {"f16": 10, "bf16": 7}[dt]
    tiny = {"f16": 2.0 ** -14, "bf16": 2.0 ** -126}[dt]
    e = np.floor(np.log2(np.maximum(x, tiny)))
    return (2.0 ** (e - mant)).astype(np.float32)


@pytest.fixture(scope="session")
def ie():
    import infengine_b200
    infengine_b200.lib()
    return infengine_b200


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available()
    torch.cuda.init()
    return torch
