"""Host-side inputs the reference's callers prepare for the hot path.

rope_tables() builds the RoPE cos/sin tables that the reference's
init_rope_buffer (kernels/rope.cu:68-103) uploads once per model and passes
to attn()/decode_attn(); ie_qkv reads them in its epilogue.
"""
from __future__ import annotations

import math

import numpy as np


def rope_tables(max_pos: int = 8192, head_dim: int = 128, theta: float = 500000.0, factor: float = 8.0,
                low_freq_factor: float = 1.0, high_freq_factor: float = 4.0, original_max_pos: int = 8192):
    """fp32 cos/sin tables [max_pos, head_dim/2] with Llama-3.1 frequency
    scaling (long wavelengths divided by `factor`, short ones kept, a linear
    blend in between), angle = position * frequency."""
    i = np.arange(head_dim // 2, dtype=np.float64)
    freq = 1.0 / np.power(theta, 2.0 * i / head_dim)
    wavelength = 2.0 * math.pi / freq
    low_wl = original_max_pos / low_freq_factor
    high_wl = original_max_pos / high_freq_factor
    smooth = (original_max_pos / wavelength - low_freq_factor) / (high_freq_factor - low_freq_factor)
    scaled = np.where(wavelength > low_wl, freq / factor,
                      np.where(wavelength < high_wl, freq, (1 - smooth) * freq / factor + smooth * freq))
    angle = np.arange(max_pos, dtype=np.float32)[:, None] * scaled.astype(np.float32)[None, :]
    return np.cos(angle).astype(np.float32), np.sin(angle).astype(np.float32)
