"""CPU: the safetensors header reader of the loader (ie_st_*), against files
written here in the format's published layout (8-byte little-endian header
length, JSON header of {dtype, shape, data_offsets}, data)."""
import json
import struct

import numpy as np
import pytest


def test_header_roundtrip(tmp_path):
    from infengine_b200.loader import SafeTensors, write_safetensors
    rng = np.random.default_rng(0)
    t = {"a.weight": rng.standard_normal((3, 8)).astype(np.float32), "norm": np.ones(8, np.float32),
         "model.layers.0.x": rng.standard_normal((16,)).astype(np.float32)}
    p = tmp_path / "m.safetensors"
    write_safetensors(p, t, "bf16", metadata={"format": "pt"})
    f = SafeTensors(p)
    assert sorted(f.names()) == sorted(t)
    assert f.info("a.weight") == {"dtype": "bf16", "shape": (3, 8), "nbytes": 48}
    assert f.info("norm")["shape"] == (8,)
    f.close()
    write_safetensors(p, t, "f32")
    f = SafeTensors(p)
    assert f.info("a.weight") == {"dtype": "f32", "shape": (3, 8), "nbytes": 96}
    f.close()


def _raw(path, header: bytes, data: bytes = b"\0" * 64):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header)))
        f.write(header)
        f.write(data)


@pytest.mark.parametrize("header", [
    b"{",                                                                          # truncated JSON
    b'{"x": {"dtype": "BF16", "shape": [4], "data_offsets": [0, 100]}}',          # past the data
    b'{"x": {"dtype": "BF16", "shape": [4], "data_offsets": [0, 6]}}',            # wrong byte count
    b'{"x": {"dtype": "BF16", "shape": [4]}}',                                     # no offsets
    b'{"x": {"dtype": "BF16", "shape": [-1], "data_offsets": [0, 2]}}',           # negative dimension
    b'[1, 2]',                                                                     # not an object
    # an element count that wraps 64 bits to 0 must not match an empty range
    b'{"x": {"dtype": "BF16", "shape": [4294967296, 4294967296], "data_offsets": [0, 0]}}',
])
def test_bad_headers_rejected(tmp_path, header):
    from infengine_b200 import IEError
    from infengine_b200.loader import SafeTensors
    p = tmp_path / "bad.safetensors"
    _raw(p, header)
    with pytest.raises(IEError):
        SafeTensors(p)


def test_header_length_beyond_file(tmp_path):
    from infengine_b200 import IEError
    from infengine_b200.loader import SafeTensors
    p = tmp_path / "bad.safetensors"
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", 1 << 40))
        f.write(b"{}")
    with pytest.raises(IEError):
        SafeTensors(p)
