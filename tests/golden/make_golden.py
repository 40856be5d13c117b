"""Generate the committed golden fixtures from the reference's own generator.

Run in the build container (it needs the reference tree; the GPU box does not
have it and only reads the committed outputs):

    python tests/golden/make_golden.py /path/to/infengine

It imports scripts/generate_test_data.py of the reference and calls the two
generator functions that need no Llama checkpoint:

  * save_swiglu_data        (scripts/generate_test_data.py:113-124)
  * save_sampling_amax_data (scripts/generate_test_data.py:163-168)

plus save_rope_data (:29-56) on a random-init model of the Llama-3.1-8B
configuration (only its rotary embedding is used, which depends on the
config, not on weights). The .bin outputs are raw little-endian tensors as
the reference's tests/test_utils.cpp reads them.

Inputs are seeded with torch.manual_seed(42) on the CPU generator and can be
regenerated bit-identically on any machine with the same torch build, so the
fixtures keep only SHA-256 digests of the inputs, the small outputs in full
and a strided sample of the 3.7 MB SwiGLU output (every 97th element).
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SWIGLU_SAMPLE_STRIDE = 97


def sha256(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def main(ref_root: str) -> None:
    spec = importlib.util.spec_from_file_location("generate_test_data",
                                                  os.path.join(ref_root, "scripts", "generate_test_data.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    out = {}
    with tempfile.TemporaryDirectory() as td:
        cwd = os.getcwd()
        os.chdir(td)
        try:
            os.makedirs("test_data")
            gen.save_swiglu_data()
            gen.save_sampling_amax_data()
            import torch
            from transformers import LlamaConfig, LlamaForCausalLM
            cfg = LlamaConfig(hidden_size=4096, intermediate_size=64, num_hidden_layers=1,
                              num_attention_heads=32, num_key_value_heads=8, vocab_size=64,
                              max_position_embeddings=131072, rope_theta=500000.0,
                              rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                            "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
                              rms_norm_eps=1e-5)
            torch.manual_seed(0)
            model = LlamaForCausalLM(cfg)
            gen.save_rope_data(model)
            td_path = Path(td) / "test_data"
            sw_out = np.fromfile(td_path / "swiglu_out.bin", dtype=np.float16)
            out["swiglu"] = {
                "source": "scripts/generate_test_data.py:113-124 (save_swiglu_data)",
                "seed": 42, "shape": [128, 14336], "dtype": "float16",
                "gate_sha256": sha256(td_path / "swiglu_gate.bin"),
                "up_sha256": sha256(td_path / "swiglu_up.bin"),
                "out_sha256": sha256(td_path / "swiglu_out.bin"),
                "sample_stride": SWIGLU_SAMPLE_STRIDE,
            }
            np.save(HERE / "swiglu_out_sample.npy", sw_out[::SWIGLU_SAMPLE_STRIDE].copy())
            amax_in = td_path / "sampling_amax_input.bin"
            out["sampling_amax"] = {
                "source": "scripts/generate_test_data.py:163-168 (save_sampling_amax_data)",
                "seed": 42, "shape": [128256], "dtype": "float16",
                "input_sha256": sha256(amax_in),
                "argmax": int(np.fromfile(td_path / "sampling_amax_output.bin", dtype=np.int32)[0]),
            }
            cos = np.fromfile(td_path / "rope_cos.bin", dtype=np.float32).reshape(128, 64)
            sin = np.fromfile(td_path / "rope_sin.bin", dtype=np.float32).reshape(128, 64)
            np.savez_compressed(HERE / "rope_tables_128.npz", cos=cos, sin=sin)
            out["rope"] = {
                "source": "scripts/generate_test_data.py:29-56 (save_rope_data), Llama-3.1 rope_scaling",
                "positions": 128, "tolerance": 1e-3,
                "note": "reference tests/test_rope.cu compares its own tables to these within 1e-3",
            }
        finally:
            os.chdir(cwd)
    (HERE / "reference_golden.json").write_text(json.dumps(out, indent=1) + "\n")
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("INFENGINE_REF")
    if not tree:
        sys.exit("usage: make_golden.py <reference tree> (or set INFENGINE_REF)")
    main(tree)
