"""GPU: the safetensors loader (ie_llama_load) — a tiny Llama written here as
a two-file Hugging Face checkpoint, loaded to the device and decoded by the
engine against the CPU model oracle; dtype conversion and tensor-parallel
shards read back bit-exact."""
import numpy as np
import pytest

from conftest import oracle, to_dev

pytestmark = pytest.mark.gpu


def _read(ptr: int, nbytes: int) -> np.ndarray:
    from cuda.bindings import runtime as rt
    buf = np.empty(nbytes, np.uint8)
    err, = rt.cudaMemcpy(buf.ctypes.data, ptr, nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess
    return buf


def _checkpoint(tmp_path, weights, dtype="bf16"):
    from infengine_b200.loader import hf_names, write_safetensors
    named = hf_names(weights)
    keys = sorted(named)
    half = len(keys) // 2
    paths = [tmp_path / "model-00001-of-00002.safetensors", tmp_path / "model-00002-of-00002.safetensors"]
    write_safetensors(paths[0], {k: named[k] for k in keys[:half]}, dtype)
    write_safetensors(paths[1], {k: named[k] for k in keys[half:]}, dtype)
    return paths


def test_loaded_model_decodes_like_the_oracle(ie, cuda, tmp_path):
    from infengine_b200.loader import LlamaModel
    from tiny_model import engine_vs_oracle, tiny_weights
    weights = tiny_weights(oracle, layers=2, seed=17)
    model = LlamaModel(_checkpoint(tmp_path, weights), "bf16", max_ctx=256)
    assert model.dims()["n_layers"] == 2 and model.dims()["n_q_heads"] == 2 and model.dims()["vocab"] == 1000
    eng = model.engine(max_batch=1, max_ctx=256, max_prefill=64)
    prompt = np.random.default_rng(2).integers(0, 1000, size=24).astype(np.int32)
    got, want, margin = engine_vs_oracle(oracle, to_dev, weights, prompt, 10, eng=eng)
    bad = got != want
    assert (~bad).mean() >= 0.8 and np.all(margin[bad] < 0.03), (got, want, margin)
    # RoPE tables built by the loader
    cos, sin = oracle.rope_tables(256)
    d = model.desc
    assert np.abs(_read(d.rope_cos, cos.nbytes).view(np.float32).reshape(cos.shape) - cos).max() < 2e-6
    assert np.abs(_read(d.rope_sin, sin.nbytes).view(np.float32).reshape(sin.shape) - sin).max() < 2e-6
    model.close()


def test_conversion_bf16_file_to_f16(ie, cuda, tmp_path):
    from infengine_b200.loader import LlamaModel
    from tiny_model import tiny_weights
    weights = tiny_weights(oracle, layers=1, seed=5)
    model = LlamaModel(_checkpoint(tmp_path, weights), "f16", max_ctx=64)
    wq = weights["layers"][0]["wq"]
    got = _read(model.desc.layers[0].wq, wq.size * 2).view(np.uint16)
    assert np.array_equal(got, oracle.to_bits(oracle.round_dt(wq, "f16"), "f16").view(np.uint16).ravel())
    model.close()


def test_tensor_parallel_shards(ie, cuda, tmp_path):
    """world=2: every rank's slab holds exactly its rows / columns."""
    from infengine_b200.loader import LlamaModel, hf_names, write_safetensors
    rng = np.random.default_rng(3)
    H, F, V, Q, KV = 256, 512, 1000, 512, 256

    def w(*s):
        return oracle.round_dt(rng.standard_normal(s).astype(np.float32) * np.float32(0.02), "bf16")

    weights = dict(embedding=w(V, H), final_norm=w(H), lm_head=w(V, H),
                   layers=[dict(attn_norm=w(H), wq=w(Q, H), wk=w(KV, H), wv=w(KV, H), wo=w(H, Q), ffn_norm=w(H),
                                w_gate=w(F, H), w_up=w(F, H), w_down=w(H, F))])
    p = tmp_path / "m.safetensors"
    write_safetensors(p, hf_names(weights), "bf16")

    def bits(a):
        return oracle.to_bits(a, "bf16").view(np.uint16)

    for rank in range(2):
        m = LlamaModel([p], "bf16", world=2, rank=rank, max_ctx=64)
        d, lw = m.desc, weights["layers"][0]
        assert (d.n_q_heads, d.n_kv_heads, d.ffn_dim, d.vocab) == (2, 1, 256, V)
        assert (m.lm_rows, m.lm_offset) == (500, 500 * rank)
        L0 = d.layers[0]
        checks = [(L0.wq, lw["wq"][256 * rank:256 * (rank + 1)]), (L0.wk, lw["wk"][128 * rank:128 * (rank + 1)]),
                  (L0.wv, lw["wv"][128 * rank:128 * (rank + 1)]), (L0.wo, lw["wo"][:, 256 * rank:256 * (rank + 1)]),
                  (L0.w_gate, lw["w_gate"][256 * rank:256 * (rank + 1)]),
                  (L0.w_up, lw["w_up"][256 * rank:256 * (rank + 1)]),
                  (L0.w_down, lw["w_down"][:, 256 * rank:256 * (rank + 1)]), (L0.attn_norm, lw["attn_norm"]),
                  (d.embedding, weights["embedding"]), (d.lm_head, weights["lm_head"][500 * rank:500 * (rank + 1)])]
        for ptr, want in checks:
            want = np.ascontiguousarray(want)
            got = _read(ptr, want.size * 2).view(np.uint16)
            assert np.array_equal(got, bits(want).ravel())
        # Q, K and V rows of a layer are one contiguous block
        assert L0.wk == L0.wq + 256 * H * 2 and L0.wv == L0.wk + 128 * H * 2
        m.close()
