"""GPU: the allocation-free lm_head + argmax entry point.

ie_lm_head_argmax_noalloc serves callers that cannot give the library a
workspace (code bound to the reference's lm_head / sample_token_amax
signatures, processes whose device memory belongs to a pool allocator, decode
loops that must not call cudaMalloc because it can synchronize the device).
It keeps its scratch in a fixed array inside the library. These tests call it
through the C-ABI and check that two calls in a row give exactly what the
workspace entry point gives on the same inputs, and that it refuses more rows
than its fixed scratch holds. The file is named to be collected last and
passes both alone and after the rest of the suite.
"""
import numpy as np
import pytest

from conftest import from_dev, oracle, to_dev, torch_dtype

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M,V", [(1, 128256), (8, 50000), (64, 32000)])
def test_noalloc_matches_workspace_entry_point(ie, cuda, dt, M, V):
    K = 4096
    d = oracle.seeded_inputs(700 + M, {"x": (M, K), "w": (V, K)}, dt)
    x, w = to_dev(d["x"], dt), to_dev(d["w"], dt)
    T = torch_dtype(dt)

    # the existing entry point, with a caller workspace
    ws = cuda.zeros(ie.lm_head_workspace_bytes(M), dtype=cuda.uint8, device="cuda")
    ref_logits = cuda.empty((M, V), dtype=T, device="cuda")
    ref_idx = cuda.full((M,), -1, dtype=cuda.int32, device="cuda")
    ref_keys = cuda.zeros((M,), dtype=cuda.int64, device="cuda")
    ie.lm_head_argmax(x, w, ws, logits=ref_logits, idx_out=ref_idx, key_out=ref_keys)
    cuda.cuda.synchronize()
    want_logits, want_idx, want_keys = from_dev(ref_logits), ref_idx.cpu().numpy(), ref_keys.cpu().numpy()
    # sanity against the oracle's tie rule on the kernel's own logits
    for m in range(M):
        assert want_idx[m] == oracle.argmax_reference_fast(want_logits[m])

    for call in range(2):  # two calls in a row share the library's scratch
        logits = cuda.full((M, V), float("nan"), dtype=T, device="cuda")
        idx = cuda.full((M,), -1, dtype=cuda.int32, device="cuda")
        keys = cuda.zeros((M,), dtype=cuda.int64, device="cuda")
        ie.lm_head_argmax_noalloc(x, w, logits=logits, idx_out=idx, key_out=keys)
        cuda.cuda.synchronize()
        # same kernel on the same inputs: identical to the workspace entry point
        # (the decode tests' bar for ids is bit-exact; logits are compared exactly too)
        assert np.array_equal(idx.cpu().numpy(), want_idx), f"call {call}"
        assert np.array_equal(keys.cpu().numpy(), want_keys), f"call {call}"
        assert np.array_equal(from_dev(logits), want_logits), f"call {call}"

    # ids only (no logits buffer), as a decode step would call it
    idx = cuda.full((M,), -1, dtype=cuda.int32, device="cuda")
    ie.lm_head_argmax_noalloc(x, w, idx_out=idx)
    cuda.cuda.synchronize()
    assert np.array_equal(idx.cpu().numpy(), want_idx)


def test_noalloc_rejects_more_rows_than_its_scratch(ie, cuda):
    x = cuda.zeros((65, 64), dtype=cuda.bfloat16, device="cuda")
    w = cuda.zeros((16, 64), dtype=cuda.bfloat16, device="cuda")
    idx = cuda.zeros((65,), dtype=cuda.int32, device="cuda")
    with pytest.raises(ie.IEError) as e:
        ie.lm_head_argmax_noalloc(x, w, idx_out=idx)
    assert e.value.status == -3  # IE_ERR_UNSUPPORTED
