"""GPU parity of the prefill-path (tcgen05/TMEM) kernels against the oracle.

Every call goes through the C-ABI. The bar is the same as for the decode
kernels: each output within one rounding step of the exact sum, per-GEMM max
relative error <= 1e-2 against the fp32 golden, argmax ids bit-exact. The
projections are checked twice: whole tiles (ie_gemm, ie_qkv, ...) and with
the tail split of the *_ws entry points, which must also be deterministic
and leave its workspace flags zeroed.
"""
import numpy as np
import pytest

from conftest import from_dev, oracle, to_dev, torch_dtype, ulp
from test_gpu_decode import assert_within_one_rounding, rope_tol

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device_status_clean(ie, cuda):
    ie.device_status(clear=True)
    yield
    assert ie.device_status(clear=True) == 0, "a bounded device wait timed out"


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M,N,K", [
    (17, 256, 64),        # smallest tensor-core case: one tile, one k-block
    (128, 512, 4096),
    (300, 1000, 520),     # ragged M, N (not a multiple of 256) and K (not of 64)
    (2048, 4096, 4096),   # O projection
    (2048, 4096, 14336),  # down projection
    (1024, 4000, 1024),   # ragged last tile
    (1536, 800, 256),     # the last tile's second half lies wholly past N
])
def test_gemm_tensor_core(ie, cuda, dt, M, N, K):
    d = oracle.seeded_inputs(M + 7 * N + K, {"x": (M, K), "w": (N, K)}, dt)
    gold = oracle.gemm_fp32(d["x"], d["w"])
    x, w = to_dev(d["x"], dt), to_dev(d["w"], dt)
    ws = ie.split_workspace()
    for workspace in (None, ws):
        y = cuda.full((M, N), float("nan"), dtype=torch_dtype(dt), device="cuda")
        ie.gemm(x, w, y, workspace=workspace)
        got = from_dev(y)
        assert not np.isnan(got).any()
        assert_within_one_rounding(got, gold, dt)
    assert_split_workspace_clean(ie, cuda, ws)


def assert_split_workspace_clean(ie, cuda, ws):
    """Every completed call leaves the split workspace's flag words zeroed."""
    cuda.cuda.synchronize()
    n = (cuda.cuda.get_device_properties(0).multi_processor_count * 16 + 255) // 256 * 256
    assert int(ws[:n].count_nonzero().item()) == 0


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M,N,K", [
    (2048, 4096, 4096),   # O: 256 tiles on 148 SMs, 108 of them split
    (2048, 6144, 4096),   # QKV-sized plain GEMM: 384 tiles
    (256, 4096, 4096),    # 32 tiles, every one split
    (40, 4096, 14336),    # an engine prefill chunk through the down projection
    (300, 1000, 520),     # ragged: partial tiles in M, N and K
])
def test_gemm_tail_split_deterministic_and_residual(ie, cuda, dt, M, N, K):
    """The tail split is deterministic (repeated calls give the same bits),
    stays within one rounding step of the exact sum, and its residual form
    equals round(y + round(split result)) exactly."""
    d = oracle.seeded_inputs(5 * M + N + K, {"x": (M, K), "w": (N, K), "r": (M, N)}, dt)
    x, w = to_dev(d["x"], dt), to_dev(d["w"], dt)
    ws = ie.split_workspace()
    T = torch_dtype(dt)
    y1, y2 = (cuda.empty((M, N), dtype=T, device="cuda") for _ in range(2))
    ie.gemm(x, w, y1, workspace=ws)
    ie.gemm(x, w, y2, workspace=ws)
    cuda.cuda.synchronize()
    assert cuda.equal(y1, y2)
    assert_within_one_rounding(from_dev(y1), oracle.gemm_fp32(d["x"], d["w"]), dt)
    res = to_dev(d["r"], dt)
    y3 = res.clone()
    ie.gemm_add(x, w, y3, workspace=ws)
    cuda.cuda.synchronize()
    assert cuda.equal(y3, (res.float() + y1.float()).to(T))
    assert_split_workspace_clean(ie, cuda, ws)


def test_gemm_tensor_core_strided_output(ie, cuda):
    dt = "bf16"
    d = oracle.seeded_inputs(3, {"x": (200, 256), "w": (384, 256)}, dt)
    Y = cuda.zeros((200, 520), dtype=torch_dtype(dt), device="cuda")
    ie.gemm(to_dev(d["x"], dt), to_dev(d["w"], dt), Y[:, 8:392], M=200, N=384, K=256)
    got = from_dev(Y)
    assert_within_one_rounding(got[:, 8:392], oracle.gemm_fp32(d["x"], d["w"]), dt)
    assert np.all(got[:, :8] == 0) and np.all(got[:, 392:] == 0)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M", [128, 2048])
def test_ffn_gate_up_swiglu_tensor_core(ie, cuda, dt, M):
    """Gate/up GEMMs with the SwiGLU epilogue (BASELINE config 3 gate+up at M=2048;
    M=128 is the shape of the reference's own test_ffn.cu)."""
    H, F = 4096, 14336
    d = oracle.seeded_inputs(60 + M, {"x": (M, H), "wg": (F, H), "wu": (F, H)}, dt)
    g = oracle.gemm_fp32(d["x"], d["wg"])
    u = oracle.gemm_fp32(d["x"], d["wu"])
    want = oracle.swiglu(oracle.round_dt(g, dt), oracle.round_dt(u, dt), dt)
    x, wg, wu = to_dev(d["x"], dt), to_dev(d["wg"], dt), to_dev(d["wu"], dt)
    ws = ie.split_workspace()
    for workspace in (None, ws):  # whole tiles, then the tail split
        h = cuda.empty((M, F), dtype=torch_dtype(dt), device="cuda")
        ie.ffn_gate_up(x, wg, wu, h, workspace=workspace)
        got = from_dev(h)
        # g/u may round one step differently from the oracle's exact sums
        close = np.abs(got - want) <= 2 * ulp(want, dt) + 1e-5 * np.abs(want).max()
        assert close.mean() > 0.999
        assert oracle.normwise_rel_err(got, want) < 2e-3
    assert_split_workspace_clean(ie, cuda, ws)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_ffn_block_reference_test_shape(ie, cuda, dt):
    """The reference's test_ffn.cu configuration (S=128 tokens) on random
    weights: whole block vs the oracle chain and vs the fp32 golden."""
    M, H, F = 128, 4096, 14336
    d = oracle.seeded_inputs(77, {"x": (M, H), "wg": (F, H), "wu": (F, H), "wd": (H, F)}, dt)
    ws = cuda.empty(ie.ffn_workspace_size(M), dtype=cuda.uint8, device="cuda")
    out = cuda.empty((M, H), dtype=torch_dtype(dt), device="cuda")
    ie.ffn(M, to_dev(d["x"], dt), out, to_dev(d["wu"], dt), to_dev(d["wd"], dt), to_dev(d["wg"], dt), ws)
    got = from_dev(out)
    ref = oracle.ffn(d["x"], d["wg"], d["wu"], d["wd"], dt)
    assert oracle.normwise_rel_err(got, ref) <= (1e-2 if dt == "bf16" else 2e-3)
    h_gpu = from_dev(ws[: M * F * 2].view(torch_dtype(dt)).reshape(M, F))
    assert_within_one_rounding(got, oracle.gemm_fp32(h_gpu, d["wd"]), dt)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M,pos0,nq,nkv", [(128, 0, 32, 8), (2048, 0, 32, 8), (200, 37, 4, 1), (64, 5, 3, 1)])
def test_qkv_tensor_core(ie, cuda, dt, M, pos0, nq, nkv):
    """Fused QKV + RoPE at prefill (BASELINE config 3 QKV at M=2048; TP shards
    of 4+1+1 heads; an odd head count)."""
    H, hd, ctx = 4096, 128, 8192
    d = oracle.seeded_inputs(13 + M + nq, {"x": (M, H), "wq": (nq * hd, H), "wk": (nkv * hd, H),
                                           "wv": (nkv * hd, H)}, dt)
    cos, sin = oracle.rope_tables(ctx)
    T = torch_dtype(dt)
    c_t, s_t = cuda.from_numpy(cos).cuda(), cuda.from_numpy(sin).cuda()
    qr, kr, vr = oracle.qkv(d["x"], d["wq"], d["wk"], d["wv"], dt, pos0, cos, sin)
    tols = rope_tol(d["x"], d["wq"], d["wk"], d["wv"], dt, True)
    x, wq, wk, wv = (to_dev(d[k], dt) for k in ("x", "wq", "wk", "wv"))
    ws = ie.split_workspace()
    for workspace in (None, ws):  # whole tiles, then the tail split
        q = cuda.empty((nq, M, hd), dtype=T, device="cuda")
        kc = cuda.zeros((nkv, ctx, hd), dtype=T, device="cuda")
        vc = cuda.zeros((nkv, ctx, hd), dtype=T, device="cuda")
        ie.qkv(x, wq, wk, wv, q, kc, vc, ctx * hd, pos0, c_t, s_t, n_q_heads=nq, n_kv_heads=nkv, workspace=workspace)
        for got, want, tol in zip((from_dev(q), from_dev(kc)[:, pos0:pos0 + M], from_dev(vc)[:, pos0:pos0 + M]),
                                  (qr, kr, vr), tols):
            err = np.abs(got - want)
            assert np.all(err <= tol), f"max err {err.max():.3g}, worst excess {(err - tol).max():.3g}"
        kall = from_dev(kc)
        mask = np.ones(ctx, bool)
        mask[pos0:pos0 + M] = False
        assert np.all(kall[:, mask] == 0)
    assert_split_workspace_clean(ie, cuda, ws)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M", [17, 64])
def test_lm_head_argmax_tensor_core(ie, cuda, dt, M):
    """BASELINE config 4 at B=64: ids bit-exact under the reference's tie rule
    on the kernel's own rounded logits; logits within one rounding step."""
    K, V = 4096, 128256
    d = oracle.seeded_inputs(90 + M, {"x": (M, K), "w": (V, K)}, dt)
    T = torch_dtype(dt)
    logits = cuda.empty((M, V), dtype=T, device="cuda")
    idx = cuda.full((M,), -1, dtype=cuda.int32, device="cuda")
    keys = cuda.zeros((M,), dtype=cuda.int64, device="cuda")
    ws = cuda.zeros(ie.lm_head_workspace_bytes(M), dtype=cuda.uint8, device="cuda")
    x, w = to_dev(d["x"], dt), to_dev(d["w"], dt)
    for _ in range(2):
        ie.lm_head_argmax(x, w, ws, logits=logits, idx_out=idx, key_out=keys)
        cuda.cuda.synchronize()
        got_logits, got_idx = from_dev(logits), idx.cpu().numpy()
        for m in range(M):
            assert got_idx[m] == oracle.argmax_reference_fast(got_logits[m])
        assert int(ws.sum().item()) == 0
    assert_within_one_rounding(got_logits, oracle.gemm_fp32(d["x"], d["w"]), dt)
    # without a logits buffer (the fused path the decode step uses)
    idx2 = cuda.full((M,), -1, dtype=cuda.int32, device="cuda")
    ie.lm_head_argmax(x, w, ws, idx_out=idx2)
    assert np.array_equal(idx2.cpu().numpy(), got_idx)
