"""GPU parity of the decode-path kernels (M <= 16) against the oracle.

Every call goes through the C-ABI (libinfengine_b200.so). Tolerances:
  * each output is within one rounding step (one ulp of the storage type at
    the output's magnitude, plus 1e-5 of the output scale for cancellations)
    of the exact sum: fp32 accumulation order is the only difference;
  * per-GEMM max relative error vs the fp32 golden <= 1e-2 (the BASELINE bar);
  * argmax ids are bit-exact.
"""
import numpy as np
import pytest

from conftest import from_dev, oracle, to_dev, torch_dtype, ulp

pytestmark = pytest.mark.gpu

DTS = ["bf16", "f16"]


def rope_tol(x, wq, wk, wv, dt, rope):
    """Per-element bound for Q/K/V after RoPE: the rotation of a stored pair
    (a, b) can cancel, so the error is bounded by the pair's magnitude
    |a| + |b| (two rounding steps at that scale), not by the output's."""
    out = []
    for w, rot in ((wq, rope), (wk, rope), (wv, False)):
        pre = np.abs(oracle.gemm_fp32(x, w)).reshape(x.shape[0], -1, 128).transpose(1, 0, 2)
        mag = pre + np.concatenate([pre[..., 64:], pre[..., :64]], axis=-1) if rot else pre
        out.append(2 * ulp(mag, dt) + 1e-5 * mag.max())
    return out


def assert_within_one_rounding(got, gold_fp32, dt):
    scale = float(np.abs(gold_fp32).max()) if gold_fp32.size else 0.0
    err = np.abs(got.astype(np.float64) - gold_fp32.astype(np.float64))
    bound = ulp(gold_fp32, dt).astype(np.float64) + 1e-5 * scale
    bad = err > bound
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside one rounding step; max err {err.max():.3g}"
    assert oracle.max_rel_err(got, gold_fp32) <= 1e-2


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("M,N,K", [
    (1, 4096, 4096),      # BASELINE config 1 (multiply_by_weight GEMV)
    (1, 1000, 4096),      # N not a multiple of the 16-row tile
    (3, 4096, 14336),     # down-projection shape, odd M
    (5, 6144, 4096),      # verify pass M=5 on the fused-QKV width
    (8, 4096, 4096),
    (9, 272, 520),        # second n8 tile, K not a multiple of 32
    (16, 128, 8),         # smallest legal K
    (7, 33, 1032),
    # few tiles: the K range is split over a cluster of 2 or 4 CTAs
    (1, 512, 4096),       # 32 tiles, 4-way (a Q shard of 4 heads)
    (8, 1792, 4096),      # 112 tiles, 2-way (a gate or up shard at 8 GPUs)
    (3, 1024, 14336),     # 64 tiles, 4-way, long K
    (16, 240, 2056),      # 15 tiles, 2-way, K not a multiple of the chunk
])
def test_gemm_skinny(ie, cuda, dt, M, N, K):
    d = oracle.seeded_inputs(M * 1000 + N + K, {"x": (M, K), "w": (N, K)}, dt)
    y = cuda.full((M, N), float("nan"), dtype=torch_dtype(dt), device="cuda")
    ie.gemm(to_dev(d["x"], dt), to_dev(d["w"], dt), y)
    got = from_dev(y)
    assert_within_one_rounding(got, oracle.gemm_fp32(d["x"], d["w"]), dt)


@pytest.mark.parametrize("N,K", [(512, 4096), (1792, 4096), (4096, 4096)])
def test_gemm_skinny_rows_batch_invariant(ie, cuda, N, K):
    """A row gets the same bits alone and inside batches of 3, 8 and 16 rows,
    with and without the cluster K split (which depends on N and K only)."""
    dt = "bf16"
    d = oracle.seeded_inputs(N + K, {"x": (16, K), "w": (N, K)}, dt)
    x, w = to_dev(d["x"], dt), to_dev(d["w"], dt)
    T = torch_dtype(dt)
    alone = cuda.empty((1, N), dtype=T, device="cuda")
    ie.gemm(x[:1], w, alone)
    for M in (3, 8, 16):
        y = cuda.empty((M, N), dtype=T, device="cuda")
        ie.gemm(x[:M], w, y)
        cuda.cuda.synchronize()
        assert cuda.equal(y[0], alone[0]), M


@pytest.mark.parametrize("dt", DTS)
def test_gemm_config1_seed0(ie, cuda, dt):
    """x [1,4096] ~N(0,1), W [4096,4096] ~N(0,0.02), seed 0."""
    d = oracle.seeded_inputs(0, {"x": (1, 4096), "w": (4096, 4096)}, dt)
    y = cuda.empty((1, 4096), dtype=torch_dtype(dt), device="cuda")
    ie.multiply_by_weight(1, 4096, 4096, to_dev(d["x"], dt), to_dev(d["w"], dt), y)
    got = from_dev(y)
    gold = oracle.gemm_fp32(d["x"], d["w"])
    assert oracle.max_rel_err(got, gold) <= 1e-2
    assert oracle.normwise_rel_err(got, gold) <= 5e-3
    assert_within_one_rounding(got, gold, dt)


def test_gemm_strided_operands(ie, cuda):
    """Leading dimensions larger than the row length (sub-matrix views)."""
    dt = "bf16"
    d = oracle.seeded_inputs(11, {"x": (4, 264), "w": (300, 272)}, dt)
    X = to_dev(d["x"], dt)
    W = to_dev(d["w"], dt)
    Y = cuda.zeros((4, 312), dtype=torch_dtype(dt), device="cuda")
    ie.gemm(X[:, :256], W[:100, :256], Y[:, :100], M=4, N=100, K=256)
    got = from_dev(Y)
    assert_within_one_rounding(got[:, :100], oracle.gemm_fp32(d["x"][:, :256], d["w"][:100, :256]), dt)
    assert np.all(got[:, 100:] == 0)  # nothing written past N


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("M,F", [(1, 14336), (4, 14336), (8, 14336), (1, 1792), (8, 3584)])
def test_ffn_decode_config2(ie, cuda, dt, M, F):
    """Llama-3.1-8B FFN at decode, M in {1,4,8}; and the
    FFN shards of 8 and 4 GPUs (gate/up split over 2-CTA clusters)."""
    H = 4096
    d = oracle.seeded_inputs(100 + M, {"x": (M, H), "wg": (F, H), "wu": (F, H), "wd": (H, F)}, dt,
                             scales={"wg": 0.02, "wu": 0.02, "wd": 0.02})
    ws = cuda.empty(ie.ffn_workspace_bytes(M, F), dtype=cuda.uint8, device="cuda")
    out = cuda.empty((M, H), dtype=torch_dtype(dt), device="cuda")
    ie.ffn_fused(to_dev(d["x"], dt), to_dev(d["wu"], dt), to_dev(d["wd"], dt), to_dev(d["wg"], dt), out, ws)
    got = from_dev(out)
    # h the kernel produced (workspace) vs the reference's rounding chain
    h_gpu = from_dev(ws[: M * F * 2].view(torch_dtype(dt)).reshape(M, F))
    g = oracle.gemm_fp32(d["x"], d["wg"])
    u = oracle.gemm_fp32(d["x"], d["wu"])
    h_ref = oracle.swiglu(oracle.round_dt(g, dt), oracle.round_dt(u, dt), dt)
    hdiff = np.abs(h_gpu - h_ref)
    assert np.mean(hdiff <= ulp(h_ref, dt) * 2 + 1e-6) > 0.999
    # down projection of the kernel's own h: one rounding step from exact
    assert_within_one_rounding(got, oracle.gemm_fp32(h_gpu, d["wd"]), dt)
    # whole block vs the oracle's chain and vs the unrounded fp32 golden
    ref = oracle.ffn(d["x"], d["wg"], d["wu"], d["wd"], dt)
    assert oracle.normwise_rel_err(got, ref) <= (1e-2 if dt == "bf16" else 2e-3)
    gold = oracle.gemm_fp32(oracle.swiglu(g, u, "f32"), d["wd"])
    assert oracle.max_rel_err(got, gold) <= 1e-2 * 3


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("M,pos0,rope,nq,nkv", [(1, 2047, True, 32, 8), (5, 100, True, 32, 8), (3, 0, False, 32, 8),
                                                (16, 8000, True, 32, 8),
                                                (1, 2047, True, 4, 1),    # 8-GPU shard: 48 tiles, 4-way K split
                                                (5, 300, True, 8, 2)])    # 4-GPU shard: 96 tiles, 2-way
def test_qkv_fused(ie, cuda, dt, M, pos0, rope, nq, nkv):
    H, hd, ctx = 4096, 128, 8192
    d = oracle.seeded_inputs(7 + M, {"x": (M, H), "wq": (nq * hd, H), "wk": (nkv * hd, H), "wv": (nkv * hd, H)}, dt)
    cos, sin = oracle.rope_tables(ctx)
    T = torch_dtype(dt)
    q = cuda.empty((nq, M, hd), dtype=T, device="cuda")
    kc = cuda.zeros((nkv, ctx, hd), dtype=T, device="cuda")
    vc = cuda.zeros((nkv, ctx, hd), dtype=T, device="cuda")
    c_t = cuda.from_numpy(cos).cuda() if rope else None
    s_t = cuda.from_numpy(sin).cuda() if rope else None
    ie.qkv(to_dev(d["x"], dt), to_dev(d["wq"], dt), to_dev(d["wk"], dt), to_dev(d["wv"], dt), q, kc, vc,
           ctx * hd, pos0, c_t, s_t, n_q_heads=nq, n_kv_heads=nkv)
    qr, kr, vr = oracle.qkv(d["x"], d["wq"], d["wk"], d["wv"], dt, pos0, cos if rope else None,
                            sin if rope else None)
    got_q = from_dev(q)
    got_k = from_dev(kc)[:, pos0:pos0 + M]
    got_v = from_dev(vc)[:, pos0:pos0 + M]
    for got, want, tol in zip((got_q, got_k, got_v), (qr, kr, vr),
                              rope_tol(d["x"], d["wq"], d["wk"], d["wv"], dt, rope)):
        err = np.abs(got - want)
        assert np.all(err <= tol), f"max err {err.max():.3g}, worst excess {(err - tol).max():.3g}"
    # no cache row outside [pos0, pos0+M) was touched
    kall = from_dev(kc)
    mask = np.ones(ctx, bool)
    mask[pos0:pos0 + M] = False
    assert np.all(kall[:, mask] == 0)


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("M", [1, 8, 16])
def test_lm_head_argmax(ie, cuda, dt, M):
    """BASELINE config 4 at B in {1,8} (and 16): ids bit-exact under the
    reference's tie rule applied to the kernel's own rounded logits."""
    K, V = 4096, 128256
    d = oracle.seeded_inputs(40 + M, {"x": (M, K), "w": (V, K)}, dt)
    T = torch_dtype(dt)
    logits = cuda.empty((M, V), dtype=T, device="cuda")
    idx = cuda.full((M,), -1, dtype=cuda.int32, device="cuda")
    keys = cuda.zeros((M,), dtype=cuda.int64, device="cuda")
    ws = cuda.zeros(ie.lm_head_workspace_bytes(M), dtype=cuda.uint8, device="cuda")
    x, w = to_dev(d["x"], dt), to_dev(d["w"], dt)
    for rep in range(2):  # the workspace must come back zeroed for the next call
        ie.lm_head_argmax(x, w, ws, logits=logits, idx_out=idx, key_out=keys)
        cuda.cuda.synchronize()
        got_logits = from_dev(logits)
        got_idx = idx.cpu().numpy()
        for m in range(M):
            assert got_idx[m] == oracle.argmax_reference_fast(got_logits[m])
            assert ie.key_index(int(keys[m].item()) & 0xFFFFFFFFFFFFFFFF) == got_idx[m]
        assert int(ws.sum().item()) == 0
    gold = oracle.gemm_fp32(d["x"], d["w"])
    assert_within_one_rounding(got_logits, gold, dt)
    # vs the oracle's own rounding: ids agree unless the top-2 margin is < 1 ulp
    ref_logits = oracle.round_dt(gold, dt)
    for m in range(M):
        want = oracle.argmax_reference_fast(ref_logits[m])
        if got_idx[m] != want:
            top2 = np.sort(gold[m])[-2:]
            assert top2[1] - top2[0] <= 2 * ulp(top2[1:], dt)[0]


@pytest.mark.parametrize("n_shards", [2, 4, 8])
@pytest.mark.parametrize("M", [3, 64])
def test_lm_head_vocab_shards_merge_by_key_max(ie, cuda, n_shards, M):
    """Vocabulary split as tensor parallelism splits it at 2 / 4 / 8 ranks
    (64128 / 32064 / 16032 rows per shard; 16032 is not a multiple of the
    tensor-core kernel's 128-row tiles), on the decode kernel (M = 3) and the
    tensor-core kernel (M = 64): the max of the shards' packed keys is the
    full-vocabulary id. Each row's winning weight row is first copied into
    the next shard at the same offset, so the merge also has to resolve
    exact cross-shard ties in the reference's order."""
    dt, K, V = "bf16", 4096, 128256
    d = oracle.seeded_inputs(5 + M, {"x": (M, K), "w": (V, K)}, dt)
    x, w = to_dev(d["x"], dt), to_dev(d["w"], dt)
    ws = cuda.zeros(ie.lm_head_workspace_bytes(M), dtype=cuda.uint8, device="cuda")
    shard = V // n_shards
    full_idx = cuda.empty((M,), dtype=cuda.int32, device="cuda")
    ie.lm_head_argmax(x, w, ws, idx_out=full_idx)
    for i in set(full_idx.cpu().tolist()):  # plant the ties
        w[(i + shard) % V] = w[i]
    logits = cuda.empty((M, V), dtype=cuda.bfloat16, device="cuda")
    ie.lm_head_argmax(x, w, ws, logits=logits, idx_out=full_idx)
    keys = []
    for s in range(n_shards):
        k = cuda.zeros((M,), dtype=cuda.int64, device="cuda")
        ie.lm_head_argmax(x, w[s * shard:(s + 1) * shard], ws, key_out=k, vocab_offset=s * shard)
        keys.append(k.cpu().numpy().view(np.uint64))
    cuda.cuda.synchronize()
    merged = np.max(np.stack(keys), axis=0)
    got_logits = from_dev(logits)
    for m in range(M):
        want = int(full_idx[m].item())
        assert want == oracle.argmax_reference_fast(got_logits[m])
        assert ie.key_index(int(merged[m])) == want, (m, want)
    assert int(ws.sum().item()) == 0


GOLD_AMAX = 75177  # tests/golden/reference_golden.json


def test_argmax_reference_golden(ie, cuda):
    """The reference's own sampling golden (torch seed 42, 128256 fp16 logits)."""
    cuda.manual_seed(0)
    import torch
    torch.manual_seed(42)
    logits = torch.randn(128256, dtype=torch.float16).cuda()
    out = cuda.full((1,), -1, dtype=cuda.int32, device="cuda")
    ie.sample_token_amax(logits, out)
    assert int(out.item()) == GOLD_AMAX


@pytest.mark.parametrize("dt", DTS)
def test_argmax_tie_vectors(ie, cuda, dt):
    """Crafted ties across residues and quotients, rows of odd length."""
    rng = np.random.default_rng(9)
    rows = []
    for V in (128256, 4096, 1001, 1024, 8200):
        v = oracle.round_dt(rng.integers(-3, 4, size=V) * 0.25, dt)
        rows.append(v)
    v = np.zeros(8192, np.float32)
    v[3074] = v[512] = 1.0
    rows.append(v)
    v = np.zeros(4096, np.float32)
    v[5] = v[1024] = 3.0
    rows.append(v)
    v = np.full(2048, -1.0, np.float32)
    v[100] = 0.0
    v[1500] = -0.0
    rows.append(v)
    for v in rows:
        V = v.size
        ld = (V + 7) // 8 * 8
        buf = np.zeros((2, ld), np.float32)
        buf[0, :V] = v
        buf[1, :V] = v[::-1]
        t = to_dev(buf, dt)
        out = cuda.full((2,), -1, dtype=cuda.int32, device="cuda")
        ie.argmax(t[:, :V], out)
        got = out.cpu().numpy()
        # rows shorter than 1024 have no reference behaviour (it reads past the
        # buffer); the oracle then gives absent threads -inf, as the kernel does
        assert got[0] == oracle.argmax_reference(v)
        assert got[1] == oracle.argmax_reference(v[::-1].copy())
        assert got[0] == oracle.argmax_reference_fast(v)


@pytest.mark.parametrize("dt", DTS)
def test_swiglu_standalone(ie, cuda, dt):
    import json
    from pathlib import Path
    import torch
    gold = json.loads((Path(__file__).parent / "golden" / "reference_golden.json").read_text())["swiglu"]
    torch.manual_seed(42)
    g = torch.randn(128, 14336, dtype=torch.float16)
    u = torch.randn(128, 14336, dtype=torch.float16)
    gf, uf = g.float().numpy(), u.float().numpy()
    if dt == "f16":
        G, U = g.cuda(), u.cuda()
    else:
        gf, uf = oracle.round_dt(gf, "bf16"), oracle.round_dt(uf, "bf16")
        G, U = to_dev(gf, dt), to_dev(uf, dt)
    out = cuda.empty_like(G)
    ie.swiglu(128, G, U, out)
    got = from_dev(out)
    want = oracle.swiglu(gf, uf, dt)
    # tests/test_swiglu.cu:33-36 thresholds, against the oracle
    r = oracle.compare(got, want, atol=2e-5 if dt == "f16" else 2e-2)
    assert r["max_abs_err"] < (1e-3 if dt == "f16" else 2e-2)
    assert r["pct_within_tol"] > 99.0
    if dt == "f16":
        sample = np.load(Path(__file__).parent / "golden" / "swiglu_out_sample.npy").astype(np.float32)
        r = oracle.compare(got.ravel()[:: gold["sample_stride"]], sample, atol=2e-5)
        assert r["max_abs_err"] < 1e-3 and r["pct_within_tol"] > 99.0
        # in place (out aliases gate), as ffn.cu:57 calls it
        ie.swiglu(128, G, U, G)
        assert np.array_equal(from_dev(G), got)


def test_empty_and_error_paths_on_device(ie, cuda):
    x = cuda.zeros((1, 64), dtype=cuda.bfloat16, device="cuda")
    w = cuda.zeros((16, 64), dtype=cuda.bfloat16, device="cuda")
    y = cuda.zeros((1, 16), dtype=cuda.bfloat16, device="cuda")
    ie.gemm(x, w, y, M=0)  # no-op
    with pytest.raises(ie.IEError):
        ie.gemm(x, w, y, K=60, ldx=64, ldw=64)  # K % 8
    with pytest.raises(ie.IEError):
        ie.gemm(x, w, y, ldy=8)  # ldy < N


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("B", [8, 24])
def test_qkv_batched_independent_sequences(ie, cuda, dt, B):
    """Batched decode (BASELINE config 5 at batch 8; 24 rows run on the
    tensor-core kernel): every row at its own position in its own cache."""
    H, nq, nkv, hd, rows = 4096, 32, 8, 128, 512
    d = oracle.seeded_inputs(200 + B, {"x": (B, H), "wq": (nq * hd, H), "wk": (nkv * hd, H), "wv": (nkv * hd, H)}, dt)
    cos, sin = oracle.rope_tables(rows)
    rng = np.random.default_rng(B)
    pos = rng.integers(0, rows, size=B).astype(np.int32)
    T = torch_dtype(dt)
    q = cuda.empty((nq, B, hd), dtype=T, device="cuda")
    kc = cuda.zeros((B, nkv, rows, hd), dtype=T, device="cuda")
    vc = cuda.zeros((B, nkv, rows, hd), dtype=T, device="cuda")
    ie.device_status(clear=True)
    ie.qkv_batched(to_dev(d["x"], dt), to_dev(d["wq"], dt), to_dev(d["wk"], dt), to_dev(d["wv"], dt), q, kc, vc,
                   cuda.from_numpy(pos).cuda(), cuda.from_numpy(cos).cuda(), cuda.from_numpy(sin).cuda())
    assert ie.device_status(clear=True) == 0
    got_q, got_k, got_v = from_dev(q), from_dev(kc), from_dev(vc)
    for b in range(B):
        qr, kr, vr = oracle.qkv(d["x"][b:b + 1], d["wq"], d["wk"], d["wv"], dt, int(pos[b]), cos, sin)
        tq, tk, tv = rope_tol(d["x"][b:b + 1], d["wq"], d["wk"], d["wv"], dt, True)
        assert np.all(np.abs(got_q[:, b:b + 1] - qr) <= tq)
        assert np.all(np.abs(got_k[b][:, pos[b]:pos[b] + 1] - kr) <= tk)
        assert np.all(np.abs(got_v[b][:, pos[b]:pos[b] + 1] - vr) <= tv)
        others = np.ones(rows, bool)
        others[pos[b]] = False
        assert np.all(got_k[b][:, others] == 0)


def test_qkv_batched_rejects_out_of_range_position(ie, cuda):
    H, nq, nkv, rows = 4096, 32, 8, 64
    T = cuda.bfloat16
    x = cuda.zeros((2, H), dtype=T, device="cuda")
    wq = cuda.zeros((nq * 128, H), dtype=T, device="cuda")
    wk = cuda.zeros((nkv * 128, H), dtype=T, device="cuda")
    q = cuda.empty((nq, 2, 128), dtype=T, device="cuda")
    kc = cuda.zeros((2, nkv, rows, 128), dtype=T, device="cuda")
    vc = cuda.zeros_like(kc)
    pos = cuda.tensor([3, rows], dtype=cuda.int32, device="cuda")  # second row out of range
    ie.device_status(clear=True)
    ie.qkv_batched(x, wq, wk, wk, q, kc, vc, pos)
    assert ie.device_status(clear=True) == -1  # IE_ERR_INVALID_ARG, row skipped
