"""GPU: the attention core behind the drop-in attn / decode_attn (ie_attention)
against the oracle's restatement of the reference's chain."""
import numpy as np
import pytest

from conftest import from_dev, oracle, to_dev, torch_dtype, ulp

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("S,pos0,nq,nkv", [(1, 0, 32, 8), (1, 300, 32, 8), (37, 0, 32, 8), (16, 50, 8, 2),
                                           (5, 2043, 4, 1), (17, 0, 8, 2), (64, 0, 8, 2), (65, 3, 8, 2),
                                           (300, 100, 32, 8), (1024, 0, 8, 2), (129, 0, 4, 4), (200, 1900, 8, 2),
                                           (2048, 64, 8, 1)])
def test_attention_core(ie, cuda, dt, S, pos0, nq, nkv):
    """S <= 16: split-KV kernel; S > 16: tensor-core flash kernel (chunked
    prefill when pos0 > 0; ragged last query and key blocks)."""
    ctx = 2048 + 64
    rng = np.random.default_rng(S * 1000 + pos0 + nq)
    q = oracle.round_dt(rng.standard_normal((nq, S, 128), dtype=np.float32), dt)
    k = np.zeros((nkv, ctx, 128), np.float32)
    v = np.zeros((nkv, ctx, 128), np.float32)
    k[:, :pos0 + S] = oracle.round_dt(rng.standard_normal((nkv, pos0 + S, 128), dtype=np.float32), dt)
    v[:, :pos0 + S] = oracle.round_dt(rng.standard_normal((nkv, pos0 + S, 128), dtype=np.float32), dt)
    out = cuda.full((S, nq * 128), float("nan"), dtype=torch_dtype(dt), device="cuda")
    ie.attention(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), out, pos0, n_kv_heads=nkv)
    got = from_dev(out)
    assert ie.device_status() == 0
    want = oracle.attention(q, k, v, pos0, dt)
    assert not np.isnan(got).any()
    # a rounding flip of one probability moves an output by about one p-ulp
    # times |V|; bound: two output rounding steps plus 2 % of the output scale
    err = np.abs(got - want)
    assert np.all(err <= 2 * ulp(want, dt) + 0.02 * np.abs(want).max()), err.max()
    assert oracle.normwise_rel_err(got, want) < (5e-3 if dt == "f16" else 2e-2)


def _check_close(got, want, dt):
    err = np.abs(got - want)
    assert not np.isnan(got).any()
    assert np.all(err <= 2 * ulp(want, dt) + 0.02 * np.abs(want).max()), err.max()
    assert oracle.normwise_rel_err(got, want) < (5e-3 if dt == "f16" else 2e-2)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("pos,nq,nkv,rows", [(0, 32, 8, 2048), (5, 32, 8, 2048), (300, 32, 8, 2048),
                                             (2047, 32, 8, 2048), (8191, 32, 8, 8192), (1000, 8, 8, 1024),
                                             (777, 16, 2, 1024), (130, 8, 4, 256)])
def test_attention_decode_one_row(ie, cuda, dt, pos, nq, nkv, rows):
    """Split-KV decode attention, one query row over its whole cache (slices
    of fewer than 8 rows, exact 64-row chunks, ragged tails, groups 1-8)."""
    rng = np.random.default_rng(pos * 7 + nq + rows)
    q = oracle.round_dt(rng.standard_normal((nq, 1, 128), dtype=np.float32), dt)
    k = np.zeros((nkv, rows, 128), np.float32)
    v = np.zeros((nkv, rows, 128), np.float32)
    k[:, :pos + 1] = oracle.round_dt(rng.standard_normal((nkv, pos + 1, 128), dtype=np.float32), dt)
    v[:, :pos + 1] = oracle.round_dt(rng.standard_normal((nkv, pos + 1, 128), dtype=np.float32), dt)
    out = cuda.full((1, nq * 128), float("nan"), dtype=torch_dtype(dt), device="cuda")
    positions = cuda.tensor([pos], dtype=cuda.int32, device="cuda")
    ie.attention_decode(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), out, positions=positions)
    assert ie.device_status() == 0
    _check_close(from_dev(out), oracle.attention(q, k, v, pos, dt), dt)


@pytest.mark.parametrize("dt", ["bf16"])
def test_attention_decode_batched_and_verify(ie, cuda, dt):
    """Eight sequences with their own positions (batched decode), then five
    causal rows of one sequence (speculative verify, positions from pos0)."""
    rng = np.random.default_rng(3)
    B, nq, nkv, rows = 8, 32, 8, 1024
    pos = np.array([0, 1, 63, 64, 500, 1000, 1023, 7], dtype=np.int32)
    q = oracle.round_dt(rng.standard_normal((nq, B, 128), dtype=np.float32), dt)
    k = oracle.round_dt(rng.standard_normal((B, nkv, rows, 128), dtype=np.float32), dt)
    v = oracle.round_dt(rng.standard_normal((B, nkv, rows, 128), dtype=np.float32), dt)
    out = cuda.full((B, nq * 128), float("nan"), dtype=torch_dtype(dt), device="cuda")
    ie.attention_decode(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), out,
                        positions=cuda.from_numpy(pos).cuda())
    assert ie.device_status() == 0
    got = from_dev(out)
    for b in range(B):
        want = oracle.attention(q[:, b:b + 1], k[b], v[b], int(pos[b]), dt)
        _check_close(got[b:b + 1], want, dt)
    # verify pass: 5 rows of sequence 0 at positions 900..904
    qv = oracle.round_dt(rng.standard_normal((nq, 5, 128), dtype=np.float32), dt)
    outv = cuda.full((5, nq * 128), float("nan"), dtype=torch_dtype(dt), device="cuda")
    ie.attention_decode(to_dev(qv, dt), to_dev(k[0], dt), to_dev(v[0], dt), outv, pos0=900, rows_per_seq=5)
    assert ie.device_status() == 0
    _check_close(from_dev(outv), oracle.attention(qv, k[0], v[0], 900, dt), dt)


@pytest.mark.parametrize("nq,nkv", [(32, 8), (8, 2)])
def test_attention_decode_batch_invariant(ie, cuda, nq, nkv):
    """A row gets the same bits alone as inside a batch of four (the key split
    and the order of the partial sums do not depend on the batch)."""
    dt = "bf16"
    rng = np.random.default_rng(11)
    B, rows = 4, 2048
    pos = np.array([2047, 5, 700, 1500], dtype=np.int32)
    q = oracle.round_dt(rng.standard_normal((nq, B, 128), dtype=np.float32), dt)
    k = to_dev(oracle.round_dt(rng.standard_normal((B, nkv, rows, 128), dtype=np.float32), dt), dt)
    v = to_dev(oracle.round_dt(rng.standard_normal((B, nkv, rows, 128), dtype=np.float32), dt), dt)
    out = cuda.empty((B, nq * 128), dtype=torch_dtype(dt), device="cuda")
    ie.attention_decode(to_dev(q, dt), k, v, out, positions=cuda.from_numpy(pos).cuda())
    for b in range(B):
        one = cuda.empty((1, nq * 128), dtype=torch_dtype(dt), device="cuda")
        ie.attention_decode(to_dev(np.ascontiguousarray(q[:, b:b + 1]), dt), k[b:b + 1], v[b:b + 1], one,
                            positions=cuda.from_numpy(pos[b:b + 1]).cuda())
        assert cuda.equal(one[0], out[b]), b
    assert ie.device_status() == 0


def test_attention_decode_bad_position(ie, cuda):
    """A device position outside the cache: that row is zero, the status word
    says IE_ERR_INVALID_ARG, the other rows are unaffected."""
    dt = "bf16"
    rng = np.random.default_rng(5)
    nq, nkv, rows = 8, 2, 256
    q = oracle.round_dt(rng.standard_normal((nq, 2, 128), dtype=np.float32), dt)
    k = oracle.round_dt(rng.standard_normal((2, nkv, rows, 128), dtype=np.float32), dt)
    v = oracle.round_dt(rng.standard_normal((2, nkv, rows, 128), dtype=np.float32), dt)
    out = cuda.full((2, nq * 128), float("nan"), dtype=torch_dtype(dt), device="cuda")
    pos = cuda.tensor([100, rows], dtype=cuda.int32, device="cuda")
    ie.attention_decode(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), out, positions=pos)
    assert ie.device_status() == -1  # IE_ERR_INVALID_ARG
    got = from_dev(out)
    assert np.all(got[1] == 0)
    _check_close(got[0:1], oracle.attention(q[:, 0:1], k[0], v[0], 100, dt), dt)
    assert ie.device_status() == 0  # cleared by the read above


def test_prefill_attention_mma_kernel_selectable(tmp_path):
    """IE_PREFILL_ATTN=mma runs prefill attention on the mma.sync kernel (kept
    for A/B measurements); it meets the same bound against the oracle. Run in a
    child process because the switch is read once per process."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    dt, S, pos0, nq, nkv = "bf16", 300, 100, 8, 2
    rng = np.random.default_rng(77)
    q = oracle.round_dt(rng.standard_normal((nq, S, 128), dtype=np.float32), dt)
    k = oracle.round_dt(rng.standard_normal((nkv, pos0 + S, 128), dtype=np.float32), dt)
    v = oracle.round_dt(rng.standard_normal((nkv, pos0 + S, 128), dtype=np.float32), dt)
    np.savez(tmp_path / "in.npz", q=q, k=k, v=v)
    root = Path(__file__).resolve().parent.parent
    code = f"""
import sys, numpy as np, torch
sys.path.insert(0, {str(root)!r})
import infengine_b200 as ie
d = np.load({str(tmp_path / 'in.npz')!r})
t = lambda a: torch.from_numpy(a).cuda().to(torch.bfloat16)
out = torch.empty({S}, {nq * 128}, dtype=torch.bfloat16, device="cuda")
ie.attention(t(d["q"]), t(d["k"]), t(d["v"]), out, {pos0}, n_kv_heads={nkv})
torch.cuda.synchronize()
assert ie.device_status() == 0
np.save({str(tmp_path / 'out.npy')!r}, out.float().cpu().numpy())
"""
    env = dict(os.environ, IE_PREFILL_ATTN="mma")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    _check_close(np.load(tmp_path / "out.npy"), oracle.attention(q, k, v, pos0, dt), dt)


def test_attention_decode_ring_depth_changes_no_bit(tmp_path):
    """The decode kernel's ring depth (2-6 slots of 64 cache rows, chosen per
    launch from the grid size; IE_FD_STAGES fixes it) only changes how many
    copies are in flight: the same rows meet the same MMAs in the same order,
    so every depth gives the same bits. Eight sequences (512 CTAs, 3 slots by
    default) with ragged lengths, run in child processes at depths 2, 5 and
    the default, because the switch is read once per process; the default
    run is also checked against the oracle."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    dt, B, nq, nkv, rows = "bf16", 8, 32, 8, 2048
    rng = np.random.default_rng(91)
    pos = np.array([2047, 1000, 5, 64, 700, 1999, 130, 1500], dtype=np.int32)
    q = oracle.round_dt(rng.standard_normal((nq, B, 128), dtype=np.float32), dt)
    k = oracle.round_dt(rng.standard_normal((B, nkv, rows, 128), dtype=np.float32), dt)
    v = oracle.round_dt(rng.standard_normal((B, nkv, rows, 128), dtype=np.float32), dt)
    np.savez(tmp_path / "in.npz", q=q, k=k, v=v, pos=pos)
    root = Path(__file__).resolve().parent.parent
    outs = {}
    for depth in ("2", "5", None):
        out_file = tmp_path / f"out_{depth}.npy"
        code = f"""
import sys, numpy as np, torch
sys.path.insert(0, {str(root)!r})
import infengine_b200 as ie
d = np.load({str(tmp_path / 'in.npz')!r})
t = lambda a: torch.from_numpy(a).cuda().to(torch.bfloat16)
out = torch.empty({B}, {nq * 128}, dtype=torch.bfloat16, device="cuda")
ie.attention_decode(t(d["q"]), t(d["k"]), t(d["v"]), out, positions=torch.from_numpy(d["pos"]).cuda())
torch.cuda.synchronize()
assert ie.device_status() == 0
np.save({str(out_file)!r}, out.view(torch.int16).cpu().numpy())
"""
        env = dict(os.environ)
        env.pop("IE_FD_STAGES", None)
        if depth:
            env["IE_FD_STAGES"] = depth
        r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        outs[depth] = np.load(out_file)
    assert np.array_equal(outs["2"], outs[None])
    assert np.array_equal(outs["5"], outs[None])
    got = outs[None].view(np.uint16).astype(np.uint32) << 16
    got = got.view(np.float32)
    for b in range(B):
        _check_close(got[b:b + 1], oracle.attention(q[:, b:b + 1], k[b], v[b], int(pos[b]), dt), dt)
