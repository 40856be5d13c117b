"""CPU (gloo, world size 2): the tensor-parallel host logic.

The shard plan of infengine_b200.tp is exercised with the oracle standing in
for the kernels: each rank computes its shard's Q/K/V heads, O and down
partial sums, SwiGLU rows and lm_head keys; gloo sums the partials and merges
the keys; the result must equal the unsharded computation. Failure handling
is tested on the host: a rank that dies before a collective makes the
survivor's collective fail within the process-group timeout.
"""
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

from infengine_b200.tp import ShardPlan  # noqa: E402

SMALL = dict(hidden=64, ffn=96, n_q_heads=8, n_kv_heads=4, head_dim=16, vocab=3000)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _full_problem(seed=0):
    import ie_oracle as oracle
    c = SMALL
    hd, H, F = c["head_dim"], c["hidden"], c["ffn"]
    return oracle.seeded_inputs(seed, {
        "x": (1, H), "wq": (c["n_q_heads"] * hd, H), "wk": (c["n_kv_heads"] * hd, H), "wv": (c["n_kv_heads"] * hd, H),
        "wo": (H, c["n_q_heads"] * hd), "wg": (F, H), "wu": (F, H), "wd": (H, F), "lm": (c["vocab"], H)}, "f32")


def test_shards_cover_every_row_once():
    for world in (1, 2, 4):
        plans = [ShardPlan(world, r, **SMALL) for r in range(world)]
        for fn, n in (("q_rows", SMALL["n_q_heads"] * 16), ("kv_rows", SMALL["n_kv_heads"] * 16),
                      ("ffn_slice", SMALL["ffn"]), ("vocab_slice", SMALL["vocab"])):
            cover = np.zeros(n, int)
            for p in plans:
                cover[getattr(p, fn)()] += 1
            assert np.all(cover == 1), (world, fn)


def test_llama_plan_sizes():
    for world, (q, kv, f, v) in {1: (32, 8, 14336, 128256), 2: (16, 4, 7168, 64128), 4: (8, 2, 3584, 32064),
                                 8: (4, 1, 1792, 16032)}.items():
        p = ShardPlan(world, world - 1)
        assert (p.q_heads, p.kv_heads, p.ffn_rows) == (q, kv, f)
        s = p.vocab_slice()
        assert s.stop - s.start == v and s.stop == 128256


def test_invalid_plans_rejected():
    with pytest.raises(ValueError):
        ShardPlan(3, 0)  # 8 KV heads do not split over 3 ranks
    with pytest.raises(ValueError):
        ShardPlan(2, 2)
    with pytest.raises(ValueError):
        ShardPlan(16, 0)  # one KV head cannot be split


def _tp_worker(rank, world, port, out):
    import torch
    import torch.distributed as dist
    import ie_oracle as oracle
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    d = _full_problem()
    plan = ShardPlan(world, rank, **SMALL)
    w = plan.shard_layer(d)
    x = d["x"]
    # local Q/K/V heads (exact sums, no rounding: the point is the sharding)
    q = oracle.gemm_fp32(x, w["wq"])
    # O: partial over this rank's heads, summed over ranks
    o_part = torch.from_numpy(oracle.gemm_fp32(q, w["wo"]).astype(np.float64))
    dist.all_reduce(o_part)
    # FFN: local SwiGLU rows, partial down, summed
    h = oracle.swiglu(oracle.gemm_fp32(x, w["wg"]), oracle.gemm_fp32(x, w["wu"]), "f32")
    d_part = torch.from_numpy(oracle.gemm_fp32(h, w["wd"]).astype(np.float64))
    dist.all_reduce(d_part)
    # lm_head: keys of the local vocabulary rows with global ids, merged by max
    lm = plan.shard_lm_head(d["lm"])
    logits = oracle.gemm_fp32(x, lm)[0]
    off = plan.vocab_slice().start
    key = max(oracle.argmax_key(float(v), off + i) for i, v in enumerate(logits))
    keys = [None] * world
    dist.all_gather_object(keys, key)
    qs = [None] * world
    dist.all_gather_object(qs, q)
    if rank == 0:
        out.put({"o": o_part.numpy(), "down": d_part.numpy(), "id": oracle.key_index(max(keys)),
                 "q": np.concatenate(qs, axis=1)})
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_sharded_step_equals_unsharded(world):
    import torch.multiprocessing as mp
    import ie_oracle as oracle
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    d = _full_problem()
    x = d["x"]
    q_full = oracle.gemm_fp32(x, d["wq"])
    np.testing.assert_allclose(res["q"], q_full, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(res["o"], oracle.gemm_fp32(q_full, d["wo"]), rtol=1e-5, atol=1e-5)
    h = oracle.swiglu(oracle.gemm_fp32(x, d["wg"]), oracle.gemm_fp32(x, d["wu"]), "f32")
    np.testing.assert_allclose(res["down"], oracle.gemm_fp32(h, d["wd"]), rtol=1e-5, atol=1e-5)
    assert res["id"] == oracle.argmax_reference_fast(oracle.gemm_fp32(x, d["lm"])[0])


def _dying_worker(rank, world, port, out):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # dies between steps, before the next collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        out.put("no error")
    except Exception as e:  # noqa: BLE001
        out.put(f"error: {type(e).__name__}")


def test_lost_rank_fails_the_survivors_collective():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg.startswith("error"), msg
