"""GPU, 2 devices: the tensor-parallel decode step against the single-GPU path.

Two ranks (spawned processes, NCCL) each hold half of every projection of a
2-layer Llama-3.1-8B-width model (plus the vocabulary-split lm_head) drawn
from the same seeded generator. After one step rank 0 compares with the
single-GPU kernels on the full weights:
  * its own Q heads and K/V cache rows are bit-identical to the full QKV's;
  * O and down outputs (fp32 partials summed over ranks, rounded once) are
    within one rounding step of the single-GPU outputs;
  * the merged greedy id equals the single-GPU id.
Skipped where fewer than two GPUs are visible.
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

pytestmark = pytest.mark.gpu


def _two_gpus():
    try:
        import torch
        return torch.cuda.device_count() >= 2
    except Exception:  # noqa: BLE001
        return False


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outq, mode, M):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import infengine_b200 as ie
    from infengine_b200.host import rope_tables
    from infengine_b200.tp import Comm, P2PExchange, ShardPlan, TPDecodeStep
    from conftest import from_dev, ulp
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=120), device_id=dev)
        H, F, V, NQ, NKV, HD, CTX, POS = 4096, 14336, 128256, 32, 8, 128, 256, 100
        g = torch.Generator(device=dev)
        g.manual_seed(11)

        def w(*shape):
            return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).mul_(0.02).to(torch.bfloat16)

        fulls = [{"wq": w(NQ * HD, H), "wk": w(NKV * HD, H), "wv": w(NKV * HD, H), "wo": w(H, H), "wg": w(F, H),
                  "wu": w(F, H), "wd": w(H, F)} for _ in range(2)]
        lm = w(V, H)
        x = torch.randn(M, H, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
        cos, sin = (torch.from_numpy(t).to(dev) for t in rope_tables(CTX))
        plan = ShardPlan(world, rank)
        comm = Comm(world, rank)
        exchange = P2PExchange(world, rank) if mode == "p2p" else None
        pos = POS if M == 1 else 0
        step = TPDecodeStep(plan, comm, [plan.shard_layer(f) for f in fulls], plan.shard_lm_head(lm), cos, sin, pos,
                            batch=M, ctx=CTX, exchange=exchange, lm_rows=1)
        step.x.copy_(x)
        for _ in range(3):  # repeated calls exercise both exchange parities
            step()
        torch.cuda.synchronize()
        res = {"ok": True}
        if rank == 0:
            # single-GPU path on the full weights (last layer is what the buffers hold)
            f = fulls[-1]
            q = torch.empty(NQ, M, HD, device=dev, dtype=torch.bfloat16)
            kc = torch.zeros(NKV, CTX, HD, device=dev, dtype=torch.bfloat16)
            vc = torch.zeros_like(kc)
            ie.qkv(x, f["wq"], f["wk"], f["wv"], q, kc, vc, CTX * HD, pos, cos, sin)
            attn = torch.empty(M, H, device=dev, dtype=torch.bfloat16)
            ie.gemm(q.view(1, H) if M == 1 else q.permute(1, 0, 2).reshape(M, H), f["wo"], attn)
            h = torch.empty(M, F, device=dev, dtype=torch.bfloat16)
            ie.ffn_gate_up(x, f["wg"], f["wu"], h)
            down = torch.empty(M, H, device=dev, dtype=torch.bfloat16)
            ie.gemm(h, f["wd"], down)
            ws = torch.zeros(ie.lm_head_workspace_bytes(1), dtype=torch.uint8, device=dev)
            tok = torch.zeros(1, dtype=torch.int32, device=dev)
            ie.lm_head_argmax(x[M - 1:], lm, ws, idx_out=tok)
            torch.cuda.synchronize()
            res["q_equal"] = bool(torch.equal(step.q, q[: plan.q_heads]))
            res["k_equal"] = bool(torch.equal(step.kc[-1][:, pos:pos + M], kc[: plan.kv_heads, pos:pos + M]))
            for name, tp, single in (("attn", step.attn_out, attn), ("down", step.ffn_out, down)):
                a, b = from_dev(tp), from_dev(single)
                # rounding steps, with the 1e-5-of-scale floor the other tests use
                # for outputs that cancel to near zero
                res[name + "_steps"] = float((np.abs(a - b) / (ulp(b, "bf16") + 1e-5 * np.abs(b).max())).max())
            res["tok_tp"], res["tok_single"] = int(step.tok.item()), int(tok.item())
        res["status"] = ie.device_status()
        outq.put((rank, res))
        dist.barrier()
        if exchange is not None:
            exchange.close()
        comm.close()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        outq.put((rank, {"ok": False, "error": repr(e)}))


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
@pytest.mark.parametrize("mode,M", [("p2p", 1), ("nccl", 1), ("nccl", 128)])
def test_tp2_step_matches_single_gpu(mode, M):
    """M=1: decode step (fused NVLink exchange or NCCL); M=128: a prefill
    chunk on the tensor-core kernels with the NCCL exchange."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    outq = ctx.Queue()
    port = _port()
    env_nvls = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    procs = [ctx.Process(target=_worker, args=(r, 2, port, outq, mode, M)) for r in range(2)]
    try:
        for p in procs:
            p.start()
        results = dict(outq.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=120)
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
        if env_nvls is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = env_nvls
    assert all(r["ok"] for r in results.values()), results
    r0 = results[0]
    assert r0["q_equal"] and r0["k_equal"], r0
    assert r0["attn_steps"] <= 1.0 and r0["down_steps"] <= 1.0, r0
    assert r0["tok_tp"] == r0["tok_single"], r0
    assert all(r["status"] == 0 for r in results.values()), results
