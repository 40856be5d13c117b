"""GPU, 2 devices: the tensor-parallel decode engine (ie_engine_create_tp)
against the single-GPU engine on the same weights.

Two ranks (spawned processes, NCCL) each hold half of every projection of a
2-layer Llama-3.1-8B-width model (plus their vocabulary half of lm_head),
built from the same seeded generator; rank 0 also runs the single-GPU engine
on the full weights. Both see the same prompt, then the same teacher-forced
tokens through ie_engine_step. O and down partial sums are reduced over the
ranks before their one rounding, so an id may differ from the single-GPU one
only at a near tie; at least 80 % must agree. Modes: the fused NVLink
exchange for decode rows (p2p) and NCCL for everything. Skipped where fewer
than two GPUs are visible.
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


def _worker(rank, world, port, outq, mode):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    from infengine_b200.engine import LlamaEngine
    from infengine_b200.host import rope_tables
    from infengine_b200.tp import Comm, P2PExchange, ShardPlan
    eng = single = comm = ex = None
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=120), device_id=dev)
        H, F, V, NQ, NKV, LAYERS = 4096, 14336, 128256, 32, 8, 2
        g = torch.Generator(device=dev)
        g.manual_seed(21)

        def w(*shape, std=0.02):
            return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).mul_(std).to(torch.bfloat16)

        ones = torch.ones(H, dtype=torch.bfloat16, device=dev)
        full = [{"wq": w(NQ * 128, H), "wk": w(NKV * 128, H), "wv": w(NKV * 128, H), "wo": w(H, H),
                 "wg": w(F, H), "wu": w(F, H), "wd": w(H, F)} for _ in range(LAYERS)]
        emb, lm = w(V, H, std=1.0), w(V, H)
        cos, sin = (torch.from_numpy(t).to(dev) for t in rope_tables(512))
        plan = ShardPlan(world, rank)

        def engine_weights(layers, lm_w):
            return dict(embedding=emb, final_norm=ones, lm_head=lm_w, rope_cos=cos, rope_sin=sin,
                        layers=[dict(attn_norm=ones, wq=l["wq"], wk=l["wk"], wv=l["wv"], wo=l["wo"], ffn_norm=ones,
                                     w_gate=l["wg"], w_up=l["wu"], w_down=l["wd"]) for l in layers])

        comm = Comm(world, rank)
        ex = P2PExchange(world, rank) if mode == "p2p" else None
        vs = plan.vocab_slice()
        dims = dict(n_layers=LAYERS, hidden=H, n_q_heads=NQ // world, n_kv_heads=NKV // world, head_dim=128,
                    ffn_dim=F // world, vocab=V)
        eng = LlamaEngine(engine_weights([plan.shard_layer(l) for l in full], plan.shard_lm_head(lm)), dims,
                          max_batch=1, max_ctx=512, max_prefill=128,
                          tp=dict(world=world, rank=rank, comm=comm, exchange=ex, lm_rows=vs.stop - vs.start,
                                  lm_offset=vs.start))
        prompt = np.random.default_rng(5).integers(0, V, size=70).astype(np.int32)  # tensor-core prefill
        tp_ids = [eng.prefill(0, prompt)]
        res = {"ok": True}
        if rank == 0:
            single = LlamaEngine(engine_weights(full, lm), dict(dims, n_q_heads=NQ, n_kv_heads=NKV, ffn_dim=F),
                                 max_batch=1, max_ctx=512, max_prefill=128)
            one_ids = [single.prefill(0, prompt)]
        forced = np.random.default_rng(6).integers(0, V, size=10).astype(np.int32)
        for t in forced:  # the same inputs on both sides
            tp_ids.append(int(eng.step(np.array([t], np.int32))[0]))
            if rank == 0:
                one_ids.append(int(single.step(np.array([t], np.int32))[0]))
        nxt = eng.decode(5)[:, 0]  # graph replays on the device-resident ids
        if rank == 0:
            res["tp"], res["single"] = tp_ids, one_ids
        res["decode"] = nxt.tolist()
        import infengine_b200 as ie
        res["status"] = ie.device_status()
        outq.put((rank, res))
        dist.barrier()
    except Exception as e:  # noqa: BLE001
        outq.put((rank, {"ok": False, "error": repr(e)}))
    finally:
        for obj in (eng, single):
            if obj is not None:
                obj.close()
        if ex is not None:
            ex.close()
        if comm is not None:
            comm.close()
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["p2p", "nccl"])
def test_tp2_engine_matches_single_gpu(mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    outq = ctx.Queue()
    port = _port()
    env_nvls = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    procs = [ctx.Process(target=_worker, args=(r, 2, port, outq, mode)) for r in range(2)]
    try:
        for p in procs:
            p.start()
        results = dict(outq.get(timeout=600) for _ in procs)
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
    agree = np.mean(np.array(r0["tp"]) == np.array(r0["single"]))
    print(f"tp2 ({mode}) vs single GPU: {agree:.2f} of ids equal; tp {r0['tp']} single {r0['single']}")
    assert agree >= 0.8, r0
    assert results[0]["decode"] == results[1]["decode"]  # every rank holds the merged ids
    assert all(r["status"] == 0 for r in results.values()), results
