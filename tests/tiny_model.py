"""A tiny random-init Llama (head_dim 128, the engine's only head size) for
comparing the decode engine with the CPU model oracle (oracle/ie_oracle.py
LlamaOracle). Test infrastructure: used by tests/ and __graft_entry__.smoke."""
from __future__ import annotations

import numpy as np

TINY = dict(hidden=256, n_q_heads=2, n_kv_heads=1, head_dim=128, ffn_dim=512, vocab=1000, rms_eps=1e-5)


def tiny_weights(oracle, layers: int, seed: int, dt: str = "bf16"):
    rng = np.random.default_rng(seed)
    H, F, V = TINY["hidden"], TINY["ffn_dim"], TINY["vocab"]
    q, kv = TINY["n_q_heads"] * 128, TINY["n_kv_heads"] * 128

    def w(*shape, std=0.02):
        return oracle.round_dt(rng.standard_normal(shape).astype(np.float32) * np.float32(std), dt)

    def norm():
        return oracle.round_dt((1 + 0.1 * rng.standard_normal(H)).astype(np.float32), dt)

    return dict(embedding=w(V, H, std=1.0), final_norm=norm(), lm_head=w(V, H, std=0.05),
                layers=[dict(attn_norm=norm(), wq=w(q, H), wk=w(kv, H), wv=w(kv, H), wo=w(H, q), ffn_norm=norm(),
                             w_gate=w(F, H), w_up=w(F, H), w_down=w(H, F)) for _ in range(layers)])


def engine_vs_oracle(oracle, to_dev, weights: dict, prompt, n_steps: int, dt: str = "bf16", max_ctx: int = 256,
                     eng=None):
    """Prefill `prompt`, then n_steps teacher-forced steps (both sides fed the
    oracle's ids); `eng`: an engine on these weights (default: one built
    here from device copies). Returns (engine ids, oracle ids, oracle margins)."""
    import torch
    from infengine_b200.engine import LlamaEngine
    layers = weights["layers"]
    if eng is None:
        dev_w = {k: to_dev(v, dt) for k, v in weights.items() if k != "layers"}
        dev_w["layers"] = [{k: to_dev(v, dt) for k, v in lw.items()} for lw in layers]
        cos, sin = oracle.rope_tables(max_ctx)
        dev_w["rope_cos"] = torch.from_numpy(cos).cuda()
        dev_w["rope_sin"] = torch.from_numpy(sin).cuda()
        dims = dict(TINY, n_layers=len(layers))
        eng = LlamaEngine(dev_w, dims, dtype=dt, max_batch=1, max_ctx=max_ctx, max_prefill=max(len(prompt), 16))
    ref = oracle.LlamaOracle(weights, TINY["n_q_heads"], TINY["n_kv_heads"], dt, max_ctx=max_ctx)
    got = [eng.prefill(0, prompt)]
    want, margin = [], []
    t, m = ref.pick(ref.forward(prompt)[-1])
    want.append(t)
    margin.append(m)
    for _ in range(n_steps):
        fed = want[-1]
        got.append(int(eng.step(np.array([fed], np.int32))[0]))
        t, m = ref.pick(ref.forward([fed])[-1])
        want.append(t)
        margin.append(m)
    eng.close()
    return np.array(got), np.array(want), np.array(margin)
