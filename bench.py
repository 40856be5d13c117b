#!/usr/bin/env python
"""Benchmark of infengine's decode on B200 (bs=1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one greedy decode token of random-init Llama-3.1-8B (bf16,
N(0,0.02) weights from a fixed seed, RMSNorm weights 1) right after a
2048-token prompt: embedding, 32 x [RMSNorm, fused QKV+RoPE into the KV
cache, split-KV attention, O projection + residual, RMSNorm, FFN gate/up +
SwiGLU, FFN down + residual], final RMSNorm, lm_head + greedy argmax. Our arm
runs it through the decode engine (ie_engine_decode: one CUDA graph per step,
the id kept on the device); 15.01 GB of weights are streamed per step (far
above the 126 MB L2, so no flush is needed). `value` is device-timed tok/s;
`e2e` is the same through ie_engine_step with the token copied in from and
the id copied out to the host every step.

Also reported: the weight-matmul path alone (`matmul_path`: the projections
and lm_head without attention, norms or residuals, one graph of 129 launches;
the north star's >= 80 % of HBM target) with the `roofline` of its dominant
kernel (FFN gate/up + SwiGLU); BASELINE configs 1-4 one by one (`configs`);
the M=2048 prefill projection chain against the sustained bf16 peak
(`prefill`); batch-8 decode and the M=5 verify pass through the engine; the
CPU golden of the path (`cpu_baseline`).

The reference arm (--impl reference) runs the reference's own decode loop
(prefill.cu / decode.cu with its kernels and cuBLAS, built from its sources
for sm_100a by oracle/Makefile; fp16, its only dtype) on random-init weights:
decode_step per token, eager on the legacy default stream, each step ending
in its blocking copy of the token to the host.

For N > 1 (torchrun) the same token stream is split by tensor parallelism
(one engine per rank: Q/K/V and gate/up column-split, O and down row-split
and reduced over NVLink with the residual add fused, lm_head
vocabulary-split with a max over packed argmax keys); the value is tok/s of
the one stream (strong scaling), timed as the max over ranks. The reference
arm has one GPU: rank 0 runs it, the other ranks exit.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s bs1 & matmul HBM GB/s, prefill GEMM TFLOPS vs B200 roofline"
H, F, V, L = 4096, 14336, 128256, 32
NQ, NKV, HD, CTX = 32, 8, 128, 8192
POS = 2047  # the 2048th token: decode right after a 2048-token prompt
PROMPT = 2048
JSON_OUT = None  # the original stdout (see main)
LAYER_WEIGHT_ELEMS = (NQ + 2 * NKV) * HD * H + H * H + 3 * F * H
WEIGHT_BYTES = 2 * (L * LAYER_WEIGHT_ELEMS + V * H)
GATE_UP_BYTES = 2 * (2 * F * H + H + F)  # one gate/up+SwiGLU launch at M=1


def load_peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, source)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def load_traffic():
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get("gate_up_swiglu_m1_bytes_per_launch")
        except Exception:
            return None
    return None


# ------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (200 ms) of this rank's GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(parts)
            except ValueError:
                pass
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------- weights
def make_weights(torch, dev, dtype, seed: int):
    """Random-init Llama-3.1-8B projection weights: N(0,0.02) drawn in fp32
    from a seeded generator, rounded to bf16 (then to the arm's dtype)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def w(*shape):
        t = torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).mul_(0.02)
        t = t.to(torch.bfloat16)
        return t if dtype == torch.bfloat16 else t.to(dtype)

    layers = []
    for _ in range(L):
        layers.append({"wq": w(NQ * HD, H), "wk": w(NKV * HD, H), "wv": w(NKV * HD, H), "wo": w(H, H),
                       "wg": w(F, H), "wu": w(F, H), "wd": w(H, F)})
    lm = w(V, H)
    return layers, lm


# ---------------------------------------------------------------- our arm
class OursStep:
    def __init__(self, torch, dev, seed, batch: int = 1, layers=None):
        import infengine_b200 as ie
        from infengine_b200.host import rope_tables
        self.ie, self.torch = ie, torch
        dt = torch.bfloat16
        self.M = batch
        self.layers, self.lm = layers if layers is not None else make_weights(torch, dev, dt, seed)
        g = torch.Generator(device=dev)
        g.manual_seed(seed + 1)
        self.x = torch.randn(batch, H, generator=g, device=dev, dtype=torch.float32).to(dt)
        self.q = torch.empty(NQ, batch, HD, device=dev, dtype=dt)
        self.attn_out = torch.empty(batch, H, device=dev, dtype=dt)
        self.h = torch.empty(batch, F, device=dev, dtype=dt)
        self.ffn_out = torch.empty(batch, H, device=dev, dtype=dt)
        self.kc = torch.zeros(L, NKV, CTX, HD, device=dev, dtype=dt)
        self.vc = torch.zeros(L, NKV, CTX, HD, device=dev, dtype=dt)
        cos, sin = rope_tables(CTX)
        self.cos = torch.from_numpy(cos).to(dev)
        self.sin = torch.from_numpy(sin).to(dev)
        self.ws = torch.zeros(ie.lm_head_workspace_bytes(batch), dtype=torch.uint8, device=dev)
        self.tok = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.launches_per_step = L * 4 + 1

    def __call__(self):
        ie = self.ie
        for l, w in enumerate(self.layers):
            ie.qkv(self.x, w["wq"], w["wk"], w["wv"], self.q, self.kc[l], self.vc[l], CTX * HD, POS, self.cos,
                   self.sin)
            # stand-in for the attention output: the Q rows ([heads, M, 128] read as [M, 4096])
            ie.gemm(self.q.view(self.M, H), w["wo"], self.attn_out)
            ie.ffn_gate_up(self.x, w["wg"], w["wu"], self.h)
            ie.gemm(self.h, w["wd"], self.ffn_out)
        ie.lm_head_argmax(self.x, self.lm, self.ws, idx_out=self.tok)

    def gate_up_only(self):
        for w in self.layers:
            self.ie.ffn_gate_up(self.x, w["wg"], w["wu"], self.h)

    def setup_prefill(self, S: int):
        """Buffers for the M=S prefill projection chain over the same weights."""
        torch, dev = self.torch, self.x.device
        g = torch.Generator(device=dev)
        g.manual_seed(7)
        self.S = S
        self.xp = torch.randn(S, H, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
        self.qp = torch.empty(NQ, S, HD, device=dev, dtype=torch.bfloat16)
        self.ap = torch.empty(S, H, device=dev, dtype=torch.bfloat16)
        self.hp = torch.empty(S, F, device=dev, dtype=torch.bfloat16)
        self.op = torch.empty(S, H, device=dev, dtype=torch.bfloat16)
        self.split_ws = self.ie.split_workspace(dev)  # the tail split of the *_ws entry points

    def release_prefill(self):
        self.xp = self.qp = self.ap = self.hp = self.op = self.split_ws = None

    def prefill(self, workspace="split"):
        """32 x [fused QKV+RoPE, O, gate/up+SwiGLU, down] at M = S tokens
        (positions 0..S-1), with the tail split (the engine's prefill path)
        or, workspace=None, whole tiles only."""
        ie, S = self.ie, self.S
        ws = self.split_ws if workspace == "split" else None
        for l, w in enumerate(self.layers):
            ie.qkv(self.xp, w["wq"], w["wk"], w["wv"], self.qp, self.kc[l], self.vc[l], CTX * HD, 0, self.cos,
                   self.sin, workspace=ws)
            ie.gemm(self.qp.view(S, H), w["wo"], self.ap, workspace=ws)  # stand-in for the attention output
            ie.ffn_gate_up(self.xp, w["wg"], w["wu"], self.hp, workspace=ws)
            ie.gemm(self.hp, w["wd"], self.op, workspace=ws)

    def prefill_flops(self):
        return 2.0 * self.S * L * LAYER_WEIGHT_ELEMS


# ------------------------------------------------------ our arm, N GPUs (TP)
class TPStep:
    """Tensor-parallel decode step (infengine_b200.tp): rank r holds 1/N of
    every projection; O and down partial sums are allreduced in fp32 over
    NCCL and the vocabulary-split lm_head is merged by a max over packed
    argmax keys. Every rank draws the full seeded weights layer by layer and
    keeps its shard, so the model is the one the single-GPU arm runs."""

    def __init__(self, torch, dev, seed, world, rank):
        import infengine_b200 as ie
        from infengine_b200.host import rope_tables
        from infengine_b200.tp import Comm, P2PExchange, ShardPlan, TPDecodeStep
        self.ie, self.torch = ie, torch
        self.plan = ShardPlan(world, rank)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)

        def w(*shape):
            return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).mul_(0.02).to(torch.bfloat16)

        layers = []
        for _ in range(L):
            full = {"wq": w(NQ * HD, H), "wk": w(NKV * HD, H), "wv": w(NKV * HD, H), "wo": w(H, H),
                    "wg": w(F, H), "wu": w(F, H), "wd": w(H, F)}
            layers.append(self.plan.shard_layer(full))
            del full
        lm = self.plan.shard_lm_head(w(V, H))
        torch.cuda.empty_cache()
        cos, sin = rope_tables(CTX)
        self.comm = Comm(world, rank)
        # O and down: one fused GEMV + NVLink exchange kernel each (default), or
        # fp32 partial + NCCL allreduce + cast (IE_TP_EXCHANGE=nccl)
        self.mode = os.environ.get("IE_TP_EXCHANGE", "p2p")
        self.exchange = P2PExchange(world, rank) if self.mode == "p2p" else None
        self.inner = TPDecodeStep(self.plan, self.comm, layers, lm, torch.from_numpy(cos).to(dev),
                                  torch.from_numpy(sin).to(dev), POS, exchange=self.exchange)
        g2 = torch.Generator(device=dev)
        g2.manual_seed(seed + 1)
        self.inner.x.copy_(torch.randn(1, H, generator=g2, device=dev, dtype=torch.float32).to(torch.bfloat16))
        self.x, self.tok = self.inner.x, self.inner.tok
        self.launches_per_step = self.inner.launches_per_step
        self.layers = layers
        self.h = self.inner.h

    def __call__(self):
        self.inner()

    def gate_up_only(self):
        for w in self.layers:
            self.ie.ffn_gate_up(self.x, w["wg"], w["wu"], self.h)

    def setup_prefill(self, S: int):
        """M=S prefill over the same shards (tensor-core kernels, NCCL allreduce)."""
        from infengine_b200.tp import TPDecodeStep
        inner = self.inner
        self.pre = TPDecodeStep(self.plan, self.comm, self.layers, self.inner.lm, inner.cos, inner.sin, 0,
                                batch=S, ctx=CTX, exchange=None, lm_rows=1)
        g = self.torch.Generator(device=inner.x.device)
        g.manual_seed(7)
        self.pre.x.copy_(self.torch.randn(S, H, generator=g, device=inner.x.device).to(self.torch.bfloat16))

    def prefill(self):
        self.pre()

    def prefill_flops(self):
        return self.pre.flops()

    def close(self):
        if self.exchange is not None:
            self.exchange.close()
        self.comm.close()


# ---------------------------------------------------------- reference arm
class RefStep:
    def __init__(self, torch, dev, seed):
        sys.path.insert(0, str(ROOT / "tests"))
        from ref_lib import p, ref
        from infengine_b200.host import rope_tables
        self.R, self.p, self.torch = ref(), p, torch
        dt = torch.float16
        self.layers, self.lm = make_weights(torch, dev, dt, seed)  # bf16 -> fp16 as model_weights.cu:61-78
        g = torch.Generator(device=dev)
        g.manual_seed(seed + 1)
        self.x = torch.randn(1, H, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16).to(dt)
        self.q = torch.empty(NQ, 1, HD, device=dev, dtype=dt)
        self.attn_out = torch.empty(1, H, device=dev, dtype=dt)
        self.ffn_out = torch.empty(1, H, device=dev, dtype=dt)
        self.kc = torch.zeros(L, NKV, CTX, HD, device=dev, dtype=dt)
        self.vc = torch.zeros(L, NKV, CTX, HD, device=dev, dtype=dt)
        cos, sin = rope_tables(CTX)
        self.cos = torch.from_numpy(cos).to(dev)
        self.sin = torch.from_numpy(sin).to(dev)
        self.ws = torch.empty(self.R.ref_ffn_workspace_size(1), dtype=torch.uint8, device=dev)
        self.logits = torch.empty(V, device=dev, dtype=dt)
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
        self.R.ref_set_stream(None)  # legacy default stream, as manager.cpp:58-59 leaves it
        self.launches_per_step = None  # cuBLAS chooses its own kernels

    def __call__(self):
        R, p = self.R, self.p
        for l, w in enumerate(self.layers):
            kdst, vdst = self.kc[l][:, POS], self.vc[l][:, POS]
            R.ref_qkv_proj(1, p(self.x), p(w["wq"]), p(w["wk"]), p(w["wv"]), p(self.q), p(kdst), p(vdst), NQ, NKV)
            R.ref_apply_rope(POS, NKV, 1, p(self.cos), p(self.sin), p(kdst), 1)
            R.ref_apply_rope(POS, NQ, 1, p(self.cos), p(self.sin), p(self.q), 0)
            R.ref_o_proj(1, p(self.q), p(w["wo"]), p(self.attn_out))
            R.ref_ffn(1, p(self.x), p(self.ffn_out), p(w["wu"]), p(w["wd"]), p(w["wg"]), p(self.ws))
        R.ref_lm_head(1, p(self.x), p(self.lm), p(self.logits))
        R.ref_sample_token_amax(p(self.logits), p(self.tok))


# ------------------------------------------------- per-config measurements
def per_config(torch, step, stream, hbm_peak, tf_peak):
    """BASELINE configs 1-4 one by one on the already-resident model weights
    (each timed over all 32 layers' copies, or 4 lm_head launches, so the
    weights stream from HBM, not L2): GB/s for the HBM-bound decode shapes,
    TFLOP/s for the prefill GEMMs."""
    import infengine_b200 as ie
    dev, bf = step.x.device, torch.bfloat16
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn, reps=5):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            fn()
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=stream):
            fn()
        with torch.cuda.stream(stream):
            g.replay()
            ev0.record(stream)
            for _ in range(reps):
                g.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
        t = ev0.elapsed_time(ev1) / 1e3 / reps
        g.reset()
        return t

    out = {}
    Ls = step.layers
    # config 1: y[1,4096] = x . W[4096,4096]^T (the O weights of the 32 layers)
    x1, y1 = step.x[:1], torch.empty(1, H, device=dev, dtype=bf)
    t = timed(lambda: [ie.gemm(x1, w["wo"], y1) for w in Ls]) / L
    b = 2 * (H * H + 2 * H)
    out["c1_gemv_4096x4096"] = {"us": round(t * 1e6, 2), "gbs": round(b / t / 1e9, 1),
                                "frac_hbm": round(b / t / 1e9 / hbm_peak, 4)}
    # config 2: FFN block at M in {1,4,8}
    c2 = {}
    for m in (1, 4, 8):
        xm = torch.randn(m, H, device=dev).to(bf)
        om = torch.empty(m, H, device=dev, dtype=bf)
        ws = torch.empty(ie.ffn_workspace_bytes(m, F), dtype=torch.uint8, device=dev)
        t = timed(lambda: [ie.ffn_fused(xm, w["wu"], w["wd"], w["wg"], om, ws) for w in Ls]) / L
        b = 2 * (3 * F * H + 2 * m * H)
        c2[f"m{m}"] = {"us": round(t * 1e6, 2), "gbs": round(b / t / 1e9, 1), "frac_hbm": round(b / t / 1e9 / hbm_peak, 4)}
    out["c2_ffn_decode"] = c2
    # config 4: lm_head + argmax at B in {1,8,64}
    c4 = {}
    for B in (1, 8, 64):
        xb = torch.randn(B, H, device=dev).to(bf)
        wsb = torch.zeros(ie.lm_head_workspace_bytes(B), dtype=torch.uint8, device=dev)
        ib = torch.zeros(B, dtype=torch.int32, device=dev)
        t = timed(lambda: [ie.lm_head_argmax(xb, step.lm, wsb, idx_out=ib) for _ in range(4)]) / 4
        b = 2 * (V * H + B * H)
        c4[f"b{B}"] = {"us": round(t * 1e6, 2), "gbs": round(b / t / 1e9, 1), "frac_hbm": round(b / t / 1e9 / hbm_peak, 4),
                       "tflops": round(2 * B * V * H / t / 1e12, 2)}
    out["c4_lm_head_argmax"] = c4
    # config 3: each prefill projection at M=2048 over the 32 layers, with
    # the tail split (the engine's path) and with whole tiles only
    S = step.S
    c3 = {}

    def c3_cases(ws):
        return (
            ("qkv_6144x4096", lambda: [ie.qkv(step.xp, w["wq"], w["wk"], w["wv"], step.qp, step.kc[l], step.vc[l],
                                              CTX * HD, 0, step.cos, step.sin, workspace=ws) for l, w in enumerate(Ls)],
             2 * S * 6144 * H),
            ("o_4096x4096", lambda: [ie.gemm(step.qp.view(S, H), w["wo"], step.ap, workspace=ws) for w in Ls],
             2 * S * H * H),
            ("gate_up_2x14336x4096", lambda: [ie.ffn_gate_up(step.xp, w["wg"], w["wu"], step.hp, workspace=ws)
                                              for w in Ls], 2 * S * 2 * F * H),
            ("down_4096x14336", lambda: [ie.gemm(step.hp, w["wd"], step.op, workspace=ws) for w in Ls], 2 * S * H * F),
        )
    for (name, fn, flops), (_, fn_whole, _) in zip(c3_cases(step.split_ws), c3_cases(None)):
        t = timed(fn, reps=2) / L
        tw = timed(fn_whole, reps=2) / L
        c3[name] = {"us": round(t * 1e6, 1), "tflops": round(flops / t / 1e12, 1),
                    "frac_burst": round(flops / t / 1e12 / tf_peak, 4), "whole_tiles_us": round(tw * 1e6, 1)}
    out["c3_prefill_m2048"] = c3
    return out


# -------------------------------------------------------------- CPU baseline
def cpu_baseline(seed: int):
    """The CPU golden of the same step (oracle/ie_oracle.py restatement of
    the reference generator's fp32 math) on the host cores, on a bounded
    sample: one decoder layer's projections and the lm_head, each timed
    (best of 3) and scaled to a 32-layer token."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import ie_oracle as oracle
    cores = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(seed)

    def w(*shape):
        return oracle.round_dt(rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02), "bf16")

    x = oracle.round_dt(rng.standard_normal((1, H), dtype=np.float32), "bf16")
    layer = {"wq": w(NQ * HD, H), "wk": w(NKV * HD, H), "wv": w(NKV * HD, H), "wo": w(H, H), "wg": w(F, H),
             "wu": w(F, H), "wd": w(H, F)}
    cos, sin = oracle.rope_tables(CTX)

    def one_layer():
        q, k, v = oracle.qkv_cpu(x, layer["wq"], layer["wk"], layer["wv"], "bf16", POS, cos, sin)
        oracle.gemm_cpu(q.transpose(1, 0, 2).reshape(1, H), layer["wo"], "bf16")
        oracle.ffn_cpu(x, layer["wg"], layer["wu"], layer["wd"], "bf16")

    def best(fn, n=3):
        ts = []
        for _ in range(n):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return min(ts)

    t_layer = best(one_layer)

    # the same golden per BASELINE config 1-4, each shape timed on its own
    # (best of 2): C1 the 4096x4096 GEMV, C2 the FFN block at M = 1/4/8, C3
    # the four prefill projections at M = 2048 (QKV with RoPE), C4 lm_head +
    # the reference's argmax at B = 1/8/64
    def xs(m):
        return oracle.round_dt(rng.standard_normal((m, H), dtype=np.float32), "bf16")

    def entry(t, nbytes=None, flops=None):
        e = {"ms": round(t * 1e3, 2)}
        if nbytes:
            e["gbs"] = round(nbytes / t / 1e9, 2)
        if flops:
            e["gflops"] = round(flops / t / 1e9, 1)
        return e

    configs = {"c1_gemv_4096x4096": entry(best(lambda: oracle.gemm_cpu(x, layer["wo"], "bf16"), 2), 2 * H * H)}
    c2 = {}
    for m in (1, 4, 8):
        xm = xs(m)
        c2[f"m{m}"] = entry(best(lambda: oracle.ffn_cpu(xm, layer["wg"], layer["wu"], layer["wd"], "bf16"), 2),
                            2 * 3 * F * H)
    configs["c2_ffn_decode"] = c2
    # C3 on a bounded sample: rows 0..255 of the 2048-token prefill, the
    # time scaled by 2048 / 256 (the golden is row-independent)
    rows, scale = 256, 2048 // 256
    xp = xs(rows)
    hp = oracle.round_dt(rng.standard_normal((rows, F), dtype=np.float32), "bf16")

    def c3(fn, flops):
        return entry(best(fn, 2) * scale, flops=flops)
    configs["c3_prefill_m2048"] = {
        "qkv_6144x4096": c3(lambda: oracle.qkv_cpu(xp, layer["wq"], layer["wk"], layer["wv"], "bf16", 0, cos, sin),
                            2 * 2048 * 6144 * H),
        "o_4096x4096": c3(lambda: oracle.gemm_cpu(xp, layer["wo"], "bf16"), 2 * 2048 * H * H),
        "gate_up_2x14336x4096": c3(lambda: oracle.swiglu(oracle.gemm_cpu(xp, layer["wg"], "bf16"),
                                                         oracle.gemm_cpu(xp, layer["wu"], "bf16"), "bf16"),
                                   2 * 2048 * 2 * F * H),
        "down_4096x14336": c3(lambda: oracle.gemm_cpu(hp, layer["wd"], "bf16"), 2 * 2048 * H * F),
        "sample": f"rows 0-{rows - 1} of 2048, time x {scale}",
    }
    del layer, xp, hp
    lm = w(V, H)
    t_lm = best(lambda: oracle.lm_head_argmax_cpu(x, lm, "bf16"))
    c4 = {"b1": entry(t_lm, 2 * V * H)}
    for B in (8, 64):
        xb = xs(B)
        c4[f"b{B}"] = entry(best(lambda: oracle.lm_head_argmax_cpu(xb, lm, "bf16"), 2), 2 * V * H)
    configs["c4_lm_head_argmax"] = c4
    t_tok = L * t_layer + t_lm
    return {"value": round(1.0 / t_tok, 4), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"1 decoder layer (QKV+RoPE, O, FFN) best of 3 = {t_layer * 1e3:.1f} ms and lm_head+argmax "
                      f"best of 3 = {t_lm * 1e3:.1f} ms, fp32 numpy BLAS on bf16-valued weights, scaled to "
                      f"{L} layers + lm_head per token; `configs` times the same golden at BASELINE configs 1-4 "
                      f"shape by shape (best of 2; C3 on 256 of the 2048 rows, scaled; gbs counts bf16 weight bytes)",
            "configs": configs}


# --------------------------------------------------------- single-kernel cases
def single_case(torch, name: str, steps: int, seed: int):
    """A few launches of one hot-path kernel on one layer's weights (a small
    workload for ncu captures; inputs still exceed the L2)."""
    import infengine_b200 as ie
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    bf = torch.bfloat16

    def w(*shape):
        return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).mul_(0.02).to(bf)

    x = torch.randn(1, H, generator=g, device=dev, dtype=torch.float32).to(bf)
    if name == "gate_up":
        wg, wu, h = w(F, H), w(F, H), torch.empty(1, F, device=dev, dtype=bf)
        fn = lambda: ie.ffn_gate_up(x, wg, wu, h)
    elif name == "down":
        wd, hh, out = w(H, F), torch.randn(1, F, device=dev).to(bf), torch.empty(1, H, device=dev, dtype=bf)
        fn = lambda: ie.gemm(hh, wd, out)
    elif name == "o":
        wo, out = w(H, H), torch.empty(1, H, device=dev, dtype=bf)
        fn = lambda: ie.gemm(x, wo, out)
    elif name == "qkv":
        from infengine_b200.host import rope_tables
        wq, wk, wv = w(NQ * HD, H), w(NKV * HD, H), w(NKV * HD, H)
        q = torch.empty(NQ, 1, HD, device=dev, dtype=bf)
        kc, vc = torch.zeros(NKV, CTX, HD, device=dev, dtype=bf), torch.zeros(NKV, CTX, HD, device=dev, dtype=bf)
        cos, sin = (torch.from_numpy(t).to(dev) for t in rope_tables(CTX))
        fn = lambda: ie.qkv(x, wq, wk, wv, q, kc, vc, CTX * HD, POS, cos, sin)
    elif name == "lm_head":
        lm = w(V, H)
        ws = torch.zeros(ie.lm_head_workspace_bytes(1), dtype=torch.uint8, device=dev)
        tok = torch.zeros(1, dtype=torch.int32, device=dev)
        fn = lambda: ie.lm_head_argmax(x, lm, ws, idx_out=tok)
    elif name in ("engine_decode", "engine_small", "engine_decode_bs8"):
        # the whole model through the engine: a 2048-token prefill (of each
        # of 8 sequences for engine_decode_bs8), then `steps` decode steps
        # (graph replays); engine_small keeps 2 of the 32 layers so that a
        # full ncu capture holds a few GB, not 17
        n_layers = 2 if name == "engine_small" else L
        batch = 8 if name == "engine_decode_bs8" else 1
        layers = [{"wq": w(NQ * HD, H), "wk": w(NKV * HD, H), "wv": w(NKV * HD, H), "wo": w(H, H),
                   "wg": w(F, H), "wu": w(F, H), "wd": w(H, F)} for _ in range(n_layers)]
        weights = full_model_weights(torch, dev, seed, layers, w(V, H))
        from infengine_b200.engine import LlamaEngine
        dims = dict(n_layers=n_layers, hidden=H, n_q_heads=NQ, n_kv_heads=NKV, head_dim=HD, ffn_dim=F, vocab=V)
        eng = LlamaEngine(weights, dims, max_batch=batch, max_ctx=PROMPT + steps + 16, max_prefill=PROMPT)
        for b, pr in enumerate(prompts(seed, batch)):
            eng.prefill(b, pr)
        eng.decode(steps)
        eng.close()
        torch.cuda.synchronize()
        print(json.dumps({"case": name, "layers": n_layers, "batch": batch, "decode_steps": steps}))
        return
    elif name in ("decode_attention_bs1", "decode_attention_bs8"):
        # the decode attention core of one step at position 2047 (after the
        # 2048-token prompt): B sequences x 8 KV heads, 32 layers' caches so
        # that the keys and values stream from HBM as in the engine (67 MB a
        # layer at B = 8); timed as one graph of 32 launches
        B = 8 if name.endswith("bs8") else 1
        rows = PROMPT + 64
        q = torch.randn(NQ, B, HD, generator=g, device=dev, dtype=torch.float32).to(bf)
        kcs = [torch.randn(B, NKV, rows, HD, generator=g, device=dev, dtype=torch.float32).to(bf) for _ in range(L)]
        vcs = [torch.randn(B, NKV, rows, HD, generator=g, device=dev, dtype=torch.float32).to(bf) for _ in range(L)]
        pos = torch.full((B,), PROMPT - 1, dtype=torch.int32, device=dev)
        out = torch.empty(B, NQ * HD, device=dev, dtype=bf)
        st = torch.cuda.Stream()
        run = lambda: [ie.attention_decode(q, kcs[l], vcs[l], out, positions=pos, stream=st) for l in range(L)]
        with torch.cuda.stream(st):
            run()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=st):
            run()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            gr.replay()
            e0.record(st)
            for _ in range(steps):
                gr.replay()
            e1.record(st)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (steps * L)
        kv = 2 * B * NKV * PROMPT * HD * 2
        print(json.dumps({"case": name, "launches": (steps + 1) * L, "us_per_launch": round(us, 2),
                          "kv_bytes": kv, "gbs": round(kv / us / 1e3, 1)}))
        return
    elif name == "prefill_attention":
        # the attention core of a 2048-token prefill: causal 2048 x 2048, 32
        # query / 8 KV heads (K/V of one layer: 8 MB, L2-resident like in the
        # engine, where the QKV projection has just written them)
        S = PROMPT
        q = torch.randn(NQ, S, HD, generator=g, device=dev, dtype=torch.float32).to(bf)
        kc = torch.randn(NKV, S, HD, generator=g, device=dev, dtype=torch.float32).to(bf)
        vc = torch.randn(NKV, S, HD, generator=g, device=dev, dtype=torch.float32).to(bf)
        out = torch.empty(S, NQ * HD, device=dev, dtype=bf)
        fn = lambda: ie.attention(q, kc, vc, out, 0, n_kv_heads=NKV)
        flops = 4.0 * NQ * HD * S * (S + 1) / 2
    elif name.startswith("prefill_"):
        S = 2048
        xs = torch.randn(S, H, generator=g, device=dev, dtype=torch.float32).to(bf)
        kind = name[len("prefill_"):]
        if kind == "o":
            wo, out = w(H, H), torch.empty(S, H, device=dev, dtype=bf)
            fn = lambda: ie.gemm(xs, wo, out)
        elif kind == "down":
            wd, hs, out = w(H, F), torch.randn(S, F, device=dev).to(bf), torch.empty(S, H, device=dev, dtype=bf)
            fn = lambda: ie.gemm(hs, wd, out)
        elif kind == "gate_up":
            wg, wu, hs = w(F, H), w(F, H), torch.empty(S, F, device=dev, dtype=bf)
            fn = lambda: ie.ffn_gate_up(xs, wg, wu, hs)
        elif kind == "qkv":
            from infengine_b200.host import rope_tables
            wq, wk, wv = w(NQ * HD, H), w(NKV * HD, H), w(NKV * HD, H)
            q = torch.empty(NQ, S, HD, device=dev, dtype=bf)
            kc, vc = torch.zeros(NKV, CTX, HD, device=dev, dtype=bf), torch.zeros(NKV, CTX, HD, device=dev, dtype=bf)
            cos, sin = (torch.from_numpy(t).to(dev) for t in rope_tables(CTX))
            fn = lambda: ie.qkv(xs, wq, wk, wv, q, kc, vc, CTX * HD, 0, cos, sin)
        else:
            raise SystemExit(f"unknown case {name}")
    else:
        raise SystemExit(f"unknown case {name}")
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / max(steps, 1)
    res = {"case": name, "launches": steps + 1, "us_per_launch": round(us, 2)}
    if name == "prefill_attention":
        res["tflops"] = round(flops / us / 1e6, 1)
    print(json.dumps(res))


# ------------------------------------------------ full model through the engine
def full_model_weights(torch, dev, seed, layers, lm):
    """Engine weights of the random-init model: the projection weights of
    make_weights (or their tensor-parallel shards), a seeded N(0,0.02)
    embedding table, RMSNorm weights of 1 (the HF initialisation) and the
    Llama-3.1 RoPE tables."""
    from infengine_b200.host import rope_tables
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 2)
    emb = torch.randn(V, H, generator=g, device=dev, dtype=torch.float32).mul_(0.02).to(torch.bfloat16)
    ones = torch.ones(H, dtype=torch.bfloat16, device=dev)
    cos, sin = (torch.from_numpy(t).to(dev) for t in rope_tables(CTX))
    return dict(embedding=emb, final_norm=ones, lm_head=lm, rope_cos=cos, rope_sin=sin,
                layers=[dict(attn_norm=ones, wq=w["wq"], wk=w["wk"], wv=w["wv"], wo=w["wo"], ffn_norm=ones,
                             w_gate=w["wg"], w_up=w["wu"], w_down=w["wd"]) for w in layers])


def make_engine(weights, world, rank, batch, ctx, comm=None, exchange=None, plan=None):
    from infengine_b200.engine import LlamaEngine
    dims = dict(n_layers=L, hidden=H, n_q_heads=NQ // world, n_kv_heads=NKV // world, head_dim=HD,
                ffn_dim=F // world, vocab=V, rms_eps=1e-5)
    tp = None
    if world > 1:
        vs = plan.vocab_slice()
        tp = dict(world=world, rank=rank, comm=comm, exchange=exchange, lm_rows=vs.stop - vs.start,
                  lm_offset=vs.start)
    return LlamaEngine(weights, dims, dtype="bf16", max_batch=batch, max_ctx=ctx, max_prefill=PROMPT, tp=tp)


def prompts(seed, n):
    return np.random.default_rng(seed + 3).integers(0, V, size=(n, PROMPT)).astype(np.int32)


def reference_decode(seed, steps, warmup):
    """The reference's own decode loop (prefill.cu / decode.cu with its
    kernels, built from its sources by oracle/Makefile) on random-init fp16
    weights: tok/s of `steps` decode steps after a PROMPT-token prompt."""
    import ctypes
    R = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libref_model_ref.so"))
    R.model_init.argtypes = [ctypes.c_ulonglong]
    dbl = ctypes.POINTER(ctypes.c_double)
    R.model_generate_timed.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p, dbl, dbl]
    assert R.model_init(seed) == 0
    prompt = prompts(seed, 1)[0]
    pm, dm = ctypes.c_double(), ctypes.c_double()
    out = np.zeros(steps + 1, np.int32)
    vp = ctypes.c_void_p
    assert R.model_generate_timed(prompt.ctypes.data_as(vp), PROMPT, warmup + 1, None, out.ctypes.data_as(vp), None,
                                  ctypes.byref(pm), ctypes.byref(dm)) == 0
    assert R.model_generate_timed(prompt.ctypes.data_as(vp), PROMPT, steps + 1, None, out.ctypes.data_as(vp), None,
                                  ctypes.byref(pm), ctypes.byref(dm)) == 0
    R.model_free()
    return {"decode_ms": dm.value, "prefill_ms": pm.value, "tokens": out}


# ------------------------------------- the reference's kernels, per config
def reference_configs(torch, dev, seed):
    """Baseline leg, not part of our path: the reference's own hot-path code
    (kernels/ffn.cu, attn.cu, lm_head.cu, swiglu.cu, rope.cu, sampling.cu with
    cuBLAS 12.9, built unchanged for sm_100a by oracle/Makefile) at BASELINE
    configs 1-4, in fp16 (its only dtype), launched eagerly on the legacy
    default stream as the reference launches them, timed with CUDA events on
    that stream. Weights: the same seeded random-init model (bf16 values
    stored as fp16), each kernel timed over the 32 layers' copies (or 4 lm_head
    launches), so weights stream from HBM. Each prefill entry gives the cuBLAS
    calls alone (`gemm_us`) and with the elementwise kernels the reference
    runs right after them (`path_us`: RoPE after Q/K/V, SwiGLU after gate and
    up), which our fused kernels fold into their epilogues."""
    sys.path.insert(0, str(ROOT / "tests"))
    from ref_lib import p, ref
    from infengine_b200.host import rope_tables
    R = ref()
    R.ref_set_stream(None)
    f16 = torch.float16
    layers, lm = make_weights(torch, dev, f16, seed)
    ds = torch.cuda.default_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed_eager(fn, reps):
        fn()
        torch.cuda.synchronize()
        e0.record(ds)
        for _ in range(reps):
            fn()
        e1.record(ds)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / reps

    out = {}
    x1, y1 = torch.randn(1, H, device=dev).to(f16), torch.empty(1, H, device=dev, dtype=f16)
    t = timed_eager(lambda: [R.ref_multiply_by_weight(1, H, H, p(x1), p(w["wo"]), p(y1)) for w in layers], 5) / L
    b = 2 * (H * H + 2 * H)
    out["c1_gemv_4096x4096"] = {"us": round(t * 1e6, 2), "gbs": round(b / t / 1e9, 1), "call": "multiply_by_weight"}
    c2 = {}
    for m in (1, 4, 8):
        xm, om = torch.randn(m, H, device=dev).to(f16), torch.empty(m, H, device=dev, dtype=f16)
        ws = torch.empty(R.ref_ffn_workspace_size(m), dtype=torch.uint8, device=dev)
        t = timed_eager(lambda: [R.ref_ffn(m, p(xm), p(om), p(w["wu"]), p(w["wd"]), p(w["wg"]), p(ws))
                                 for w in layers], 5) / L
        b = 2 * (3 * F * H + 2 * m * H)
        c2[f"m{m}"] = {"us": round(t * 1e6, 2), "gbs": round(b / t / 1e9, 1)}
    out["c2_ffn_decode"] = dict(c2, call="ffn (3 cuBLAS GEMMs + swiglu)")
    c4 = {}
    for B in (1, 8, 64):
        xb = torch.randn(B, H, device=dev).to(f16)
        logits = torch.empty(B, V, device=dev, dtype=f16)
        tok = torch.zeros(B, dtype=torch.int32, device=dev)
        if B == 1:  # lm_head (its row seq_len - 1) + sample_token_amax, as decode.cu:41-42
            fn = lambda: [(R.ref_lm_head(1, p(xb), p(lm), p(logits)), R.ref_sample_token_amax(p(logits), p(tok)))
                          for _ in range(4)]
        else:  # no batched lm_head in the reference: one GEMM over B rows + amax per row
            fn = lambda: [(R.ref_multiply_by_weight(B, H, V, p(xb), p(lm), p(logits)),
                           [R.ref_sample_token_amax(ctypes_ptr(logits, r * V), ctypes_ptr(tok, r)) for r in range(B)])
                          for _ in range(4)]
        t = timed_eager(fn, 2) / 4
        b = 2 * (V * H + B * H)
        c4[f"b{B}"] = {"us": round(t * 1e6, 2), "gbs": round(b / t / 1e9, 1)}
    out["c4_lm_head_argmax"] = dict(c4, call="lm_head + sample_token_amax (B=1); multiply_by_weight + B x "
                                             "sample_token_amax (B>1)")
    S = 2048
    xs = torch.randn(S, H, device=dev).to(f16)
    hs = torch.randn(S, F, device=dev).to(f16)
    q = torch.empty(NQ, S, HD, device=dev, dtype=f16)
    kc, vc = (torch.zeros(NKV, CTX, HD, device=dev, dtype=f16) for _ in range(2))
    G, U = torch.empty(S, F, device=dev, dtype=f16), torch.empty(S, F, device=dev, dtype=f16)
    o = torch.empty(S, H, device=dev, dtype=f16)
    cos, sin = (torch.from_numpy(a).to(dev) for a in rope_tables(CTX))

    def qkv(w, rope):
        R.ref_qkv_proj(S, p(xs), p(w["wq"]), p(w["wk"]), p(w["wv"]), p(q), p(kc), p(vc), NQ, NKV)
        if rope:  # attn.cu:351-352
            R.ref_apply_rope(0, NKV, S, p(cos), p(sin), p(kc), 1)
            R.ref_apply_rope(0, NQ, S, p(cos), p(sin), p(q), 0)

    def gate_up(w, act):
        R.ref_multiply_by_weight(S, H, F, p(xs), p(w["wg"]), p(G))
        R.ref_multiply_by_weight(S, H, F, p(xs), p(w["wu"]), p(U))
        if act:  # ffn.cu:57
            R.ref_swiglu(S, p(G), p(U), p(G))

    c3 = {}
    for name, gemm, path, flops in (
        ("qkv_6144x4096", lambda: [qkv(w, False) for w in layers], lambda: [qkv(w, True) for w in layers],
         2 * S * 6144 * H),
        ("o_4096x4096", lambda: [R.ref_o_proj(S, p(xs), p(w["wo"]), p(o)) for w in layers], None, 2 * S * H * H),
        ("gate_up_2x14336x4096", lambda: [gate_up(w, False) for w in layers], lambda: [gate_up(w, True) for w in layers],
         2 * S * 2 * F * H),
        ("down_4096x14336", lambda: [R.ref_multiply_by_weight(S, F, H, p(hs), p(w["wd"]), p(o)) for w in layers], None,
         2 * S * H * F),
    ):
        tg = timed_eager(gemm, 2) / L
        tp = timed_eager(path, 2) / L if path is not None else tg
        c3[name] = {"gemm_us": round(tg * 1e6, 1), "gemm_tflops": round(flops / tg / 1e12, 1),
                    "path_us": round(tp * 1e6, 1), "path_tflops": round(flops / tp / 1e12, 1)}
    out["c3_prefill_m2048"] = c3
    out["timing"] = ("eager on the legacy default stream (the reference's launch mode), CUDA events; fp16; weights "
                     "rotated over the 32 layers' copies")
    del layers, lm
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def ctypes_ptr(t, offset_elems):
    import ctypes
    return ctypes.c_void_p(t.data_ptr() + offset_elems * t.element_size())


def versus_reference(ours, ref):
    """Speed-up of our per-config times over the reference's (same box)."""
    def r(a, b):
        return round(b / a, 3) if a and b else None
    vs = {"c1_gemv_4096x4096": r(ours["c1_gemv_4096x4096"]["us"], ref["c1_gemv_4096x4096"]["us"])}
    vs["c2_ffn_decode"] = {k: r(ours["c2_ffn_decode"][k]["us"], ref["c2_ffn_decode"][k]["us"]) for k in ("m1", "m4", "m8")}
    vs["c4_lm_head_argmax"] = {k: r(ours["c4_lm_head_argmax"][k]["us"], ref["c4_lm_head_argmax"][k]["us"])
                               for k in ("b1", "b8", "b64")}
    vs["c3_prefill_m2048"] = {
        k: {"vs_path": r(ours["c3_prefill_m2048"][k]["us"], ref["c3_prefill_m2048"][k]["path_us"]),
            "vs_gemm_only": r(ours["c3_prefill_m2048"][k]["us"], ref["c3_prefill_m2048"][k]["gemm_us"])}
        for k in ours["c3_prefill_m2048"]}
    return vs


# ----------------------------------------------------------- parity checker
def fp16_spacing(x: float) -> float:
    """Spacing of fp16 numbers at |x| (one unit in the last place)."""
    import math
    a = max(abs(x), 2.0 ** -14)
    return 2.0 ** (math.floor(math.log2(a)) - 10)


def parity_leg(torch, dev, seed, n_steps, batch=8):
    """Checker leg (untimed): greedy ids of BASELINE config 5 at its full
    length against the reference's own decode loop.

    The reference (prefill.cu / decode.cu with its kernels and cuBLAS, built
    unchanged by oracle/Makefile; manager.cpp:79-86's loop) runs on its
    random-init fp16 model, once per prompt: PROMPT tokens, then n_steps
    greedy ids, with its top-2 logit margin and top logit at every step. Our
    engine runs in fp16 on the same weights:
      * bs1 - teacher-forced (each step fed the reference's previous id, so
        every step is scored on the same context) and free-running;
      * bs8 - `batch` prompts decoded together, each against its own bs1
        reference run;
      * verify M=5 - one verify pass over the reference's ids 0..4, compared
        with its ids 1..5.
    Every disagreement is listed with the reference's margin in fp16 units of
    its top logit."""
    import ctypes
    from infengine_b200.engine import LlamaEngine
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    R = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libref_model_ref.so"))
    R.model_init.argtypes = [ctypes.c_ulonglong]
    R.model_generate_ex.argtypes = [vp, i32, i32, vp, vp, vp, vp, vp, vp]
    R.model_weight_ptrs.argtypes = [vp, i32]
    t_start = time.perf_counter()
    assert R.model_init(seed) == 0
    ps = prompts(seed, batch)  # the prompts of the timed runs (bs1 uses the first)
    ref_ids, ref_m, ref_top = [], [], []
    for b in range(batch):
        ids, m, top = np.zeros(n_steps, np.int32), np.zeros(n_steps, np.float32), np.zeros(n_steps, np.float32)
        assert R.model_generate_ex(ps[b].ctypes.data_as(vp), PROMPT, n_steps, None, ids.ctypes.data_as(vp),
                                   m.ctypes.data_as(vp), top.ctypes.data_as(vp), None, None) == 0
        ref_ids.append(ids)
        ref_m.append(m)
        ref_top.append(top)
    n = 5 + 9 * L
    ptrs = (ctypes.c_void_p * n)()
    assert R.model_weight_ptrs(ptrs, n) == n
    v = [int(x) for x in ptrs]
    names = ["attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "w_gate", "w_up", "w_down"]
    weights = dict(embedding=v[0], final_norm=v[1], lm_head=v[2], rope_cos=v[3], rope_sin=v[4],
                   layers=[dict(zip(names, v[5 + 9 * l: 14 + 9 * l])) for l in range(L)])
    dims = dict(n_layers=L, hidden=H, n_q_heads=NQ, n_kv_heads=NKV, head_dim=HD, ffn_dim=F, vocab=V, rms_eps=1e-5)

    def misses(seq, got):
        bad = np.nonzero(got != ref_ids[seq])[0]
        return [{"seq": seq, "step": int(i), "ref_margin": float(ref_m[seq][i]), "ref_top": float(ref_top[seq][i]),
                 "margin_in_ulps": round(float(ref_m[seq][i]) / fp16_spacing(float(ref_top[seq][i])), 2)}
                for i in bad]

    def first_difference(a, b):
        d = np.nonzero(a != b)[0]
        return int(d[0]) if len(d) else len(a)

    out = {"checker": "the reference's decode loop (prefill.cu, decode.cu, kernels/*.cu + cuBLAS 12.9, compiled "
                      "unchanged for sm_100a) on its random-init fp16 model; ours: the decode engine in fp16 on the "
                      "same weights", "prompt": PROMPT, "steps": n_steps}
    try:
        eng = LlamaEngine(weights, dims, dtype="f16", max_batch=1, max_ctx=PROMPT + n_steps + 8, max_prefill=PROMPT)
        r0 = ref_ids[0]
        first = eng.prefill(0, ps[0])
        tf = [first]
        for i in range(n_steps - 1):
            eng.set_position(0, PROMPT + i, int(r0[i]))
            tf.append(int(eng.decode(1)[0, 0]))
        tf = np.array(tf, np.int32)
        eng.set_position(0, PROMPT, first)
        free = np.concatenate([[first], eng.decode(n_steps - 1)[:, 0]]).astype(np.int32)
        eng.set_position(0, PROMPT, int(r0[0]))
        ver = eng.verify(0, r0[:5])
        eng.close()
        m1 = misses(0, tf)
        out["bs1"] = {"teacher_forced_equal": int((tf == r0).sum()), "of": n_steps,
                      "free_running_identical_steps": first_difference(free, r0), "misses": m1}
        out["verify_m5"] = {"equal": int((ver == r0[1:6]).sum()), "of": 5, "ids": ver.tolist(),
                            "reference": r0[1:6].tolist()}
        eng = LlamaEngine(weights, dims, dtype="f16", max_batch=batch, max_ctx=PROMPT + n_steps + 8,
                          max_prefill=PROMPT)
        firsts = [eng.prefill(b, ps[b]) for b in range(batch)]
        tf8 = np.zeros((n_steps, batch), np.int32)
        tf8[0] = firsts
        for i in range(n_steps - 1):
            for b in range(batch):
                eng.set_position(b, PROMPT + i, int(ref_ids[b][i]))
            tf8[i + 1] = eng.decode(1)[0]
        for b in range(batch):
            eng.set_position(b, PROMPT, firsts[b])
        free8 = np.concatenate([np.array(firsts, np.int32)[None], eng.decode(n_steps - 1)]).astype(np.int32)
        eng.close()
        m8 = [x for b in range(batch) for x in misses(b, tf8[:, b])]
        out["bs8"] = {"teacher_forced_equal": int(sum((tf8[:, b] == ref_ids[b]).sum() for b in range(batch))),
                      "of": n_steps * batch,
                      "free_running_identical_steps": [first_difference(free8[:, b], ref_ids[b]) for b in range(batch)],
                      "bs8_row0_equals_bs1_free_run": bool(np.array_equal(free8[:, 0], free)),
                      "misses": m8}
        allm = m1 + m8
        out["max_miss_margin_ulps"] = max((x["margin_in_ulps"] for x in allm), default=None)
    finally:
        R.model_free()
    out["reference_vs_itself"] = reference_noise_floor(seed, ps[0], ref_ids[0], ref_m[0], ref_top[0])
    out["seconds"] = round(time.perf_counter() - t_start, 1)
    return out


def reference_noise_floor(seed, prompt, ids, margin, top):
    """The reference's decode loop once more, in a second process whose
    cuBLAS runs with CUBLAS_WORKSPACE_CONFIG=:0:0 (so it chooses other
    kernels and split-K reductions), teacher-forced on the first run's ids
    (oracle/ref_replay.py): how many greedy ids the reference itself changes
    when only its fp32 summation order changes."""
    with tempfile.TemporaryDirectory() as td:
        pp, fp, op = (os.path.join(td, n) for n in ("prompt.npy", "forced.npy", "out.npz"))
        np.save(pp, prompt)
        np.save(fp, ids)
        env = dict(os.environ, CUBLAS_WORKSPACE_CONFIG=":0:0")
        r = subprocess.run([sys.executable, str(ROOT / "oracle" / "ref_replay.py"), str(seed), pp, fp, op], env=env,
                           stdout=subprocess.DEVNULL, stderr=subprocess.PIPE, text=True)
        if r.returncode != 0:
            return {"error": r.stderr.strip().splitlines()[-1:] or ["replay failed"]}
        got = np.load(op)["ids"]
    bad = np.nonzero(got != ids)[0]
    return {"teacher_forced_equal": int(len(ids) - len(bad)), "of": int(len(ids)),
            "miss_margins_in_ulps": [round(float(margin[i]) / fp16_spacing(float(top[i])), 2) for i in bad],
            "how": "the reference's loop in a second process with CUBLAS_WORKSPACE_CONFIG=:0:0, fed the first "
                   "run's ids: the ids that change when only cuBLAS's kernel choice (summation order) changes"}


def tp_parity(torch, dist, dev, seed, rank, prompt, tp_eng, tp_ids, ctx):
    """Untimed, after the timed steps: rank 0 runs the single-GPU engine on
    the full model from the same seeded generator (the same prompt, as many
    greedy steps as the tensor-parallel run made) and broadcasts its ids.
    Reported: the tensor-parallel run's own ids against them (free-running),
    and a teacher-forced pass in which every rank's engine is fed the
    single-GPU ids step by step, so that each step is scored on the same
    context. The O and down partial sums meet in another order across ranks
    than inside one GPU, so an id can flip where two logits tie to within a
    rounding step."""
    n = len(tp_ids)
    ref = torch.zeros(n, dtype=torch.int32, device=dev)
    if rank == 0:
        layers, lm = make_weights(torch, dev, torch.bfloat16, seed)
        weights = full_model_weights(torch, dev, seed, layers, lm)
        eng = make_engine(weights, 1, 0, 1, ctx)
        eng.prefill(0, prompt[:256])  # the same warm-up the TP run made
        eng.set_position(0, 0, 0)
        first = eng.prefill(0, prompt)
        ids = np.concatenate([[first], eng.decode(n - 1)[:, 0]]).astype(np.int32)
        eng.close()
        del eng, weights, layers, lm
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        ref.copy_(torch.from_numpy(ids))
    dist.broadcast(ref, 0)
    ref = ref.cpu().numpy()
    tf = [int(tp_ids[0])]
    for i in range(n - 1):  # every rank, in lockstep (the step holds collectives)
        tp_eng.set_position(0, PROMPT + i, int(ref[i]))
        tf.append(int(tp_eng.decode(1)[0, 0]))
    tf = np.array(tf, np.int32)
    d = np.nonzero(ref != tp_ids)[0]
    return {"ids": n, "free_running_equal": int((ref == tp_ids).sum()), "identical": bool(len(d) == 0),
            "free_running_first_difference": int(d[0]) if len(d) else None,
            "teacher_forced_equal": int((tf == ref).sum()),
            "against": "single-GPU engine, same seeded bf16 model and prompt"}


# ------------------------------------------------------------------- main
def timed(torch, stream, fn, world, dev):
    """Device time (ms) of fn() on `stream`, max over ranks."""
    import torch.distributed as dist
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    fn()
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--parity-steps", type=int, default=256,
                    help="greedy steps of the parity checker leg (N=1; 0 skips it)")
    ap.add_argument("--no-reference-configs", action="store_true",
                    help="skip timing the reference's own kernels per BASELINE config")
    ap.add_argument("--case", default=None,
                    help="for profiling: one kernel (gate_up|down|o|qkv|lm_head|prefill_{qkv,o,gate_up,down}|"
                         "prefill_attention|decode_attention_bs1|decode_attention_bs8) "
                         "--steps times, or the engine (engine_decode: 32 layers, engine_small: 2 layers, "
                         "engine_decode_bs8: 32 layers, 8 sequences) with a 2048-token prefill per sequence and "
                         "--steps decode steps")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    import torch
    import torch.distributed as dist

    if args.case:
        single_case(torch, args.case, args.steps, args.seed)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # stdout carries only the JSON line: whatever the libraries print on file
    # descriptor 1 (NCCL's version banner, for one) goes to stderr instead
    global JSON_OUT
    sys.stdout.flush()
    JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.impl == "reference":
        if rank != 0:  # the reference runs on one GPU; other ranks have no work
            return
        world = 1
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    hbm_peak, tf_peak, tf_peak_sus, peak_src = load_peaks()
    if args.impl == "reference":
        run_reference(torch, dev, args)
        return
    run_ours(torch, dist, dev, args, world, rank, local, hbm_peak, tf_peak, tf_peak_sus, peak_src)


def base_result(args, world, value, ms_step, clk, e2e, dtype):
    return {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": dtype,
        "data": "synthetic: random-init Llama-3.1-8B weights N(0,0.02) (seeded), RMSNorm weights 1, "
                f"{PROMPT}-token prompt uniform over the vocabulary (seeded)",
        "config": {
            "workload": f"BASELINE config 5 at batch 1: greedy decode of random-init Llama-3.1-8B (32 layers, "
                        f"hidden 4096, 32/8 heads, FFN 14336, vocab 128256) right after a {PROMPT}-token prompt",
            "batch": 1, "prompt": PROMPT, "layers": L, "hidden": H, "ffn": F, "vocab": V,
            "weight_bytes_per_step": WEIGHT_BYTES,
            "l2": "inputs larger than L2 (15.01 GB of weights streamed per step)",
            "parallelism": f"tp{world}" if world > 1 else "single",
        },
        "e2e": e2e,
        "clocks": clk,
    }


def run_reference(torch, dev, args):
    clocks = ClockSampler(0)
    clocks.start()
    time.sleep(0.3)
    r = reference_decode(args.seed, args.steps, args.warmup)
    clk = clocks.stop()
    ms_step = r["decode_ms"] / args.steps
    tok_s = args.steps / (r["decode_ms"] / 1e3)
    e2e = {"value": round(tok_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4}
    result = base_result(args, 1, tok_s, ms_step, clk, e2e, "f16")
    result["impl"] = "reference"
    result["config"]["launch"] = "the reference's decode_step loop: eager, legacy default stream, blocking D2H per token"
    result["reference_build"] = ("Aryan470/infengine prefill.cu, decode.cu and kernels/*.cu compiled unchanged for "
                                 "sm_100a (oracle/Makefile), cuBLAS 12.9; fp16 (its only dtype)")
    result["prefill"] = {"prompt": PROMPT, "ms": round(r["prefill_ms"], 3),
                         "tok_per_s": round(PROMPT / (r["prefill_ms"] / 1e3), 1)}
    result["timing"] = "host wall clock around the reference's decode_step calls (each ends in a blocking copy)"
    # the reference's weight-matmul path alone (its cuBLAS projections, RoPE,
    # SwiGLU, lm_head and argmax kernels), eager on the legacy default stream
    step = RefStep(torch, dev, args.seed)
    ds = torch.cuda.default_stream(dev)
    for _ in range(args.warmup):
        step()
    ms_mm = timed(torch, ds, lambda: [step() for _ in range(args.steps)], 1, dev) / args.steps
    result["matmul_path"] = {"tok_per_s": round(1e3 / ms_mm, 3), "ms_per_step": round(ms_mm, 4),
                             "hbm_gbs_per_gpu": round(WEIGHT_BYTES / (ms_mm / 1e3) / 1e9, 1)}
    del step
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if not args.no_reference_configs:
        result["configs"] = reference_configs(torch, dev, args.seed)
    if not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args.seed)
    emit(result)


def emit(result):
    out = JSON_OUT if JSON_OUT is not None else sys.stdout
    out.write(json.dumps(result) + "\n")
    out.flush()


def run_ours(torch, dist, dev, args, world, rank, local, hbm_peak, tf_peak, tf_peak_sus, peak_src):
    stream = torch.cuda.Stream(device=dev)
    step = TPStep(torch, dev, args.seed, world, rank) if world > 1 else OursStep(torch, dev, args.seed)
    torch.cuda.synchronize()
    weights = full_model_weights(torch, dev, args.seed, step.layers, step.lm if world == 1 else step.inner.lm)
    e2e_steps = max(5, args.steps // 2)
    ctx = PROMPT + args.warmup + args.steps + e2e_steps + 64
    eng = make_engine(weights, world, rank, 1, ctx, comm=getattr(step, "comm", None),
                      exchange=getattr(step, "exchange", None), plan=getattr(step, "plan", None))
    es = torch.cuda.ExternalStream(eng.stream, device=dev)
    prompt = prompts(args.seed, 1)[0]
    # untimed warm-up prefill (first-call setup: tensor maps, NCCL connections)
    eng.prefill(0, prompt[:256])
    eng.set_position(0, 0, 0)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    first = eng.prefill(0, prompt)
    prefill_s = time.perf_counter() - t0
    warm_ids = eng.decode(args.warmup)  # captures the step graph, then replays it

    # ---------------- timed region: K decode steps (graph replays), device events
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    timed_ids = {}
    ms_total = timed(torch, es, lambda: timed_ids.__setitem__("ids", eng.decode(args.steps)), world, dev)
    clk = clocks.stop()
    run_ids = np.concatenate([[first], warm_ids[:, 0], timed_ids["ids"][:, 0]]).astype(np.int32)
    ms_step = ms_total / args.steps
    tok_s = args.steps / (ms_total / 1e3)

    # ---------------- e2e: ie_engine_step, host token in and host id out per step
    tok = np.array([first], np.int32)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        tok = eng.step(tok)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = {"value": round(e2e_steps / e2e_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
           "api": "ie_engine_step"}
    result = base_result(args, world, tok_s, ms_step, clk, e2e, "bf16")
    result["config"]["launch"] = "one CUDA graph per decode step (ie_engine_decode), ids kept on the device"
    result["config"]["tp_exchange"] = getattr(step, "mode", None)
    result["gpu_launches"] = (L * 7 + 4 + (1 if world > 1 else 0)) * args.steps
    result["prefill_engine"] = {"prompt": PROMPT, "ms": round(prefill_s * 1e3, 3),
                                "tok_per_s": round(PROMPT / prefill_s, 1), "timing": "host wall clock, blocking call"}
    if world > 1:
        # the N-rank engine's ids of this run against the single-GPU engine's
        result["tp_parity"] = tp_parity(torch, dist, dev, args.seed, rank, prompt, eng, run_ids, ctx)
    eng.close()
    del eng, es
    torch.cuda.synchronize()

    # ---------------- the weight-matmul path alone (north-star target: >= 80 % of HBM)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        step()  # eager warm-up on the capture stream
    torch.cuda.synchronize()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()

    def replays():
        for _ in range(args.steps):
            graph.replay()
    with torch.cuda.stream(stream):
        ms_mm = timed(torch, stream, replays, world, dev) / args.steps
    result["matmul_path"] = {
        "workload": "32 x [fused QKV+RoPE (KV cache row 2047), O, FFN gate/up+SwiGLU, FFN down] + lm_head+argmax, "
                    "bs=1 (no attention core, norms or residual adds)",
        "tok_per_s": round(1e3 / ms_mm, 3), "ms_per_step": round(ms_mm, 4),
        "hbm_gbs_per_gpu": round(WEIGHT_BYTES / world / (ms_mm / 1e3) / 1e9, 1),
        "frac_of_hbm": round(WEIGHT_BYTES / world / (ms_mm / 1e3) / 1e9 / hbm_peak, 4),
        "gpu_launches_per_step": step.launches_per_step,
    }

    # dominant kernel (FFN gate/up + SwiGLU, 54% of the bytes): 32 launches over
    # distinct layer weights per replay, timed with events on its stream
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=stream):
        step.gate_up_only()
    reps = 10
    with torch.cuda.stream(stream):
        for _ in range(3):
            g2.replay()

        def gu():
            for _ in range(reps):
                g2.replay()
        per_launch_s = timed(torch, stream, gu, world, dev) / 1e3 / (reps * L)
    f_local = step.h.shape[1]
    gate_up_bytes = 2 * (2 * f_local * H + H + f_local)
    achieved = gate_up_bytes / per_launch_s / 1e9
    traffic = load_traffic()
    result["roofline"] = {
        "kernel": f"skinny_kernel<bf16,1,EPI_SWIGLU> (FFN gate/up + SwiGLU, M=1, {f_local} rows)",
        "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
        "frac": round(achieved / hbm_peak, 4), "peak_source": peak_src,
        "traffic": traffic if world == 1 else None, "algorithmic_bytes_per_launch": gate_up_bytes,
        "avg_launch_us": round(per_launch_s * 1e6, 2),
    }
    del g2

    if world > 1:
        # BASELINE config 3 under tensor parallelism: M=2048 projection chain,
        # per-rank shards on the tensor-core kernels, NCCL allreduce of the
        # fp32 O / down partials (32 MB each); aggregate TFLOP/s over ranks
        step.setup_prefill(2048)
        gp = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            step.prefill()
        torch.cuda.synchronize()
        with torch.cuda.graph(gp, stream=stream):
            step.prefill()
        with torch.cuda.stream(stream):
            gp.replay()

            def pre():
                for _ in range(3):
                    gp.replay()
            pre_s = timed(torch, stream, pre, world, dev) / 1e3 / 3
        tflops = step.prefill_flops() * world / pre_s / 1e12
        result["prefill"] = {"workload": f"M=2048 tokens, tp{world}: 32 x [QKV+RoPE, O+allreduce, gate/up+SwiGLU, "
                                         f"down+allreduce] + lm_head(last row)", "ms": round(pre_s * 1e3, 3),
                             "tflops_aggregate": round(tflops, 1),
                             "frac_of_n_x_burst": round(tflops / (world * tf_peak), 4)}
        gp.reset()
        del gp
    else:
        # prefill projection GEMMs at M=2048 over all 32 layers
        step.setup_prefill(2048)
        # BASELINE configs 1-4 one by one (before the long prefill chain, which
        # leaves the GPU warm and power-capped)
        result["configs"] = per_config(torch, step, stream, hbm_peak, tf_peak)
        if not args.no_reference_configs:
            ref_cfg = reference_configs(torch, dev, args.seed)
            result["configs_reference"] = ref_cfg
            result["configs_speedup_vs_reference"] = versus_reference(result["configs"], ref_cfg)
        gp = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            step.prefill()
        torch.cuda.synchronize()
        with torch.cuda.graph(gp, stream=stream):
            step.prefill()
        reps = 3
        with torch.cuda.stream(stream):
            gp.replay()

            def pre():
                for _ in range(reps):
                    gp.replay()
            pre_s = timed(torch, stream, pre, world, dev) / 1e3 / reps
        tflops = step.prefill_flops() / pre_s / 1e12
        # the timed region is a few chains of ~25 ms, not a seconds-long loop:
        # the burst peak is the denominator (the sustained figure is shown too)
        result["prefill"] = {
            "workload": "M=2048 tokens: 32 x [fused QKV+RoPE 6144x4096, O 4096x4096, gate/up+SwiGLU 2x14336x4096, "
                        "down 4096x14336]", "ms": round(pre_s * 1e3, 3), "tflops": round(tflops, 1),
            "peak_tflops": tf_peak, "frac": round(tflops / tf_peak, 4),
            "peak_source": f"{peak_src} bf16 burst ({reps} chains of {pre_s * 1e3:.0f} ms)",
            "frac_of_sustained": round(tflops / tf_peak_sus, 4),
            "gpu_launches": 4 * L,
        }
        del gp
        step.release_prefill()
        torch.cuda.empty_cache()
        # BASELINE config 5 at batch 8 and the M=5 verify pass, full model
        # warm-up of at least 20 steps: the first ~20 steps after the eight
        # 2048-token prefills run at ~3.9 ms, the following ones at ~3.65
        B8, n8, w8 = 8, 20, max(args.warmup, 20)
        eng8 = make_engine(weights, 1, 0, B8, PROMPT + w8 + n8 + 16)
        ps = prompts(args.seed, B8)
        for b in range(B8):
            eng8.prefill(b, ps[b])
        eng8.decode(w8)
        es8 = torch.cuda.ExternalStream(eng8.stream, device=dev)
        ms8 = timed(torch, es8, lambda: eng8.decode(n8), 1, dev) / n8
        result["decode_bs8"] = {"batch": B8, "ms_per_step": round(ms8, 4), "tok_per_s": round(B8 / (ms8 / 1e3), 1),
                                "steps": n8, "warmup_steps": w8, "context": f"{PROMPT}-token prompts"}
        eng8.close()
        del eng8, es8
        torch.cuda.synchronize()
        eng5 = make_engine(weights, 1, 0, 1, PROMPT + 16)
        nxt = eng5.prefill(0, prompt)
        draft = np.concatenate([[nxt], prompts(args.seed + 1, 1)[0][:4]]).astype(np.int32)
        for _ in range(3):
            eng5.verify(0, draft)
        es5 = torch.cuda.ExternalStream(eng5.stream, device=dev)
        n5 = 20

        def ver():
            for _ in range(n5):
                eng5.verify(0, draft)
        ms5 = timed(torch, es5, ver, 1, dev) / n5
        result["verify_m5"] = {"rows": 5, "ms_per_pass": round(ms5, 4), "tok_per_s": round(5 / (ms5 / 1e3), 1),
                               "timing": "device events around blocking ie_engine_verify calls (host ids out)"}
        eng5.close()
        del eng5, es5
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        if args.parity_steps > 0:
            result["parity"] = parity_leg(torch, dev, args.seed, args.parity_steps)
        if not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline(args.seed)

    if rank == 0:
        emit(result)
    # graphs holding NCCL work are released before the communicators
    graph.reset()
    del graph
    torch.cuda.synchronize()
    if hasattr(step, "close"):
        step.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
