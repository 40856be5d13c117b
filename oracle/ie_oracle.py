"""CPU oracle for the infengine weight-matmul hot path — TEST INFRASTRUCTURE.

This module restates, in numpy, what the reference (Aryan470/infengine)
computes on the hot path, so that tests/ can check the CUDA kernels of
infengine_b200 against it. Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg may import it; the product path never does.

Pinning (how the oracle itself is checked):
  * swiglu and argmax: against golden vectors produced by the reference's own
    generator functions (scripts/generate_test_data.py:113-124 and :163-168,
    run in the build container by tests/golden/make_golden.py);
  * argmax tie order: against the reference's own amax_kern compiled from its
    sources (oracle/_ref, GPU tests) on crafted tie vectors;
  * GEMM / FFN / lm_head: the reference does this arithmetic in cuBLAS
    (CUDA 12.9); the oracle computes the exact sum in float64 and rounds once
    to fp32 and then to the storage type. Bit-level parity with cuBLAS is not
    defined; tests compare within stated tolerances and against the reference
    library run on the same inputs (oracle/_ref).

Every value in and out is a numpy float32 array holding numbers exactly
representable in the storage dtype ("f16" or "bf16").
"""
from __future__ import annotations

import math

import numpy as np

HIDDEN_SIZE = 4096
FFN_DIM = 14336
VOCAB_SIZE = 128256
HEAD_DIM = 128
MAX_CONTEXT_LENGTH = 8192


# ----------------------------------------------------------- storage types
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (NaN kept quiet)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    rounded = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    out = np.where(nan, (b >> 16) | 0x40, rounded).astype(np.uint16)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_dt(x, dt: str) -> np.ndarray:
    """Value of fp32 x after storing it as dt (one rounding, RNE)."""
    x = np.asarray(x, dtype=np.float32)
    if dt == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dt == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if dt == "f32":
        return x
    raise ValueError(dt)


def to_bits(x: np.ndarray, dt: str) -> np.ndarray:
    """uint16 storage bits of values representable in dt."""
    if dt == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)
    return f32_to_bf16_bits(x)


def from_bits(b: np.ndarray, dt: str) -> np.ndarray:
    if dt == "f16":
        return np.asarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)
    return bf16_bits_to_f32(b)


# -------------------------------------------------------- a1 / a5: GEMM
def multiply_by_weight(x: np.ndarray, w: np.ndarray, dt: str) -> np.ndarray:
    """y[m,n] = x[m,k] . w[n,k]^T with exact accumulation, one rounding.

    Follows kernels/ffn.cu:7-33 (cublasGemmEx, fp16 in/out, CUDA_R_32F
    compute, alpha=1, beta=0) and the BASELINE fp32 golden (x @ W.T).
    """
    acc = np.asarray(x, dtype=np.float64) @ np.asarray(w, dtype=np.float64).T
    return round_dt(acc.astype(np.float32), dt)


def gemm_fp32(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Unrounded fp32 golden (the normwise-error reference)."""
    return (np.asarray(x, dtype=np.float64) @ np.asarray(w, dtype=np.float64).T).astype(np.float32)


# ---------------------------------------------------------- a3: SwiGLU
def swiglu(gate: np.ndarray, up: np.ndarray, dt: str) -> np.ndarray:
    """out = g * (1 / (1 + exp(-g))) * u in fp32, rounded to dt.

    kernels/swiglu.cu:26-29; the golden generator computes
    silu(gate.float()) * up.float() (scripts/generate_test_data.py:121).
    """
    g = np.asarray(gate, dtype=np.float32)
    u = np.asarray(up, dtype=np.float32)
    with np.errstate(over="ignore"):
        s = np.float32(1.0) / (np.float32(1.0) + np.exp(-g))
    return round_dt(g * s * u, dt)


# ------------------------------------------------------------- a2: FFN
def ffn(x, w_gate, w_up, w_down, dt: str) -> np.ndarray:
    """kernels/ffn.cu:39-64: U = x.Wu^T, G = x.Wg^T (each rounded to dt),
    H = swiglu(G, U) (rounded), out = H.Wd^T (rounded)."""
    g = multiply_by_weight(x, w_gate, dt)
    u = multiply_by_weight(x, w_up, dt)
    h = swiglu(g, u, dt)
    return multiply_by_weight(h, w_down, dt)


# ------------------------------------------------------------------ RoPE
def rope_tables(max_pos: int = MAX_CONTEXT_LENGTH, head_dim: int = HEAD_DIM):
    """cos/sin tables [max_pos, head_dim/2] fp32 as built by init_rope_buffer
    (kernels/rope.cu:68-103): Llama-3.1 frequency scaling, theta 500000,
    factor 8, low/high frequency factors 1/4, original context 8192."""
    theta, factor, low, high, orig = 500000.0, 8, 1, 4, 8192
    low_wl, high_wl = orig // low, orig // high
    freqs = np.empty(head_dim // 2, dtype=np.float32)
    for i in range(head_dim // 2):
        freq = np.float32(1.0 / math.pow(theta, 2.0 * i / head_dim))
        wavelength = np.float32(2 * math.pi / float(freq))
        if wavelength > low_wl:
            freqs[i] = np.float32(freq / np.float32(factor))
        elif wavelength < high_wl:
            freqs[i] = freq
        else:
            smoothed = np.float32((np.float32(orig) / wavelength - np.float32(low)) / np.float32(high - low))
            freqs[i] = np.float32((np.float32(1) - smoothed) * (freq / np.float32(factor)) + smoothed * freq)
    pos = np.arange(max_pos, dtype=np.float32)[:, None]
    angle = (pos * freqs[None, :]).astype(np.float32)
    return np.cos(angle).astype(np.float32), np.sin(angle).astype(np.float32)


def apply_rope(xh: np.ndarray, positions: np.ndarray, cos: np.ndarray, sin: np.ndarray, dt: str) -> np.ndarray:
    """Rotate-half RoPE on [..., S, 128] rows (kernels/rope.cu:30-66): pair
    (d, d+64) with table column d at the row's position; fp32 math on the
    stored values, result rounded to dt."""
    half = xh.shape[-1] // 2
    a = xh[..., :half].astype(np.float32)
    b = xh[..., half:].astype(np.float32)
    c = cos[positions][..., :half]
    s = sin[positions][..., :half]
    out = np.empty_like(xh, dtype=np.float32)
    out[..., :half] = round_dt(a * c - b * s, dt)
    out[..., half:] = round_dt(a * s + b * c, dt)
    return out


# ---------------------------------------------------------- a4: Q/K/V
def qkv(x, wq, wk, wv, dt: str, pos0: int = 0, cos=None, sin=None, head_dim: int = HEAD_DIM):
    """Three per-head projections (kernels/attn.cu:12-39) written head-major
    [heads, M, head_dim], then RoPE on Q and K (kernels/attn.cu:351-352 /
    :419-420) when tables are given. Returns (q, k, v) as [heads, M, 128]."""
    M = x.shape[0]
    out = []
    for w in (wq, wk, wv):
        y = multiply_by_weight(x, w, dt)  # [M, heads*128]
        out.append(y.reshape(M, -1, head_dim).transpose(1, 0, 2).copy())
    q, k, v = out
    if cos is not None:
        positions = np.arange(pos0, pos0 + M)
        q = apply_rope(q, positions, cos, sin, dt)
        k = apply_rope(k, positions, cos, sin, dt)
    return q, k, v


# ---------------------------------------------------------- a7: argmax
def argmax_reference(logits: np.ndarray, threads: int = 1024) -> int:
    """Exact restatement of sample_token_amax (kernels/sampling.cu:8-58).

    Thread t starts with (logits[t], t), scans t+threads, t+2*threads, ...
    replacing on a strictly greater value (:36-45); then a shared-memory
    tree keeps [i] unless [i+delta] is strictly greater (:16-24). The
    comparisons follow IEEE semantics, so NaNs never win a comparison.

    With fewer than `threads` logits the reference reads past the buffer
    (every thread starts at logits[t]); here those threads hold -inf, which
    is the rule infengine_b200 applies.
    """
    v = np.asarray(logits, dtype=np.float32).ravel()
    n = v.size
    loc_val = np.full(threads, -np.inf, dtype=np.float32)
    loc_idx = np.arange(threads, dtype=np.int64)
    for t in range(min(threads, n)):
        col = v[t::threads]
        best_v, best_i = col[0], t
        # strict '>' scan, first occurrence of a new maximum wins
        with np.errstate(invalid="ignore"):
            for j in range(1, col.size):
                if col[j] > best_v:
                    best_v, best_i = col[j], t + j * threads
        loc_val[t], loc_idx[t] = best_v, best_i
    delta = threads // 2
    while delta > 0:
        for i in range(delta):
            if loc_val[i] < loc_val[i + delta]:
                loc_val[i], loc_idx[i] = loc_val[i + delta], loc_idx[i + delta]
        delta //= 2
    return int(loc_idx[0])


def bitrev(r, bits: int = 10):
    r = np.asarray(r, dtype=np.int64)
    out = np.zeros_like(r)
    for b in range(bits):
        out |= ((r >> b) & 1) << (bits - 1 - b)
    return out


def argmax_reference_fast(logits: np.ndarray, threads: int = 1024) -> int:
    """Vectorised equivalent of argmax_reference for NaN-free input.

    The strided scan keeps, per residue class t = id mod threads, the
    smallest id holding the class maximum; the halving tree keeps the lower
    slot on ties, and its last level compares bit 0 of t, the level before
    bit 1, ... So among equal maxima the class with the smallest bit-reversed
    t wins, then the smallest id."""
    v = np.asarray(logits, dtype=np.float32).ravel()
    if np.isnan(v).any():
        return argmax_reference(v, threads)
    mx = v.max()
    cand = np.nonzero(v == mx)[0]
    bits = int(threads).bit_length() - 1
    order = np.lexsort((cand // threads, bitrev(cand % threads, bits)))
    return int(cand[order[0]])


def argmax_key(value: float, idx: int) -> int:
    """The packed key of include/infengine_b200.h (unsigned max = winner)."""
    v = np.float32(value)
    if np.isnan(v):
        return 0
    if v == 0:
        v = np.float32(0.0)
    b = int(np.array([v], dtype=np.float32).view(np.uint32)[0])
    ordv = (~b & 0xFFFFFFFF) if (b & 0x80000000) else (b | 0x80000000)
    tie = (int(bitrev(idx & 1023)) << 21) | (idx >> 10)
    return (ordv << 32) | (~tie & 0xFFFFFFFF)


def key_index(key: int) -> int:
    tie = (~key) & 0xFFFFFFFF
    return (tie & ((1 << 21) - 1)) * 1024 + int(bitrev(tie >> 21))


# ------------------------------------------------------ a6: lm_head+argmax
def lm_head_argmax(x: np.ndarray, w: np.ndarray, dt: str, vocab_offset: int = 0):
    """kernels/lm_head.cu:5-20 then kernels/sampling.cu:54-58 for each row of
    x: rounded logits and the reference's greedy id (global ids when w is a
    vocabulary shard starting at vocab_offset)."""
    logits = multiply_by_weight(x, w, dt)
    ids = []
    for row in logits:
        if vocab_offset == 0:
            ids.append(argmax_reference_fast(row))
        else:
            full = np.full(vocab_offset + row.size, -np.inf, dtype=np.float32)
            full[vocab_offset:] = row
            ids.append(argmax_reference_fast(full))
    return logits, np.array(ids, dtype=np.int64)


# ------------------------------------------------------- error metrics
def compare(actual, expected, atol: float):
    """compare_tensors of the reference test harness (tests/test_utils.cpp:42-54):
    max_abs_err, mean_abs_err, pct_within_tol (err <= atol)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    err = np.abs(a - e)
    return {
        "max_abs_err": float(err.max()) if err.size else 0.0,
        "mean_abs_err": float(err.mean()) if err.size else 0.0,
        "pct_within_tol": float(100.0 * (err <= atol).mean()) if err.size else 100.0,
    }


def normwise_rel_err(actual, golden_fp32) -> float:
    """||actual - golden||_F / ||golden||_F (the BASELINE per-GEMM bar is 1e-2)."""
    a = np.asarray(actual, dtype=np.float64)
    g = np.asarray(golden_fp32, dtype=np.float64)
    return float(np.linalg.norm(a - g) / max(np.linalg.norm(g), 1e-30))


def max_rel_err(actual, golden_fp32) -> float:
    """max |actual - golden| / max |golden| (per-GEMM max relative error)."""
    a = np.asarray(actual, dtype=np.float64)
    g = np.asarray(golden_fp32, dtype=np.float64)
    return float(np.abs(a - g).max() / max(np.abs(g).max(), 1e-30))


# ---------------------------------------------------- seeded test inputs
def seeded_inputs(seed: int, shapes: dict, dt: str, scales: dict | None = None) -> dict:
    """Synthetic tensors of the BASELINE configs: N(0,1) activations and
    N(0,0.02) weights, drawn in fp32 from numpy's PCG64 and rounded to dt."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in shapes.items():
        s = (scales or {}).get(name, 0.02 if name.startswith("w") else 1.0)
        out[name] = round_dt(rng.standard_normal(shape, dtype=np.float32) * np.float32(s), dt)
    return out


# ----------------------------------------------- fp32 CPU golden (baseline)
# The same math with fp32 BLAS accumulation (numpy float32 matmul, all host
# threads): the CPU-side golden the reference generator computes with torch
# on the CPU, used as the timed CPU baseline. Roundings to dt as above.
def gemm_cpu(x, w, dt: str) -> np.ndarray:
    return round_dt(np.asarray(x, np.float32) @ np.asarray(w, np.float32).T, dt)


def ffn_cpu(x, w_gate, w_up, w_down, dt: str) -> np.ndarray:
    h = swiglu(gemm_cpu(x, w_gate, dt), gemm_cpu(x, w_up, dt), dt)
    return gemm_cpu(h, w_down, dt)


def qkv_cpu(x, wq, wk, wv, dt: str, pos0: int = 0, cos=None, sin=None, head_dim: int = HEAD_DIM):
    M = x.shape[0]
    out = [gemm_cpu(x, w, dt).reshape(M, -1, head_dim).transpose(1, 0, 2) for w in (wq, wk, wv)]
    q, k, v = out
    if cos is not None:
        positions = np.arange(pos0, pos0 + M)
        q = apply_rope(q, positions, cos, sin, dt)
        k = apply_rope(k, positions, cos, sin, dt)
    return q, k, v


def lm_head_argmax_cpu(x, w, dt: str):
    logits = gemm_cpu(x, w, dt)
    return logits, np.array([argmax_reference_fast(r) for r in logits], dtype=np.int64)


# ------------------------------------------------ attention (drop-in core)
def attention(q, k, v, pos0: int, dt: str):
    """Causal grouped-query attention as the reference's attn / decode_attn
    chain computes it (kernels/attn.cu:355-366, :423-431;
    kernels/softmax.cu:55-160): scores = round(q.k) (the cuBLAS QK^T output),
    t = round(score * rsqrt(128)), e = exp(t - max t) summed in fp32 and stored
    rounded, p = round(round(e) * (1/sum)), out = round(p.V) (cuBLAS A.V).
    q [nq, S, 128] (positions pos0..pos0+S-1), k/v [nkv, >= pos0+S, 128].
    Returns the token-major [S, nq*128] output (attn_permute's layout)."""
    nq, S, D = q.shape
    nkv = k.shape[0]
    group = nq // nkv
    scale = np.float32(1.0 / math.sqrt(D))
    out = np.zeros((S, nq * D), dtype=np.float32)
    for h in range(nq):
        hk = h // group
        for s in range(S):
            L = pos0 + s + 1
            sc = round_dt((q[h, s].astype(np.float64) @ k[hk, :L].astype(np.float64).T).astype(np.float32), dt)
            t = round_dt(sc * scale, dt)
            e = np.exp(t - t.max()).astype(np.float32)
            ssum = np.float32(e.sum(dtype=np.float64))
            p = round_dt(round_dt(e, dt) * (np.float32(1.0) / ssum), dt)
            out[s, h * D:(h + 1) * D] = round_dt((p.astype(np.float64) @ v[hk, :L].astype(np.float64)).astype(np.float32),
                                                 dt)
    return out


# ------------------------------------------- the decode step around the path
def rmsnorm(x, w, dt: str, eps: float = 1e-5):
    """kernels/rmsnorm.cu:29-62: scale = rsqrt(sum(x^2) / H + eps) per row,
    out = round(round(x * scale) * w). The sum is taken exactly and rounded
    once to fp32 (the reference's fp32 tree can differ in the last bit)."""
    x = np.asarray(x, dtype=np.float32)
    ss = (x.astype(np.float64) ** 2).sum(axis=-1, keepdims=True).astype(np.float32)
    scale = (np.float32(1.0) / np.sqrt(ss / np.float32(x.shape[-1]) + np.float32(eps))).astype(np.float32)
    return round_dt(round_dt(x * scale, dt) * np.asarray(w, dtype=np.float32), dt)


def residual_add(x, delta, dt: str):
    """kernels/residual_add.cu:10-20: x = round(x + delta)."""
    return round_dt(np.asarray(x, dtype=np.float32) + np.asarray(delta, dtype=np.float32), dt)


class LlamaOracle:
    """The reference's request flow on the CPU (prefill.cu:11-48 then
    decode.cu:11-49 per token, manager.cpp:31-86), built from the functions
    above, for small models: weights is a dict of float32 arrays holding
    dt-representable values (embedding [V,H], final_norm [H], lm_head [V,H],
    layers: list of dicts attn_norm, wq, wk, wv, wo, ffn_norm, w_gate, w_up,
    w_down). Keeps the K/V cache between calls."""

    def __init__(self, weights: dict, n_q_heads: int, n_kv_heads: int, dt: str, max_ctx: int = 4096,
                 eps: float = 1e-5):
        self.w, self.nq, self.nkv, self.dt, self.eps = weights, n_q_heads, n_kv_heads, dt, eps
        self.cos, self.sin = rope_tables(max_ctx)
        L = len(weights["layers"])
        self.k = np.zeros((L, n_kv_heads, max_ctx, HEAD_DIM), np.float32)
        self.v = np.zeros_like(self.k)
        self.pos = 0

    def forward(self, tokens):
        """Run the rows of `tokens` from the current position; returns the
        rounded logits of every row and advances the position."""
        dt, w = self.dt, self.w
        x = w["embedding"][np.asarray(tokens)]
        S, pos0 = len(tokens), self.pos
        for l, lw in enumerate(w["layers"]):
            a = rmsnorm(x, lw["attn_norm"], dt, self.eps)
            q, k, v = qkv(a, lw["wq"], lw["wk"], lw["wv"], dt, pos0, self.cos, self.sin)
            self.k[l, :, pos0:pos0 + S] = k
            self.v[l, :, pos0:pos0 + S] = v
            att = attention(q, self.k[l], self.v[l], pos0, dt)
            x = residual_add(x, multiply_by_weight(att, lw["wo"], dt), dt)
            a = rmsnorm(x, lw["ffn_norm"], dt, self.eps)
            x = residual_add(x, ffn(a, lw["w_gate"], lw["w_up"], lw["w_down"], dt), dt)
        self.pos += S
        return multiply_by_weight(rmsnorm(x, w["final_norm"], dt, self.eps), w["lm_head"], dt)

    @staticmethod
    def pick(logits_row):
        """Greedy id (the reference's tie order) and the top-1 minus top-2 margin."""
        top2 = np.sort(logits_row)[-2:]
        return argmax_reference_fast(logits_row), float(top2[1] - top2[0])
