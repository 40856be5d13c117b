"""Megatron-style tensor parallelism of the weight-matmul hot path.

The reference runs on one GPU; this splits its projections across the GPUs of
one machine:

* Q/K/V column-split by heads: rank r owns query heads
  [r*NQ/t, (r+1)*NQ/t) and KV heads [r*NKV/t, (r+1)*NKV/t) (ie_qkv on the
  shard writes its own heads of Q and of the KV cache);
* O row-split by its input columns (the rank's attention heads):
  ie_gemm_f32out gives an fp32 partial, summed over ranks
  (ie_allreduce_sum_f32) and rounded once (ie_cast_f32);
* gate/up column-split by FFN rows (ie_ffn_gate_up, SwiGLU stays local);
* down row-split by its input columns (the rank's FFN rows), reduced like O;
* lm_head vocab-split: ie_lm_head_argmax on the rank's vocabulary rows with
  its global offset, packed keys merged by a max over ranks
  (ie_argmax_allreduce), which reproduces the single-GPU tie order.

Every rank runs the same sequence of launches and collectives in the same
order. The exchanges are NCCL collectives issued by the library on the
caller's stream.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import (FFN_DIM, HEAD_DIM, HIDDEN_SIZE, NUM_KV_HEADS, NUM_Q_HEADS, VOCAB_SIZE, _check, _dt, _ptr, _stream,
               lib)


@dataclass(frozen=True)
class ShardPlan:
    """Slices of every weight that rank `rank` of `world` owns."""

    world: int
    rank: int
    hidden: int = HIDDEN_SIZE
    ffn: int = FFN_DIM
    n_q_heads: int = NUM_Q_HEADS
    n_kv_heads: int = NUM_KV_HEADS
    head_dim: int = HEAD_DIM
    vocab: int = VOCAB_SIZE

    def __post_init__(self):
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside a world of {self.world}")
        for name, n in (("query heads", self.n_q_heads), ("KV heads", self.n_kv_heads), ("FFN rows", self.ffn)):
            if n % self.world:
                raise ValueError(f"{name} ({n}) do not split evenly over {self.world} ranks")
        if (self.ffn // self.world) % 8:
            raise ValueError("FFN shard must be a multiple of 8 rows (16-byte aligned rows)")

    # ---- sizes
    @property
    def q_heads(self) -> int:
        return self.n_q_heads // self.world

    @property
    def kv_heads(self) -> int:
        return self.n_kv_heads // self.world

    @property
    def ffn_rows(self) -> int:
        return self.ffn // self.world

    # ---- slices (row ranges of the [out, in] weights, or input-column ranges)
    def q_rows(self) -> slice:
        n = self.q_heads * self.head_dim
        return slice(self.rank * n, (self.rank + 1) * n)

    def kv_rows(self) -> slice:
        n = self.kv_heads * self.head_dim
        return slice(self.rank * n, (self.rank + 1) * n)

    def o_cols(self) -> slice:
        return self.q_rows()  # O's inputs are the rank's attention heads

    def ffn_slice(self) -> slice:
        return slice(self.rank * self.ffn_rows, (self.rank + 1) * self.ffn_rows)

    def vocab_slice(self) -> slice:
        return slice(self.rank * self.vocab // self.world, (self.rank + 1) * self.vocab // self.world)

    def shard_layer(self, w: dict) -> dict:
        """Contiguous per-rank copies of one layer's weights (torch or numpy).
        Keys: wq wk wv wo wg wu wd (HF [out, in] layouts)."""
        def c(t):
            return t.contiguous() if hasattr(t, "contiguous") else t.copy()
        return {"wq": c(w["wq"][self.q_rows()]), "wk": c(w["wk"][self.kv_rows()]), "wv": c(w["wv"][self.kv_rows()]),
                "wo": c(w["wo"][:, self.o_cols()]), "wg": c(w["wg"][self.ffn_slice()]),
                "wu": c(w["wu"][self.ffn_slice()]), "wd": c(w["wd"][:, self.ffn_slice()])}

    def shard_lm_head(self, lm):
        s = self.vocab_slice()
        t = lm[s]
        return t.contiguous() if hasattr(t, "contiguous") else t.copy()


class Comm:
    """NCCL communicator of the library (ie_comm_*), bootstrapped over an
    initialized torch.distributed process group."""

    def __init__(self, world: int, rank: int, group=None):
        import torch.distributed as dist
        L = lib()
        L.ie_comm_unique_id.argtypes = [ctypes.c_void_p]
        L.ie_comm_create.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
        L.ie_comm_destroy.argtypes = [ctypes.c_void_p]
        L.ie_allreduce_sum_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        L.ie_argmax_allreduce.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                          ctypes.c_void_p]
        L.ie_cast_f32.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        uid = (ctypes.c_ubyte * 128)()
        if rank == 0:
            _check(L.ie_comm_unique_id(ctypes.cast(uid, ctypes.c_void_p)), "ie_comm_unique_id")
        box = [bytes(uid)]
        dist.broadcast_object_list(box, src=0, group=group)
        uid = (ctypes.c_ubyte * 128).from_buffer_copy(box[0])
        self.handle = ctypes.c_void_p()
        _check(L.ie_comm_create(world, rank, ctypes.cast(uid, ctypes.c_void_p), ctypes.byref(self.handle)),
               "ie_comm_create")
        self.world, self.rank = world, rank

    def allreduce_sum_f32(self, t, stream=None):
        _check(lib().ie_allreduce_sum_f32(self.handle, _ptr(t), t.numel(), _stream(stream)), "ie_allreduce_sum_f32")

    def argmax_allreduce(self, keys, idx_out=None, stream=None):
        _check(lib().ie_argmax_allreduce(self.handle, _ptr(keys), keys.numel(), _ptr(idx_out), _stream(stream)),
               "ie_argmax_allreduce")

    def close(self):
        if self.handle:
            lib().ie_comm_destroy(self.handle)
            self.handle = ctypes.c_void_p()


class _Exchange(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int), ("sym", ctypes.c_void_p),
                ("max_rows", ctypes.c_int), ("max_cols", ctypes.c_int)]


class P2PExchange:
    """Exchange buffers for ie_gemm_allreduce: one zeroed device buffer per
    rank, mapped into every other rank with CUDA IPC (handles distributed over
    the torch.distributed group). All ranks construct it together."""

    def __init__(self, world: int, rank: int, max_rows: int = 16, max_cols: int = HIDDEN_SIZE, group=None):
        import torch
        import torch.distributed as dist
        L = lib()
        L.ie_tp_exchange_bytes.restype = ctypes.c_size_t
        L.ie_tp_exchange_bytes.argtypes = [ctypes.c_int] * 3
        L.ie_ipc_export.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)]
        L.ie_ipc_import.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]
        L.ie_ipc_release.argtypes = [ctypes.c_void_p]
        for fn in (L.ie_gemm_allreduce, L.ie_gemm_allreduce_add):
            fn.argtypes = [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_int64] * 3 + [
                ctypes.POINTER(_Exchange), ctypes.c_void_p]
        nbytes = int(L.ie_tp_exchange_bytes(world, max_rows, max_cols))
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        handle = (ctypes.c_ubyte * 64)()
        off = ctypes.c_uint64()
        _check(L.ie_ipc_export(ctypes.c_void_p(self.buf.data_ptr()), ctypes.cast(handle, ctypes.c_void_p),
                               ctypes.byref(off)), "ie_ipc_export")
        everyone = [None] * world
        dist.all_gather_object(everyone, (bytes(handle), int(off.value)), group=group)
        self.imported = []
        ptrs = []
        for r, (h, o) in enumerate(everyone):
            if r == rank:
                ptrs.append(self.buf.data_ptr())
                continue
            hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
            p = ctypes.c_void_p()
            _check(L.ie_ipc_import(ctypes.cast(hb, ctypes.c_void_p), o, ctypes.byref(p)), "ie_ipc_import")
            self.imported.append(p)
            ptrs.append(p.value)
        self.sym = torch.tensor(ptrs, dtype=torch.int64, device="cuda")
        self.desc = _Exchange(world, rank, ctypes.c_void_p(self.sym.data_ptr()), max_rows, max_cols)
        dist.barrier(group=group)

    def gemm_allreduce(self, x, w, y, stream=None, residual=False):
        """y[M,N] = round(sum over ranks of x_r . w_r^T), one fused kernel;
        with residual, y = round(y + round(sum)) in place."""
        M, K = x.shape
        N = w.shape[0]
        fn = lib().ie_gemm_allreduce_add if residual else lib().ie_gemm_allreduce
        _check(fn(_dt(x), M, N, K, _ptr(x), x.stride(0), _ptr(w), w.stride(0), _ptr(y), y.stride(0),
                  ctypes.byref(self.desc), _stream(stream)), "ie_gemm_allreduce")

    def close(self):
        for p in self.imported:
            lib().ie_ipc_release(p)
        self.imported = []


def cast_f32(src, dst, stream=None):
    _check(lib().ie_cast_f32(_dt(dst), _ptr(src), _ptr(dst), src.numel(), _stream(stream)), "ie_cast_f32")


def gemm_f32out(x, w, y, stream=None):
    """y (fp32) [M,N] = x[M,K] . w[N,K]^T, unrounded (ie_gemm_f32out)."""
    L = lib()
    L.ie_gemm_f32out.argtypes = [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_int64] * 3 + [ctypes.c_void_p]
    M, K = x.shape
    N = w.shape[0]
    _check(L.ie_gemm_f32out(_dt(x), M, N, K, _ptr(x), x.stride(0), _ptr(w), w.stride(0), _ptr(y), y.stride(0),
                            _stream(stream)), "ie_gemm_f32out")


class TPDecodeStep:
    """One rank's share of a decode step of the weight-matmul path.

    Buffers are allocated once; __call__ launches, per layer: QKV (+RoPE) on
    the local heads, O partial + allreduce + cast, gate/up on the local FFN
    rows, down partial + allreduce + cast; then the lm_head shard and the
    argmax merge. As in the single-GPU bench, the attention core, norms and
    residual adds are outside the path: each layer's projections read the
    step input and O reads the local Q heads.
    """

    def __init__(self, plan: ShardPlan, comm: Comm, layers: list, lm_shard, rope_cos, rope_sin, pos: int,
                 batch: int = 1, ctx: int = 8192, exchange: "P2PExchange | None" = None, lm_rows: int | None = None):
        import torch
        from . import lm_head_workspace_bytes
        self.plan, self.comm, self.layers, self.lm = plan, comm, layers, lm_shard
        if exchange is not None and batch > 16:
            raise ValueError("the fused NVLink exchange serves decode batches of at most 16 rows")
        self.exchange = exchange
        # rows that reach lm_head: all of them in decode, the last one in a
        # prefill (the reference's lm_head reads row seq_len-1, lm_head.cu:7)
        self.lm_rows = batch if lm_rows is None else lm_rows
        self.cos, self.sin, self.pos, self.ctx = rope_cos, rope_sin, pos, ctx
        dev, dt = lm_shard.device, lm_shard.dtype
        M, H = batch, plan.hidden
        self.x = torch.zeros(M, H, device=dev, dtype=dt)
        self.q = torch.empty(plan.q_heads, M, plan.head_dim, device=dev, dtype=dt)
        self.kc = torch.zeros(len(layers), plan.kv_heads, ctx, plan.head_dim, device=dev, dtype=dt)
        self.vc = torch.zeros(len(layers), plan.kv_heads, ctx, plan.head_dim, device=dev, dtype=dt)
        self.part = torch.empty(M, H, device=dev, dtype=torch.float32)
        self.attn_out = torch.empty(M, H, device=dev, dtype=dt)
        self.h = torch.empty(M, plan.ffn_rows, device=dev, dtype=dt)
        self.ffn_out = torch.empty(M, H, device=dev, dtype=dt)
        self.keys = torch.zeros(self.lm_rows, device=dev, dtype=torch.int64)
        self.tok = torch.zeros(self.lm_rows, device=dev, dtype=torch.int32)
        self.ws = torch.zeros(lm_head_workspace_bytes(self.lm_rows), dtype=torch.uint8, device=dev)
        # kernels of this library per step (NCCL's own kernels not counted)
        self.launches_per_step = len(layers) * (4 if exchange else 8) + 2

    def flops(self) -> float:
        """Projection FLOPs of one call on this rank (2*M*N*K per GEMM)."""
        p, M = self.plan, self.x.shape[0]
        H, D = p.hidden, p.head_dim
        per_layer = ((p.q_heads + 2 * p.kv_heads) * D * H + H * p.q_heads * D + 3 * p.ffn_rows * H) * 2 * M
        return len(self.layers) * per_layer + 2.0 * self.lm_rows * (self.lm.shape[0]) * H

    def __call__(self):
        from . import ffn_gate_up, lm_head_argmax, qkv
        p, M = self.plan, self.x.shape[0]
        for l, w in enumerate(self.layers):
            qkv(self.x, w["wq"], w["wk"], w["wv"], self.q, self.kc[l], self.vc[l], self.ctx * p.head_dim, self.pos,
                self.cos, self.sin, n_q_heads=p.q_heads, n_kv_heads=p.kv_heads)
            a_in = self.q.view(M, -1) if M == 1 else self.q.permute(1, 0, 2).reshape(M, -1)
            if self.exchange is not None:
                # one kernel: partial O rows to every rank over NVLink, summed on arrival
                self.exchange.gemm_allreduce(a_in, w["wo"], self.attn_out)
                ffn_gate_up(self.x, w["wg"], w["wu"], self.h)
                self.exchange.gemm_allreduce(self.h, w["wd"], self.ffn_out)
                continue
            gemm_f32out(a_in, w["wo"], self.part)
            self.comm.allreduce_sum_f32(self.part)
            cast_f32(self.part, self.attn_out)
            ffn_gate_up(self.x, w["wg"], w["wu"], self.h)
            gemm_f32out(self.h, w["wd"], self.part)
            self.comm.allreduce_sum_f32(self.part)
            cast_f32(self.part, self.ffn_out)
        lm_head_argmax(self.x[M - self.lm_rows:], self.lm, self.ws, key_out=self.keys,
                       vocab_offset=p.vocab_slice().start)
        self.comm.argmax_allreduce(self.keys, self.tok)
