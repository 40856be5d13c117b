"""GPU, one device: a bounded device-side wait that runs out, and the device
afterwards.

ie_gemm_allreduce is called with world = 2 on a single process: the "peer"
buffer of rank 1 is a second zeroed buffer on this GPU that no kernel ever
fills. Every CTA pushes its partial rows, then waits for rank 1's rows, which
never arrive. With the wait limit set to 1 ms (ie_set_wait_limit_ns) each CTA
gives up after about 1 ms, records IE_ERR_TIMEOUT in the device status word,
writes none of its outputs and returns, so the call ends in milliseconds, not
at the 2 s default. After that the context is intact: the status word clears,
and the next calls (a world = 1 exchange and a plain projection) are exact.
No fault, trap or endless loop is involved: the wait is bounded and ends on
its own.
"""
import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

IE_ERR_TIMEOUT = -5


def _exchange(ie, cuda, bufs, max_rows, max_cols):
    from infengine_b200.tp import _Exchange
    L = ie.lib()
    sym = cuda.tensor([b.data_ptr() for b in bufs], dtype=cuda.int64, device="cuda")
    desc = _Exchange(len(bufs), 0, ctypes.c_void_p(sym.data_ptr()), max_rows, max_cols)
    return desc, sym


def _bind(ie):
    L = ie.lib()
    L.ie_tp_exchange_bytes.restype = ctypes.c_size_t
    L.ie_tp_exchange_bytes.argtypes = [ctypes.c_int] * 3
    from infengine_b200.tp import _Exchange
    L.ie_gemm_allreduce.argtypes = [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_int64] * 3 + [
        ctypes.POINTER(_Exchange), ctypes.c_void_p]
    return L


IE_DTYPE_BF16 = 1


def _call(L, x, w, y, desc):
    M, K = x.shape
    N = w.shape[0]
    return L.ie_gemm_allreduce(IE_DTYPE_BF16, M, N, K, x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), y.data_ptr(),
                               y.stride(0), ctypes.byref(desc), None)


def test_exchange_wait_times_out_and_device_stays_usable(ie, cuda):
    L = _bind(ie)
    M, N, K, max_rows = 2, 4096, 2048, 16
    g = cuda.Generator(device="cuda").manual_seed(5)
    x = cuda.randn(M, K, generator=g, device="cuda").to(cuda.bfloat16)
    w = (0.02 * cuda.randn(N, K, generator=g, device="cuda")).to(cuda.bfloat16)
    assert ie.device_status() == 0
    nbytes = int(L.ie_tp_exchange_bytes(2, max_rows, N))
    bufs = [cuda.zeros(nbytes, dtype=cuda.uint8, device="cuda") for _ in range(2)]
    desc, sym = _exchange(ie, cuda, bufs, max_rows, N)
    y = cuda.zeros(M, N, dtype=cuda.bfloat16, device="cuda")
    ie.set_wait_limit_ns(1_000_000)  # 1 ms
    try:
        cuda.cuda.synchronize()
        t0 = time.perf_counter()
        assert _call(L, x, w, y, desc) == 0  # the launch itself succeeds
        cuda.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        ie.set_wait_limit_ns(0)  # back to the 2 s default
    assert elapsed < 0.5, elapsed  # gave up after ~1 ms, not after the 2 s default
    assert ie.device_status(clear=True) == IE_ERR_TIMEOUT
    assert ie.device_status() == 0  # cleared
    assert not y.any()  # no row was complete, so nothing was written
    # the same context keeps working: a world = 1 exchange (own buffer only)
    # and the plain projection give the same bits, close to the fp32 product
    one = cuda.zeros(int(L.ie_tp_exchange_bytes(1, max_rows, N)), dtype=cuda.uint8, device="cuda")
    desc1, sym1 = _exchange(ie, cuda, [one], max_rows, N)
    for _ in range(2):
        y1 = cuda.empty(M, N, dtype=cuda.bfloat16, device="cuda")
        assert _call(L, x, w, y1, desc1) == 0
        y2 = cuda.empty(M, N, dtype=cuda.bfloat16, device="cuda")
        ie.gemm(x, w, y2)
        cuda.cuda.synchronize()
        assert cuda.equal(y1, y2)
        want = (x.float() @ w.float().T)
        err = ((y2.float() - want).abs().max() / want.abs().max()).item()
        assert err < 1e-2, err
    assert ie.device_status() == 0
    del sym, sym1


def test_wait_limit_argument_checks(ie, cuda):
    from infengine_b200 import IEError
    with pytest.raises(IEError):
        ie.set_wait_limit_ns(61 * 10**9)  # above the 60 s ceiling
    ie.set_wait_limit_ns(0)
    assert ie.device_status() == 0
