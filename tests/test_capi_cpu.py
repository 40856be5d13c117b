"""CPU: the C-ABI library loads, exports what include/infengine_b200.h
declares, and rejects bad arguments before touching a device."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "infengine_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(ie_\w+)\s*\(", text, flags=re.M)
    static_inline = set(re.findall(r"static inline [\w\s\*]+?\b(ie_\w+)\s*\(", text))
    return sorted(set(names) - static_inline)


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("ie_gemm", "ie_ffn", "ie_qkv", "ie_lm_head_argmax", "ie_argmax", "ie_swiglu"):
        assert n in names


@pytest.mark.parametrize("compiler,std", [("gcc", "-std=c99"), ("g++", "-std=c++11")])
def test_header_compiles_cleanly(tmp_path, compiler, std):
    """The public header is plain C (and C++): no CUDA or torch types, and no
    warnings under -Wall -Wextra for a caller that builds with -Werror."""
    src = tmp_path / ("use.c" if compiler == "gcc" else "use.cpp")
    src.write_text('#include "infengine_b200.h"\nint main(void) { return ie_version() ? 0 : 1; }\n')
    r = subprocess.run([compiler, std, "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", str(HEADER.parent), "-c",
                        str(src), "-o", str(tmp_path / "use.o")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_library_exports_every_declared_symbol(ie):
    lib = ie.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(ie.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert set(declared_functions()) <= exported
    assert set(ie.EXPORTED_SYMBOLS) <= exported


def test_dropin_library_exports_reference_signatures(ie):
    out = subprocess.run(["nm", "-DC", "--defined-only", str(ie.DROPIN_PATH)], capture_output=True,
                         text=True).stdout
    for sig in (
        "multiply_by_weight(cublasContext*, int, int, int, __half const*, __half const*, __half*)",
        "ffn(cublasContext*, int, __half*, __half*, __half*, __half*, __half*, void*)",
        "ffn_workspace_size(int)",
        "swiglu(int, __half*, __half*, __half*)",
        "lm_head(cublasContext*, int, __half*, __half*, __half*)",
        "sample_token_amax(__half const*, int*)",
        "attn(cublasContext*, float const*, float const*, int, __half*, __half*, __half*, __half*, __half*, __half*, "
        "void*, void*, int)",
        "decode_attn(cublasContext*, float const*, float const*, int, __half*, __half*, __half*, __half*, __half*, "
        "__half*, void*, void*, int)",
        "attn_workspace_size(int)",
        "kv_cache_size()",
    ):
        assert sig in out, sig


def test_status_strings(ie):
    lib = ie.lib()
    assert lib.ie_status_string(0) == b"ok"
    for code, text in ie.STATUS.items():
        assert lib.ie_status_string(code).decode() == text
    assert lib.ie_version().decode().count(".") == 2


def test_invalid_arguments_rejected_without_device(ie):
    lib = ie.lib()
    vp = ctypes.c_void_p
    fake = vp(0x1000)  # never dereferenced: validation fails first
    # bad dtype
    assert lib.ie_gemm(7, 1, 16, 16, fake, 16, fake, 16, fake, 16, None) == -1
    # null operands
    assert lib.ie_gemm(1, 1, 16, 16, None, 16, fake, 16, fake, 16, None) == -1
    # K not a multiple of 8
    assert lib.ie_gemm(1, 1, 16, 12, fake, 12, fake, 12, fake, 16, None) == -2
    # misaligned pointer
    assert lib.ie_gemm(1, 1, 16, 16, vp(0x1002), 16, fake, 16, fake, 16, None) == -2
    # leading dimension smaller than K
    assert lib.ie_gemm(1, 1, 16, 16, fake, 8, fake, 16, fake, 16, None) == -1
    # empty problems are a no-op
    assert lib.ie_gemm(1, 0, 16, 16, fake, 16, fake, 16, fake, 16, None) == 0
    # head_dim other than 128
    assert lib.ie_qkv(1, 1, 4096, 32, 8, 64, fake, fake, fake, fake, fake, fake, fake, 8192 * 64, 0,
                      None, None, None) == -3
    # ffn workspace too small
    assert lib.ie_ffn(1, 1, 4096, 14336, fake, fake, fake, fake, fake, fake, 16, None) == -7
    # lm_head workspace missing
    assert lib.ie_lm_head_argmax(1, 1, 4096, 128256, 0, fake, 4096, fake, None, 0, None, None, None, 0,
                                 None) == -7
    # vocab ids must fit the packed key (id < 2^31)
    assert lib.ie_lm_head_argmax(1, 1, 4096, 16, 2 ** 31, fake, 4096, fake, None, 0, None, None, fake, 4096,
                                 None) == -3
    # argmax leading dimension smaller than V
    assert lib.ie_argmax(0, 1, 100, fake, 50, fake, None) == -1
    # wait limit above the 60 s ceiling (checked before the device is touched)
    assert lib.ie_set_wait_limit_ns(61 * 10**9) == -1


def test_attention_rejects_bad_arguments_without_device(ie):
    """ie_attention (prefill / chunk) and ie_attention_decode validate shapes,
    strides and alignment before any launch."""
    lib = ie.lib()
    vp = ctypes.c_void_p
    f = vp(0x1000)
    chs = 2048 * 128  # cache head stride: 2048 positions
    # ie_attention(dt, S, pos0, nq, nkv, head_dim, q, q_hs, k, v, chs, out, ld_out, stream)
    ok = lambda **kw: dict(dict(dt=1, S=300, pos0=0, nq=32, nkv=8, hd=128, q=f, qhs=300 * 128, k=f, v=f, chs=chs,
                                out=f, ldo=4096), **kw)
    call = lambda a: lib.ie_attention(a["dt"], a["S"], a["pos0"], a["nq"], a["nkv"], a["hd"], a["q"], a["qhs"],
                                      a["k"], a["v"], a["chs"], a["out"], a["ldo"], None)
    assert call(ok(dt=5)) == -1                        # unknown dtype
    assert call(ok(S=-1)) == -1                        # negative length
    assert call(ok(hd=64)) == -3                       # head_dim other than 128
    assert call(ok(nq=30)) == -3                       # query heads not a multiple of KV heads
    assert call(ok(S=0)) == 0                          # empty chunk: no-op
    assert call(ok(q=None)) == -1                      # null operand
    assert call(ok(k=vp(0x1008))) == -2                # cache not 16-byte aligned
    assert call(ok(ldo=4000)) == -1                    # output row shorter than the heads
    assert call(ok(qhs=100 * 128)) == -1               # q head stride shorter than S rows
    assert call(ok(pos0=1900)) == -1                   # chunk runs past the cache (1900 + 300 > 2048)
    big = 2**31 - 2                                    # pos0 + S would wrap a 32-bit int
    assert call(ok(pos0=big, chs=1 << 62)) == -1
    assert call(ok(pos0=big, S=16, chs=1 << 62)) == -1
    # ie_attention_decode(dt, R, rows_per_seq, nq, nkv, hd, q, q_hs, k, v, chs, cbs, cache_rows, positions,
    #                     pos0, out, ld_out, stream)
    dec = lambda R=1, rps=1, nq=32, nkv=8, rows=2048, pos0=0, k=f, q=f, qhs=None: lib.ie_attention_decode(
        1, R, rps, nq, nkv, 128, q, qhs if qhs is not None else 128 * max(R, 1), k, f, chs, 0, rows, None, pos0, f,
        4096, None)
    assert dec(nq=24) == -3                            # group of 3 query heads per KV head
    assert dec(R=3, rps=2) == -1                       # rows not a whole number of sequences
    assert dec(rows=4096) == -1                        # cache rows beyond the head stride
    assert dec(pos0=2048) == -1                        # position outside the cache
    assert dec(R=2, pos0=2**31 - 1) == -1              # pos0 + R would wrap a 32-bit int
    assert dec(k=vp(0x1004)) == -2                     # cache not 16-byte aligned
    assert dec(q=vp(0x1004)) == -2                     # q not 16-byte aligned (read with 16-byte loads)
    assert dec(qhs=128 * 2 + 4) == -2                  # q head stride not a multiple of 8
    assert dec(R=0) == 0                               # no rows: no-op


def test_norm_embed_add_reject_bad_arguments_without_device(ie):
    """ie_rmsnorm, ie_embed and ie_add_f32 validate before any launch."""
    from infengine_b200.engine import _bind
    _bind()
    lib = ie.lib()
    vp = ctypes.c_void_p
    f = vp(0x1000)
    rms = lambda dt=1, M=1, H=4096, x=f, ldx=4096, w=f, out=f, ldo=4096: lib.ie_rmsnorm(dt, M, H, x, ldx, w, out, ldo,
                                                                                     1e-5, None)
    assert rms(dt=9) == -1                 # unknown dtype
    assert rms(M=0) == 0                   # no rows: no-op
    assert rms(w=None) == -1               # null weight
    assert rms(ldx=4000) == -1             # row stride shorter than the row
    assert rms(H=4092, ldx=4096) == -2     # row not a whole number of 16-byte chunks
    assert rms(x=vp(0x1004)) == -2         # misaligned input
    assert rms(H=20480, ldx=20480, ldo=20480) == -3  # wider than one CTA's 16-byte chunks
    emb = lambda M=1, H=4096, V=128256, tok=f, ldo=4096: lib.ie_embed(1, M, H, V, tok, f, f, ldo, None)
    assert emb(V=0) == -1                  # empty vocabulary
    assert emb(M=0) == 0                   # no tokens: no-op
    assert emb(tok=None) == -1             # null token array
    assert emb(H=4100, ldo=4104) == -2     # row not a whole number of 16-byte chunks
    lib.ie_add_f32.argtypes = [ctypes.c_int, vp, vp, ctypes.c_size_t, vp]
    assert lib.ie_add_f32(1, None, f, 16, None) == -1   # null input
    assert lib.ie_add_f32(1, None, None, 0, None) == 0  # empty: no-op


def test_workspace_sizes(ie):
    assert ie.ffn_workspace_bytes(1, 14336) >= 14336 * 2
    assert ie.ffn_workspace_size(5) == 2 * 5 * 14336 * 2  # reference ffn.cu:35-37
    assert ie.lm_head_workspace_bytes(64) >= 64 * 8 + 4


def test_key_index_roundtrip(ie):
    from conftest import oracle
    for idx in (0, 1, 1023, 1024, 75177, 128255, 2 ** 31 - 1):
        assert ie.key_index(oracle.argmax_key(1.5, idx)) == idx


def test_python_mirror_fails_loudly_without_library(monkeypatch, ie, tmp_path):
    monkeypatch.setattr(ie, "LIB_PATH", tmp_path / "missing.so")
    monkeypatch.setattr(ie, "_lib_handle", None)
    with pytest.raises(RuntimeError, match="missing"):
        ie.lib()


def test_engine_and_loader_reject_bad_arguments_without_device(ie):
    """Engine creation and the loader validate before any device work."""
    lib = ie.lib()
    vp = ctypes.c_void_p
    out = vp()
    from infengine_b200.engine import LlamaDesc, _bind
    _bind()
    # null descriptor
    assert lib.ie_engine_create(1, None, 1, 128, 16, None, ctypes.byref(out)) == -1
    # descriptor with missing weights
    d = LlamaDesc()
    d.n_layers, d.hidden, d.n_q_heads, d.n_kv_heads, d.head_dim, d.ffn_dim, d.vocab = 1, 256, 2, 1, 128, 512, 100
    assert lib.ie_engine_create(1, ctypes.byref(d), 1, 128, 16, None, ctypes.byref(out)) == -1
    assert not out.value
    # engine calls on a null engine
    assert lib.ie_engine_decode(None, 1, None) == -1
    assert lib.ie_engine_step(None, None, None) == -1
    # loader: missing file
    from infengine_b200.loader import _bind as bind_loader
    bind_loader()
    arr = (ctypes.c_char_p * 1)(b"/nonexistent/model.safetensors")
    assert lib.ie_llama_load(arr, 1, 1, 1, 0, 128, 1e-5, None, ctypes.byref(out)) == -1
    # world / rank out of range
    assert lib.ie_llama_load(arr, 1, 1, 2, 2, 128, 1e-5, None, ctypes.byref(out)) == -1
