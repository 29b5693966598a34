"""The C-ABI library: it loads, exports every entry point include/exl3_b200.h
declares, and rejects bad arguments on the host with a status code and a
message before any CUDA call (so these run without a GPU)."""
from __future__ import annotations

import ctypes as C

import pytest

from dsv4_carve_b200 import _lib


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _lib.declared_symbols()
    assert len(declared) >= 11
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/exl3_b200.h but not exported"
    assert set(declared) == set(_lib._SIGS), "ctypes signature table out of sync with the header"


def test_abi_version():
    assert _lib.load().exl3_abi_version() == 2


def test_scratch_size_queries_are_host_only():
    lib = _lib.load()
    assert lib.exl3_moe_max_rows() == 32
    a = lib.exl3_moe_scratch_bytes(4, 8, 4096, 2048)
    b = lib.exl3_moe_scratch_bytes(16, 8, 4096, 2048)
    assert _lib.MOE_CTRL_BYTES < a < b
    assert lib.exl3_moe_scratch_bytes(0, 8, 4096, 2048) == -1
    assert lib.exl3_linear_scratch_bytes(4, 4096, 4096, 6) >= _lib.LINEAR_CTRL_BYTES
    assert lib.exl3_linear_scratch_bytes(4, 100, 4096, 6) == -1


def _err(code: int, fragment: str):
    assert code == _lib.EXL3_ERR_ARG or code == _lib.EXL3_ERR_UNSUPPORTED
    assert fragment in _lib.last_error()


def test_linear_argument_checks():
    lib = _lib.load()
    buf = (C.c_uint8 * 64)()
    p = C.addressof(buf)
    _err(lib.exl3_linear(None, 0, 1, 128, 128, p, 2, 1, p, p, p, 0, p, 64, 1, None), "null pointer")
    _err(lib.exl3_linear(p, 0, 0, 128, 128, p, 2, 1, p, p, p, 0, p, 64, 1, None), "rows must be")
    _err(lib.exl3_linear(p, 0, 1, 100, 128, p, 2, 1, p, p, p, 0, p, 64, 1, None), "multiples of 128")
    _err(lib.exl3_linear(p, 0, 1, 128, 128, p, 9, 1, p, p, p, 0, p, 64, 1, None), "K must be")
    _err(lib.exl3_linear(p, 0, 1, 128, 128, p, 2, 5, p, p, p, 0, p, 64, 1, None), "codebook")
    _err(lib.exl3_linear(p, 7, 1, 128, 128, p, 2, 1, p, p, p, 0, p, 64, 1, None), "dtype")
    _err(lib.exl3_linear(p, 0, 1, 128, 128, p + 2, 2, 1, p, p, p, 0, p, 64, 1, None), "16-byte aligned")


def test_dequant_argument_checks():
    lib = _lib.load()
    buf = (C.c_uint8 * 64)()
    p = C.addressof(buf)
    _err(lib.exl3_dequant(None, 8, 8, 2, 1, p, p, p, 1, None), "null")
    _err(lib.exl3_dequant(p, 8, 8, 0, 1, p, p, p, 1, None), "K must be")
    _err(lib.exl3_dequant(p, 8, 8, 2, 3, p, p, p, 1, None), "codebook")
    _err(lib.exl3_dequant(p, 4, 8, 2, 1, p, p, p, 1, None), "Hadamard")
    _err(lib.exl3_dequant(p, 8, 8, 2, 1, None, p, p, 1, None), "suh and svh")


def test_moe_argument_checks():
    lib = _lib.load()
    buf = (C.c_uint8 * 64)()
    p = C.addressof(buf)
    tabs = [p] * 9

    def call(m=4, H=4096, I=256, E=256, ktab=None, K=2, kmax=2, cb=1, topk=8, limit=10.0, scratch_bytes=1 << 30,
             x=p, tables=tabs, scratch=p):
        return lib.exl3_moe_decode(x, 0, p, 0, m, H, I, *tables, E, ktab, K, kmax, cb, p, p, topk,
                                   C.c_float(limit), scratch, scratch_bytes, 0, None)

    _err(call(x=None), "null pointer")
    _err(call(tables=[p] * 8 + [None]), "null pointer table 8")
    _err(call(m=0), "row count")
    _err(call(m=33), "row count")
    _err(call(topk=17), "topk")
    _err(call(m=32, topk=9), "topk")
    _err(call(E=0), "expert count")
    _err(call(H=4000), "hidden")
    _err(call(I=100), "intermediate")
    _err(call(K=5), "K must be")
    _err(call(ktab=p, kmax=6), "kmax")
    _err(call(limit=0.0), "SwiGLU")
    _err(call(limit=float("inf")), "SwiGLU")
    _err(call(scratch=p + 4), "16-byte aligned")
    _err(call(scratch_bytes=1024), "scratch too small")


def test_moe_prefill_argument_checks_and_sizes():
    lib = _lib.load()
    buf = (C.c_uint8 * 64)()
    p = C.addressof(buf)
    tabs = [p] * 9

    def call(m=512, H=4096, I=256, E=256, ktab=None, K=2, kmax=2, cb=1, topk=8, limit=10.0,
             scratch_bytes=1 << 40, x=p, tables=tabs, scratch=p, x_dtype=0):
        return lib.exl3_moe_prefill(x, x_dtype, p, 0, m, H, I, *tables, E, ktab, K, kmax, cb, p, p, topk,
                                    C.c_float(limit), scratch, scratch_bytes, None)

    _err(call(x=None), "null pointer")
    _err(call(tables=[p] * 8 + [None]), "null pointer table")
    _err(call(m=0), "m must be")
    _err(call(topk=17), "topk")
    _err(call(E=0), "n_experts")
    _err(call(E=1025), "n_experts")
    _err(call(H=4000), "multiples of 128")
    _err(call(kmax=5), "kmax")
    _err(call(K=3, kmax=2), "K must be")
    _err(call(cb=3), "codebook")
    _err(call(x_dtype=2), "fp16/bf16")
    _err(call(limit=0.0), "swiglu_limit")
    _err(call(scratch=p + 4), "16-byte aligned")
    _err(call(scratch_bytes=1024), "scratch too small")
    # sizes: one chunk of at most 2048 tokens at 256 experts, 512 at 1024
    assert lib.exl3_moe_prefill_chunk_tokens(256) == 2048
    assert lib.exl3_moe_prefill_chunk_tokens(1024) == 512
    assert lib.exl3_moe_prefill_chunk_tokens(0) == -1
    a = lib.exl3_moe_prefill_scratch_bytes(512, 8, 4096, 2048, 256)
    b = lib.exl3_moe_prefill_scratch_bytes(4096, 8, 4096, 2048, 256)
    c = lib.exl3_moe_prefill_scratch_bytes(2048, 8, 4096, 2048, 256)
    assert 0 < a < b and b == c
    assert lib.exl3_moe_prefill_scratch_bytes(512, 17, 4096, 2048, 256) == -1


def test_status_word_checks():
    lib = _lib.load()
    _err(lib.exl3_scratch_status(None, 1, 0, None, None), "null")


def test_python_layer_raises_without_cuda_tensors():
    import torch

    from dsv4_carve_b200 import vllm_exl3_c as ext

    t = torch.zeros((8, 8, 32), dtype=torch.int16)
    su = torch.ones(128, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ext.dequant_trellis(t, su, su, 2, True)
    with pytest.raises(RuntimeError, match="K must be"):
        ext.dequant_trellis(t, su, su, 9, True)
    x = torch.zeros((1, 128), dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ext.exl3_gemv(x, t, su, su, 2, True)
    with pytest.raises(RuntimeError, match="1 <= m <= 8"):
        ext.exl3_gemv(torch.zeros((9, 128), dtype=torch.float16), t, su, su, 2, True)


def test_decode_roof_argument_checks():
    lib = _lib.load()
    n = C.c_int64(0)
    buf = C.c_void_p(16)
    for K, cb, iters in ((0, 1, 1), (9, 1, 1), (2, 2, 1), (2, 1, 0)):
        assert lib.exl3_decode_roof(K, cb, iters, buf, 4096, buf, 1 << 20, C.byref(n), None) == _lib.EXL3_ERR_ARG
    assert lib.exl3_decode_roof(2, 1, 1, None, 4096, buf, 1 << 20, C.byref(n), None) == _lib.EXL3_ERR_ARG
    # too few tile words for K = 3 (32 tiles x 24 words)
    assert lib.exl3_decode_roof(3, 1, 1, buf, 767, buf, 1 << 20, C.byref(n), None) == _lib.EXL3_ERR_ARG
    assert "words" in _lib.last_error()


def test_linear_group_argument_checks():
    lib = _lib.load()
    buf = (C.c_uint8 * 64)()
    p = C.addressof(buf)
    ptr = lambda *v: (C.c_void_p * len(v))(*v)   # noqa: E731
    n2 = (C.c_int64 * 2)(128, 256)
    t2, s2 = ptr(p, p), ptr(p, p)

    def call(nmat=2, n=n2, t=t2, rows=1, k=128, K=2, cb=1, x=p, scratch_bytes=1 << 30):
        return lib.exl3_linear_group(x, 0, rows, k, nmat, n, t, K, cb, s2, s2, s2, 0, p, scratch_bytes, 1, None)

    _err(call(x=None), "null pointer")
    _err(call(nmat=0), "1 to 8 matrices")
    _err(call(nmat=9), "1 to 8 matrices")
    _err(call(rows=0), "rows must be")
    _err(call(k=100), "multiples of 128")
    _err(call(n=(C.c_int64 * 2)(128, 200)), "matrix 1")
    _err(call(t=ptr(p, p + 2)), "16-byte aligned")
    _err(call(t=ptr(p, None)), "matrix 1")
    _err(call(K=0), "K must be")
    _err(call(scratch_bytes=64), "scratch too small")
    assert lib.exl3_linear_group_scratch_bytes(4, 1024, 2, n2, 3) > _lib.LINEAR_CTRL_BYTES
    assert lib.exl3_linear_group_scratch_bytes(4, 1024, 9, n2, 3) == -1
    assert lib.exl3_linear_group_scratch_bytes(4, 1024, 2, (C.c_int64 * 2)(128, 100), 3) == -1
    one = (C.c_int64 * 1)(4096)
    assert lib.exl3_linear_group_scratch_bytes(4, 4096, 1, one, 6) == lib.exl3_linear_scratch_bytes(4, 4096, 4096, 6)
