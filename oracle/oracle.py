"""NumPy-facing wrapper of the C oracle (oracle/exl3_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the product.  Arrays are numpy; fp16 and
bf16 data travel as their uint16 bit patterns.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import build_oracle as _b

_lib = None

F16, BF16, F32 = 0, 1, 2
CB_3INST, CB_MCG, CB_MUL1 = 0, 1, 2

_P = C.c_void_p
_I64 = C.c_int64


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = _b.ORACLE_SO
        if not path.exists():
            _b.build_oracle()
        L = C.CDLL(str(path))
        L.exo_window.restype = C.c_uint32
        L.exo_window.argtypes = [_P, C.c_int, C.c_int]
        L.exo_codebook.restype = C.c_uint16
        L.exo_codebook.argtypes = [C.c_uint32, C.c_int, C.c_int]
        L.exo_half_from_double.restype = C.c_uint16
        L.exo_half_from_double.argtypes = [C.c_double]
        L.exo_decode.restype = None
        L.exo_decode.argtypes = [_P, _I64, _I64, C.c_int, C.c_int, C.c_int, _P]
        L.exo_reconstruct.restype = None
        L.exo_reconstruct.argtypes = [_P, _P, _P, _I64, _I64, _P]
        L.exo_input_transform.restype = None
        L.exo_input_transform.argtypes = [_P, C.c_int, _I64, _I64, _P, _P]
        L.exo_gemv.restype = None
        L.exo_gemv.argtypes = [_P, C.c_int, _I64, _P, _P, _P, _I64, _I64, C.c_int, C.c_int, _P]
        L.exo_gemv_ex.restype = None
        L.exo_gemv_ex.argtypes = [_P, C.c_int, _I64, _P, _P, _P, _I64, _I64, C.c_int, C.c_int, C.c_int, _P]
        L.exo_moe.restype = _I64
        L.exo_moe.argtypes = ([_P, C.c_int, _I64, _I64, _I64] + [_P] * 9
                              + [_P, C.c_int, _I64, _P, _P, _I64, C.c_double, _P])
        L.exo_moe_ex.restype = _I64
        L.exo_moe_ex.argtypes = ([_P, C.c_int, _I64, _I64, _I64] + [_P] * 9
                                 + [_P, C.c_int, _I64, _P, _P, _I64, C.c_double, C.c_int, _P])
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def _bits16(a: np.ndarray) -> np.ndarray:
    """fp16 / bf16 / uint16 / int16 array -> contiguous uint16 bit view."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return a.view(np.uint16)
    if a.dtype in (np.uint16, np.int16):
        return a.view(np.uint16)
    raise TypeError(f"expected 16-bit data, got {a.dtype}")


def _act(x: np.ndarray, dtype_code: int | None):
    """Activation array -> (contiguous array, dtype code)."""
    x = np.ascontiguousarray(x)
    if x.dtype == np.float16:
        return x.view(np.uint16), F16
    if x.dtype == np.float32:
        return x, F32
    if x.dtype == np.uint16 and dtype_code in (F16, BF16):
        return x, dtype_code
    raise TypeError("x must be float16, float32, or uint16 bits with dtype_code")


def window(tile: np.ndarray, K: int, t: int) -> int:
    tile = _bits16(tile)
    return int(lib().exo_window(_ptr(tile), K, t))


def codebook(window_value: int, cb: int, trunc: bool = False) -> int:
    return int(lib().exo_codebook(window_value, cb, int(trunc)))


def codebook_table(cb: int, trunc: bool = False) -> np.ndarray:
    """fp16 bits of the codebook value of every 16-bit window (65536 entries)."""
    L = lib()
    return np.array([L.exo_codebook(w, cb, int(trunc)) for w in range(65536)], dtype=np.uint16)


def decode(trellis: np.ndarray, K: int, cb: int = CB_MCG, trunc: bool = False) -> np.ndarray:
    """Packed trellis [k/16, n/16, 16K] -> W' [k, n] float16 (inner weights)."""
    t = _bits16(trellis)
    kt, nt, last = t.shape
    assert last == 16 * K
    out = np.empty((kt * 16, nt * 16), dtype=np.uint16)
    lib().exo_decode(_ptr(t), kt, nt, K, cb, int(trunc), _ptr(out))
    return out.view(np.float16)


def reconstruct(wprime: np.ndarray, suh: np.ndarray, svh: np.ndarray) -> np.ndarray:
    """W = diag(suh) H W' H diag(svh) / 128 -> float16, reference float order."""
    wp = _bits16(wprime)
    k, n = wp.shape
    out = np.empty((k, n), dtype=np.uint16)
    lib().exo_reconstruct(_ptr(wp), _ptr(_bits16(suh)), _ptr(_bits16(svh)), k, n, _ptr(out))
    return out.view(np.float16)


def dequant(trellis, suh, svh, K: int, cb: int = CB_MCG, trunc: bool = False) -> np.ndarray:
    return reconstruct(decode(trellis, K, cb, trunc), suh, svh)


def input_transform(x: np.ndarray, suh: np.ndarray, dtype_code: int | None = None) -> np.ndarray:
    xa, code = _act(x, dtype_code)
    R, k = xa.shape
    out = np.empty((R, k), dtype=np.uint16)
    lib().exo_input_transform(_ptr(xa), code, R, k, _ptr(_bits16(suh)), _ptr(out))
    return out.view(np.float16)


def gemv(x: np.ndarray, trellis: np.ndarray, suh: np.ndarray, svh: np.ndarray, K: int,
         cb: int = CB_MCG, dtype_code: int | None = None, exact: bool = False) -> np.ndarray:
    """Dense EXL3 linear in GEMV form; returns float64 [R, n].

    exact=False multiplies by the fp16-rounded weights (the reference's
    decoder); exact=True by lo + hi unrounded (the fast kernel path)."""
    xa, code = _act(x, dtype_code)
    R, k = xa.shape
    t = _bits16(trellis)
    n = t.shape[1] * 16
    y = np.empty((R, n), dtype=np.float64)
    lib().exo_gemv_ex(_ptr(xa), code, R, _ptr(t), _ptr(_bits16(suh)), _ptr(_bits16(svh)), k, n, K, cb,
                      int(exact), _ptr(y))
    return y


def moe(x: np.ndarray, experts: list[dict], Ktab, ids: np.ndarray, weights: np.ndarray,
        limit: float, cb: int = CB_MCG, dtype_code: int | None = None, exact: bool = False):
    """Routed-MoE decode layer.  experts[e] has keys gate/up/down -> (trellis, suh, svh).

    Returns (out float64 [T, H], number of unique (expert,row) pairs).
    """
    xa, code = _act(x, dtype_code)
    T, H = xa.shape
    E = len(experts)
    I = experts[0]["gate"][0].shape[1] * 16
    keep = []

    def table(proj, idx):
        arrs = [_bits16(experts[e][proj][idx]) for e in range(E)]
        keep.extend(arrs)
        return (C.c_void_p * E)(*[a.ctypes.data for a in arrs])

    tabs = [table(p, i) for p in ("gate", "up", "down") for i in range(3)]
    ktab = np.ascontiguousarray(np.asarray(Ktab, dtype=np.int32))
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    weights = np.ascontiguousarray(weights, dtype=np.float32)
    topk = ids.shape[1]
    out = np.empty((T, H), dtype=np.float64)
    pairs = lib().exo_moe_ex(_ptr(xa), code, T, H, I, *[C.cast(t, C.c_void_p) for t in tabs],
                             _ptr(ktab), cb, E, _ptr(ids), _ptr(weights), topk, float(limit), int(exact),
                             _ptr(out))
    return out, int(pairs)


# ---------------------------------------------------------------- reference pins

_ref = None


def ref_pin_lib():
    """ctypes handle on the reference's own host helpers (oracle/_ref), or None."""
    global _ref
    if _ref is None:
        path = _b.REF_PIN_SO
        if not path.exists():
            return None
        L = C.CDLL(str(path))
        L.ref_read_window.restype = C.c_uint16
        L.ref_read_window.argtypes = [_P, C.c_size_t, C.c_size_t]
        L.ref_decode_codebook_bits.restype = C.c_uint16
        L.ref_decode_codebook_bits.argtypes = [C.c_uint16, C.c_int]
        L.ref_decode_mcg.restype = C.c_float
        L.ref_decode_mcg.argtypes = [C.c_uint16]
        L.ref_decode_mul1.restype = C.c_float
        L.ref_decode_mul1.argtypes = [C.c_uint16]
        L.ref_decode_weight.restype = C.c_float
        L.ref_decode_weight.argtypes = [_P, C.c_size_t, C.c_int, C.c_int, C.c_int]
        L.ref_hadamard.restype = None
        L.ref_hadamard.argtypes = [_P, C.c_int]
        _ref = L
    return _ref


def ref_ext():
    """The reference's bindings.cpp built CPU-only (module vllm_exl3_c_ref), or None."""
    import importlib.util
    import sys

    path = _b.ref_ext_path()
    if not path.exists():
        return None
    if _b.REF_EXT_NAME in sys.modules:
        return sys.modules[_b.REF_EXT_NAME]
    import torch  # noqa: F401  (libtorch must be loaded first)

    spec = importlib.util.spec_from_file_location(_b.REF_EXT_NAME, str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[_b.REF_EXT_NAME] = mod
    return mod
