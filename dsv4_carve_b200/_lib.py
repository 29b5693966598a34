"""ctypes binding of the C-ABI library libexl3b200.so (include/exl3_b200.h).

The library is required: importing a compute entry point without it raises.
There is no CPU fallback anywhere in the product.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("EXL3_B200_LIB", PKG / "libexl3b200.so"))
HEADER = PKG.parent / "include" / "exl3_b200.h"

EXL3_OK, EXL3_ERR_ARG, EXL3_ERR_CUDA, EXL3_ERR_UNSUPPORTED, EXL3_ERR_DEVICE = range(5)
DT_F16, DT_BF16, DT_F32 = 0, 1, 2
CB_3INST, CB_MCG, CB_MUL1 = 0, 1, 2
LINEAR_CTRL_BYTES = 4096
MOE_CTRL_BYTES = 262144
MOE_STATIC_SCRATCH_BYTES = 8 << 20

_P = C.c_void_p
_I64 = C.c_int64
_I = C.c_int

# name -> (restype, argtypes), mirroring include/exl3_b200.h
_SIGS = {
    "exl3_abi_version": (_I, []),
    "exl3_last_error": (C.c_char_p, []),
    "exl3_dequant": (_I, [_P, _I64, _I64, _I, _I, _P, _P, _P, _I, _P]),
    "exl3_linear_scratch_bytes": (_I64, [_I64, _I64, _I64, _I]),
    "exl3_linear": (_I, [_P, _I, _I64, _I64, _I64, _P, _I, _I, _P, _P, _P, _I, _P, _I64, _I, _P]),
    "exl3_linear_group_scratch_bytes": (_I64, [_I64, _I64, _I, _P, _I]),
    "exl3_linear_group": (_I, [_P, _I, _I64, _I64, _I, _P, _P, _I, _I, _P, _P, _P, _I, _P, _I64, _I, _P]),
    "exl3_moe_scratch_bytes": (_I64, [_I64, _I64, _I64, _I64]),
    "exl3_moe_max_rows": (_I64, []),
    "exl3_moe_decode": (_I, [_P, _I, _P, _I, _I64, _I64, _I64] + [_P] * 9
                        + [_I64, _P, _I, _I, _I, _P, _P, _I64, C.c_float, _P, _I64, _I, _P]),
    "exl3_moe_decode_noalloc": (_I, [_P, _I, _P, _I, _I64, _I64, _I64] + [_P] * 9
                                + [_I64, _P, _I, _I, _I, _P, _P, _I64, C.c_float, _I, _P]),
    "exl3_tp_buffer_bytes": (_I64, [_I, _I64, _I64]),
    "exl3_tp_buffer_alloc": (_I, [_I, _I64, _I64, _P]),
    "exl3_tp_buffer_free": (_I, [_P]),
    "exl3_tp_ipc_handle": (_I, [_P, _P]),
    "exl3_tp_ipc_open": (_I, [_P, _P]),
    "exl3_tp_ipc_close": (_I, [_P]),
    "exl3_moe_decode_tp": (_I, [_P, _I, _P, _I, _I64, _I64, _I64] + [_P] * 9
                           + [_I64, _P, _I, _I, _I, _P, _P, _I64, C.c_float, _P, _I64, _I, _P, _I, _I, _I64, _P]),
    "exl3_moe_decode_routed": (_I, [_P, _I, _P, _I, _I64, _I64, _I64] + [_P] * 9
                               + [_I64, _P, _I, _I, _I, _P, _I64, C.c_float, _P, _I64, _I, _P, _I, _I, _I64, _P]),
    "exl3_moe_prefill_routed": (_I, [_P, _I, _P, _I, _I64, _I64, _I64] + [_P] * 9
                                + [_I64, _P, _I, _I, _I, _P, _I64, C.c_float, _P, _I64, _P]),
    "exl3_moe_prefill_scratch_bytes": (_I64, [_I64, _I64, _I64, _I64, _I64]),
    "exl3_moe_prefill_chunk_tokens": (_I64, [_I64]),
    "exl3_moe_prefill": (_I, [_P, _I, _P, _I, _I64, _I64, _I64] + [_P] * 9
                         + [_I64, _P, _I, _I, _I, _P, _P, _I64, C.c_float, _P, _I64, _P]),
    "exl3_moe_prepare": (_I, [_I]),
    "exl3_moe_info": (_I, [_I, _P]),
    "exl3_scratch_status": (_I, [_P, _I, _I, _P, _P]),
    "exl3_decode_roof_out_floats": (_I64, []),
    "exl3_decode_roof": (_I, [_I, _I, _I, _P, _I64, _P, _I64, _P, _P]),
}


class MoeRoute(C.Structure):
    """exl3_moe_route of include/exl3_b200.h."""
    _fields_ = [("ids", C.c_void_p), ("ids_dtype", C.c_int), ("weights", C.c_void_p), ("weights_dtype", C.c_int),
                ("expert_map", C.c_void_p), ("n_global", C.c_int64)]


_lib = None


class Exl3Error(RuntimeError):
    """A C-ABI call returned a non-zero exl3_status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def load() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"exl3 B200 library not found at {LIB_PATH}; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` (no CPU fallback exists)")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def declared_symbols() -> list[str]:
    """Function names declared in include/exl3_b200.h."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(exl3_[a-z0-9_]+)\s*\(", text)))


def last_error() -> str:
    return load().exl3_last_error().decode()


def check(code: int) -> None:
    if code != EXL3_OK:
        raise Exl3Error(code, last_error())


def call(name: str, *args) -> int:
    """Call a status-returning entry point; raise RuntimeError with its message."""
    fn = getattr(load(), name)
    check(fn(*args))
    return 0
