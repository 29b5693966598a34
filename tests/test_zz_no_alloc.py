"""exl3_moe_decode_noalloc: the routed-MoE layer for callers that may not
allocate device memory (code inside CUDA graph capture, hosts whose device
memory belongs to another allocator, callers that cannot take cudaMalloc's
synchronization).  Its scratch is an 8 MiB array compiled into the library.

Called through the C ABI twice in a row (the array keeps the first call's
contents, which the second call must not depend on); each result is compared
with the existing entry point exl3_moe_decode run with a caller-provided
scratch, at the MoE tests' tolerance (fp32 output, max-abs 2e-3).  This file
is collected last on purpose, and passes alone in a fresh process as well.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from dsv4_carve_b200 import _lib, synth

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _layer(dev):
    E, H, I = 16, 1024, 256
    cpu = synth.make_moe_layer(E, H, I, synth.expert_bits(E, 31), seed=31)
    L = synth.MoeLayer(E=E, H=H, I=I, kbits=cpu.kbits, cb=cpu.cb)
    L.experts = [{p: w.to(dev) for p, w in ex.items()} for ex in cpu.experts]
    L.build_tables()
    return L


def _args(L, x, out, ids, w):
    return (x.data_ptr(), _lib.DT_F16, out.data_ptr(), _lib.DT_F32, x.shape[0], L.H, L.I,
            *[t.data_ptr() for t in L.table_list()], L.E, L.ktab.data_ptr(), max(L.kbits), max(L.kbits), L.cb,
            ids.data_ptr(), w.data_ptr(), ids.shape[1], ctypes.c_float(10.0))


def test_noalloc_matches_scratch_entry_point_twice(cuda):
    lib = _lib.load()
    L = _layer(cuda)
    T, topk = 4, 4
    ids, w = synth.route_uniform(T, L.E, topk, seed=32, device=cuda)
    x = synth.activations(T, L.H, seed=33, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream

    ref = torch.empty((T, L.H), dtype=torch.float32, device=cuda)
    scratch = torch.zeros(lib.exl3_moe_scratch_bytes(T, topk, L.H, L.I), dtype=torch.uint8, device=cuda)
    _lib.check(lib.exl3_moe_decode(*_args(L, x, ref, ids, w), scratch.data_ptr(), scratch.numel(), 0, stream))

    for _ in range(2):
        got = torch.full((T, L.H), float("nan"), dtype=torch.float32, device=cuda)
        _lib.check(lib.exl3_moe_decode_noalloc(*_args(L, x, got, ids, w), 0, stream))
        torch.cuda.synchronize(cuda)
        assert torch.isfinite(got).all()
        assert (got - ref).abs().max().item() <= TOL


def test_noalloc_rejects_geometry_beyond_its_maximum(cuda):
    lib = _lib.load()
    need = lib.exl3_moe_scratch_bytes(32, 8, 4096, 2048)
    assert need > _lib.MOE_STATIC_SCRATCH_BYTES
    dummy = torch.zeros(64, dtype=torch.uint8, device=cuda)
    p = dummy.data_ptr()
    rc = lib.exl3_moe_decode_noalloc(p, 0, p, 0, 32, 4096, 2048, *[p] * 9, 256, None, 2, 2, 1, p, p, 8,
                                     ctypes.c_float(10.0), 0, torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == _lib.EXL3_ERR_ARG
    assert "static maximum" in _lib.last_error()
