"""exl3_moe_decode_noalloc: the routed-MoE layer for callers that cannot
allocate device memory -- a plugin loaded into a serving process whose
device memory belongs to the host's own allocator (it may hand out no buffer
of its own), and latency-critical callers that cannot take cudaMalloc's
implicit device-wide synchronization.  Its scratch is an 8 MiB array compiled
into the library, shared by every call on a device and keeping the previous
call's contents.

Two calls in a row through the C ABI: first a larger geometry (8 rows,
top-8), then a smaller one with different experts, activations and row
count (3 rows, top-4), so that anything the second call wrongly took from
what the first left in the shared array would show.  Each output is compared
with the existing entry point exl3_moe_decode given a fresh caller scratch:
both run the same deterministic kernel (fixed-order sums), so they must agree
bit for bit, which is inside the MoE tests' 2e-3 bound.  This file is
collected last on purpose, and passes alone in a fresh process as well.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from dsv4_carve_b200 import _lib, synth

pytestmark = pytest.mark.gpu


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


def _with_scratch(lib, L, x, ids, w, stream):
    T, topk = ids.shape
    out = torch.empty((T, L.H), dtype=torch.float32, device=x.device)
    scratch = torch.zeros(lib.exl3_moe_scratch_bytes(T, topk, L.H, L.I), dtype=torch.uint8, device=x.device)
    _lib.check(lib.exl3_moe_decode(*_args(L, x, out, ids, w), scratch.data_ptr(), scratch.numel(), 0, stream))
    return out


def test_noalloc_matches_scratch_entry_point_twice(cuda):
    lib = _lib.load()
    L = _layer(cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    calls = [(8, 8, 32), (3, 4, 35)]          # (rows, topk, seed): larger first, then smaller
    for T, topk, seed in calls:
        assert lib.exl3_moe_scratch_bytes(T, topk, L.H, L.I) <= _lib.MOE_STATIC_SCRATCH_BYTES
        ids, w = synth.route_uniform(T, L.E, topk, seed=seed, device=cuda)
        x = synth.activations(T, L.H, seed=seed + 1, device=cuda)
        got = torch.full((T, L.H), float("nan"), dtype=torch.float32, device=cuda)
        _lib.check(lib.exl3_moe_decode_noalloc(*_args(L, x, got, ids, w), 0, stream))
        ref = _with_scratch(lib, L, x, ids, w, stream)
        torch.cuda.synchronize(cuda)
        assert torch.isfinite(got).all()
        assert torch.equal(got, ref), (got - ref).abs().max().item()


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
