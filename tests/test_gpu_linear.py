"""Dense EXL3 linear (GEMV form) on the GPU against the oracle.

Tolerance: max-abs error <= 2e-3 against the oracle's
fp64 result on unit-scale inputs, fp32 output.  fp16 / bf16 outputs add one
rounding of the output: per-row relative <= 2e-3 (fp16) / 6e-3 (bf16), the
reference's own gates (recipe-lna/lna2/parity_native.py:48-58).

precise=True multiplies by the fp16-rounded weights the reference decodes and
is compared with the oracle in that mode.  precise=False (the fast path)
multiplies by lo + hi unrounded: it is compared at max-abs 2e-3 with the
oracle in the same arithmetic (exact=True), and separately bounded against
the fp16-rounded reference by the reference's per-row relative gate.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from dsv4_carve_b200 import synth
from dsv4_carve_b200 import vllm_exl3_c as ext
from dsv4_carve_b200.linear import LinearEXL3
from tests.helpers import dense_np, max_abs, oracle_x, row_rel

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _run(cuda, oracle, k, n, K, cb, rows, precise, x_dtype=torch.float16, out_dtype=torch.float32, seed=0):
    w = synth.make_dense(k, n, K, seed=seed + 31 * K + n, cb=cb)
    x = synth.activations(rows, k, seed=seed + 7, dtype=x_dtype)
    wd = w.to(cuda)
    y = ext.linear_forward(x.to(cuda), wd.trellis, wd.suh, wd.svh, K, cb, out_dtype, precise)
    xa, code = oracle_x(x)
    want = oracle.gemv(xa, *dense_np(w), K, cb, dtype_code=code, exact=not precise)
    return y.float().cpu().numpy(), want


@pytest.mark.parametrize("precise", [True, False])
def test_config0_4096x4096_k4_3inst(cuda, oracle, precise):
    got, want = _run(cuda, oracle, 4096, 4096, 4, 0, 1, precise)
    assert max_abs(got, want) <= TOL


def test_fast_path_against_rounded_reference(cuda, oracle):
    """The fast path's distance from the fp16-rounded reference weights is
    the weights' own rounding: per-row relative <= 2e-3."""
    w = synth.make_dense(4096, 4096, 4, seed=3, cb=0)
    x = synth.activations(4, 4096, seed=4)
    wd = w.to(cuda)
    y = ext.linear_forward(x.to(cuda), wd.trellis, wd.suh, wd.svh, 4, 0, torch.float32, precise=False)
    want = oracle.gemv(x.numpy(), *dense_np(w), 4, 0)
    assert row_rel(y.cpu().numpy(), want) <= 2e-3


@pytest.mark.parametrize("rows", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("k,n", [(4096, 4096), (4096, 1536), (1536, 4096)])
def test_config1_k6(cuda, oracle, k, n, rows):
    got, want = _run(cuda, oracle, k, n, 6, 0, rows, True, seed=rows)
    assert max_abs(got, want) <= TOL


@pytest.mark.parametrize("K", [1, 2, 3, 5, 7, 8])
@pytest.mark.parametrize("cb", [1, 2])
def test_other_bit_widths(cuda, oracle, K, cb):
    got, want = _run(cuda, oracle, 1024, 512, K, cb, 3, K % 2 == 0)
    assert max_abs(got, want) <= TOL


@pytest.mark.parametrize("rows", [9, 32, 33, 70])
def test_row_blocks(cuda, oracle, rows):
    got, want = _run(cuda, oracle, 512, 384, 3, 1, rows, False)
    assert max_abs(got, want) <= TOL


def test_fp16_and_bf16_io(cuda, oracle):
    got, want = _run(cuda, oracle, 2048, 1024, 6, 1, 4, True, out_dtype=torch.float16)
    assert row_rel(got, want) <= 2e-3
    got, want = _run(cuda, oracle, 2048, 1024, 6, 1, 4, True, x_dtype=torch.bfloat16, out_dtype=torch.bfloat16)
    assert row_rel(got, want) <= 6e-3


def test_zero_input_gives_zero(cuda):
    w = synth.make_dense(512, 256, 4, seed=1).to(cuda)
    x = torch.zeros((2, 512), dtype=torch.float16, device=cuda)
    y = ext.linear_forward(x, w.trellis, w.suh, w.svh, 4, 1, torch.float32)
    assert torch.count_nonzero(y).item() == 0


def test_bitwise_deterministic(cuda):
    w = synth.make_dense(4096, 1536, 6, seed=5).to(cuda)
    x = synth.activations(8, 4096, seed=9, device=cuda)
    a = ext.linear_forward(x, w.trellis, w.suh, w.svh, 6, 1, torch.float32)
    b = ext.linear_forward(x, w.trellis, w.suh, w.svh, 6, 1, torch.float32)
    assert torch.equal(a, b)


def test_reference_entry_points(cuda, oracle):
    """exl3_gemv / exl3_gemm with the reference's positional signature."""
    w = synth.make_dense(1024, 512, 3, seed=12, cb=1)
    x = synth.activations(4, 1024, seed=2)
    wd = w.to(cuda)
    y1 = ext.exl3_gemv(x.to(cuda), wd.trellis, wd.suh, wd.svh, 3, True, 1)
    y2 = ext.exl3_gemm(x.to(cuda).view(2, 2, 1024), wd.trellis, wd.suh, wd.svh, 3, True)
    want = oracle.gemv(x.numpy(), *dense_np(w), 3, 1)
    assert y1.dtype == torch.float16 and y2.shape == (4, 512)   # bindings.cpp:104-109 flattens rows
    assert row_rel(y1.float().cpu().numpy(), want) <= 2e-3
    assert torch.equal(y1, y2)


def test_linear_exl3_class(cuda, oracle):
    w = synth.make_dense(1024, 768 - 640 + 640, 6, seed=3, cb=0)
    wd = w.to(cuda)
    lin = LinearEXL3(None, 1024, w.out_features, suh=wd.suh, svh=wd.svh, trellis=wd.trellis)
    x = synth.activations(5, 1024, seed=4)
    y = lin.forward(x.to(cuda), {}, out_dtype=torch.float32)
    want = oracle.gemv(x.numpy(), *dense_np(w), 6, 0)
    assert max_abs(y.cpu().numpy(), want) <= TOL
    full = lin.get_weight_tensor()
    want_w = oracle.dequant(*dense_np(w), 6, 0)
    np.testing.assert_array_equal(full.cpu().numpy().view(np.uint16), want_w.view(np.uint16))


def test_status_word_clean(cuda):
    w = synth.make_dense(1024, 512, 4, seed=1).to(cuda)
    x = synth.activations(3, 1024, seed=1, device=cuda)
    ext.linear_forward(x, w.trellis, w.suh, w.svh, 4, 1, torch.float32)
    scratch = ext._linear_scratch(cuda, 0)
    import ctypes

    from dsv4_carve_b200 import _lib

    word = ctypes.c_uint32(7)
    _lib.call("exl3_scratch_status", scratch.data_ptr(), 0, 0, ctypes.addressof(word),
              torch.cuda.current_stream().cuda_stream)
    assert word.value == 0


@pytest.mark.parametrize("rows", [64, 130, 256, 300, 512, 600])
@pytest.mark.parametrize("K,cb", [(2, 1), (6, 0)])
def test_tensor_core_rows(cuda, oracle, rows, K, cb):
    """64 rows or more go through the tcgen05 path (weights rounded to fp16 as
    the reference decodes them, fp32 accumulation in tensor memory).  130 and
    300 rows end inside an MMA N block; 300 and 512 use the second
    accumulator; 600 takes two 512-row passes."""
    got, want = _run(cuda, oracle, 1024, 512, K, cb, rows, True, seed=rows)
    assert max_abs(got, want) <= TOL


def test_tensor_core_single_chunk_and_repeat(cuda, oracle):
    """A 128-column, 256-k matrix is one strip of one k-chunk (no partial
    sum); the split-k case (1024 x 512) run twice gives bitwise the same
    result, so the strip counters are left zero between calls."""
    got, want = _run(cuda, oracle, 256, 128, 4, 1, 96, True)
    assert max_abs(got, want) <= TOL
    w = synth.make_dense(1024, 512, 5, seed=8, cb=0).to(cuda)
    x = synth.activations(200, 1024, seed=9, device=cuda)
    a = ext.linear_forward(x, w.trellis, w.suh, w.svh, 5, 0, torch.float32)
    b = ext.linear_forward(x, w.trellis, w.suh, w.svh, 5, 0, torch.float32)
    assert torch.equal(a, b)


def test_tensor_core_config1_shape(cuda, oracle):
    """A prefill-sized block through the tensor cores at the config-1 shape."""
    got, want = _run(cuda, oracle, 4096, 4096, 6, 0, 128, True)
    assert max_abs(got, want) <= TOL
