"""Grouped dense EXL3 linear (one launch, several matrices sharing the input:
exllamav3_ext.exl3_mgemm with a broadcast input,
recipe-lna/exllamav3/exl3_gemm.cu.lna:659-679) on the GPU.

Every output of a group is checked against the oracle's GEMV of its own
matrix at max-abs 2e-3 (fp32 out, unit-scale inputs), and is bit-identical to
the single-matrix entry point on the same matrix (same units, same chunk
count when the widths match, fixed-order sums) where the chunking agrees;
row counts cover the GEMV engine (< 64 rows) and a mixed group where the
tensor-core path takes every matrix (>= 64 rows)."""
from __future__ import annotations

import pytest
import torch

from dsv4_carve_b200 import synth
from dsv4_carve_b200 import vllm_exl3_c as ext
from tests.helpers import dense_np, max_abs, oracle_x

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _group(cuda, oracle, k, ns, K, cb, rows, precise, seed=0, x_dtype=torch.float16):
    ws = [synth.make_dense(k, n, K, seed=seed + 17 * j + n, cb=cb) for j, n in enumerate(ns)]
    x = synth.activations(rows, k, seed=seed + 5, dtype=x_dtype)
    wd = [w.to(cuda) for w in ws]
    ys = ext.linear_group_forward(x.to(cuda), [(w.trellis, w.suh, w.svh) for w in wd], K, cb, torch.float32,
                                  precise)
    torch.cuda.synchronize()
    xa, code = oracle_x(x)
    for j, (w, y) in enumerate(zip(ws, ys)):
        assert tuple(y.shape) == (rows, ns[j])
        want = oracle.gemv(xa, *dense_np(w), K, cb, dtype_code=code, exact=not precise)
        assert max_abs(y.cpu().numpy(), want) <= TOL, (j, max_abs(y.cpu().numpy(), want))
    return x, wd, ys


@pytest.mark.parametrize("rows", [1, 4, 16])
def test_config1_set_in_one_launch(cuda, oracle, rows):
    """q/k/v-like group: [2048 -> 2048], [2048 -> 768], [2048 -> 1024], K6."""
    _group(cuda, oracle, 2048, [2048, 768, 1024], 6, 0, rows, True, seed=rows)


@pytest.mark.parametrize("precise", [True, False])
@pytest.mark.parametrize("K,cb", [(2, 1), (3, 1), (4, 0), (5, 2)])
def test_bit_widths_codebooks(cuda, oracle, K, cb, precise):
    _group(cuda, oracle, 1024, [512, 256, 384, 128], K, cb, 3, precise, seed=K)


def test_eight_matrices_bf16_input(cuda, oracle):
    _group(cuda, oracle, 512, [128, 256, 128, 384, 128, 256, 512, 128], 4, 1, 5, True, x_dtype=torch.bfloat16)


def test_same_as_single_matrix_calls(cuda, oracle):
    """Equal widths: the group's chunking equals each single call's only if the
    chunk count agrees, so compare values at the tolerance and, for a
    one-matrix group, bit for bit."""
    x, wd, ys = _group(cuda, oracle, 1024, [512, 512], 3, 1, 2, True, seed=9)
    for w, y in zip(wd, ys):
        single = ext.linear_forward(x.to(cuda), w.trellis, w.suh, w.svh, 3, 1, torch.float32, True)
        assert max_abs(single.cpu().numpy(), y.cpu().numpy()) <= 1e-4
    one = ext.linear_group_forward(x.to(cuda), [(wd[0].trellis, wd[0].suh, wd[0].svh)], 3, 1, torch.float32, True)
    single = ext.linear_forward(x.to(cuda), wd[0].trellis, wd[0].suh, wd[0].svh, 3, 1, torch.float32, True)
    assert torch.equal(one[0], single)


def test_tensor_core_rows(cuda, oracle):
    """>= 64 rows: every matrix takes the tensor-core path, one after another."""
    _group(cuda, oracle, 1024, [512, 256], 6, 0, 64, True, seed=3)


def test_mgemm_shim_and_repeat(cuda, oracle):
    ws = [synth.make_dense(512, n, 2, seed=50 + n, cb=1) for n in (256, 128)]
    x = synth.activations(4, 512, seed=51)
    wd = [w.to(cuda) for w in ws]
    outs = [ext.exl3_mgemm(x.to(cuda), [w.trellis for w in wd], [w.suh for w in wd], [w.svh for w in wd], 2, True)
            for _ in range(2)]
    for a, b in zip(*outs):
        assert torch.equal(a, b)                      # deterministic across calls (control words restored)
    for w, y in zip(ws, outs[0]):
        assert y.dtype == torch.float32
        assert max_abs(y.cpu().numpy(), oracle.gemv(x.numpy(), *dense_np(w), 2, 1)) <= TOL
