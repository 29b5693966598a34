"""GPU trellis decode and full dequant against the oracle, bit for bit.

The device decoder rounds lo + hi to fp16 once (nearest even, as __hadd),
and the full reconstruct keeps the reference's float operation order
(recipe-lna/lna2/bindings.cpp:79-99), so both must equal the oracle exactly.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from dsv4_carve_b200 import _lib, synth
from dsv4_carve_b200 import vllm_exl3_c as ext
from tests.helpers import np16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cb", [0, 1, 2])
@pytest.mark.parametrize("K", range(1, 9))
def test_inner_decode_bitexact(cuda, oracle, K, cb):
    w = synth.make_dense(256, 384, K, seed=100 + 10 * K + cb)
    t = w.trellis.to(cuda)
    got = ext.dequant_trellis(t, w.suh.to(cuda), w.svh.to(cuda), K, True, codebook=cb, inner_only=True)
    want = oracle.decode(np16(w.trellis), K, cb)
    np.testing.assert_array_equal(np16(got).view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("K,cb", [(2, 1), (3, 1), (4, 0), (6, 0), (6, 1), (8, 2), (2, 2)])
def test_full_dequant_bitexact(cuda, oracle, K, cb):
    w = synth.make_dense(256, 512, K, seed=7 + K + cb)
    got = ext.dequant_trellis(w.trellis.to(cuda), w.suh.to(cuda), w.svh.to(cuda), K, True, codebook=cb)
    want = oracle.dequant(np16(w.trellis), np16(w.suh), np16(w.svh), K, cb)
    np.testing.assert_array_equal(np16(got).view(np.uint16), want.view(np.uint16))


def test_reference_codebook_selection(cuda, oracle):
    """mcg=True -> MCG, mcg=False -> MUL1 (bindings.cpp:49)."""
    w = synth.make_dense(128, 128, 3, seed=3)
    a = ext.dequant_trellis(w.trellis.to(cuda), w.suh.to(cuda), w.svh.to(cuda), 3, False)
    want = oracle.dequant(np16(w.trellis), np16(w.suh), np16(w.svh), 3, oracle.CB_MUL1)
    np.testing.assert_array_equal(np16(a).view(np.uint16), want.view(np.uint16))


def test_every_window_value(cuda, oracle):
    """A K=16-equivalent sweep: one tile per 16-bit window value pattern is
    impractical, so decode a trellis whose tiles cover all 65536 windows at
    K=8 (each tile yields 256 windows; 256 tiles with rolling patterns)."""
    K = 8
    rng = np.random.default_rng(0)
    tr = rng.integers(-32768, 32768, size=(16, 32, 16 * K), dtype=np.int16)
    t = torch.from_numpy(tr).to(cuda)
    ones = torch.ones(16 * 32, dtype=torch.float16, device=cuda)
    for cb in (0, 1, 2):
        got = ext.dequant_trellis(t, ones[:256], ones, K, True, codebook=cb, inner_only=True)
        want = oracle.decode(tr, K, cb)
        np.testing.assert_array_equal(np16(got).view(np.uint16), want.view(np.uint16))


def test_library_is_the_native_path(cuda):
    """The ctypes handle is libexl3b200.so from this tree (no fallback)."""
    lib = _lib.load()
    assert _lib.LIB_PATH.name == "libexl3b200.so"
    assert lib.exl3_abi_version() == 2
