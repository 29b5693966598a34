"""exl3_decode_roof (the decode-issue roof bench.py reports) on the GPU: it
runs, decodes the weight count it reports, and its per-thread sums are
finite and deterministic for the same tile words."""
from __future__ import annotations

import ctypes as C

import pytest
import torch

from dsv4_carve_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("K,cb", [(2, 1), (3, 1), (4, 0), (6, 0)])
def test_decode_roof_runs_and_counts(cuda, K, cb):
    lib = _lib.load()
    g = torch.Generator(device="cpu").manual_seed(K)
    words = torch.randint(-2**31, 2**31 - 1, (32 * 8 * K,), generator=g, dtype=torch.int32).to(cuda)
    nout = int(lib.exl3_decode_roof_out_floats())
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    assert nout == sms * 2 * 256
    outs = []
    for _ in range(2):
        out = torch.empty(nout, dtype=torch.float32, device=cuda)
        n = C.c_int64(0)
        _lib.check(lib.exl3_decode_roof(K, cb, 3, C.c_void_p(words.data_ptr()), words.numel(),
                                        C.c_void_p(out.data_ptr()), out.numel(), C.byref(n),
                                        C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        torch.cuda.synchronize()
        assert n.value == sms * 2 * 8 * 3 * 8 * 256
        assert torch.isfinite(out).all()
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
