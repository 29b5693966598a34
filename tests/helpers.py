"""Test helpers: move synthetic layers between torch (product) and numpy
(oracle) and compare results with the tolerances the tests state."""
from __future__ import annotations

import numpy as np
import torch


def np16(t: torch.Tensor) -> np.ndarray:
    """fp16 / bf16 / int16 tensor -> numpy array of the same bits."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float16:
        return t.numpy()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.int16:
        return t.numpy()
    raise TypeError(t.dtype)


def dense_np(w) -> tuple:
    return np16(w.trellis), np16(w.suh), np16(w.svh)


def moe_np(layer) -> list:
    return [{p: dense_np(ex[p]) for p in ("gate", "up", "down")} for ex in layer.experts]


def oracle_x(x: torch.Tensor):
    """Activation tensor -> (numpy array, oracle dtype code or None)."""
    if x.dtype == torch.bfloat16:
        return np16(x), 1
    if x.dtype == torch.float16:
        return np16(x), None
    return x.detach().cpu().float().numpy(), None


def max_abs(a, b) -> float:
    return float(np.abs(np.asarray(a, dtype=np.float64) - np.asarray(b, dtype=np.float64)).max())


def row_rel(got, want) -> float:
    """Largest per-row error relative to that row's largest magnitude (the
    reference's per-row relative gate, recipe-lna/lna2/parity_native.py:48-58)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    worst = 0.0
    for r in range(want.shape[0]):
        scale = max(np.abs(want[r]).max(), 1e-30)
        worst = max(worst, float(np.abs(got[r] - want[r]).max() / scale))
    return worst


def routed_subset(layer, ids) -> tuple:
    """(experts as numpy, their bit widths, ids renumbered into that list)
    for only the experts that `ids` routes to: the oracle then decodes ~30
    experts of a 256-expert layer instead of all of them.  Ids outside the
    layer become -1 (skipped, as in the kernel).  The oracle's result does
    not depend on how experts are numbered: pairs are per (expert, row) and
    the output sums slots in slot order."""
    ids = np.asarray(ids.cpu() if hasattr(ids, "cpu") else ids).astype(np.int64)
    used = sorted({int(e) for e in ids.flatten().tolist() if 0 <= int(e) < layer.E})
    remap = {e: j for j, e in enumerate(used)}
    local = np.vectorize(lambda v: remap.get(int(v), -1), otypes=[np.int32])(ids) if ids.size else ids
    experts = [{p: dense_np(layer.experts[e][p]) for p in ("gate", "up", "down")} for e in used]
    return experts, [int(layer.kbits[e]) for e in used], np.ascontiguousarray(local, dtype=np.int32)
