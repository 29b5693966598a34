"""The CPU oracle against the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from the reference built from source) and
against the algebraic invariants of the EXL3 format.  No GPU."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

from tests.golden import make_golden as MG

GOLD = Path(__file__).resolve().parent / "golden"


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ----------------------------------------------------------------- pins
@pytest.mark.parametrize("K,mcg", MG.DEQUANT_CASES)
def test_dequant_matches_reference_bitwise(oracle, K, mcg):
    """trunc=True reproduces the reference's dequant_cpu bit for bit
    (recipe-lna/lna2/bindings.cpp:16-101; its half conversion truncates)."""
    g = np.load(GOLD / "ref_dequant.npz")
    t, su, sv = MG.inputs(K, MG.case_seed(K, mcg))
    w = oracle.dequant(t, su, sv, K, oracle.CB_MCG if mcg else oracle.CB_MUL1, trunc=True).view(np.uint16)
    tag = f"K{K}_{'mcg' if mcg else 'mul1'}"
    if f"w_{tag}" in g.files:
        np.testing.assert_array_equal(w, g[f"w_{tag}"])
    assert _sha(w) == str(g[f"sha_{tag}"])


@pytest.mark.parametrize("cb", [0, 1, 2])
def test_codebook_table_matches_reference(oracle, cb):
    g = np.load(GOLD / "ref_codebook.npz")
    assert _sha(oracle.codebook_table(cb, trunc=True)) == str(g[f"sha_cb{cb}"])


def test_codebook_rn_is_the_exact_sum(oracle):
    """The oracle's default (RN) value is the nearest fp16 of the reference's
    exact float sum decode_mcg (exl3_dequant.cuh:95-100), which is what the
    device __hadd returns."""
    g = np.load(GOLD / "ref_codebook.npz")
    wins = g["windows"].astype(np.int64)
    rn = oracle.codebook_table(oracle.CB_MCG)[wins].view(np.float16)
    np.testing.assert_array_equal(rn, g["mcg_float"].astype(np.float16))
    rn1 = oracle.codebook_table(oracle.CB_MUL1)[wins].view(np.float16)
    np.testing.assert_array_equal(rn1, g["mul1_float"].astype(np.float16))


@pytest.mark.parametrize("K", range(1, 9))
def test_windows_match_reference(oracle, K):
    g = np.load(GOLD / "ref_window.npz")
    tiles, want = g[f"tiles_K{K}"], g[f"windows_K{K}"]
    for i in range(tiles.shape[0]):
        got = [oracle.window(tiles[i], K, t) for t in range(256)]
        np.testing.assert_array_equal(np.array(got, dtype=np.uint16), want[i])


@pytest.mark.parametrize("K,mcg,rows", MG.GEMV_CASES)
def test_gemv_form_matches_reference_linear(oracle, K, mcg, rows):
    """GEMV form y = out_T(in_T(x) W') equals the reference's x @ dequant(W)
    (bindings.cpp:135-148) up to the fp16 roundings each side makes."""
    g = np.load(GOLD / "ref_gemv.npz")
    t, su, sv = MG.inputs(K, MG.case_seed(K, mcg) + 500)
    x = MG.gemv_x(rows, t.shape[0] * 16, 4000 + K)
    y = oracle.gemv(x, t, su, sv, K, oracle.CB_MCG if mcg else oracle.CB_MUL1)
    ref = g[f"y_K{K}_{int(mcg)}_{rows}"].view(np.float16).astype(np.float64)
    scale = max(1.0, float(np.abs(ref).max()))
    assert np.abs(y - ref).max() <= 6e-3 * scale


def test_reference_build_still_agrees(oracle):
    """When the reference build is present (oracle/_ref), compare live too."""
    ref = oracle.ref_ext()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    import torch

    t, su, sv = MG.inputs(3, 42, kt=16, nt=8)
    w = ref.dequant_trellis(torch.from_numpy(t), torch.from_numpy(su), torch.from_numpy(sv), 3, True).numpy()
    np.testing.assert_array_equal(oracle.dequant(t, su, sv, 3, oracle.CB_MCG, trunc=True), w)


# ------------------------------------------------------------ invariants
def _hadamard(n: int) -> np.ndarray:
    h = np.array([[1.0]])
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    return h


def test_rn_and_trunc_differ_by_at_most_one_ulp(oracle):
    for cb in (0, 1):
        a = oracle.codebook_table(cb).astype(np.int32)
        b = oracle.codebook_table(cb, trunc=True).astype(np.int32)
        assert np.abs(a - b).max() <= 1


def test_codebook_halves_have_forced_exponents(oracle):
    """(x & 0x8fff8fff) ^ 0x3b603b60 leaves each half with exponent field in
    [14, 15] | [6..] such that lo + hi is exact in fp32."""
    w = np.arange(65536, dtype=np.uint64)
    for mul, add in ((89226354, 64248484), (0xCBAC1FED, 0)):
        x = ((w * mul + add) & 0xFFFFFFFF).astype(np.uint32)
        y = (x & np.uint32(0x8FFF8FFF)) ^ np.uint32(0x3B603B60)
        lo = (y & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float64)
        hi = (y >> 16).astype(np.uint16).view(np.float16).astype(np.float64)
        s = lo + hi
        assert np.all(np.abs(lo) < 2) and np.all(np.abs(hi) < 2)
        assert np.array_equal(s.astype(np.float32).astype(np.float64), s)


def test_decode_layout_matches_reference_swizzle(oracle):
    """exo_decode places lane l, value j at the position bindings.cpp:52-76
    assigns (own/peer lane pairs); restated here independently."""
    K = 3
    t, _, _ = MG.inputs(K, 9, kt=1, nt=1)
    tile = t[0, 0].view(np.uint16)
    vals = [oracle.codebook(oracle.window(tile, K, i), 1) for i in range(256)]
    want = np.zeros((16, 16), dtype=np.uint16)
    for l in range(32):
        if l & 4:
            continue
        row0, col0 = (l % 4) * 2, (l // 8) * 2
        own, peer = vals[8 * l:8 * l + 8], vals[8 * (l + 4):8 * (l + 4) + 8]
        for j, (r, c) in enumerate([(row0, col0), (row0 + 1, col0), (row0 + 8, col0), (row0 + 9, col0),
                                    (row0, col0 + 8), (row0 + 1, col0 + 8), (row0 + 8, col0 + 8),
                                    (row0 + 9, col0 + 8)]):
            want[r, c], want[r, c + 1] = own[j], peer[j]
    np.testing.assert_array_equal(oracle.decode(t, K).view(np.uint16), want)


def test_reconstruct_is_two_sided_hadamard(oracle):
    t, su, sv = MG.inputs(2, 5, kt=8, nt=16)
    wp = oracle.decode(t, 2).astype(np.float64)
    H = _hadamard(128)
    blk = np.kron(np.eye(1), H)
    W = np.zeros_like(wp)
    for r in range(0, 128, 128):
        for c in range(0, 256, 128):
            W[r:r + 128, c:c + 128] = blk @ wp[r:r + 128, c:c + 128] @ blk / 128.0
    W = su.astype(np.float64)[:, None] * W * sv.astype(np.float64)[None, :]
    got = oracle.dequant(t, su, sv, 2).astype(np.float64)
    assert np.abs(got - W).max() <= 2e-3 * np.abs(W).max()


def test_gemv_form_equals_x_times_w(oracle):
    """in/out transforms on activations == multiplying by the reconstructed W."""
    K, k, n = 3, 256, 384
    t, su, sv = MG.inputs(K, 11, kt=k // 16, nt=n // 16)
    x = np.random.default_rng(3).standard_normal((3, k)).astype(np.float16)
    y = oracle.gemv(x, t, su, sv, K)
    W = oracle.dequant(t, su, sv, K).astype(np.float64)
    ref = x.astype(np.float64) @ W
    assert np.abs(y - ref).max() <= 5e-3 * max(1.0, np.abs(ref).max())


def test_moe_oracle_equals_explicit_loop(oracle):
    """exo_moe == the plugin's Python loop semantics restated with oracle.gemv
    (recipe-lna/vllm_exl3_exl3.py.lna:988-1027), including duplicates and
    skipped ids."""
    rng = np.random.default_rng(8)
    E, H, I, T, topk = 6, 256, 128, 3, 3
    kt = [2, 3, 2, 3, 2, 2]
    experts = []
    for e in range(E):
        d = {}
        for p, (k, n) in (("gate", (H, I)), ("up", (H, I)), ("down", (I, H))):
            d[p] = MG.inputs(kt[e], 100 * e + len(p), kt=k // 16, nt=n // 16)
        experts.append(d)
    ids = np.array([[0, 3, 3], [5, -1, 2], [6, 0, 1]], dtype=np.int32)   # dup, -1, out of range
    w = rng.random((T, topk)).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float16)
    out, pairs = oracle.moe(x, experts, kt, ids, w, 10.0)
    want = np.zeros((T, H))
    for r in range(T):
        for s in range(topk):
            e = int(ids[r, s])
            if not 0 <= e < E:
                continue
            g = oracle.gemv(x[r:r + 1], *experts[e]["gate"], kt[e])[0]
            u = oracle.gemv(x[r:r + 1], *experts[e]["up"], kt[e])[0]
            g = np.minimum(g, 10.0)
            u = np.clip(u, -10.0, 10.0)
            a = (g / (1.0 + np.exp(-g)) * u).astype(np.float16)
            d = oracle.gemv(a[None, :], *experts[e]["down"], kt[e])[0]
            want[r] += float(w[r, s]) * d
    np.testing.assert_allclose(out, want, rtol=0, atol=1e-9)
    assert pairs == 6   # (0,r0) (3,r0) (5,r1) (2,r1) (0,r2) (1,r2)


def reference_loop_cases():
    from tests.golden import make_moe_golden as MGL

    return list(MGL.CASES)


def local_ids(ids: np.ndarray, emap: np.ndarray | None, n_local: int) -> np.ndarray:
    """Global ids -> local ids, -1 for every slot the plugin's mapping sends
    to its sentinel (negative, past the map, mapped off this rank, or past the
    local experts)."""
    if emap is not None:
        inside = (ids >= 0) & (ids < emap.size)
        ids = np.where(inside, emap[np.clip(ids, 0, emap.size - 1)], -1)
    return np.where((ids >= 0) & (ids < n_local), ids, -1).astype(np.int32)


@pytest.mark.parametrize("name", reference_loop_cases())
def test_moe_oracle_matches_reference_loop(oracle, name):
    """exo_moe against the reference's own apply_exl3_python_loop
    (recipe-lna/vllm_exl3_exl3.py.lna:988-1027), run unchanged over the
    reference's CPU dequant_trellis + fp32 matmul by
    tests/golden/make_moe_golden.py: duplicates, skipped and unmapped ids, an
    expert map, the SwiGLU clamp, MUL1, bf16 input, one row.  The loop
    multiplies x by the fully reconstructed fp16 W (with the reference's
    truncating fp16 conversion), the oracle runs the GEMV form with
    nearest-even weights, so the two differ by weight rounding only: max-abs
    <= 2e-3 (the bound for outputs on unit-scale inputs) and per-row relative
    <= 4e-3 (measured 2.5e-3 at most, on rows with few valid slots)."""
    from tests.golden import make_moe_golden as MGL
    from tests.helpers import moe_np, row_rel

    fx = np.load(GOLD / "ref_moe_loop.npz")
    layer, x, ids, w, emap = MGL.make_case(name)
    assert MGL.layer_sha(layer) == str(fx[f"{name}_sha"]), "regenerated layer differs from the fixture's"
    assert np.array_equal(ids.numpy(), fx[f"{name}_ids"])
    emap_np = fx[f"{name}_map"] if f"{name}_map" in fx else None
    loc = local_ids(fx[f"{name}_ids"], emap_np, layer.E)
    meta = fx[f"{name}_meta"]
    limit = float(meta[6]) / 1000.0
    code = 1 if int(meta[5]) else 0
    want = fx[f"{name}_out"].astype(np.float64)
    got, _ = oracle.moe(fx[f"{name}_x"], moe_np(layer), layer.kbits, loc, fx[f"{name}_w"], limit, cb=layer.cb,
                        dtype_code=code)
    assert np.abs(got - want).max() <= 2e-3
    assert row_rel(got, want) <= 4e-3
