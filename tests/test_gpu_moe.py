"""Routed-MoE decode layer on the GPU against the oracle.

Mirrors the reference's parity suite (recipe-lna/lna2/parity_native.py):
route profiles unique / hot / zipf / within-row duplicates / invalid ids /
boundary rows, inputs zero / unit / amplified past the SwiGLU clamp,
bitwise determinism over two runs, NaN-poisoned scratch replay, and the
device status word.  Tolerances: fp32 output max-abs <= 2e-3 against the
oracle's fp64 result on unit-scale inputs and per-row relative <= 2e-3.
The fast path (precise=False, lo + hi unrounded in the MMA) is compared with
the oracle in the same arithmetic (exact=True); precise=True with the
fp16-rounded reference weights.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from dsv4_carve_b200 import moe as M
from dsv4_carve_b200 import synth
from dsv4_carve_b200 import vllm_exl3_c as ext
from tests.helpers import max_abs, moe_np, oracle_x, row_rel

pytestmark = pytest.mark.gpu

TOL = 2e-3
M_CTRL = 262144   # EXL3_MOE_CTRL_BYTES
_LAYERS: dict = {}


def layer(E, H, I, kbits, seed, cb=1, device="cpu"):
    key = (E, H, I, tuple(kbits), seed, cb)
    if key not in _LAYERS:
        cpu = synth.make_moe_layer(E, H, I, kbits, seed, device="cpu", cb=cb)
        _LAYERS[key] = cpu
    return _LAYERS[key]


def to_device(cpu_layer, dev):
    L = synth.MoeLayer(E=cpu_layer.E, H=cpu_layer.H, I=cpu_layer.I, kbits=cpu_layer.kbits, cb=cpu_layer.cb)
    L.experts = [{p: w.to(dev) for p, w in ex.items()} for ex in cpu_layer.experts]
    L.build_tables()
    return L


def run_kernel(L, x, ids, w, limit=10.0, out_dtype=torch.float32, precise=False, scratch=None, kscalar=None):
    dev = L.ktab.device
    T, topk = ids.shape
    if scratch is None:
        scratch = torch.zeros(ext.lna2_moe_scratch_bytes(T, topk, L.H, L.I), dtype=torch.uint8, device=dev)
    out = torch.empty((T, L.H), dtype=out_dtype, device=dev)
    ktab = None if kscalar else L.ktab
    K = kscalar or max(L.kbits)
    ext.lna2_moe_decode(x.to(dev), out, *L.table_list(), ids.to(dev), w.to(dev), K, limit, scratch,
                        intermediate=L.I, k_table=ktab, codebook=L.cb, precise=precise)
    return out, scratch


def run_oracle(oracle, L, x, ids, w, limit=10.0, exact=True):
    xa, code = oracle_x(x)
    return oracle.moe(xa, moe_np(L), L.kbits, ids.numpy(), w.numpy(), limit, cb=L.cb, dtype_code=code,
                      exact=exact)


def check(got, want):
    got = got.float().cpu().numpy()
    assert max_abs(got, want) <= TOL, max_abs(got, want)
    assert row_rel(got, want) <= 2e-3


@pytest.mark.parametrize("cb", [1, 0])
@pytest.mark.parametrize("precise", [False, True])
def test_small_mixed_k(cuda, oracle, cb, precise):
    E, H, I, T, topk = 16, 1024, 256, 4, 4
    L0 = layer(E, H, I, synth.expert_bits(E, 3), 3, cb=cb)
    ids, w = synth.route_uniform(T, E, topk, seed=5)
    x = synth.activations(T, H, seed=6)
    got, scratch = run_kernel(to_device(L0, cuda), x, ids, w, precise=precise)
    want, _ = run_oracle(oracle, L0, x, ids, w, exact=not precise)
    check(got, want)
    assert ext.lna2_moe_status(scratch) == 0
    if not precise:
        rounded, _ = run_oracle(oracle, L0, x, ids, w, exact=False)
        assert row_rel(got.cpu().numpy(), rounded) <= 2e-3


@pytest.mark.parametrize("profile", ["unique", "hot", "zipf", "dup", "invalid", "single"])
def test_route_profiles(cuda, oracle, profile):
    E, H, I, topk = 32, 512, 256, 8
    T = 16 if profile != "single" else 1
    L0 = layer(E, H, I, synth.expert_bits(E, 11), 11)
    rng = np.random.default_rng(sum(map(ord, profile)))
    if profile == "zipf":
        ids, w = synth.route_zipf(T, E, topk, seed=3)
    else:
        ids, w = synth.route_uniform(T, E, topk, seed=4)
        ids = ids.clone()
        if profile == "unique":
            ids = torch.arange(T * topk, dtype=torch.int32).view(T, topk) % E
        elif profile == "hot":
            ids[:, 0] = 7
            ids[:, 1] = 9
        elif profile == "dup":
            ids[:, 1] = ids[:, 0]
        elif profile == "invalid":
            ids[0, 2] = -1
            ids[1, 3] = E
            ids[2, :] = -5
        ids = ids.contiguous()
    x = synth.activations(T, H, seed=int(rng.integers(100)))
    got, _ = run_kernel(to_device(L0, cuda), x, ids, w)
    want, _ = run_oracle(oracle, L0, x, ids, w)
    check(got, want)


def test_all_ids_invalid_gives_zero(cuda):
    L = to_device(layer(8, 256, 128, [2] * 8, 1), cuda)
    ids = torch.full((3, 2), -1, dtype=torch.int32)
    w = torch.ones((3, 2), dtype=torch.float32)
    x = synth.activations(3, 256, seed=1)
    got, scratch = run_kernel(L, x, ids, w, out_dtype=torch.float16)
    assert torch.count_nonzero(got).item() == 0
    assert ext.lna2_moe_status(scratch) == 0


@pytest.mark.parametrize("scale,limit", [(0.0, 10.0), (8.0, 10.0), (8.0, 1.0)])
def test_inputs_and_clamp(cuda, oracle, scale, limit):
    E, H, I, T, topk = 8, 512, 128, 4, 3
    L0 = layer(E, H, I, [2, 3] * 4, 21)
    ids, w = synth.route_uniform(T, E, topk, seed=2)
    x = synth.activations(T, H, seed=8, scale=scale)
    got, _ = run_kernel(to_device(L0, cuda), x, ids, w, limit=limit)
    want, _ = run_oracle(oracle, L0, x, ids, w, limit=limit)
    got = got.cpu().numpy()
    s = max(1.0, float(np.abs(want).max()))
    assert max_abs(got, want) <= TOL * s


def test_bf16_in_bf16_out(cuda, oracle):
    E, H, I, T, topk = 16, 1024, 256, 4, 6
    L0 = layer(E, H, I, synth.expert_bits(E, 4), 4)
    ids, w = synth.route_uniform(T, E, topk, seed=1)
    x = synth.activations(T, H, seed=2, dtype=torch.bfloat16)
    got, _ = run_kernel(to_device(L0, cuda), x, ids, w, out_dtype=torch.bfloat16)
    want, _ = run_oracle(oracle, L0, x, ids, w)
    assert row_rel(got.float().cpu().numpy(), want) <= 6e-3


def test_max_rows_and_scalar_k(cuda, oracle):
    """32 rows (the build's ceiling), topk 8, the reference's scalar-K ABI."""
    E, H, I, T, topk = 64, 512, 256, 32, 8
    L0 = layer(E, H, I, [3] * E, 9)
    ids, w = synth.route_uniform(T, E, topk, seed=6)
    x = synth.activations(T, H, seed=7)
    got, _ = run_kernel(to_device(L0, cuda), x, ids, w, kscalar=3)
    want, _ = run_oracle(oracle, L0, x, ids, w)
    check(got, want)


def test_config2_shape_tp8(cuda, oracle):
    """Config 2 at its TP8 shard: 256 experts, hidden 4096, I_local 256,
    T = 4, top-8, K in {2, 3}."""
    E, H, I, T, topk = 256, 4096, 256, 4, 8
    L0 = layer(E, H, I, synth.expert_bits(E, 2), 2)
    ids, w = synth.route_uniform(T, E, topk, seed=12)
    x = synth.activations(T, H, seed=13)
    got, scratch = run_kernel(to_device(L0, cuda), x, ids, w)
    want, pairs = run_oracle(oracle, L0, x, ids, w)
    check(got, want)
    assert pairs == T * topk


def test_config3_shape_zipf_one_gpu(cuda, oracle):
    """Config 3 routes (T = 16, Zipf 1.1) with the single-GPU expert width
    I = 2048, over 32 experts to keep the oracle fast."""
    E, H, I, T, topk = 32, 4096, 2048, 16, 8
    L0 = layer(E, H, I, synth.expert_bits(E, 5), 5)
    ids, w = synth.route_zipf(T, E, topk, seed=14)
    x = synth.activations(T, H, seed=15)
    got, _ = run_kernel(to_device(L0, cuda), x, ids, w)
    want, _ = run_oracle(oracle, L0, x, ids, w)
    check(got, want)


def test_deterministic_and_nan_poisoned_scratch(cuda):
    """Two runs are bitwise equal, also when everything after the control
    region of the scratch was filled with NaN (parity_native.py:369-393)."""
    E, H, I, T, topk = 32, 1024, 256, 8, 8
    L = to_device(layer(E, H, I, synth.expert_bits(E, 6), 6), cuda)
    ids, w = synth.route_zipf(T, E, topk, seed=2)
    x = synth.activations(T, H, seed=3)
    a, scratch = run_kernel(L, x, ids, w)
    b, _ = run_kernel(L, x, ids, w, scratch=scratch)
    assert torch.equal(a, b)
    scratch[M_CTRL:] = 0xFF   # 0xFFFFFFFF is a NaN in fp32 and in fp16 pairs
    for _ in range(3):
        c, _ = run_kernel(L, x, ids, w, scratch=scratch)
        assert torch.equal(a, c)
    assert ext.lna2_moe_status(scratch) == 0



def test_plugin_dispatch(cuda, oracle):
    """apply_moe_decode: local id mapping, shared scratch, call counter."""
    E, H, I, T, topk = 16, 512, 128, 4, 4
    L0 = layer(E, H, I, synth.expert_bits(E, 8), 8)
    L = to_device(L0, cuda)
    state = M.build_moe_state(L.experts, codebook=1)
    M.prepare(state, cuda, max_rows=T, topk=topk)
    ids, w = synth.route_uniform(T, E, topk, seed=9)
    x = synth.activations(T, H, seed=10)
    M.reset_moe_kernel_call_counts()
    out = M.apply_moe_decode(x.to(cuda), ids.to(cuda).long(), w.to(cuda), state, out_dtype=torch.float32)
    assert M.moe_kernel_call_counts()["b200"] == 1
    want, _ = run_oracle(oracle, L0, x, ids, w)
    check(out, want)


def test_fused_tp_sum_world_of_one(cuda):
    """The in-kernel tensor-parallel sum with a world of one (the exchange
    runs against this rank's own buffer): bitwise the plain output, over
    several calls (both epoch parities)."""
    from dsv4_carve_b200.tp import MoeTpExchange

    E, H, I, T, topk = 16, 1024, 256, 4, 4
    L = to_device(layer(E, H, I, synth.expert_bits(E, 3), 3), cuda)
    ex = MoeTpExchange.single(cuda, max_rows=8, hidden=H)
    try:
        for it in range(5):
            ids, w = synth.route_uniform(T, E, topk, seed=50 + it)
            x = synth.activations(T, H, seed=60 + it, device=cuda)
            ref, _ = run_kernel(L, x, ids, w)
            got = torch.empty_like(ref)
            scratch = torch.zeros(ext.lna2_moe_scratch_bytes(T, topk, H, I), dtype=torch.uint8, device=cuda)
            ext.lna2_moe_decode(x, got, *L.table_list(), ids.to(cuda), w.to(cuda), max(L.kbits), 10.0, scratch,
                                intermediate=I, k_table=L.ktab, codebook=L.cb, tp_exchange=ex)
            torch.cuda.synchronize(cuda)
            assert torch.equal(got, ref)
            assert ext.lna2_moe_status(scratch) == 0
    finally:
        torch.cuda.synchronize(cuda)
        ex.close()


# ------------------------------------------------------------------ benchmarked shapes
@pytest.mark.parametrize("precise", [False, True])
def test_config2_full_layer(cuda, oracle, precise):
    """The benchmarked workload itself: config 2 on one GPU (256 experts,
    hidden 4096, intermediate 2048, T = 4, top-8, K2/K3 MCG).  The layer is
    generated on the device; the oracle gets only the ~30 routed experts."""
    from tests.helpers import routed_subset

    E, H, I, T, topk = 256, 4096, 2048, 4, 8
    L = synth.make_moe_layer(E, H, I, synth.expert_bits(E, 71), 71, device=cuda)
    ids, w = synth.route_uniform(T, E, topk, seed=72)
    x = synth.activations(T, H, seed=73)
    got, scratch = run_kernel(L, x, ids, w, precise=precise)
    experts, kb, loc = routed_subset(L, ids)
    want, pairs = oracle.moe(x.numpy(), experts, kb, loc, w.numpy(), 10.0, cb=L.cb, exact=not precise)
    check(got, want)
    assert ext.lna2_moe_status(scratch) == 0
    assert pairs == len({(int(e), r) for r in range(T) for e in ids[r].tolist()})


# ------------------------------------------------------------------ the reference's own MoE loop
def _loop_cases():
    from tests.golden import make_moe_golden as MGL

    return list(MGL.CASES)


@pytest.mark.parametrize("precise", [False, True])
@pytest.mark.parametrize("name", _loop_cases())
def test_kernel_matches_reference_loop(cuda, name, precise):
    """The kernel on the reference loop's fixtures (tests/golden/ref_moe_loop.npz:
    apply_exl3_python_loop, recipe-lna/vllm_exl3_exl3.py.lna:988-1027, run
    unchanged over the reference's CPU dequant_trellis + fp32 matmul), fed the
    loop's own inputs -- global int64 ids and, for the mapped case, the same
    expert_map -- through lna2_moe_decode_routed.  Weight rounding differs
    (full fp16 W with truncation there, GEMV form here): max-abs <= 2e-3,
    per-row relative <= 4e-3."""
    from pathlib import Path

    from tests.golden import make_moe_golden as MGL

    fx = np.load(Path(__file__).resolve().parent / "golden" / "ref_moe_loop.npz")
    cpu, _, _, _, _ = MGL.make_case(name)
    assert MGL.layer_sha(cpu) == str(fx[f"{name}_sha"])
    L = to_device(cpu, cuda)
    meta = fx[f"{name}_meta"]
    bf16 = bool(meta[5])
    xbits = torch.from_numpy(fx[f"{name}_x"].view(np.int16))
    x = xbits.view(torch.bfloat16 if bf16 else torch.float16).to(cuda)
    ids = torch.from_numpy(fx[f"{name}_ids"]).to(cuda)
    w = torch.from_numpy(fx[f"{name}_w"]).to(cuda)
    emap = torch.from_numpy(fx[f"{name}_map"]).to(cuda) if f"{name}_map" in fx else None
    T, topk = ids.shape
    scratch = torch.zeros(ext.lna2_moe_scratch_bytes(T, topk, L.H, L.I), dtype=torch.uint8, device=cuda)
    out = torch.empty((T, L.H), dtype=torch.float32, device=cuda)
    ext.lna2_moe_decode_routed(x, out, *L.table_list(), ids, w, max(L.kbits), float(meta[6]) / 1000.0, scratch,
                               intermediate=L.I, k_table=L.ktab, codebook=L.cb, precise=precise, expert_map=emap,
                               check_status=True)
    want = fx[f"{name}_out"].astype(np.float64)
    got = out.cpu().numpy()
    assert max_abs(got, want) <= TOL
    assert row_rel(got, want) <= 4e-3


# ------------------------------------------------------------------ routing inputs on the device
def test_routed_entry_equals_reference_abi_bitwise(cuda):
    """lna2_moe_decode_routed with int64 ids and fp32 weights == lna2_moe_decode
    with int32 ids bit for bit; bf16 / fp16 weights == the reference ABI fed
    the same values cast to fp32 (the plugin's .to(float32))."""
    E, H, I, T, topk = 32, 1024, 256, 8, 8
    L = to_device(layer(E, H, I, synth.expert_bits(E, 13), 13), cuda)
    ids, w = synth.route_zipf(T, E, topk, seed=14, device=cuda)
    x = synth.activations(T, H, seed=15, device=cuda)
    ref, _ = run_kernel(L, x, ids, w)
    for w_in in (w, w.to(torch.bfloat16), w.to(torch.float16)):
        base, _ = run_kernel(L, x, ids, w_in.float())
        out = torch.empty_like(ref)
        scratch = torch.zeros(ext.lna2_moe_scratch_bytes(T, topk, H, I), dtype=torch.uint8, device=cuda)
        ext.lna2_moe_decode_routed(x, out, *L.table_list(), ids.long(), w_in, max(L.kbits), 10.0, scratch,
                                   intermediate=I, k_table=L.ktab, codebook=L.cb)
        assert torch.equal(out, base)
        if w_in is w:
            assert torch.equal(out, ref)


def test_expert_map_and_skips_on_device(cuda, oracle):
    """Global ids through an expert map (half the experts on this rank),
    plus a negative id, an id past the map and an unmapped expert, against
    the oracle fed the host-mapped local ids."""
    E, H, I, T, topk = 16, 1024, 256, 4, 6
    n_global = 40
    L0 = layer(E, H, I, synth.expert_bits(E, 17), 17)
    L = to_device(L0, cuda)
    g = torch.Generator().manual_seed(18)
    perm = torch.randperm(n_global, generator=g)
    emap = torch.full((n_global,), -1, dtype=torch.long)
    emap[perm[:E]] = torch.arange(E)
    ids, w = synth.route_uniform(T, n_global, topk, seed=19)
    ids = ids.long()
    ids[0, 0] = -3
    ids[1, 1] = n_global + 5
    ids[2, 2] = int(perm[E])      # a global expert that lives on another rank
    x = synth.activations(T, H, seed=20)
    e = emap.numpy()
    gid = ids.numpy()
    loc = np.where((gid >= 0) & (gid < n_global), e[np.clip(gid, 0, n_global - 1)], -1).astype(np.int32)
    out = torch.empty((T, H), dtype=torch.float32, device=cuda)
    scratch = torch.zeros(ext.lna2_moe_scratch_bytes(T, topk, H, I), dtype=torch.uint8, device=cuda)
    ext.lna2_moe_decode_routed(x.to(cuda), out, *L.table_list(), ids.to(cuda), w.to(cuda), max(L.kbits), 10.0,
                               scratch, intermediate=I, k_table=L.ktab, codebook=L.cb, expert_map=emap.to(cuda))
    want, _ = run_oracle(oracle, L0, x, torch.from_numpy(loc), w)
    check(out, want)


def test_plugin_dispatch_is_one_launch(cuda, oracle):
    """apply_moe_decode on the router's raw outputs (int64 global ids, bf16
    weights, an expert map): exactly one kernel runs for the layer -- no
    mapping, cast or copy kernels around it -- and the result matches."""
    from torch.profiler import ProfilerActivity, profile

    E, H, I, T, topk = 16, 1024, 256, 4, 4
    n_global = 24
    L0 = layer(E, H, I, synth.expert_bits(E, 22), 22)
    L = to_device(L0, cuda)
    state = M.build_moe_state(L.experts, codebook=1)
    M.prepare(state, cuda, max_rows=8, topk=topk)
    emap = torch.full((n_global,), -1, dtype=torch.long)
    emap[torch.arange(E) + 8] = torch.arange(E)       # global ids 8..23 live here
    ids, w = synth.route_uniform(T, n_global, topk, seed=23)
    x = synth.activations(T, H, seed=24).to(cuda)
    ids_d, w_d, emap_d = ids.long().to(cuda), w.to(torch.bfloat16).to(cuda), emap.to(cuda)
    out = torch.empty((T, H), dtype=torch.float32, device=cuda)
    M.apply_moe_decode(x, ids_d, w_d, state, expert_map=emap_d, out=out)   # warm
    torch.cuda.synchronize(cuda)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        M.apply_moe_decode(x, ids_d, w_d, state, expert_map=emap_d, out=out)
        torch.cuda.synchronize(cuda)
    kernels = [ev.name for ev in prof.events() if ev.device_type == torch.autograd.DeviceType.CUDA]
    assert len(kernels) == 1 and "moe_kernel" in kernels[0], kernels
    gid = ids.numpy()
    loc = np.where((gid >= 8) & (gid < n_global), gid - 8, -1).astype(np.int32)
    want, _ = run_oracle(oracle, L0, x.cpu(), torch.from_numpy(loc), w.to(torch.bfloat16).float())
    check(out, want)


def test_status_word_surfaces(cuda):
    """The status word as a pollable device view (0 after a healthy call) and
    the synchronizing check, which passes on a healthy call."""
    E, H, I, T, topk = 8, 512, 128, 2, 2
    L = to_device(layer(E, H, I, [2] * E, 25), cuda)
    ids, w = synth.route_uniform(T, E, topk, seed=26)
    x = synth.activations(T, H, seed=27)
    out, scratch = run_kernel(L, x, ids, w)
    word = ext.lna2_moe_status_word(scratch)
    assert word.dtype == torch.int32 and word.numel() == 1 and int(word.item()) == 0
    ext.lna2_moe_decode(x.to(cuda), out, *L.table_list(), ids.to(cuda), w.to(cuda), 2, 10.0, scratch,
                        intermediate=I, k_table=L.ktab, codebook=L.cb, check_status=True)
