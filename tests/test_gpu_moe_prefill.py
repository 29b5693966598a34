"""Routed-MoE prefill layer (tcgen05 path) on the GPU against the oracle.

The prefill path multiplies the fp16-rounded decoded weights (the values the
reference's decoder returns), so it is compared with the oracle in that mode
(exact=False).  Tolerances as for decode: fp32 output max-abs <= 2e-3 against
the oracle's fp64 result on unit-scale inputs, per-row relative <= 2e-3.
Cases follow the reference's route profiles (recipe-lna/lna2/parity_native.py):
uniform / hot (one expert takes every token: several 128-row passes) / zipf /
within-row duplicates / invalid ids; plus token chunking (more tokens than one
device route plan holds), bf16 input, fp16 / bf16 output, bitwise
determinism, the exllamav3_ext.exl3_moe-shaped shim and the plugin dispatch.
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
_LAYERS: dict = {}


def layer(E, H, I, kbits, seed, cb=1):
    key = (E, H, I, tuple(kbits), seed, cb)
    if key not in _LAYERS:
        _LAYERS[key] = synth.make_moe_layer(E, H, I, kbits, seed, device="cpu", cb=cb)
    return _LAYERS[key]


def to_device(cpu_layer, dev):
    L = synth.MoeLayer(E=cpu_layer.E, H=cpu_layer.H, I=cpu_layer.I, kbits=cpu_layer.kbits, cb=cpu_layer.cb)
    L.experts = [{p: w.to(dev) for p, w in ex.items()} for ex in cpu_layer.experts]
    L.build_tables()
    return L


def run_prefill(L, x, ids, w, limit=10.0, out_dtype=torch.float32, kscalar=None):
    dev = L.ktab.device
    T, topk = ids.shape
    scratch = torch.empty(ext.lna2_moe_prefill_scratch_bytes(T, topk, L.H, L.I, L.E), dtype=torch.uint8,
                          device=dev)
    out = torch.empty((T, L.H), dtype=out_dtype, device=dev)
    ktab = None if kscalar else L.ktab
    K = kscalar or max(L.kbits)
    ext.lna2_moe_prefill(x.to(dev), out, *L.table_list(), ids.to(dev), w.to(dev), K, limit, scratch,
                         intermediate=L.I, k_table=ktab, codebook=L.cb)
    return out, scratch


def run_oracle(oracle, L, x, ids, w, limit=10.0):
    xa, code = oracle_x(x)
    want, _ = oracle.moe(xa, moe_np(L), L.kbits, ids.numpy(), w.numpy(), limit, cb=L.cb, dtype_code=code,
                         exact=False)
    return want


def check(got, want, rel=2e-3):
    got = got.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert max_abs(got, want) <= TOL, max_abs(got, want)
    assert row_rel(got, want) <= rel, row_rel(got, want)


@pytest.mark.parametrize("cb", [1, 0])
@pytest.mark.parametrize("T", [1, 20, 160])
def test_uniform_mixed_k(cuda, oracle, cb, T):
    E, H, I, topk = 16, 1024, 256, 4
    L0 = layer(E, H, I, synth.expert_bits(E, 3), 3, cb=cb)
    ids, w = synth.route_uniform(T, E, topk, seed=5 + T)
    x = synth.activations(T, H, seed=6 + T)
    got, scratch = run_prefill(to_device(L0, cuda), x, ids, w)
    check(got, run_oracle(oracle, L0, x, ids, w))
    assert ext.lna2_moe_status(scratch) == 0


def test_hot_expert_several_passes(cuda, oracle):
    """Every token routes slot 0 to expert 3: 300 rows = 3 passes of 128."""
    E, H, I, T, topk = 16, 1024, 256, 300, 2
    L0 = layer(E, H, I, synth.expert_bits(E, 7), 7)
    ids, w = synth.route_uniform(T, E, topk, seed=8)
    ids[:, 0] = 3
    ids[:, 1] = torch.where(ids[:, 1] == 3, torch.full_like(ids[:, 1], 4), ids[:, 1])
    x = synth.activations(T, H, seed=9)
    got, _ = run_prefill(to_device(L0, cuda), x, ids, w)
    check(got, run_oracle(oracle, L0, x, ids, w))


def test_zipf_duplicates_invalid(cuda, oracle):
    """Zipf-skewed routes, a row that lists one expert twice, ids outside
    [0, E) (skipped), all in one call."""
    E, H, I, T, topk = 32, 512, 384, 96, 4
    L0 = layer(E, H, I, synth.expert_bits(E, 11), 11)
    ids, w = synth.route_zipf(T, E, topk, seed=12)
    ids[5, 1] = ids[5, 0]
    ids[7, 2] = -1
    ids[9, 3] = E + 5
    x = synth.activations(T, H, seed=13)
    got, _ = run_prefill(to_device(L0, cuda), x, ids, w)
    check(got, run_oracle(oracle, L0, x, ids, w))


def test_token_chunks(cuda, oracle):
    """1024 experts: one device route plan holds 512 tokens, so 600 tokens
    run as two chunks on one scratch."""
    E, H, I, T, topk = 1024, 256, 128, 600, 2
    assert ext.lna2_moe_prefill_chunk_tokens(E) == 512
    L0 = layer(E, H, I, [2] * E, 17)
    ids, w = synth.route_uniform(T, E, topk, seed=18)
    x = synth.activations(T, H, seed=19)
    got, _ = run_prefill(to_device(L0, cuda), x, ids, w, kscalar=2)
    check(got, run_oracle(oracle, L0, x, ids, w))


def test_bf16_in_and_half_outputs(cuda, oracle):
    E, H, I, T, topk = 16, 1024, 256, 48, 4
    L0 = layer(E, H, I, synth.expert_bits(E, 3), 3)
    ids, w = synth.route_uniform(T, E, topk, seed=21)
    x = synth.activations(T, H, seed=22, dtype=torch.bfloat16)
    L = to_device(L0, cuda)
    want = run_oracle(oracle, L0, x, ids, w)
    got, _ = run_prefill(L, x, ids, w, out_dtype=torch.float16)
    assert row_rel(got.float().cpu().numpy(), want) <= 2e-3
    got, _ = run_prefill(L, x, ids, w, out_dtype=torch.bfloat16)
    assert row_rel(got.float().cpu().numpy(), want) <= 6e-3


def test_amplified_input_past_clamp(cuda, oracle):
    E, H, I, T, topk = 16, 1024, 256, 40, 4
    L0 = layer(E, H, I, synth.expert_bits(E, 3), 3)
    ids, w = synth.route_uniform(T, E, topk, seed=23)
    x = synth.activations(T, H, seed=24) * 8
    got, _ = run_prefill(to_device(L0, cuda), x, ids, w, limit=1.0)
    want = run_oracle(oracle, L0, x, ids, w, limit=1.0)
    assert row_rel(got.float().cpu().numpy(), want) <= 2e-3


def test_bitwise_deterministic(cuda):
    E, H, I, T, topk = 16, 1024, 256, 200, 4
    L = to_device(layer(E, H, I, synth.expert_bits(E, 3), 3), cuda)
    ids, w = synth.route_uniform(T, E, topk, seed=25)
    x = synth.activations(T, H, seed=26)
    a, _ = run_prefill(L, x, ids, w)
    b, _ = run_prefill(L, x, ids, w)
    assert torch.equal(a, b)


def test_matches_decode_kernel_precise(cuda):
    """Both kernels in the precise arithmetic on a decode-sized call: same
    weights, same boundaries; only the accumulation order differs."""
    E, H, I, T, topk = 16, 1024, 256, 4, 4
    L = to_device(layer(E, H, I, synth.expert_bits(E, 3), 3), cuda)
    ids, w = synth.route_uniform(T, E, topk, seed=27)
    x = synth.activations(T, H, seed=28, device=cuda)
    pre, _ = run_prefill(L, x, ids, w)
    dec = torch.empty_like(pre)
    scratch = torch.zeros(ext.lna2_moe_scratch_bytes(T, topk, H, I), dtype=torch.uint8, device=cuda)
    ext.lna2_moe_decode(x, dec, *L.table_list(), ids.to(cuda), w.to(cuda), max(L.kbits), 10.0, scratch,
                        intermediate=I, k_table=L.ktab, codebook=L.cb, precise=True)
    assert (pre - dec).abs().max().item() <= 1e-4


def test_exl3_moe_shim(cuda, oracle):
    """exllamav3_ext.exl3_moe's signature, fed the sorted-slot arrays the
    plugin builds (recipe-lna/vllm_exl3_exl3.py.lna:1617-1629); the output
    is accumulated into output_state."""
    E, H, I, T, topk = 16, 1024, 256, 64, 4
    L0 = layer(E, H, I, [2] * E, 29)
    L = to_device(L0, cuda)
    ids, w = synth.route_uniform(T, E, topk, seed=30)
    ids[3, 1] = E          # an id past the local experts: the slot is skipped
    x = synth.activations(T, H, seed=31)
    local = ids.to(cuda).reshape(-1).long()
    flat_token = torch.arange(T, device=cuda).repeat_interleave(topk)
    flat_weight = w.to(cuda).reshape(-1).to(torch.float16)
    order = local.argsort()
    expert_count = torch.zeros(E + 1, dtype=torch.long, device=cuda)
    expert_count.scatter_add_(0, local, torch.ones_like(local))
    out = torch.ones((T, H), dtype=torch.float32, device=cuda)
    temps = [torch.empty((1, 8, n), dtype=torch.float16, device=cuda) for n in (H, H, I, I)]
    t = L.table_list()
    ext.exl3_moe(x.to(cuda), out, expert_count, flat_token[order], flat_weight[order], *temps, 0, 2, 2, 2,
                 *t, True, False, True, False, True, False, 10.0, -1)
    w16 = w.to(torch.float16).to(torch.float32)
    ids_ref = ids.clone()
    ids_ref[3, 1] = -1
    want = run_oracle(oracle, L0, x, ids_ref, w16) + 1.0
    check(out, want)


def test_plugin_dispatch_routes_by_rows(cuda, oracle):
    """apply_moe: the decode kernel up to its row ceiling, prefill above it."""
    E, H, I = 16, 1024, 256
    L0 = layer(E, H, I, [3] * E, 33)
    L = to_device(L0, cuda)
    state = M.build_moe_state(L.experts, codebook=1)
    for T in (4, 100):
        ids, w = synth.route_uniform(T, E, 4, seed=40 + T)
        x = synth.activations(T, H, seed=41 + T)
        y = M.apply_moe(x.to(cuda), ids.to(cuda).long(), w.to(cuda), state, out_dtype=torch.float32)
        assert y is not None
        want = run_oracle(oracle, L0, x, ids, w)
        assert row_rel(y.float().cpu().numpy(), want) <= 2e-3


@pytest.mark.parametrize("I,rows_checked", [(256, 64), (2048, 8)])
def test_config4b_shape(cuda, oracle, I, rows_checked):
    """The config-4b prefill chunk: 512 tokens, bf16 activations N(0,1),
    top-8 of 256 experts, hidden 4096, K2/K3 MCG, at the TP8 shard's
    intermediate width (256) and at the full single-GPU width (2048).  The
    kernel runs all 512 tokens; the oracle checks `rows_checked` of them,
    spread over the chunk (a token's output depends only on its own routes)."""
    from tests.helpers import routed_subset

    E, H, T, topk = 256, 4096, 512, 8
    L = synth.make_moe_layer(E, H, I, synth.expert_bits(E, 81), 81, device=cuda)
    ids, w = synth.route_uniform(T, E, topk, seed=82)
    x = synth.activations(T, H, seed=83, dtype=torch.bfloat16)
    out, scratch = run_prefill(L, x, ids, w)
    rows = torch.from_numpy(np.linspace(0, T - 1, rows_checked).round().astype(np.int64))
    experts, kb, loc = routed_subset(L, ids[rows])
    xa, code = oracle_x(x[rows])
    want, _ = oracle.moe(xa, experts, kb, loc, w[rows].numpy(), 10.0, cb=L.cb, dtype_code=code, exact=False)
    check(out[rows.to(cuda)], want)
    assert ext.lna2_moe_status(scratch) == 0


def test_prefill_expert_map_on_device(cuda, oracle):
    """lna2_moe_prefill with int64 global ids, fp16 routing weights and an
    expert map, read by the device route plan, against the oracle fed the
    host-mapped ids."""
    E, H, I, T, topk = 16, 1024, 256, 80, 4
    n_global = 32
    L0 = layer(E, H, I, synth.expert_bits(E, 34), 34)
    L = to_device(L0, cuda)
    emap = torch.full((n_global,), -1, dtype=torch.long)
    emap[1::2] = torch.arange(E)                       # odd global ids live here
    ids, w = synth.route_uniform(T, n_global, topk, seed=35)
    ids = ids.long()
    ids[0, 0] = -1
    ids[5, 1] = n_global
    x = synth.activations(T, H, seed=36)
    w16 = w.to(torch.float16)
    scratch = torch.empty(ext.lna2_moe_prefill_scratch_bytes(T, topk, H, I, E), dtype=torch.uint8, device=cuda)
    out = torch.empty((T, H), dtype=torch.float32, device=cuda)
    ext.lna2_moe_prefill(x.to(cuda), out, *L.table_list(), ids.to(cuda), w16.to(cuda), max(L.kbits), 10.0, scratch,
                         intermediate=I, k_table=L.ktab, codebook=L.cb, expert_map=emap.to(cuda),
                         check_status=True)
    gid = ids.numpy()
    e = emap.numpy()
    loc = np.where((gid >= 0) & (gid < n_global), e[np.clip(gid, 0, n_global - 1)], -1).astype(np.int32)
    want = run_oracle(oracle, L0, x, torch.from_numpy(loc), w16.float())
    check(out, want)
