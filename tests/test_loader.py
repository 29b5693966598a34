"""The EXL3 checkpoint loader (dsv4_carve_b200/loader.py) on small packs
written here with safetensors: the reference's tensor names
(layers.L.ffn.experts.E.w1|w2|w3.trellis|suh|svh|mcg, recipe-lna/lna2/
parity_native.py:138-147), quantization_config.json with per-layer bits and
non-routed modules (recipe-lna/vllm_exl3_exl3.py.lna:1797-1930), codebook
markers (:50-54, :1357-1366) and TP slicing (:805-871).  The CPU tests check
what is loaded against the synthetic tensors that were written; the GPU test
runs the decode kernel on a loaded layer against the oracle."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

from dsv4_carve_b200 import loader as LD
from dsv4_carve_b200 import synth

E, H, I = 4, 256, 512


def _marker(cb: int):
    return {synth.CB_MCG: ("mcg", LD.MCG_MARKER), synth.CB_MUL1: ("mul1", LD.MUL1_MARKER)}.get(cb)


def _put(tensors: dict, prefix: str, w: synth.DenseWeight):
    tensors[f"{prefix}.trellis"] = w.trellis.contiguous()
    tensors[f"{prefix}.suh"] = w.suh.contiguous()
    tensors[f"{prefix}.svh"] = w.svh.contiguous()
    m = _marker(w.cb)
    if m is not None:
        tensors[f"{prefix}.{m[0]}"] = torch.tensor([m[1]], dtype=torch.int32)


def write_pack(root, layer_k=(2, 3), cb=synth.CB_MCG, split=False, config=None, dense_k=6):
    """Two MoE layers (layer L all at bit width layer_k[L]) and one dense
    module; returns {layer: synth.MoeLayer (full width, CPU)} and the dense weight."""
    tensors, layers = {}, {}
    for L, K in enumerate(layer_k):
        full = synth.make_moe_layer(E, H, I, [K] * E, seed=40 + L, cb=cb)
        layers[L] = full
        for e in range(E):
            for proj, wn in LD.EXPERT_PROJ.items():
                _put(tensors, f"layers.{L}.ffn.experts.{e}.{wn}", full.experts[e][proj])
    dense = synth.make_dense(H, 384, dense_k, seed=7, cb=cb)
    _put(tensors, "layers.0.self_attn.o_proj", dense)
    names = sorted(tensors)
    if split:
        half = len(names) // 2
        parts = {"model-00001.safetensors": names[:half], "model-00002.safetensors": names[half:]}
        for fname, ns in parts.items():
            save_file({n: tensors[n] for n in ns}, str(root / fname))
        wm = {n: f for f, ns in parts.items() for n in ns}
        (root / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wm}))
    else:
        save_file(tensors, str(root / "model.safetensors"))
    cfg = config if config is not None else {
        "quant_method": "exl3", "bits": layer_k[0], "codebook": "mcg",
        "layer_bits": {str(L): K for L, K in enumerate(layer_k) if K != layer_k[0]},
        "non_routed_exl3": {"modules": ["self_attn.o_proj"], "bits": dense_k}}
    (root / "quantization_config.json").write_text(json.dumps(cfg))
    return layers, dense


def _same(a: synth.DenseWeight, b: synth.DenseWeight):
    assert a.K == b.K and a.cb == b.cb
    for x, y in ((a.trellis, b.trellis), (a.suh, b.suh), (a.svh, b.svh)):
        assert x.dtype == y.dtype and tuple(x.shape) == tuple(y.shape)
        assert torch.equal(x.cpu(), y.cpu())


def test_config_bits_and_non_routed():
    c = LD.Exl3QuantConfig.from_dict({"quant_method": "exl3", "bits": 2, "codebook": "mcg",
                                      "layer_bits": {"42": 3, "27": 3},
                                      "non_routed_exl3": {"modules": ["self_attn.o_proj", "mlp.shared"],
                                                          "bits": 6, "layer_bits": {"mlp.shared": 5},
                                                          "layers": {"model.layers.1.attn.wq": {"bits": 4}}}})
    assert c.bits_for_prefix("model.layers.42.ffn.experts.3.w1") == 3
    assert c.bits_for_prefix("model.layers.4.ffn.experts.3.w1") == 2
    assert c.bits_for_prefix("lm_head") == 2
    assert c.matches_non_routed("model.layers.3.self_attn.o_proj")
    assert not c.matches_non_routed("model.layers.3.self_attn.o_proj_x")
    assert c.bits_for_non_routed("model.layers.3.self_attn.o_proj") == 6
    assert c.bits_for_non_routed("model.layers.9.mlp.shared") == 5
    assert c.bits_for_non_routed("model.layers.1.attn.wq") == 4


@pytest.mark.parametrize("bad", [{"bits": 7}, {"codebook": "3inst"}, {"layer_bits": {"1": 9}},
                                 {"non_routed_exl3": {"bits": 1}}, {"non_routed_exl3": {"codebook": "x"}},
                                 {"non_routed_exl3": {"layers": {"a": 3}}}])
def test_config_rejects_what_the_plugin_rejects(bad):
    with pytest.raises(ValueError):
        LD.Exl3QuantConfig.from_dict({"bits": 2, **bad})


@pytest.mark.parametrize("split", [False, True])
def test_moe_layer_loads_as_written(tmp_path, split):
    layers, _ = write_pack(tmp_path, split=split)
    ck = LD.Checkpoint(tmp_path)
    for L, want in layers.items():
        got = LD.load_moe_layer(ck, L, E, device="cpu")
        assert got.kbits == [(2, 3)[L]] * E and got.cb == synth.CB_MCG and (got.H, got.I) == (H, I)
        for e in range(E):
            for proj in ("gate", "up", "down"):
                _same(got.experts[e][proj], want.experts[e][proj])
        assert [int(v) for v in got.tables["gate_trellis"]] == [got.experts[e]["gate"].trellis.data_ptr()
                                                                for e in range(E)]
        assert got.ktab.tolist() == got.kbits


@pytest.mark.parametrize("world", [2, 4])
def test_tp_shards_match_the_plugin_slicing(tmp_path, world):
    layers, _ = write_pack(tmp_path)
    ck = LD.Checkpoint(tmp_path)
    full = layers[1]
    for rank in range(world):
        got = LD.load_moe_layer(ck, 1, E, rank=rank, world=world, device="cpu")
        assert got.I == I // world
        for e in range(E):
            _same(got.experts[e]["gate"], synth.shard_col(full.experts[e]["gate"], rank, world))
            _same(got.experts[e]["up"], synth.shard_col(full.experts[e]["up"], rank, world))
            _same(got.experts[e]["down"], synth.shard_row(full.experts[e]["down"], rank, world))


def test_codebooks_from_markers(tmp_path):
    for cb in (synth.CB_3INST, synth.CB_MUL1):
        d = tmp_path / f"cb{cb}"
        d.mkdir()
        write_pack(d, cb=cb, config={"bits": 2, "layer_bits": {"1": 3}})
        assert LD.load_moe_layer(LD.Checkpoint(d), 0, E, device="cpu").cb == cb


def test_bad_marker_bits_mismatch_and_shapes_raise(tmp_path):
    write_pack(tmp_path, config={"bits": 2})          # layer 1 holds K3 but the config says 2
    ck = LD.Checkpoint(tmp_path)
    with pytest.raises(ValueError, match="K=3"):
        LD.load_moe_layer(ck, 1, E, device="cpu")
    with pytest.raises(ValueError, match="not divisible"):
        LD.load_moe_layer(ck, 0, E, rank=0, world=3, device="cpu")
    d = tmp_path / "badmarker"
    d.mkdir()
    write_pack(d)
    from safetensors.torch import load_file
    t = load_file(str(d / "model.safetensors"))
    t["layers.0.ffn.experts.2.w3.mcg"] = torch.tensor([LD.MUL1_MARKER], dtype=torch.int32)
    save_file(t, str(d / "model.safetensors"))
    with pytest.raises(ValueError, match="marker"):
        LD.load_moe_layer(LD.Checkpoint(d), 0, E, device="cpu")
    with pytest.raises(KeyError):
        LD.load_moe_layer(ck, 0, E + 1, device="cpu")


def test_dense_module_loads_as_linear(tmp_path):
    _, dense = write_pack(tmp_path)
    ck = LD.Checkpoint(tmp_path)
    lin = LD.load_linear(ck, "layers.0.self_attn.o_proj", device="cpu")
    assert (lin.in_features, lin.out_features, lin.K, lin.codebook) == (H, 384, 6, synth.CB_MCG)
    assert torch.equal(lin.trellis, dense.trellis) and lin.mcg_tensor is not None
    bad = tmp_path / "bad"
    bad.mkdir()
    write_pack(bad, config={"bits": 2, "layer_bits": {"1": 3},
                            "non_routed_exl3": {"modules": ["self_attn.o_proj"], "bits": 4}})
    with pytest.raises(ValueError, match="K=6"):
        LD.load_linear(LD.Checkpoint(bad), "layers.0.self_attn.o_proj", device="cpu")


@pytest.mark.gpu
def test_loaded_layer_decodes_like_the_oracle(tmp_path, cuda, oracle):
    from dsv4_carve_b200 import vllm_exl3_c as ext
    from tests.helpers import max_abs, moe_np

    layers, _ = write_pack(tmp_path)
    ck = LD.Checkpoint(tmp_path)
    L = LD.load_moe_layer(ck, 1, E, rank=1, world=2, device=cuda)
    ref = synth.MoeLayer(E=E, H=H, I=I // 2, kbits=[3] * E, cb=synth.CB_MCG)
    ref.experts = [{p: (synth.shard_col if p != "down" else synth.shard_row)(layers[1].experts[e][p], 1, 2)
                    for p in ("gate", "up", "down")} for e in range(E)]
    T, topk = 4, 2
    ids, w = synth.route_uniform(T, E, topk, seed=3)
    x = synth.activations(T, H, seed=4)
    scratch = torch.zeros(ext.lna2_moe_scratch_bytes(T, topk, H, L.I), dtype=torch.uint8, device=cuda)
    out = torch.empty((T, H), dtype=torch.float32, device=cuda)
    ext.lna2_moe_decode(x.to(cuda), out, *L.table_list(), ids.to(cuda), w.to(cuda), 3, 10.0, scratch,
                        intermediate=L.I, k_table=L.ktab, codebook=L.cb)
    torch.cuda.synchronize()
    want, _ = oracle.moe(x.numpy(), moe_np(ref), ref.kbits, ids.numpy(), w.numpy(), 10.0, cb=ref.cb)
    assert max_abs(out.cpu().numpy(), want) <= 2e-3
    assert np.isfinite(out.cpu().numpy()).all()
