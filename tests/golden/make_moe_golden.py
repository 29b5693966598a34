"""Golden MoE outputs of the reference's own semantic MoE loop.

Run where the reference tree is (REF_ROOT names it; required):

    REF_ROOT=<reference tree> python tests/golden/make_moe_golden.py

What it runs: the function ``apply_exl3_python_loop`` exactly as written in
the reference (recipe-lna/vllm_exl3_exl3.py.lna:988-1027), taken from that
file by name with ``ast`` and executed unchanged.  Its ``pack["gate"|"up"|
"down"].forward(x, {}, out_dtype=torch.float32)`` calls go to a LinearEXL3
stand-in whose forward is the reference's own CPU linear: the weight decoded
by the reference's ``dequant_trellis`` (recipe-lna/lna2/bindings.cpp:118-133
-> dequant_cpu :16-101, built from source into oracle/_ref by
oracle/build_oracle.py) and an fp32 matmul, the arithmetic of the reference's
CPU ``exl3_gemv`` (bindings.cpp:135-148) with the fp32 output the plugin asks
for.  The stand-in is the only piece that is not the reference's code: the
reference's LinearEXL3 needs exllamav3's CUDA extension, which is absent.

Layers, routes and activations come from dsv4_carve_b200.synth with the
seeds stored in ref_moe_loop.npz (torch CPU generators, reproducible), and a
sha256 of every case's packed weights is stored so that a test notices if the
regenerated layer ever differs.  Fixture keys per case <name>:
  <name>_out      fp32 [T, hidden]  the reference loop's output
  <name>_ids      int64 [T, topk]   global expert ids handed to the loop
  <name>_w        fp32 [T, topk]    routing weights
  <name>_x        uint16 [T, hidden] activation bits (fp16 or bf16)
  <name>_map      int64 [n_global]  expert_map (only for mapped cases)
  <name>_meta     int64 [..]        E, H, I, layer seed, codebook, bf16 flag,
                                     limit * 1000
  <name>_sha      str               sha256 of the layer's trellis/suh/svh bytes
"""
from __future__ import annotations

import __future__ as _future
import ast
import hashlib
import os
import sys
from pathlib import Path
from typing import Any

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

PLUGIN_FILE = "recipe-lna/vllm_exl3_exl3.py.lna"
FIXTURE = HERE / "ref_moe_loop.npz"

# name: (E, H, I, layer seed, codebook, T, topk, route seed, x seed, x scale, limit, bf16, kind)
CASES = {
    "mcg_mixed": (12, 1024, 256, 41, 1, 4, 4, 42, 43, 1.0, 10.0, False, "uniform"),
    "dup_invalid": (12, 1024, 256, 41, 1, 4, 4, 44, 45, 1.0, 10.0, False, "dup_invalid"),
    "expert_map": (12, 1024, 256, 41, 1, 4, 6, 46, 47, 1.0, 10.0, False, "mapped"),
    "clamp": (8, 512, 256, 48, 1, 3, 3, 49, 50, 8.0, 1.0, False, "uniform"),
    "mul1": (8, 512, 128, 51, 2, 4, 3, 52, 53, 1.0, 10.0, False, "uniform"),
    "bf16_in": (12, 1024, 256, 41, 1, 4, 4, 57, 58, 1.0, 10.0, True, "uniform"),
    "single_row": (16, 1024, 256, 59, 1, 1, 8, 60, 61, 1.0, 10.0, False, "uniform"),
}


def layer_sha(layer) -> str:
    h = hashlib.sha256()
    for ex in layer.experts:
        for p in ("gate", "up", "down"):
            for t in (ex[p].trellis, ex[p].suh, ex[p].svh):
                h.update(t.contiguous().view(-1).view(dtype=t.dtype).numpy().tobytes())
    return h.hexdigest()


def make_case(name: str):
    """Inputs of one case from its seeds: (layer, x, ids int64, weights, expert_map or None)."""
    import torch

    from dsv4_carve_b200 import synth

    E, H, I, seed, cb, T, topk, rseed, xseed, xscale, limit, bf16, kind = CASES[name]
    layer = synth.make_moe_layer(E, H, I, synth.expert_bits(E, seed, choices=(2, 3, 4)), seed, cb=cb)
    x = synth.activations(T, H, seed=xseed, scale=xscale, dtype=torch.bfloat16 if bf16 else torch.float16)
    emap = None
    if kind == "mapped":
        n_global = 2 * E
        ids, w = synth.route_uniform(T, n_global, topk, seed=rseed)
        g = torch.Generator().manual_seed(rseed)
        perm = torch.randperm(n_global, generator=g)
        emap = torch.full((n_global,), -1, dtype=torch.long)
        emap[perm[:E]] = torch.arange(E)          # half the global experts live on this rank
    else:
        ids, w = synth.route_uniform(T, E, topk, seed=rseed)
    ids = ids.long()
    if kind == "dup_invalid":
        ids[0, 1] = ids[0, 0]                     # an expert listed twice in one row
        ids[1, 2] = -1                            # a skipped slot
        ids[2, 3] = E                             # an id past the local experts
        ids[3, :] = -1                            # a row with no valid slot
    return layer, x, ids.contiguous(), w.contiguous(), emap


def load_reference_loop(ref_root: Path):
    """apply_exl3_python_loop from the reference's plugin file, unchanged."""
    import torch
    import torch.nn.functional as F

    path = ref_root / PLUGIN_FILE
    text = path.read_text()
    tree = ast.parse(text)
    node = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "apply_exl3_python_loop")
    src = ast.get_source_segment(text, node)
    code = compile(src, f"{path}:{node.lineno}", "exec", flags=_future.annotations.compiler_flag,
                   dont_inherit=True)
    ns = {"torch": torch, "F": F, "Any": Any}
    exec(code, ns)
    return ns["apply_exl3_python_loop"], node.lineno, node.end_lineno


class RefCpuLinear:
    """LinearEXL3 stand-in: forward = the reference's dequant_trellis (CPU,
    built from source) then an fp32 matmul, cast to out_dtype."""

    def __init__(self, ref, weight):
        self.ref = ref
        self.w = weight
        self._W = None

    def forward(self, x, params, out_dtype=None):
        import torch

        if self._W is None:
            if self.w.cb == 0:
                raise RuntimeError("the reference's dequant_trellis has no 3INST mode (bindings.cpp:49)")
            mcg = self.w.cb == 1
            self._W = self.ref.dequant_trellis(self.w.trellis, self.w.suh, self.w.svh, self.w.K, mcg).float()
        y = x.float() @ self._W
        return y.to(out_dtype or x.dtype)


def main() -> None:
    import torch

    ref_root = os.environ.get("REF_ROOT")
    if not ref_root:
        raise SystemExit("set REF_ROOT to the reference tree")
    from oracle import build_oracle as B
    from oracle import oracle as O

    B.build_all()
    ref = O.ref_ext()
    if ref is None:
        raise SystemExit("the reference's CPU extension (oracle/_ref) could not be built")
    loop, l0, l1 = load_reference_loop(Path(ref_root))
    print(f"apply_exl3_python_loop taken from {PLUGIN_FILE}:{l0}-{l1}")
    out = {}
    for name in CASES:
        layer, x, ids, w, emap = make_case(name)
        inners = [{p: RefCpuLinear(ref, ex[p]) for p in ("gate", "up", "down")} for ex in layer.experts]
        E, H, I, seed, cb = CASES[name][:5]
        limit, bf16 = CASES[name][10], CASES[name][11]
        y = loop(x, ids, w, inners, emap, limit)
        out[f"{name}_out"] = y.numpy().astype(np.float32)
        out[f"{name}_ids"] = ids.numpy().astype(np.int64)
        out[f"{name}_w"] = w.numpy().astype(np.float32)
        out[f"{name}_x"] = x.view(torch.int16).numpy().view(np.uint16)
        if emap is not None:
            out[f"{name}_map"] = emap.numpy().astype(np.int64)
        out[f"{name}_meta"] = np.array([E, H, I, seed, cb, int(bf16), int(round(limit * 1000))], dtype=np.int64)
        out[f"{name}_sha"] = np.array(layer_sha(layer))
        print(f"{name}: |out| max {float(y.abs().max()):.3f}")
    np.savez_compressed(FIXTURE, **out)
    print("written", FIXTURE)


if __name__ == "__main__":
    main()
