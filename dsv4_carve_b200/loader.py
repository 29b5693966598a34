"""EXL3 checkpoint loader: the on-disk format the reference's packs use.

A pack is a directory of safetensors files, optionally with a
``*.safetensors.index.json`` weight map, and a ``quantization_config.json``.
Each EXL3 linear is stored under a module prefix as ``<prefix>.trellis``
(int16 [in/16, out/16, 16K]), ``<prefix>.suh`` (fp16 [in]), ``<prefix>.svh``
(fp16 [out]) and, for the MCG / MUL1 codebooks, a marker tensor
``<prefix>.mcg`` / ``<prefix>.mul1`` holding the multiplier as int32
(-877912083 / -2082680531); neither marker means the 3INST codebook
(recipe-lna/vllm_exl3_exl3.py.lna:50-54, exllamav3 1.4.5's LinearEXL3 attributes
read at :1337-1366).  Routed experts live at
``layers.<L>.ffn.experts.<E>.w1|w2|w3`` -- w1 the gate, w3 the up and w2 the
down projection (recipe-lna/lna2/parity_native.py:138-147).

The quantization config restates the plugin's Exl3Config
(recipe-lna/vllm_exl3_exl3.py.lna:1797-1930): base ``bits`` and ``codebook``,
per-layer ``layer_bits`` for mixed-K packs, and ``non_routed_exl3`` for
quantized dense modules (``modules`` suffixes, ``bits``, ``layer_bits`` per
suffix, ``layers`` per prefix).  Tensor-parallel slicing follows
``shard_exl3_col`` / ``shard_exl3_row`` (:855-871): gate and up keep columns
``[r*I/N, (r+1)*I/N)`` (trellis dim 1 and svh), down keeps those rows (trellis
dim 0 and suh).

What is built is what the kernels bind to: a ``synth.MoeLayer`` with the nine
device pointer tables and the per-expert K table of ``lna2_moe_decode``, and
``LinearEXL3`` for dense modules.  Nothing here touches the GPU kernels.
"""
from __future__ import annotations

import json
import re
from pathlib import Path
from typing import Any

import torch

from . import synth
from .linear import LinearEXL3

MCG_MARKER = -877912083
MUL1_MARKER = -2082680531
EXL3_SUFFIXES = ("trellis", "suh", "svh", "mcg", "mul1")
EXPERT_PROJ = {"gate": "w1", "up": "w3", "down": "w2"}
SUPPORTED_BITS = (2, 3, 4, 5, 6)
_LAYER_RE = re.compile(r"(?:^|\.)layers\.(\d+)(?:\.|$)")


def _prefix_has_suffix(prefix: str, suffix: str) -> bool:
    """Module-path suffix match on whole components ("self_attn.o_proj"
    matches "model.layers.3.self_attn.o_proj", not "x.self_attn.o_proj_b")."""
    return prefix == suffix or prefix.endswith("." + suffix)


class Exl3QuantConfig:
    """The pack's quantization_config.json (routed experts + optional
    non-routed dense modules), validated as the plugin validates it."""

    def __init__(self, bits: int = 4, codebook: str = "mcg", layer_bits: dict | None = None,
                 non_routed_exl3: dict | None = None, **extra: Any):
        self.bits = int(bits)
        self.codebook = str(codebook)
        if self.bits not in SUPPORTED_BITS:
            raise ValueError(f"unsupported EXL3 bits={self.bits}")
        if self.codebook not in ("mcg", "mul1"):
            raise ValueError(f"unsupported codebook={self.codebook!r}; must be 'mcg' or 'mul1'")
        self.layer_bits = {int(k): int(v) for k, v in dict(layer_bits or {}).items()}
        for layer, k in self.layer_bits.items():
            if k not in SUPPORTED_BITS:
                raise ValueError(f"unsupported EXL3 bits={k} for layer {layer}")
        self.non_routed = dict(non_routed_exl3 or {})
        nr_bits = self.non_routed.get("bits")
        if nr_bits is not None and int(nr_bits) not in SUPPORTED_BITS:
            raise ValueError(f"unsupported non_routed_exl3 bits={nr_bits}")
        for suffix, k in (self.non_routed.get("layer_bits") or {}).items():
            if int(k) not in SUPPORTED_BITS:
                raise ValueError(f"unsupported non_routed_exl3 bits={k} for suffix {suffix}")
        for prefix, cfg in (self.non_routed.get("layers") or {}).items():
            if not isinstance(cfg, dict):
                raise ValueError(f"non_routed_exl3 layers[{prefix}] must be a dict, got {type(cfg)}")
            if cfg.get("bits") is not None and int(cfg["bits"]) not in SUPPORTED_BITS:
                raise ValueError(f"unsupported non_routed_exl3 layers[{prefix}] bits={cfg['bits']}")
        if self.non_routed.get("codebook", "mcg") not in ("mcg", "mul1"):
            raise ValueError(f"unsupported non_routed_exl3 codebook={self.non_routed['codebook']!r}")
        self.extra = extra

    @classmethod
    def from_dict(cls, cfg: dict) -> "Exl3QuantConfig":
        skip = {"quant_method", "scope", "tensor_storage", "non_routed_quantization", "mtp_experts",
                "mtp_experts_start_layer"}
        kw = {k: v for k, v in cfg.items() if k not in skip}
        return cls(**kw)

    @classmethod
    def from_file(cls, path: str | Path) -> "Exl3QuantConfig":
        return cls.from_dict(json.loads(Path(path).read_text()))

    def bits_for_prefix(self, prefix: str) -> int:
        """Routed-expert K of the layer the prefix belongs to (layer_bits, else bits)."""
        m = _LAYER_RE.search(prefix or "")
        if m is None or not self.layer_bits:
            return self.bits
        return self.layer_bits.get(int(m.group(1)), self.bits)

    def matches_non_routed(self, prefix: str) -> bool:
        layers = self.non_routed.get("layers") or {}
        if prefix in layers:
            return True
        return any(_prefix_has_suffix(prefix, s) for s in self.non_routed.get("modules") or [])

    def bits_for_non_routed(self, prefix: str) -> int:
        layers = self.non_routed.get("layers") or {}
        default = int(self.non_routed.get("bits", self.bits))
        if prefix in layers:
            return int(layers[prefix].get("bits", default))
        for suffix in self.non_routed.get("modules") or []:
            if _prefix_has_suffix(prefix, suffix):
                return int((self.non_routed.get("layer_bits") or {}).get(suffix, default))
        return self.bits


class Checkpoint:
    """Name -> tensor access over a directory of safetensors files."""

    def __init__(self, root: str | Path):
        from safetensors import safe_open

        self.root = Path(root)
        self._open = safe_open
        index = sorted(self.root.glob("*.safetensors.index.json"))
        self.weight_map: dict[str, str] = {}
        if index:
            self.weight_map = dict(json.loads(index[0].read_text())["weight_map"])
        else:
            for f in sorted(self.root.glob("*.safetensors")):
                with safe_open(str(f), framework="pt") as h:
                    for name in h.keys():
                        self.weight_map[name] = f.name
        if not self.weight_map:
            raise FileNotFoundError(f"no safetensors tensors under {self.root}")
        self._handles: dict[str, Any] = {}
        cfg = self.root / "quantization_config.json"
        self.config = Exl3QuantConfig.from_file(cfg) if cfg.exists() else None

    def has(self, name: str) -> bool:
        return name in self.weight_map

    def get(self, name: str, device="cpu") -> torch.Tensor:
        if name not in self.weight_map:
            raise KeyError(name)
        fname = self.weight_map[name]
        if fname not in self._handles:
            self._handles[fname] = self._open(str(self.root / fname), framework="pt")
        return self._handles[fname].get_tensor(name).to(device)


def codebook_of(ckpt: Checkpoint, prefix: str) -> int:
    """Codebook from the marker tensors: MCG / MUL1 when their marker is
    present (every element must hold the multiplier), else 3INST."""
    for suffix, marker, cb in (("mcg", MCG_MARKER, synth.CB_MCG), ("mul1", MUL1_MARKER, synth.CB_MUL1)):
        name = f"{prefix}.{suffix}"
        if ckpt.has(name):
            t = ckpt.get(name).reshape(-1)
            if t.numel() == 0 or not bool(torch.all(t.to(torch.int64) == marker)):
                raise ValueError(f"{name} is not the {suffix.upper()} marker {marker}")
            return cb
    return synth.CB_3INST


def load_dense(ckpt: Checkpoint, prefix: str, device="cpu", bits: int | None = None) -> synth.DenseWeight:
    """One EXL3 linear as stored, with the shape / dtype checks the plugin makes
    before binding it (recipe-lna/vllm_exl3_exl3.py.lna:1339-1356)."""
    trellis = ckpt.get(f"{prefix}.trellis", device)
    suh = ckpt.get(f"{prefix}.suh", device)
    svh = ckpt.get(f"{prefix}.svh", device)
    if trellis.dtype != torch.int16 or trellis.dim() != 3 or trellis.shape[-1] % 16:
        raise ValueError(f"{prefix}.trellis must be int16 [in/16, out/16, 16K], got {trellis.dtype} {tuple(trellis.shape)}")
    K = int(trellis.shape[-1]) // 16
    if bits is not None and K != int(bits):
        raise ValueError(f"{prefix}: trellis holds K={K}, the quantization config says K={bits}")
    if suh.dtype != torch.float16 or suh.numel() != trellis.shape[0] * 16:
        raise ValueError(f"{prefix}.suh must be fp16[{trellis.shape[0] * 16}]")
    if svh.dtype != torch.float16 or svh.numel() != trellis.shape[1] * 16:
        raise ValueError(f"{prefix}.svh must be fp16[{trellis.shape[1] * 16}]")
    return synth.DenseWeight(trellis.contiguous(), suh.contiguous(), svh.contiguous(), K, codebook_of(ckpt, prefix))


def _narrow(t: torch.Tensor, dim: int, rank: int, world: int, what: str) -> torch.Tensor:
    """The plugin's even TP narrow (recipe-lna/vllm_exl3_exl3.py.lna:805-814)."""
    if world <= 1:
        return t
    size = int(t.shape[dim])
    if size % world:
        raise ValueError(f"EXL3 TP shard: {what} dim {dim} size {size} is not divisible by tp={world}")
    chunk = size // world
    return t.narrow(dim, chunk * rank, chunk).contiguous()


def shard_expert(proj: str, w: synth.DenseWeight, rank: int, world: int) -> synth.DenseWeight:
    """Gate / up: trellis dim 1 and svh are column-parallel; down: trellis dim 0
    and suh are row-parallel (shard_exl3_col / shard_exl3_row, :855-871)."""
    if world <= 1:
        return w
    if proj in ("gate", "up"):
        return synth.DenseWeight(_narrow(w.trellis, 1, rank, world, proj), w.suh,
                                 _narrow(w.svh, 0, rank, world, proj), w.K, w.cb)
    return synth.DenseWeight(_narrow(w.trellis, 0, rank, world, proj), _narrow(w.suh, 0, rank, world, proj),
                             w.svh, w.K, w.cb)


def expert_prefix(layer: int, expert: int, fmt: str = "layers.{layer}.ffn.experts.{expert}") -> str:
    return fmt.format(layer=layer, expert=expert)


def load_moe_layer(ckpt: Checkpoint, layer: int, n_experts: int, rank: int = 0, world: int = 1, device="cuda",
                   config: Exl3QuantConfig | None = None,
                   prefix_fmt: str = "layers.{layer}.ffn.experts.{expert}") -> synth.MoeLayer:
    """All routed experts of one layer, this rank's TP shard, on `device`, with
    the nine pointer tables and the K table that lna2_moe_decode /
    lna2_moe_prefill take.  Every expert must use the same codebook (one
    launch decodes one); bit widths may differ per expert (k_table)."""
    config = config or ckpt.config
    experts, kbits, cbs = [], [], set()
    H = I = None
    for e in range(n_experts):
        base = expert_prefix(layer, e, prefix_fmt)
        want = config.bits_for_prefix(base) if config is not None else None
        ex = {}
        for proj, wname in EXPERT_PROJ.items():
            w = load_dense(ckpt, f"{base}.{wname}", "cpu", want)
            ex[proj] = shard_expert(proj, w, rank, world).to(device)
            cbs.add(w.cb)
        h, i = ex["gate"].in_features, ex["gate"].out_features
        if ex["up"].in_features != h or ex["up"].out_features != i or ex["down"].in_features != i \
                or ex["down"].out_features != h:
            raise ValueError(f"{base}: gate/up/down shapes disagree")
        if not (ex["gate"].K == ex["up"].K == ex["down"].K):
            raise ValueError(f"{base}: gate/up/down bit widths disagree")
        if H is None:
            H, I = h, i
        elif (h, i) != (H, I):
            raise ValueError(f"{base}: expert shape ({h}, {i}) differs from ({H}, {I})")
        if I % 128 or H % 128:
            raise ValueError(f"{base}: hidden {H} and intermediate shard {I} must be multiples of 128")
        experts.append(ex)
        kbits.append(ex["gate"].K)
    if len(cbs) != 1:
        raise ValueError(f"layer {layer}: experts mix codebooks {sorted(cbs)}")
    L = synth.MoeLayer(E=n_experts, H=H, I=I, kbits=kbits, cb=cbs.pop())
    L.experts = experts
    L.build_tables()
    return L


def load_linear(ckpt: Checkpoint, prefix: str, device="cuda", config: Exl3QuantConfig | None = None) -> LinearEXL3:
    """A dense EXL3 module (attention / shared expert) as the LinearEXL3 the
    plugin's dense branch calls; K is checked against non_routed_exl3 when the
    config lists the module."""
    config = config or ckpt.config
    bits = None
    if config is not None and config.matches_non_routed(prefix):
        bits = config.bits_for_non_routed(prefix)
    w = load_dense(ckpt, prefix, device, bits)
    mcg = ckpt.get(f"{prefix}.mcg", device) if w.cb == synth.CB_MCG else None
    mul1 = ckpt.get(f"{prefix}.mul1", device) if w.cb == synth.CB_MUL1 else None
    return LinearEXL3(None, w.in_features, w.out_features, None, None, None, w.suh, w.svh, w.trellis, mcg, mul1,
                      key=prefix)
