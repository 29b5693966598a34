"""Plugin-side glue of the routed-MoE decode path.

Covers what the vllm-exl3 plugin does around the native kernel
(recipe-lna/vllm_exl3_exl3.py.lna): the load-time pointer-table contract
(:1318-1374, :1552-1570), one shared zeroed scratch per device created
before any graph capture (:1276-1296), the strict / call-counter / decline
instrumentation (:1070-1157) and the dispatch itself (``_apply_lna2_moe``,
:1190-1248), generalised to per-expert bit widths, top-k up to 16 and any
128-multiple hidden / intermediate width.  The plugin's per-layer torch glue
-- global-to-local id mapping through ``expert_map`` and the id / weight
casts (:963-987, :1234-1236) -- is not done here at all: the router's
outputs go to the kernel as they are and the kernel's route plan maps and
converts them, so a layer is one launch.
"""
from __future__ import annotations

import logging
import os
from dataclasses import dataclass

import torch

from . import vllm_exl3_c as _ext
from .synth import MCG_MARKER_SIGNED_INT32

logger = logging.getLogger("dsv4_carve_b200.moe")

_TABLE_ORDER = ("gate_trellis", "gate_suh", "gate_svh", "up_trellis", "up_suh", "up_svh",
                "down_trellis", "down_suh", "down_svh")
_CALLS = {"b200": 0}
_DECLINED: set[str] = set()
_ACTIVE_LOGGED = False


def moe_kernel_strict() -> int:
    """VLLM_EXL3_MOE_STRICT: 1 raises when not ready, 2 also on shape declines."""
    try:
        return int(os.environ.get("VLLM_EXL3_MOE_STRICT", "0") or 0)
    except ValueError:
        return 0


def moe_kernel_call_counts() -> dict:
    return dict(_CALLS)


def reset_moe_kernel_call_counts() -> None:
    for k in _CALLS:
        _CALLS[k] = 0


def moe_kernel_declined_reasons() -> list:
    return sorted(_DECLINED)


def _decline(why: str, *, not_ready: bool = False) -> None:
    if why not in _DECLINED and len(_DECLINED) < 12:
        _DECLINED.add(why)
        logger.warning("B200 EXL3 MoE declined: %s", why)
    level = moe_kernel_strict()
    if level >= (1 if not_ready else 2):
        raise RuntimeError(f"VLLM_EXL3_MOE_STRICT={level}, but the B200 MoE kernel declined this call: {why}")


def _router_outputs(ids: torch.Tensor, weights: torch.Tensor, expert_map: torch.Tensor | None):
    """ids / weights / map as the kernel reads them; views only, unless a
    tensor comes in a layout or dtype the kernel does not read."""
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int64)
    ids = ids.reshape(ids.shape[0], -1) if ids.dim() != 2 else ids
    if not ids.is_contiguous():
        ids = ids.contiguous()
    w = weights.reshape(ids.shape)
    if w.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        w = w.to(torch.float32)
    if not w.is_contiguous():
        w = w.contiguous()
    if expert_map is not None and (expert_map.device != ids.device or expert_map.dtype != torch.long):
        raise RuntimeError("EXL3 expert_map is not pinned to the hidden-state device as int64")
    return ids, w


@dataclass
class MoeState:
    """Everything the kernel needs about one layer, built once at load time."""
    tables: dict
    ktab: torch.Tensor
    kmax: int
    hidden: int
    inter: int
    n_experts: int
    codebook: int
    precise: bool = False

    def table_list(self) -> list:
        return [self.tables[n] for n in _TABLE_ORDER]


def build_moe_state(inners: list, codebook: int | None = None) -> MoeState:
    """Validate the per-expert tensors and build the 9 pointer tables.

    `inners[e]` maps 'gate'/'up'/'down' to objects with trellis/suh/svh
    (LinearEXL3 or synth.DenseWeight).  Checks restate
    _validate_lna_pointer_contract (vllm_exl3_exl3.py.lna:1318-1374) with the
    alignment this kernel needs (16 bytes, for bulk copies)."""
    if not inners:
        raise ValueError("MoE requires at least one routed expert")
    g0 = inners[0]["gate"]
    hidden = int(g0.suh.numel())
    inter = int(g0.svh.numel())
    device = g0.trellis.device
    if hidden % 128 or inter % 128:
        raise ValueError(f"hidden/intermediate must be multiples of 128, got {hidden}/{inter}")
    kbits = []
    for e, pack in enumerate(inners):
        K = int(pack["gate"].trellis.shape[-1]) // 16
        if not 1 <= K <= 4:
            raise ValueError(f"expert {e}: K{K} is outside this build's MoE range 1..4")
        expected = {"gate": ((hidden // 16, inter // 16, 16 * K), hidden, inter),
                    "up": ((hidden // 16, inter // 16, 16 * K), hidden, inter),
                    "down": ((inter // 16, hidden // 16, 16 * K), inter, hidden)}
        for which, (shape, nsu, nsv) in expected.items():
            lin = pack[which]
            t, su, sv = lin.trellis, lin.suh, lin.svh
            if tuple(int(v) for v in t.shape) != shape:
                raise ValueError(f"expert {e} {which}.trellis shape {tuple(t.shape)} != {shape}")
            if t.dtype != torch.int16 or not t.is_contiguous():
                raise ValueError(f"expert {e} {which}.trellis must be contiguous int16")
            if su.dtype != torch.float16 or su.numel() != nsu or not su.is_contiguous():
                raise ValueError(f"expert {e} {which}.suh must be contiguous fp16[{nsu}]")
            if sv.dtype != torch.float16 or sv.numel() != nsv or not sv.is_contiguous():
                raise ValueError(f"expert {e} {which}.svh must be contiguous fp16[{nsv}]")
            marker = getattr(lin, "mcg_tensor", None)
            if marker is not None and codebook is None:
                if not bool(torch.all(marker.reshape(-1) == MCG_MARKER_SIGNED_INT32).item()):
                    raise ValueError(f"expert {e} {which}.mcg is not the MCG marker")
            for name, tensor in (("trellis", t), ("suh", su), ("svh", sv)):
                if tensor.device != device:
                    raise ValueError(f"expert {e} {which}.{name} is on the wrong device")
            if t.data_ptr() % 16:
                raise ValueError(f"expert {e} {which}.trellis is not 16-byte aligned")
        kbits.append(K)
    cb = codebook
    if cb is None:
        cb = getattr(g0, "cb", None)
        if cb is None:
            cb = getattr(g0, "codebook", 1)
    names = {"gate_trellis": ("gate", "trellis"), "gate_suh": ("gate", "suh"), "gate_svh": ("gate", "svh"),
             "up_trellis": ("up", "trellis"), "up_suh": ("up", "suh"), "up_svh": ("up", "svh"),
             "down_trellis": ("down", "trellis"), "down_suh": ("down", "suh"), "down_svh": ("down", "svh")}
    tables = {n: torch.tensor([getattr(inners[e][p], a).data_ptr() for e in range(len(inners))],
                              dtype=torch.int64, device=device) for n, (p, a) in names.items()}
    ktab = torch.tensor(kbits, dtype=torch.int32, device=device)
    return MoeState(tables, ktab, max(kbits), hidden, inter, len(inners), int(cb))


_SCRATCH: dict[int, torch.Tensor] = {}


def moe_scratch_for(device: torch.device, nbytes: int | None = None) -> torch.Tensor:
    """One zeroed scratch per device for the whole model (vllm_exl3_exl3.py.lna:1276-1296):
    the kernel restores its control region, and only one MoE launch is in
    flight per device."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    need = int(nbytes if nbytes is not None else _ext.lna2_moe_scratch_bytes())
    buf = _SCRATCH.get(idx)
    if buf is None or buf.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("B200 MoE scratch was not prewarmed for this device")
        buf = torch.zeros(need, dtype=torch.uint8, device=device)
        _SCRATCH[idx] = buf
    return buf


def prepare(state: MoeState, device: torch.device, max_rows: int | None = None, topk: int = 8) -> None:
    """Pre-capture preparation: occupancy/attributes and the shared scratch."""
    _ext.lna2_moe_prepare(state.kmax)
    rows = max_rows or _ext.lna2_moe_max_rows()
    moe_scratch_for(device, _ext.lna2_moe_scratch_bytes(rows, topk, state.hidden, state.inter))


def apply_moe_decode(x2d: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, state: MoeState,
                     expert_map: torch.Tensor | None = None, limit: float = 10.0,
                     out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None):
    """The lna2 branch of apply_exl3_experts, for any geometry this build serves.

    Returns the [T, hidden] output, or None when the call is declined."""
    global _ACTIVE_LOGGED
    T = int(x2d.shape[0])
    if (not x2d.is_cuda or x2d.dim() != 2 or not 1 <= T <= _ext.lna2_moe_max_rows()
            or int(x2d.shape[1]) != state.hidden or T * int(ids.shape[-1]) > 256 or int(ids.shape[-1]) > 16):
        _decline(f"geometry x={tuple(x2d.shape)} topk={int(ids.shape[-1])}")
        return None
    ids2, route_w = _router_outputs(ids, weights, expert_map)
    x = x2d if x2d.dtype in (torch.float16, torch.bfloat16, torch.float32) else x2d.to(torch.float16)
    x = x.contiguous()
    scratch = moe_scratch_for(x.device, _ext.lna2_moe_scratch_bytes(
        _ext.lna2_moe_max_rows(), max(8, int(ids2.shape[-1])), state.hidden, state.inter))
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or (x.dtype if x.dtype != torch.float32 else torch.float16),
                          device=x.device)
    _ext.lna2_moe_decode_routed(x, out, *state.table_list(), ids2, route_w, state.kmax, float(limit), scratch,
                                intermediate=state.inter, k_table=state.ktab, codebook=state.codebook,
                                precise=state.precise, expert_map=expert_map)
    _CALLS["b200"] += 1
    if not _ACTIVE_LOGGED:
        _ACTIVE_LOGGED = True
        logger.warning("B200 EXL3 MoE kernel ACTIVE")
    return out


def apply_moe_prefill(x2d: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, state: MoeState,
                      expert_map: torch.Tensor | None = None, limit: float = 10.0,
                      out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None):
    """The fused prefill branch of apply_exl3_experts (the reference calls
    exllamav3_ext.exl3_moe after torch argsort / count glue,
    recipe-lna/vllm_exl3_exl3.py.lna:1597-1704): one tensor-core layer per
    chunk of tokens, route plan on the device.  Returns the [T, hidden]
    output, or None when the call is declined."""
    T = int(x2d.shape[0])
    if (not x2d.is_cuda or x2d.dim() != 2 or T < 1 or int(x2d.shape[1]) != state.hidden
            or int(ids.shape[-1]) > 16 or state.kmax > 4):
        _decline(f"prefill geometry x={tuple(x2d.shape)} topk={int(ids.shape[-1])}")
        return None
    ids2, route_w = _router_outputs(ids, weights, expert_map)
    x = x2d if x2d.dtype in (torch.float16, torch.bfloat16) else x2d.to(torch.float16)
    x = x.contiguous()
    scratch = _ext._prefill_scratch(x.device, _ext.lna2_moe_prefill_scratch_bytes(
        T, int(ids2.shape[-1]), state.hidden, state.inter, state.n_experts))
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    _ext.lna2_moe_prefill(x, out, *state.table_list(), ids2, route_w, state.kmax, float(limit), scratch,
                          intermediate=state.inter, k_table=state.ktab, codebook=state.codebook,
                          expert_map=expert_map)
    _CALLS["b200"] += 1
    return out


def apply_moe(x2d: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, state: MoeState,
              expert_map: torch.Tensor | None = None, limit: float = 10.0,
              out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None):
    """Decode kernel up to its row ceiling, tensor-core prefill above it
    (the plugin's lna2 / fused-exl3_moe split, vllm_exl3_exl3.py.lna:1707-1779)."""
    if int(x2d.shape[0]) <= _ext.lna2_moe_max_rows() and int(x2d.shape[0]) * int(ids.shape[-1]) <= 256:
        return apply_moe_decode(x2d, ids, weights, state, expert_map, limit, out, out_dtype)
    return apply_moe_prefill(x2d, ids, weights, state, expert_map, limit, out, out_dtype)

