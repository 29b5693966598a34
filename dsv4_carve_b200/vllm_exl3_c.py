"""Drop-in for the reference's native extension module ``vllm_exl3_c``.

Same entry-point names, positional argument order, argument meaning and
error behaviour (RuntimeError with the reference's messages) as the
pybind11 module the vllm-exl3 plugin imports through its ``NATIVE_SO`` hook
(recipe-lna/lna2/bindings.cpp:178-224, recipe-lna/lna2/lna_moe_ticket.cu:489-581).
Every call goes to the sm_100a kernels of libexl3b200.so on the tensors'
CUDA device and the current stream; there is no CPU path (the reference's CPU
fallback of dequant_trellis / exl3_gemv is its CPU baseline, not product).

Generalisations over the reference, all optional keyword arguments:
  * lna2_moe_decode(..., intermediate=256, k_table=None, codebook=1, precise=False):
    any hidden / intermediate that are multiples of 128, top-k 1..16,
    per-expert bit widths through an int32 [experts] table (K = largest);
  * precise: round each decoded weight to fp16 before the MMA (the dense
    entries default to True, the MoE to False; see include/exl3_b200.h);
  * dequant_trellis / exl3_gemv / exl3_gemm(..., codebook=None): the
    reference maps mcg=True to MCG and mcg=False to MUL1 (bindings.cpp:49);
    ``codebook=0`` selects 3INST explicitly.
"""
from __future__ import annotations

import os

import torch

from . import _lib

__all__ = [
    "dequant_trellis", "exl3_gemv", "exl3_gemm", "exl3_mgemm", "lna2_moe_decode", "lna2_moe_scratch_bytes",
    "lna2_moe_max_rows", "lna2_moe_prepare", "lna2_moe_info", "lna2_moe_status", "lna2_moe_status_word",
    "lna2_moe_decode_routed", "lna2_moe_prefill", "lna2_moe_prefill_scratch_bytes", "exl3_linear_scratch_bytes",
]

_DT = {torch.float16: _lib.DT_F16, torch.bfloat16: _lib.DT_BF16, torch.float32: _lib.DT_F32}


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _on_device:
    """Make `device` current for the C-ABI call when it is not already."""

    def __init__(self, device: torch.device):
        self.index = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.index:
            self.prev = cur
            torch.cuda.set_device(self.index)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def _codebook(mcg: bool, codebook) -> int:
    if codebook is None:
        return _lib.CB_MCG if mcg else _lib.CB_MUL1
    _check(int(codebook) in (0, 1, 2), "codebook must be 0 (3INST), 1 (MCG) or 2 (MUL1)")
    return int(codebook)


# --------------------------------------------------------------------- dequant
def dequant_trellis(trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int, mcg: bool,
                    *, codebook: int | None = None, inner_only: bool = False) -> torch.Tensor:
    """Decode an EXL3 trellis tensor into an fp16 weight matrix [in, out].

    recipe-lna/lna2/bindings.cpp:118-133.  ``inner_only`` returns W' (no
    Hadamards or sign vectors)."""
    bits = int(K)
    _check(1 <= bits <= 8, "K must be in 1..8")
    _check(trellis.dim() == 3 and trellis.dtype == torch.int16,
           "trellis must be int16 [rows/16, cols/16, 16*K]")
    _check(trellis.size(2) == 16 * bits, "trellis last dimension must be 16*K")
    _check(trellis.size(0) > 0 and trellis.size(1) > 0, "trellis dimensions must be positive")
    _check(suh.dtype == torch.float16 and svh.dtype == torch.float16, "suh and svh must be float16")
    _check(suh.numel() >= trellis.size(0) * 16 and svh.numel() >= trellis.size(1) * 16,
           "suh/svh are too short")
    _check(trellis.is_cuda, "dequant_trellis: the B200 build decodes on CUDA tensors only")
    if not inner_only:
        _check(trellis.size(0) % 8 == 0 and trellis.size(1) % 8 == 0,
               "trellis dimensions must reconstruct whole 128-element Hadamard blocks")
    t = trellis.contiguous()
    su = suh.to(t.device).contiguous()
    sv = svh.to(t.device).contiguous()
    out = torch.empty((t.size(0) * 16, t.size(1) * 16), dtype=torch.float16, device=t.device)
    with _on_device(t.device):
        _lib.call("exl3_dequant", t.data_ptr(), t.size(0), t.size(1), bits, _codebook(mcg, codebook),
                  su.data_ptr(), sv.data_ptr(), out.data_ptr(), 0 if inner_only else 1, _stream(t.device))
    return out


# --------------------------------------------------------------------- dense
_LIN_SCRATCH: dict[tuple[int, int], torch.Tensor] = {}


def exl3_linear_scratch_bytes(rows: int, k: int, n: int, K: int) -> int:
    return int(_lib.load().exl3_linear_scratch_bytes(rows, k, n, K))


def _linear_scratch(device: torch.device, nbytes: int) -> torch.Tensor:
    """Shared per-(device, stream) linear scratch, zeroed on creation; the
    kernel restores its control words, so it is reused without a memset."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, _stream(device))
    buf = _LIN_SCRATCH.get(key)
    if buf is None or buf.numel() < nbytes:
        _check(not torch.cuda.is_current_stream_capturing(),
               "exl3 linear scratch was not prewarmed for this device/stream (graph capture)")
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _LIN_SCRATCH[key] = buf
    return buf


def linear_forward(x2: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor,
                   K: int, codebook: int, out_dtype: torch.dtype, precise: bool = True) -> torch.Tensor:
    """y[m, n] = x2[m, k] . W on the current stream (k, n multiples of 128).

    precise=True rounds every decoded weight to fp16 as the reference does;
    False feeds the codebook's half pair to the tensor core unrounded."""
    m, k = x2.shape
    n = trellis.size(1) * 16
    _check(x2.dtype in _DT and out_dtype in _DT, "exl3 linear: dtypes must be fp16, bf16 or fp32")
    y = torch.empty((m, n), dtype=out_dtype, device=x2.device)
    nbytes = exl3_linear_scratch_bytes(m, k, n, K)
    scratch = _linear_scratch(x2.device, nbytes)
    with _on_device(x2.device):
        _lib.call("exl3_linear", x2.data_ptr(), _DT[x2.dtype], m, k, n, trellis.data_ptr(), K, codebook,
                  suh.data_ptr(), svh.data_ptr(), y.data_ptr(), _DT[out_dtype], scratch.data_ptr(),
                  scratch.numel(), int(bool(precise)), _stream(x2.device))
    return y


def linear_group_forward(x2: torch.Tensor, mats: list, K: int, codebook: int, out_dtype: torch.dtype,
                         precise: bool = True) -> list:
    """[x2 . W_j for each (trellis_j, suh_j, svh_j) in mats] in one launch:
    one input, up to 8 matrices of the same k, bit width and codebook
    (exllamav3_ext.exl3_mgemm with a broadcast input,
    recipe-lna/exllamav3/exl3_gemm.cu.lna:659-679)."""
    import ctypes

    m, k = x2.shape
    nm = len(mats)
    _check(1 <= nm <= 8, "exl3 linear group: 1 to 8 matrices")
    _check(x2.dtype in _DT and out_dtype in _DT, "exl3 linear: dtypes must be fp16, bf16 or fp32")
    for t, su, sv in mats:
        _linear_checks(x2, t, su, sv, K)
    ns = [int(t.size(1)) * 16 for t, _, _ in mats]
    ys = [torch.empty((m, n), dtype=out_dtype, device=x2.device) for n in ns]
    arr_n = (ctypes.c_int64 * nm)(*ns)
    ptrs = lambda ts: (ctypes.c_void_p * nm)(*[t.data_ptr() for t in ts])   # noqa: E731
    lib = _lib.load()
    nbytes = int(lib.exl3_linear_group_scratch_bytes(m, k, nm, arr_n, K))
    _check(nbytes > 0, "exl3 linear group: unsupported shape")
    scratch = _linear_scratch(x2.device, nbytes)
    with _on_device(x2.device):
        _lib.check(lib.exl3_linear_group(x2.data_ptr(), _DT[x2.dtype], m, k, nm, arr_n,
                                         ptrs([t for t, _, _ in mats]), K, codebook, ptrs([su for _, su, _ in mats]),
                                         ptrs([sv for _, _, sv in mats]), ptrs(ys), _DT[out_dtype],
                                         scratch.data_ptr(), scratch.numel(), int(bool(precise)), _stream(x2.device)))
    return ys


def exl3_mgemm(x: torch.Tensor, trellis: list, suh: list, svh: list, K: int, mcg: bool, *,
               codebook: int | None = None, out_dtype: torch.dtype = torch.float32) -> list:
    """Grouped EXL3 GEMM over matrices sharing the input x [..., k]: returns
    one [m, n_j] output per matrix (fp32 by default, as the plugin's dense
    groups use it, recipe-lna/vllm_exl3_exl3.py.lna:546-613)."""
    bits = int(K)
    _check(len(trellis) == len(suh) == len(svh), "exl3_mgemm: trellis, suh and svh lists differ in length")
    x2 = x.contiguous().view(x.numel() // x.size(-1), x.size(-1))
    mats = [(t.contiguous(), su.contiguous(), sv.contiguous()) for t, su, sv in zip(trellis, suh, svh)]
    return linear_group_forward(x2, mats, bits, _codebook(mcg, codebook), out_dtype)


def _linear_checks(x, trellis, suh, svh, bits):
    _check(x.dim() >= 2, "x must have shape [..., in_features]")
    _check(x.size(-1) == trellis.size(0) * 16, "x feature dimension does not match trellis")
    _check(trellis.dim() == 3 and trellis.dtype == torch.int16 and trellis.size(2) == 16 * bits,
           "trellis must be int16 [rows/16, cols/16, 16*K]")
    _check(suh.dtype == torch.float16 and svh.dtype == torch.float16, "suh and svh must be float16")
    _check(x.is_cuda and trellis.is_cuda and suh.is_cuda and svh.is_cuda,
           "exl3 linear: the B200 build runs on CUDA tensors only")
    _check(x.device == trellis.device == suh.device == svh.device, "exl3 linear: tensors on different devices")


def exl3_gemv(x: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int,
              mcg: bool, mmode: int = 1, *, codebook: int | None = None) -> torch.Tensor:
    """Native small-m EXL3 GEMV, [m, k] -> [m, n] in x.dtype (bindings.cpp:135-148)."""
    bits = int(K)
    _check(x.dim() >= 2, "x must have shape [..., in_features]")
    m = x.numel() // x.size(-1)
    _check(1 <= m <= 8, "native GEMV supports 1 <= m <= 8")
    _check(int(mmode) in (0, 1), "mmode must be 0 or 1")
    _linear_checks(x, trellis, suh, svh, bits)
    x2 = x.contiguous().view(m, x.size(-1))
    return linear_forward(x2, trellis.contiguous(), suh.contiguous(), svh.contiguous(), bits,
                          _codebook(mcg, codebook), x.dtype)


def exl3_gemm(x: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int,
              mcg: bool, *, codebook: int | None = None) -> torch.Tensor:
    """Native tiled EXL3 GEMM, any row count (bindings.cpp:104-109)."""
    bits = int(K)
    _linear_checks(x, trellis, suh, svh, bits)
    x2 = x.contiguous().view(x.numel() // x.size(-1), x.size(-1))
    return linear_forward(x2, trellis.contiguous(), suh.contiguous(), svh.contiguous(), bits,
                          _codebook(mcg, codebook), x.dtype)


# --------------------------------------------------------------------- MoE
def lna2_moe_scratch_bytes(max_rows: int | None = None, topk: int = 8, hidden: int = 4096,
                           intermediate: int = 2048) -> int:
    """Scratch bytes for calls up to (max_rows, topk, hidden, intermediate).

    With no arguments: the build's row ceiling, top-8, 4096 x 2048, which
    covers every geometry of the plugin up to a single-GPU expert width."""
    rows = lna2_moe_max_rows() if max_rows is None else int(max_rows)
    return int(_lib.load().exl3_moe_scratch_bytes(rows, topk, hidden, intermediate))


def lna2_moe_max_rows() -> int:
    """Row ceiling of this build (the plugin asks, lna_moe_ticket.cu:491-492)."""
    return int(_lib.load().exl3_moe_max_rows())


def lna2_moe_prepare(K: int) -> None:
    _check(1 <= int(K) <= 4, "LNA2 supports K1..K4 in this build")
    _lib.call("exl3_moe_prepare", int(K))


def lna2_moe_info(K: int) -> list[int]:
    """14 ints; index 13 = concurrent streams (the plugin reads it, :1266-1273)."""
    import ctypes

    buf = (ctypes.c_int64 * 14)()
    _lib.call("exl3_moe_info", int(K), ctypes.addressof(buf))
    return [int(v) for v in buf]


def lna2_moe_status(scratch: torch.Tensor, clear: bool = False) -> int:
    """Device status word of a MoE scratch (0 = healthy).  Synchronizes.

    The word is sticky: kernels only OR bits into it (bit 0 dependency wait
    timed out, 1 misaligned trellis, 2 bit width out of range, 3 ring wait
    timed out, 4 plan overflow), until it is cleared here."""
    import ctypes

    word = ctypes.c_uint32(0)
    with _on_device(scratch.device):
        _lib.call("exl3_scratch_status", scratch.data_ptr(), 1, int(bool(clear)), ctypes.addressof(word),
                  _stream(scratch.device))
    return int(word.value)


def lna2_moe_status_word(scratch: torch.Tensor) -> torch.Tensor:
    """The status word of a MoE (or prefill) scratch as a 1-element int32
    device tensor, a view that stays valid as long as the scratch: a serving
    loop can copy it to pinned memory asynchronously (or test it inside a CUDA
    graph) after a layer, without a synchronization per call."""
    _check(scratch.is_cuda and scratch.dtype == torch.uint8 and scratch.numel() >= 12,
           "LNA2 scratch must be a CUDA uint8 buffer")
    return scratch[8:12].view(torch.int32)


def _raise_on_status(scratch: torch.Tensor) -> None:
    word = lna2_moe_status(scratch, clear=True)
    if word:
        raise RuntimeError(f"LNA2 device status word 0x{word:x}: a bounded wait or check failed inside the kernel "
                           "(bit 0 dependency timeout, 1 misaligned trellis, 2 bad bit width, 3 ring timeout, "
                           "4 plan overflow); the output of that call is not valid")


def check_status_default() -> bool:
    """EXL3_MOE_CHECK_STATUS=1 makes every MoE call synchronize and raise on a
    nonzero device status word (a validation mode: one sync per layer)."""
    return os.environ.get("EXL3_MOE_CHECK_STATUS", "0") not in ("", "0")


_IDS_DT = {torch.int32: 0, torch.int64: 1}


class _MoeArgs:
    """Argument checks shared by the MoE entries (lna_moe_ticket.cu:516-553)."""

    def __init__(self, x, out, tables, expert_ids, routing_weights, K, swiglu_limit, scratch, intermediate,
                 k_table, *, routed: bool, prefill: bool, expert_map=None):
        _check(x.is_cuda and x.dtype in ((torch.float16, torch.bfloat16, torch.float32) if routed and not prefill
                                          else (torch.float16, torch.bfloat16)),
               "LNA2 input must be CUDA fp16 or bf16")
        _check(x.dim() == 2 and x.size(1) % 128 == 0, "LNA2 input must be [m,hidden] with hidden % 128 == 0")
        if prefill:
            _check(x.size(0) >= 1, "LNA2 row count out of range (m >= 1)")
        else:
            _check(1 <= x.size(0) <= lna2_moe_max_rows(), "LNA2 row count out of range (1 <= m <= LNA2_MAX_M)")
        _check(x.is_contiguous(), "LNA2 input must be contiguous")
        _check(out.is_cuda and out.device == x.device and out.shape == x.shape and out.is_contiguous(),
               "LNA2 output must match x shape/device and be contiguous")
        _check(out.dtype in (torch.float16, torch.bfloat16, torch.float32), "LNA2 output must be fp16/bf16/fp32")
        topk = expert_ids.size(-1) if expert_ids.dim() == 2 else -1
        id_types = (torch.int32, torch.int64) if routed else (torch.int32,)
        _check(expert_ids.is_cuda and expert_ids.device == x.device and expert_ids.dtype in id_types
               and expert_ids.is_contiguous() and expert_ids.dim() == 2 and expert_ids.size(0) == x.size(0)
               and 1 <= topk <= 16,
               "LNA2 expert_ids must be contiguous int32 [m,topk]" if not routed
               else "LNA2 expert_ids must be contiguous int32 or int64 [m,topk]")
        w_types = (torch.float32, torch.bfloat16, torch.float16) if routed else (torch.float32,)
        _check(routing_weights.is_cuda and routing_weights.device == x.device and routing_weights.dtype in w_types
               and routing_weights.is_contiguous() and routing_weights.shape == expert_ids.shape,
               "LNA2 routing_weights must be contiguous fp32 [m,topk]" if not routed
               else "LNA2 routing_weights must be contiguous fp32/bf16/fp16 [m,topk]")
        n_experts = tables[0].numel()
        _check(1 <= n_experts <= 1024, "LNA2 pointer table has invalid expert count")
        for t in tables:
            _check(t.is_cuda and t.device == x.device and t.dtype == torch.int64 and t.is_contiguous()
                   and t.numel() == n_experts, "LNA2 pointer tables must be contiguous CUDA int64 [experts]")
        limit = float(swiglu_limit)
        _check(limit > 0.0 and limit < float("inf"), "LNA2 requires a finite positive SwiGLU limit")
        inter = int(intermediate)
        if prefill:
            need = lna2_moe_prefill_scratch_bytes(x.size(0), topk, x.size(1), inter, n_experts)
        else:
            need = int(_lib.load().exl3_moe_scratch_bytes(x.size(0), topk, x.size(1), inter))
        _check(scratch.is_cuda and scratch.device == x.device and scratch.dtype == torch.uint8
               and scratch.is_contiguous() and scratch.numel() >= need, "LNA2 scratch too small")
        if k_table is None:
            bits = int(K)
            _check(1 <= bits <= 4, "LNA2 supports K1..K4 in this build")
            kt_ptr, kmax = None, bits
        else:
            _check(k_table.is_cuda and k_table.device == x.device and k_table.dtype == torch.int32
                   and k_table.is_contiguous() and k_table.numel() == n_experts,
                   "LNA2 k_table must be contiguous CUDA int32 [experts]")
            kt_ptr, kmax = k_table.data_ptr(), int(K)
            bits = kmax
        map_ptr, n_global = None, 0
        if expert_map is not None:
            _check(expert_map.is_cuda and expert_map.device == x.device and expert_map.dtype == torch.int64
                   and expert_map.dim() == 1 and expert_map.is_contiguous() and expert_map.numel() >= 1,
                   "EXL3 expert_map must be a contiguous CUDA int64 [n_global] on the hidden-state device")
            map_ptr, n_global = expert_map.data_ptr(), expert_map.numel()
        self.topk, self.n_experts, self.limit, self.inter = topk, n_experts, limit, inter
        self.kt_ptr, self.kmax, self.bits = kt_ptr, kmax, bits
        self.tables = [t.data_ptr() for t in tables]
        self.route = _lib.MoeRoute(expert_ids.data_ptr(), _IDS_DT[expert_ids.dtype], routing_weights.data_ptr(),
                                   _DT[routing_weights.dtype], map_ptr, n_global)


def lna2_moe_decode(x: torch.Tensor, out: torch.Tensor,
                    gate_trellis: torch.Tensor, gate_suh: torch.Tensor, gate_svh: torch.Tensor,
                    up_trellis: torch.Tensor, up_suh: torch.Tensor, up_svh: torch.Tensor,
                    down_trellis: torch.Tensor, down_suh: torch.Tensor, down_svh: torch.Tensor,
                    expert_ids: torch.Tensor, routing_weights: torch.Tensor, K: int,
                    swiglu_limit: float, scratch: torch.Tensor, *, intermediate: int = 256,
                    k_table: torch.Tensor | None = None, codebook: int = 1,
                    precise: bool = False, tp_exchange=None, check_status: bool | None = None) -> torch.Tensor:
    """Routed-expert decode of one layer; writes and returns `out`.

    Argument checks follow recipe-lna/lna2/lna_moe_ticket.cu:516-553.  With
    `tp_exchange` (a dsv4_carve_b200.tp.MoeTpExchange), the tensor-parallel
    sum of the layer output over the exchange's ranks is done inside the
    kernel and every rank's `out` holds the full sum.  `check_status` (default:
    EXL3_MOE_CHECK_STATUS) synchronizes after the launch and raises
    RuntimeError if the device status word reports a failed wait or check."""
    tables = (gate_trellis, gate_suh, gate_svh, up_trellis, up_suh, up_svh, down_trellis, down_suh, down_svh)
    a = _MoeArgs(x, out, tables, expert_ids, routing_weights, K, swiglu_limit, scratch, intermediate, k_table,
                 routed=False, prefill=False)
    with _on_device(x.device):
        if tp_exchange is None:
            _lib.call("exl3_moe_decode", x.data_ptr(), _DT[x.dtype], out.data_ptr(), _DT[out.dtype],
                      x.size(0), x.size(1), a.inter, *a.tables, a.n_experts, a.kt_ptr, a.bits, a.kmax,
                      int(codebook), expert_ids.data_ptr(), routing_weights.data_ptr(), a.topk, a.limit,
                      scratch.data_ptr(), scratch.numel(), int(bool(precise)), _stream(x.device))
        else:
            _check(tp_exchange.table.device == x.device and tp_exchange.hidden == x.size(1)
                   and x.size(0) <= tp_exchange.max_rows, "LNA2 TP exchange does not match this call")
            _lib.call("exl3_moe_decode_tp", x.data_ptr(), _DT[x.dtype], out.data_ptr(), _DT[out.dtype],
                      x.size(0), x.size(1), a.inter, *a.tables, a.n_experts, a.kt_ptr, a.bits, a.kmax,
                      int(codebook), expert_ids.data_ptr(), routing_weights.data_ptr(), a.topk, a.limit,
                      scratch.data_ptr(), scratch.numel(), int(bool(precise)), tp_exchange.table.data_ptr(),
                      tp_exchange.rank, tp_exchange.world, tp_exchange.max_rows, _stream(x.device))
        if check_status_default() if check_status is None else check_status:
            _raise_on_status(scratch)
    return out


def lna2_moe_decode_routed(x: torch.Tensor, out: torch.Tensor,
                           gate_trellis: torch.Tensor, gate_suh: torch.Tensor, gate_svh: torch.Tensor,
                           up_trellis: torch.Tensor, up_suh: torch.Tensor, up_svh: torch.Tensor,
                           down_trellis: torch.Tensor, down_suh: torch.Tensor, down_svh: torch.Tensor,
                           expert_ids: torch.Tensor, routing_weights: torch.Tensor, K: int,
                           swiglu_limit: float, scratch: torch.Tensor, *, intermediate: int = 256,
                           k_table: torch.Tensor | None = None, codebook: int = 1, precise: bool = False,
                           expert_map: torch.Tensor | None = None, tp_exchange=None,
                           check_status: bool | None = None) -> torch.Tensor:
    """lna2_moe_decode on the router's raw outputs, in ONE launch: expert_ids
    int32 or int64 (global ids when `expert_map` is given), routing_weights
    fp32 / bf16 / fp16, x fp16 / bf16 / fp32.  The id mapping and casts the
    reference's plugin runs as torch operations before the kernel
    (map_topk_to_local and .to(int32) / .to(float32),
    recipe-lna/vllm_exl3_exl3.py.lna:963-987,1234-1236) happen inside it
    (exl3_moe_decode_routed)."""
    tables = (gate_trellis, gate_suh, gate_svh, up_trellis, up_suh, up_svh, down_trellis, down_suh, down_svh)
    a = _MoeArgs(x, out, tables, expert_ids, routing_weights, K, swiglu_limit, scratch, intermediate, k_table,
                 routed=True, prefill=False, expert_map=expert_map)
    tp_ptr, tp_rank, tp_world, tp_rows = None, 0, 0, 0
    if tp_exchange is not None:
        _check(tp_exchange.table.device == x.device and tp_exchange.hidden == x.size(1)
               and x.size(0) <= tp_exchange.max_rows, "LNA2 TP exchange does not match this call")
        tp_ptr, tp_rank = tp_exchange.table.data_ptr(), tp_exchange.rank
        tp_world, tp_rows = tp_exchange.world, tp_exchange.max_rows
    import ctypes

    with _on_device(x.device):
        _lib.call("exl3_moe_decode_routed", x.data_ptr(), _DT[x.dtype], out.data_ptr(), _DT[out.dtype],
                  x.size(0), x.size(1), a.inter, *a.tables, a.n_experts, a.kt_ptr, a.bits, a.kmax, int(codebook),
                  ctypes.addressof(a.route), a.topk, a.limit, scratch.data_ptr(), scratch.numel(),
                  int(bool(precise)), tp_ptr, tp_rank, tp_world, tp_rows, _stream(x.device))
        if check_status_default() if check_status is None else check_status:
            _raise_on_status(scratch)
    return out


# --------------------------------------------------------------------- prefill MoE
def lna2_moe_prefill_scratch_bytes(rows: int, topk: int = 8, hidden: int = 4096, intermediate: int = 2048,
                                   n_experts: int = 256) -> int:
    """Scratch bytes of lna2_moe_prefill for calls of up to `rows` tokens.

    Calls longer than lna2_moe_prefill_chunk_tokens(n_experts) run in chunks
    and need no more than one chunk's scratch."""
    return int(_lib.load().exl3_moe_prefill_scratch_bytes(int(rows), int(topk), int(hidden), int(intermediate),
                                                          int(n_experts)))


def lna2_moe_prefill_chunk_tokens(n_experts: int = 256) -> int:
    """Tokens per device route plan (2048 = the reference's TEMP_ROWS_FUSED at
    256 experts, recipe-lna/vllm_exl3_exl3.py.lna:57)."""
    return int(_lib.load().exl3_moe_prefill_chunk_tokens(int(n_experts)))


def lna2_moe_prefill(x: torch.Tensor, out: torch.Tensor,
                     gate_trellis: torch.Tensor, gate_suh: torch.Tensor, gate_svh: torch.Tensor,
                     up_trellis: torch.Tensor, up_suh: torch.Tensor, up_svh: torch.Tensor,
                     down_trellis: torch.Tensor, down_suh: torch.Tensor, down_svh: torch.Tensor,
                     expert_ids: torch.Tensor, routing_weights: torch.Tensor, K: int,
                     swiglu_limit: float, scratch: torch.Tensor, *, intermediate: int = 256,
                     k_table: torch.Tensor | None = None, codebook: int = 1,
                     expert_map: torch.Tensor | None = None, check_status: bool | None = None) -> torch.Tensor:
    """Routed-expert layer for prefill chunks on the tensor cores; writes and
    returns `out`.  Same arguments and checks as lna2_moe_decode, any row
    count; the weights enter the MMA rounded to fp16 (the reference's decoded
    values).  Like lna2_moe_decode_routed it also takes int64 ids, bf16 / fp16
    routing weights and an `expert_map`, read by the device route plan."""
    tables = (gate_trellis, gate_suh, gate_svh, up_trellis, up_suh, up_svh, down_trellis, down_suh, down_svh)
    routed = (expert_map is not None or expert_ids.dtype != torch.int32
              or routing_weights.dtype != torch.float32)
    a = _MoeArgs(x, out, tables, expert_ids, routing_weights, K, swiglu_limit, scratch, intermediate, k_table,
                 routed=routed, prefill=True, expert_map=expert_map)
    import ctypes

    with _on_device(x.device):
        if not routed:
            _lib.call("exl3_moe_prefill", x.data_ptr(), _DT[x.dtype], out.data_ptr(), _DT[out.dtype],
                      x.size(0), x.size(1), a.inter, *a.tables, a.n_experts, a.kt_ptr, a.bits, a.kmax,
                      int(codebook), expert_ids.data_ptr(), routing_weights.data_ptr(), a.topk, a.limit,
                      scratch.data_ptr(), scratch.numel(), _stream(x.device))
        else:
            _lib.call("exl3_moe_prefill_routed", x.data_ptr(), _DT[x.dtype], out.data_ptr(), _DT[out.dtype],
                      x.size(0), x.size(1), a.inter, *a.tables, a.n_experts, a.kt_ptr, a.bits, a.kmax,
                      int(codebook), ctypes.addressof(a.route), a.topk, a.limit, scratch.data_ptr(),
                      scratch.numel(), _stream(x.device))
        if check_status_default() if check_status is None else check_status:
            _raise_on_status(scratch)
    return out


_PREFILL_SCRATCH: dict = {}


def _prefill_scratch(device: torch.device, nbytes: int) -> torch.Tensor:
    """One scratch tensor per device, grown on demand (prefill is not captured)."""
    key = (device.type, device.index)
    buf = _PREFILL_SCRATCH.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _PREFILL_SCRATCH[key] = buf
    return buf


def exl3_moe(hidden_state, output_state, expert_count, token_sorted, weight_sorted,
             temp_state_g, temp_state_u, temp_intermediate_g, temp_intermediate_u,
             act_function, K_gate, K_up, K_down,
             gate_ptrs_trellis, gate_ptrs_suh, gate_ptrs_svh,
             up_ptrs_trellis, up_ptrs_suh, up_ptrs_svh,
             down_ptrs_trellis, down_ptrs_suh, down_ptrs_svh,
             gate_mcg, gate_mul1, up_mcg, up_mul1, down_mcg, down_mul1,
             act_limit, num_active=-1):
    """exllamav3_ext.exl3_moe with its positional signature and checks
    (orders/F1-ref/exl3_moe.cu:99-210): output_state (fp32, [T, hidden]) +=
    the routed experts' contribution of the sorted slots.  The sorted-slot
    form (expert_count [E+1] int64, token_sorted / weight_sorted [T*topk];
    slots of expert E are skipped) is turned back into per-token slots and
    handed to lna2_moe_prefill; the temp buffers are not used (this build
    keeps its own scratch)."""
    _check(hidden_state.is_cuda and hidden_state.dtype == torch.float16 and hidden_state.dim() == 2,
           "hidden_state must be CUDA fp16 [T, hidden]")
    _check(output_state.dtype == torch.float32 and output_state.shape == hidden_state.shape,
           "output_state must be fp32 with hidden_state's shape")
    _check(expert_count.dtype == torch.int64 and expert_count.dim() == 1, "expert_count must be int64 [E+1]")
    _check(token_sorted.dtype == torch.int64 and token_sorted.shape == weight_sorted.shape,
           "token_sorted / weight_sorted must be [T*topk]")
    _check(gate_mcg == up_mcg == down_mcg and gate_mul1 == up_mul1 == down_mul1,
           "MoE kernel: gate/up/down must share the same codebook")
    _check(gate_mcg != gate_mul1, "MoE kernel: Only mcg and mul1 codebooks are supported")
    _check(K_gate == K_up == K_down, "MoE kernel: gate/up/down must share one bit width in this build")
    if num_active == 0:
        return
    T, hidden = hidden_state.shape
    n_experts = expert_count.numel() - 1
    topk = token_sorted.numel() // T
    _check(topk * T == token_sorted.numel(), "token_sorted must hold T*topk slots")
    ends = torch.cumsum(expert_count, 0)
    pos = torch.arange(token_sorted.numel(), device=token_sorted.device)
    expert_of = torch.searchsorted(ends, pos, right=True)
    order = torch.argsort(token_sorted, stable=True)
    ids = expert_of[order].view(T, topk)
    ids = torch.where(ids < n_experts, ids, torch.full_like(ids, -1)).to(torch.int32).contiguous()
    w = weight_sorted[order].view(T, topk).to(torch.float32).contiguous()
    inter = int(temp_intermediate_g.size(-1))
    y = torch.empty((T, hidden), dtype=torch.float32, device=hidden_state.device)
    scratch = _prefill_scratch(hidden_state.device,
                               lna2_moe_prefill_scratch_bytes(T, topk, hidden, inter, n_experts))
    lna2_moe_prefill(hidden_state.contiguous(), y, gate_ptrs_trellis, gate_ptrs_suh, gate_ptrs_svh,
                     up_ptrs_trellis, up_ptrs_suh, up_ptrs_svh, down_ptrs_trellis, down_ptrs_suh, down_ptrs_svh,
                     ids, w, int(K_gate), float(act_limit), scratch, intermediate=inter,
                     codebook=2 if gate_mul1 else 1)
    output_state.add_(y)
