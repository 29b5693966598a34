"""LinearEXL3-compatible dense linear on the B200 kernels.

Mirrors the interface the vllm-exl3 plugin uses from exllamav3's LinearEXL3
(recipe-lna/exllamav3/exl3.py.lna:16-139; attributes read by the plugin at
recipe-lna/vllm_exl3_exl3.py.lna:1337-1366,1552-1558): constructor
arguments, ``trellis / suh / svh / K / in_features / out_features /
mcg_tensor / mul1_tensor`` attributes and ``forward(x, params, out_dtype)``.
``forward`` calls the C ABI's exl3_linear, which picks the kernel by row
count: below 64 rows the GEMV ring kernel (register decode into mma.sync,
32 rows per pass), from 64 rows the tcgen05 tensor-core path (weights decoded
once into shared memory, applied to up to 512 rows per pass) -- the B200
counterpart of the reference's GEMV / reconstruct + hgemm split at 144 rows.
"""
from __future__ import annotations

import torch

from . import vllm_exl3_c as _ext

AUTO_RECONSTRUCT_THRESHOLD = 144   # exl3.py.lna:10 (kept for interface parity)


def unpack_bf(bitfield: torch.Tensor) -> torch.Tensor:
    """Packed sign bits (int16, 16 per word, LSB first) -> +-1 fp16 vector
    (exl3.py.lna:122-139: a set bit means -1)."""
    b = bitfield.view(torch.uint16).to(torch.int32)
    masks = (1 << torch.arange(16, device=b.device, dtype=torch.int32))
    bits = ((b.unsqueeze(-1) & masks) > 0).flatten()
    return (1.0 - bits.to(torch.float16) * 2.0).contiguous()


class LinearEXL3:
    quant_type: str = "exl3"

    def __init__(self, config=None, in_features: int | None = None, out_features: int | None = None,
                 scale=None, su=None, sv=None, suh=None, svh=None, trellis=None, mcg=None, mul1=None,
                 bias=None, out_dtype=None, transformers_fix: bool = False, key: str | None = None):
        assert scale is None, "EXL3 keeps its scales in svh; a separate scale tensor is not accepted"
        assert su is not None or suh is not None, "input signs missing: give su (bit-packed) or suh (fp16)"
        assert sv is not None or svh is not None, "output signs missing: give sv (bit-packed) or svh (fp16)"
        assert trellis is not None, "the packed trellis tensor is missing"
        if su is not None: assert su.dtype == torch.int16, "su must be int16 bit words"
        if sv is not None: assert sv.dtype == torch.int16, "sv must be int16 bit words"
        if suh is not None: assert suh.dtype == torch.half, "suh must be fp16"
        if svh is not None: assert svh.dtype == torch.half, "svh must be fp16"
        assert trellis.dtype == torch.int16, "trellis must be int16"
        assert len(trellis.shape) == 3, "trellis must be [in/16, out/16, 16*K]"
        if bias is not None and bias.dtype == torch.float:
            bias = bias.to(torch.half)
        self.config = config
        self.key = key
        self.transformers_fix = transformers_fix
        self.su = None
        self.sv = None
        self.suh = (suh if suh is not None else unpack_bf(su)).contiguous()
        self.svh = (svh if svh is not None else unpack_bf(sv)).contiguous()
        self.trellis = trellis.contiguous()
        self.K = trellis.shape[-1] // 16
        self.in_features = int(in_features if in_features is not None else self.suh.numel())
        self.out_features = int(out_features if out_features is not None else self.svh.numel())
        assert self.trellis.shape[0] * 16 == self.in_features and self.trellis.shape[1] * 16 == self.out_features
        self.bias = bias
        self.out_dtype = out_dtype
        self.default_out_dtype = out_dtype or torch.half
        self.mcg_tensor = mcg
        self.mul1_tensor = mul1
        self.mcg = mcg is not None
        self.mul1 = mul1 is not None
        # exllamav3 codebook selection: MCG marker -> MCG, MUL1 marker -> MUL1, else 3INST
        self.codebook = 1 if self.mcg else (2 if self.mul1 else 0)
        # fp16-rounded weights in the MMA, as the reference decoder rounds them
        self.precise = True

    def forward(self, x: torch.Tensor, params: dict | None = None, out_dtype: torch.dtype | None = None):
        assert x.is_contiguous(), f"LinearEXL3 {self.key}: non-contiguous input {tuple(x.shape)}"
        rows = x.numel() // x.shape[-1]
        dtype = out_dtype or self.default_out_dtype
        x2 = x.view(rows, self.in_features)
        y = _ext.linear_forward(x2, self.trellis, self.suh, self.svh, self.K, self.codebook, dtype, self.precise)
        if self.bias is not None:
            y += self.bias
        return y.view(*x.shape[:-1], self.out_features)

    def get_inner_weight_tensor(self) -> torch.Tensor:
        return _ext.dequant_trellis(self.trellis, self.suh, self.svh, self.K, self.mcg,
                                    codebook=self.codebook, inner_only=True)

    def get_weight_tensor(self) -> torch.Tensor:
        return _ext.dequant_trellis(self.trellis, self.suh, self.svh, self.K, self.mcg, codebook=self.codebook)

    def unload(self):
        pass
