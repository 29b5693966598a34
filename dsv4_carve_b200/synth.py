"""Seeded synthetic EXL3 weights, activations and routes for the benchmark configs.

There is no checkpoint or dataset on the box: packed trellis words are
uniform random uint16, su / sv are +-1 Bernoulli(0.5), the per-output-channel
scale |N(0,1)| * 0.02 is folded into svh (EXL3 keeps no separate scale
tensor), activations are N(0,1).  Everything is generated from explicit seeds
with torch generators on the target device, so every rank of a TP run
produces identical full tensors and then keeps its own shard.

Shapes follow the EXL3 layout: trellis int16 [in/16, out/16, 16*K], suh fp16
[in], svh fp16 [out].
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

CB_3INST, CB_MCG, CB_MUL1 = 0, 1, 2
MCG_MARKER_SIGNED_INT32 = -877912083      # recipe-lna/vllm_exl3_exl3.py.lna:50-53


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def random_trellis(kt: int, nt: int, K: int, gen: torch.Generator, device) -> torch.Tensor:
    return torch.randint(-32768, 32768, (kt, nt, 16 * K), generator=gen, device=device, dtype=torch.int32
                         ).to(torch.int16)


def random_signs(n: int, gen: torch.Generator, device) -> torch.Tensor:
    bits = torch.randint(0, 2, (n,), generator=gen, device=device)
    return (1 - 2 * bits).to(torch.float16)


def random_svh(n: int, gen: torch.Generator, device, scale: float = 0.02) -> torch.Tensor:
    sv = random_signs(n, gen, device).float()
    mag = torch.randn(n, generator=gen, device=device).abs() * scale
    return (sv * mag).to(torch.float16)


@dataclass
class DenseWeight:
    trellis: torch.Tensor
    suh: torch.Tensor
    svh: torch.Tensor
    K: int
    cb: int

    @property
    def in_features(self) -> int:
        return self.suh.numel()

    @property
    def out_features(self) -> int:
        return self.svh.numel()

    def nbytes(self) -> int:
        return self.trellis.numel() * 2 + self.suh.numel() * 2 + self.svh.numel() * 2

    def to(self, device) -> "DenseWeight":
        return DenseWeight(self.trellis.to(device), self.suh.to(device), self.svh.to(device), self.K, self.cb)


def make_dense(k: int, n: int, K: int, seed: int, device="cpu", cb: int = CB_MCG) -> DenseWeight:
    g = _gen(device, seed)
    t = random_trellis(k // 16, n // 16, K, g, device)
    suh = random_signs(k, g, device)
    svh = random_svh(n, g, device)
    return DenseWeight(t, suh, svh, K, cb)


def shard_col(w: DenseWeight, rank: int, world: int) -> DenseWeight:
    """Column parallel: trellis dim 1 and svh dim 0 (vllm_exl3_exl3.py.lna:855-861)."""
    if world == 1:
        return w
    nt = w.trellis.size(1)
    assert nt % world == 0, "column shard must keep whole 16-wide tiles"
    c = nt // world
    return DenseWeight(w.trellis[:, rank * c:(rank + 1) * c].contiguous(), w.suh,
                       w.svh[rank * c * 16:(rank + 1) * c * 16].contiguous(), w.K, w.cb)


def shard_row(w: DenseWeight, rank: int, world: int) -> DenseWeight:
    """Row parallel: trellis dim 0 and suh dim 0 (vllm_exl3_exl3.py.lna:864-871)."""
    if world == 1:
        return w
    kt = w.trellis.size(0)
    assert kt % world == 0
    c = kt // world
    return DenseWeight(w.trellis[rank * c:(rank + 1) * c].contiguous(),
                       w.suh[rank * c * 16:(rank + 1) * c * 16].contiguous(), w.svh, w.K, w.cb)


def block_range(nblocks: int, rank: int, world: int) -> tuple:
    """Whole 128-wide Hadamard blocks of a dimension split over `world` ranks
    as evenly as possible (e.g. 1536 = 12 blocks over 8 ranks: 2,2,2,2,1,1,1,1).
    Returns (first block, block count) of `rank`."""
    base, extra = divmod(nblocks, world)
    return rank * base + min(rank, extra), base + (1 if rank < extra else 0)


def shard_col_blocks(w: DenseWeight, rank: int, world: int) -> DenseWeight:
    """Column parallel in whole 128-column blocks (uneven when the block count
    does not divide by the world size)."""
    if world == 1:
        return w
    b0, nb = block_range(w.out_features // 128, rank, world)
    assert nb > 0, "more ranks than 128-column blocks"
    t = w.trellis[:, b0 * 8:(b0 + nb) * 8].contiguous()
    return DenseWeight(t, w.suh, w.svh[b0 * 128:(b0 + nb) * 128].contiguous(), w.K, w.cb)


def shard_row_blocks(w: DenseWeight, rank: int, world: int) -> DenseWeight:
    """Row parallel in whole 128-row blocks (the partial outputs are summed)."""
    if world == 1:
        return w
    b0, nb = block_range(w.in_features // 128, rank, world)
    assert nb > 0, "more ranks than 128-row blocks"
    t = w.trellis[b0 * 8:(b0 + nb) * 8].contiguous()
    return DenseWeight(t, w.suh[b0 * 128:(b0 + nb) * 128].contiguous(), w.svh, w.K, w.cb)


@dataclass
class MoeLayer:
    """One routed-MoE layer (possibly a TP shard) with the plugin's 9 pointer tables."""
    E: int
    H: int
    I: int                      # intermediate width held by this rank
    kbits: list
    cb: int
    experts: list = field(default_factory=list)   # [{'gate'|'up'|'down': DenseWeight}]
    tables: dict = field(default_factory=dict)     # name -> int64 [E] device tensor
    ktab: torch.Tensor | None = None

    def expert_bytes(self, e: int) -> int:
        return sum(self.experts[e][p].nbytes() for p in ("gate", "up", "down"))

    def unique_bytes(self, ids: torch.Tensor) -> int:
        u = torch.unique(ids.flatten())
        return sum(self.expert_bytes(int(e)) for e in u.tolist() if 0 <= int(e) < self.E)

    def build_tables(self) -> None:
        dev = self.experts[0]["gate"].trellis.device
        names = {"gate_trellis": ("gate", "trellis"), "gate_suh": ("gate", "suh"), "gate_svh": ("gate", "svh"),
                 "up_trellis": ("up", "trellis"), "up_suh": ("up", "suh"), "up_svh": ("up", "svh"),
                 "down_trellis": ("down", "trellis"), "down_suh": ("down", "suh"),
                 "down_svh": ("down", "svh")}
        for name, (proj, attr) in names.items():
            ptrs = [getattr(self.experts[e][proj], attr).data_ptr() for e in range(self.E)]
            self.tables[name] = torch.tensor(ptrs, dtype=torch.int64, device=dev)
        self.ktab = torch.tensor(self.kbits, dtype=torch.int32, device=dev)

    def table_list(self) -> list:
        return [self.tables[n] for n in ("gate_trellis", "gate_suh", "gate_svh", "up_trellis", "up_suh",
                                          "up_svh", "down_trellis", "down_suh", "down_svh")]

    def to_cpu(self) -> "MoeLayer":
        cpu = MoeLayer(E=self.E, H=self.H, I=self.I, kbits=self.kbits, cb=self.cb)
        cpu.experts = [{p: w.to("cpu") for p, w in ex.items()} for ex in self.experts]
        return cpu


def expert_bits(E: int, seed: int, choices=(2, 3), uniform: int | None = None) -> list:
    if uniform is not None:
        return [int(uniform)] * E
    g = torch.Generator().manual_seed(int(seed) ^ 0x5EED)
    idx = torch.randint(0, len(choices), (E,), generator=g)
    return [int(choices[i]) for i in idx.tolist()]


def make_moe_layer(E: int, H: int, I_full: int, kbits: list, seed: int, device="cpu", cb: int = CB_MCG,
                   rank: int = 0, world: int = 1) -> MoeLayer:
    """Full-width experts are generated from (seed, expert) and sharded for TP:
    gate/up keep columns [rank*I/world, (rank+1)*I/world), down keeps those rows."""
    I = I_full // world
    assert I % 128 == 0, "TP shard of the intermediate dim must keep whole 128-blocks"
    layer = MoeLayer(E=E, H=H, I=I, kbits=list(kbits), cb=cb)
    for e in range(E):
        K = int(kbits[e])
        g = _gen(device, seed * 100003 + e)
        gate = DenseWeight(random_trellis(H // 16, I_full // 16, K, g, device), random_signs(H, g, device),
                           random_svh(I_full, g, device), K, cb)
        up = DenseWeight(random_trellis(H // 16, I_full // 16, K, g, device), random_signs(H, g, device),
                         random_svh(I_full, g, device), K, cb)
        down = DenseWeight(random_trellis(I_full // 16, H // 16, K, g, device), random_signs(I_full, g, device),
                           random_svh(H, g, device), K, cb)
        layer.experts.append({"gate": shard_col(gate, rank, world), "up": shard_col(up, rank, world),
                              "down": shard_row(down, rank, world)})
    layer.build_tables()
    return layer


def activations(T: int, H: int, seed: int, device="cpu", dtype=torch.float16, scale: float = 1.0) -> torch.Tensor:
    g = _gen(device, seed)
    return (torch.randn((T, H), generator=g, device=device) * scale).to(dtype)


def route_uniform(T: int, E: int, topk: int, seed: int, device="cpu"):
    """Router logits N(0,1) -> top-k -> softmax over the k selected logits."""
    g = _gen("cpu", seed)
    logits = torch.randn((T, E), generator=g)
    val, idx = torch.topk(logits, topk, dim=1)
    w = torch.softmax(val, dim=1)
    return idx.to(torch.int32).contiguous().to(device), w.float().contiguous().to(device)


def route_zipf(T: int, E: int, topk: int, seed: int, s: float = 1.1, device="cpu"):
    """Zipf(s) expert popularity over a seeded permutation; top-k distinct
    experts per token drawn without replacement in proportion to it."""
    g = _gen("cpu", seed)
    perm = torch.randperm(E, generator=g)
    mass = 1.0 / torch.arange(1, E + 1, dtype=torch.float64) ** s
    p = torch.empty(E, dtype=torch.float64)
    p[perm] = mass / mass.sum()
    idx = torch.multinomial(p.expand(T, E), topk, replacement=False, generator=g)
    logits = torch.randn((T, topk), generator=g)
    w = torch.softmax(logits, dim=1)
    return idx.to(torch.int32).contiguous().to(device), w.float().contiguous().to(device)
