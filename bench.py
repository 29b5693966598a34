"""Benchmark of the EXL3 decode hot path on B200.

Default workload (the lna2 case): one routed-MoE decode
layer -- hidden 4096, 256 experts with gate/up [4096 -> 2048] and down
[2048 -> 4096], per-expert K in {2, 3} (p = 0.5), T = 4 tokens, router logits
N(0,1) -> top-8 -> softmax over the 8, fp16 activations N(0,1), MCG codebook.
A step is one layer over one batch of T tokens.  Steps cycle over --layers
independent layers (seeded), so every step streams its experts from HBM:
one layer's unique expert bytes (~240 MB at T = 4) already exceed the 126 MB
L2, and the other layers stream through L2 between two uses of a layer.

With --gpus N (torchrun, one rank per GPU) the layer is tensor-parallel:
each rank holds the intermediate columns [r*2048/N, (r+1)*2048/N) of every
expert's gate/up and those rows of down, computes a partial [T, 4096] and one
NCCL all-reduce sums it.  Total work is fixed as N grows ("strong").

metric/value: packed-weight bytes streamed per second (algorithmic bytes:
unique experts' trellis + suh + svh of every rank's shard, plus activations),
aggregated over ranks; us_per_layer is the step time.  `e2e` is the same
metric through the public plugin call (vllm_exl3_c.lna2_moe_decode) with
pinned host inputs copied in and the output copied back every step.

--impl reference times the reference's own CPU decode + matmul
(recipe-lna/lna2/bindings.cpp:16-101,135-148, built from source into
oracle/_ref) on a bounded sample of the same workload, on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "routed-MoE decode layer: packed-weight HBM GB/s (config 2: T=4, top-8 of 256 experts, K2/K3, hidden 4096)"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0
NCU_TRAFFIC_FILE = ROOT / "profiles" / "moe_kernel_config2_traffic.json"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--stack", action="store_true",
                    help="moe: config 4(a), the decode layer stack (every 8th layer all-K2); a step is one layer, "
                         "the line adds the whole stack's time per decode step")
    ap.add_argument("--tokens", type=int, default=4)
    ap.add_argument("--route", choices=["uniform", "zipf"], default="uniform")
    ap.add_argument("--config", choices=["moe", "dense", "single", "prefill"], default="moe",
                    help="moe: config 2/3 routed-MoE layer (the headline); dense: config 1 K6 linears; "
                         "single: config 0, one 4096 x 4096 K4 3INST linear")
    ap.add_argument("--rows", type=int, default=4, help="dense: activation rows R")
    ap.add_argument("--group", action="store_true",
                    help="dense: the two 4096-input matrices in one grouped launch (exl3_linear_group)")
    ap.add_argument("--prefill-tokens", type=int, default=512, help="prefill: tokens per chunk")
    ap.add_argument("--emulate-tp", type=int, default=1,
                    help="one GPU: run rank 0's shard of a TP-N layer (intermediate / N), no collective")
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--precise", action="store_true", help="fp16-rounded weights in the MMA")
    ap.add_argument("--allreduce", choices=["fused", "nccl"], default="fused",
                    help="N > 1: TP sum inside the MoE kernel over NVLink (fused) or NCCL after it")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    return ap.parse_args()


# ----------------------------------------------------------------------------- env
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            v = float(json.loads(p.read_text())["hbm_gbs"])
            return v, "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


class NvmlClockSampler:
    """SM clock, max clock, power and clock-event reasons of this GPU read
    through NVML every few milliseconds while running (reading only), so
    that even a timed region of a few tens of milliseconds holds samples."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, bus_id: str | None, period_s: float = 0.004):
        import pynvml

        self.nv = pynvml
        pynvml.nvmlInit()
        self.h = None
        n = pynvml.nvmlDeviceGetCount()
        for i in range(n):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            pci = pynvml.nvmlDeviceGetPciInfo(h).busId
            pci = pci.decode() if isinstance(pci, bytes) else pci
            if bus_id and pci.lower().endswith(str(bus_id).lower()):
                self.h = h
        if self.h is None:
            raise RuntimeError("NVML: no device with this PCI bus id")
        self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        self.period = period_s
        self.samples: list = []
        self.run = False
        self.t = None

    def start(self):
        self.run = True
        self.t = threading.Thread(target=self._loop, daemon=True)
        self.t.start()

    def _loop(self):
        nv = self.nv
        while self.run:
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                rs = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
                self.samples.append((time.time(), sm, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def stop(self):
        self.run = False
        if self.t is not None:
            self.t.join(timeout=2)

    def summary(self, t0: float, t1: float):
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        use = inside or self.samples
        if not use:
            return None
        reasons = sorted({n for _, _, rs in use for n, b in self.REASONS if rs & b})
        return {"sm_mhz": statistics.median(sm for _, sm, _ in use), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(use), "in_region": bool(inside), "source": "nvml"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id: str | None):
        self.bus = str(bus_id or "").lower()   # "bb:dd.0" suffix of nvidia-smi's pci.bus_id
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.t is not None:
            self.t.join(timeout=2)

    def summary(self, t0: float, t1: float):
        rows = []
        for ts, line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            if self.bus and not f[1].lower().endswith(self.bus):
                continue
            rows.append((ts, f))
        inside = [f for ts, f in rows if t0 <= ts <= t1] or [f for ts, f in rows]
        if not inside:
            return None
        sm = [float(f[2]) for f in inside if f[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for f in inside for i in range(4) if f[6 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(inside[0][3]) if inside[0][3].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(inside),
                "in_region": any(t0 <= ts <= t1 for ts, _ in rows)}


# ----------------------------------------------------------------------------- workload
class MoeWorkload:
    def __init__(self, args, rank, world, dev):
        import torch

        from dsv4_carve_b200 import synth
        from dsv4_carve_b200 import vllm_exl3_c as ext

        self.torch, self.ext, self.synth = torch, ext, synth
        self.args, self.rank, self.world, self.dev = args, rank, world, dev
        self.E, self.H, self.I_full, self.T, self.topk = args.experts, 4096, 2048, args.tokens, 8
        self.shards = world if world > 1 else max(1, args.emulate_tp)
        self.I = self.I_full // self.shards
        self.layers, self.routes, self.xs, self.ubytes, self.uniq = [], [], [], [], []
        for li in range(args.layers):
            seed = 1000 + li
            kbits = synth.expert_bits(self.E, seed)
            if args.stack and li % 8 == 7:
                kbits = [2] * self.E        # config 4: K = 2 for 1 in 8 layers
            L = synth.make_moe_layer(self.E, self.H, self.I_full, kbits, seed, device=dev, cb=synth.CB_MCG,
                                     rank=rank, world=self.shards)
            if args.route == "zipf":
                ids, w = synth.route_zipf(self.T, self.E, self.topk, seed=seed + 7, device=dev)
            else:
                ids, w = synth.route_uniform(self.T, self.E, self.topk, seed=seed + 7, device=dev)
            x = synth.activations(self.T, self.H, seed=seed + 11, device=dev, dtype=torch.float16)
            self.layers.append(L)
            self.routes.append((ids, w))
            self.xs.append(x)
            act = self.T * self.H * 2 * 2   # x in, out written (fp16)
            self.ubytes.append(L.unique_bytes(ids) + act)
            self.uniq.append(int(torch.unique(ids).numel()))
        self.kmax = 3
        self.scratch = torch.zeros(ext.lna2_moe_scratch_bytes(self.T, self.topk, self.H, self.I), dtype=torch.uint8,
                                   device=dev)
        self.outs = [torch.empty((self.T, self.H), dtype=torch.float16, device=dev) for _ in self.layers]
        ext.lna2_moe_prepare(self.kmax)
        # pre-bound C-ABI calls for the device-resident path (no per-call Python checks)
        from dsv4_carve_b200 import _lib

        self._lib = _lib.load()
        self.exchange = None
        self.allreduce_note = None
        if world > 1 and args.allreduce == "fused":
            from dsv4_carve_b200.tp import MoeTpExchange

            # every rank must agree on the path: the setup outcome is all-reduced
            try:
                ex = MoeTpExchange(None, dev, max_rows=self.T, hidden=self.H)
                ok = torch.ones(1, device=dev)
            except Exception as exc:      # no peer access: NCCL after the kernel instead
                ex, ok = None, torch.zeros(1, device=dev)
                self.allreduce_note = f"fused exchange setup failed ({exc!r}); NCCL used"
            torch.distributed.all_reduce(ok, op=torch.distributed.ReduceOp.MIN)
            if ok.item() == 1:
                self.exchange = ex
            else:
                if ex is not None:
                    torch.distributed.barrier()
                    ex.close()
                self.allreduce_note = self.allreduce_note or "fused exchange setup failed on a peer rank; NCCL used"
        self._argv = [self.argv_for(li, self.xs[li].data_ptr(), self.routes[li][0].data_ptr(),
                                    self.routes[li][1].data_ptr(), self.outs[li].data_ptr(), int(args.precise))
                      for li in range(len(self.layers))]
        # End-to-end path: each step's inputs (x fp16, ids int32, weights fp32)
        # sit packed in one pinned host buffer and cross in ONE host-to-device
        # copy into a device staging buffer, the layer runs through the
        # pre-bound C-ABI call on views of it, and the output comes back.
        nx, ni = self.T * self.H * 2, self.T * self.topk * 4
        self.stage_bytes = nx + 2 * ni
        self.h_stage, self.d_stage, self.e2e_argv = [], [], []
        for li in range(len(self.layers)):
            ids, w = self.routes[li]
            h = torch.empty(self.stage_bytes, dtype=torch.uint8).pin_memory()
            h[:nx].copy_(self.xs[li].cpu().view(torch.uint8).reshape(-1))
            h[nx:nx + ni].copy_(ids.cpu().view(torch.uint8).reshape(-1))
            h[nx + ni:].copy_(w.cpu().view(torch.uint8).reshape(-1))
            d = torch.empty(self.stage_bytes, dtype=torch.uint8, device=dev)
            base = d.data_ptr()
            self.h_stage.append(h)
            self.d_stage.append(d)
            self.e2e_argv.append(self.argv_for(li, base, base + nx, base + nx + ni, self.outs[li].data_ptr(),
                                               int(args.precise)))
        self.h_out = [torch.empty((self.T, self.H), dtype=torch.float16).pin_memory() for _ in self.layers]
        self.h2d = self.stage_bytes
        self.d2h = self.T * self.H * 2

    def argv_for(self, li, x_ptr, ids_ptr, w_ptr, out_ptr, precise):
        """Arguments of exl3_moe_decode (+ the exchange of exl3_moe_decode_tp) for layer li."""
        from dsv4_carve_b200 import _lib

        L = self.layers[li]
        argv = (x_ptr, _lib.DT_F16, out_ptr, _lib.DT_F16, self.T, self.H, self.I,
                *[t.data_ptr() for t in L.table_list()], self.E, L.ktab.data_ptr(), self.kmax, self.kmax,
                self.synth.CB_MCG, ids_ptr, w_ptr, self.topk, 10.0, self.scratch.data_ptr(), self.scratch.numel(),
                precise)
        if self.exchange is not None:
            argv = argv + (self.exchange.table.data_ptr(), self.exchange.rank, self.exchange.world,
                           self.exchange.max_rows)
        return argv

    def call(self, argv, stream_handle):
        fn = self._lib.exl3_moe_decode_tp if self.exchange is not None else self._lib.exl3_moe_decode
        rc = fn(*argv, stream_handle)
        if rc:
            raise RuntimeError(self._lib.exl3_last_error().decode())

    def launch(self, i, stream_handle):
        self.call(self._argv[i % len(self.layers)], stream_handle)

    def check(self, li, snap, stream_handle):
        """Validation of the timed run (every rank, same collective steps):
        the device status word; a fresh run of layer li must equal the output
        the timed region left (`snap`) bit for bit; and the precise arithmetic
        (fp16-rounded weights, a second computation) must agree with it within
        2e-3 (times the output scale when that is above 1)."""
        torch = self.torch
        dev = self.dev
        again = torch.empty_like(self.outs[li])
        prec = torch.empty_like(self.outs[li])
        ids, w = self.routes[li]
        self.call(self.argv_for(li, self.xs[li].data_ptr(), ids.data_ptr(), w.data_ptr(), again.data_ptr(),
                                int(self.args.precise)), stream_handle)
        self.allreduce(again)
        self.call(self.argv_for(li, self.xs[li].data_ptr(), ids.data_ptr(), w.data_ptr(), prec.data_ptr(), 1),
                  stream_handle)
        self.allreduce(prec)
        torch.cuda.synchronize(dev)
        status = self.ext.lna2_moe_status(self.scratch)
        err = float((snap.float() - prec.float()).abs().max().item())
        scale = max(1.0, float(prec.float().abs().max().item()))
        return status, bool(torch.equal(again, snap)), err, 2e-3 * scale

    def allreduce(self, out):
        # the fused path has summed over the ranks inside the kernel
        if self.world > 1 and self.exchange is None:
            self.torch.distributed.all_reduce(out)

    def close(self):
        if self.exchange is not None:
            self.torch.distributed.barrier()
            self.torch.cuda.synchronize()
            self.exchange.close()
            self.exchange = None

    def step(self, i, stream_handle):
        self.launch(i, stream_handle)
        self.allreduce(self.outs[i % len(self.layers)])

    def e2e_step(self, i, stream_handle):
        li = i % len(self.layers)
        self.d_stage[li].copy_(self.h_stage[li], non_blocking=True)
        out = self.outs[li]
        self.call(self.e2e_argv[li], stream_handle)
        self.allreduce(out)
        self.h_out[li].copy_(out, non_blocking=True)

    e2e_api = "C ABI exl3_moe_decode (exl3_moe_decode_tp for N > 1), inputs in one pinned staging buffer"

    def bytes_per_step(self, i):
        return self.ubytes[i % len(self.layers)]

    def weights_by_k(self):
        """Mean weights per launch of this rank's shard, by bit width (unique
        experts of each cycled layer, gate + up + down)."""
        out: dict = {}
        for L, (ids, _) in zip(self.layers, self.routes):
            for e in self.torch.unique(ids).tolist():
                k = int(L.kbits[e])
                out[k] = out.get(k, 0.0) + 3.0 * self.H * self.I / len(self.layers)
        return out

    launches_per_step = 1
    kernel_name = "exl3::moe_kernel"
    metric = None

    def describe(self):
        a = self.args
        name = "config2_moe_decode_layer" if a.route == "uniform" else "config3_moe_decode_layer_zipf"
        if a.stack:
            name = f"config4a_moe_decode_stack_{a.layers}_layers"
        return {"workload": name,
                "tokens": a.tokens, "topk": 8, "experts": a.experts, "hidden": 4096, "intermediate": 2048,
                "intermediate_per_gpu": self.I, "route": a.route, "layers_cycled": a.layers,
                "unique_experts_per_layer": self.uniq,
                "parallelism": (f"tp{self.world}" if self.world > 1 else
                                f"rank 0 shard of tp{self.shards} on one GPU (no collective)" if self.shards > 1
                                else "single"),
                "allreduce": (("nccl" if self.args.allreduce == "nccl" or self.allreduce_note else "fused-nvlink")
                              if self.world > 1 else None),
                "allreduce_note": self.allreduce_note,
                "l2": "inputs larger than L2 (unique bytes per layer > 126 MB; layers cycled)",
                "precise": bool(a.precise)}


class PrefillWorkload:
    """Config 4b: one routed-MoE layer over a 512-token prefill chunk through
    the tensor-core path (exl3_moe_prefill): bf16 activations N(0,1), top-8 of
    256 experts (router N(0,1), softmax over the 8), per-expert K2/K3, MCG,
    hidden 4096, intermediate 2048 / N per rank.  Two layers are cycled
    (2 x ~2 GB of packed weights at one GPU, > L2).  N > 1: TP shards of the
    intermediate dim and one NCCL all-reduce of the [512, 4096] output."""

    launches_per_step = 4
    kernel_name = "exl3::pf_gemm_kernel"
    metric = ("prefill MoE layer (config 4b: 512 tokens bf16, top-8 of 256, K2/K3, hidden 4096): "
              "packed-weight HBM GB/s")

    def __init__(self, args, rank, world, dev):
        import torch

        from dsv4_carve_b200 import _lib, synth
        from dsv4_carve_b200 import vllm_exl3_c as ext

        self.torch, self.ext, self.args, self.world, self.dev = torch, ext, args, world, dev
        self.E, self.H, self.I_full, self.T, self.topk = args.experts, 4096, 2048, args.prefill_tokens, 8
        self.shards = world if world > 1 else max(1, args.emulate_tp)
        self.I = self.I_full // self.shards
        self.rows = self.T
        self.lib = _lib.load()
        self.layers, self.routes, self.xs, self.outs, self.ubytes, self.uniq, self._argv = [], [], [], [], [], [], []
        nl = max(1, min(2, args.layers))
        self.scratch = torch.empty(ext.lna2_moe_prefill_scratch_bytes(self.T, self.topk, self.H, self.I, self.E),
                                   dtype=torch.uint8, device=dev)
        for li in range(nl):
            seed = 3000 + li
            kbits = synth.expert_bits(self.E, seed)
            L = synth.make_moe_layer(self.E, self.H, self.I_full, kbits, seed, device=dev, cb=synth.CB_MCG,
                                     rank=rank, world=self.shards)
            ids, w = synth.route_uniform(self.T, self.E, self.topk, seed=seed + 7, device=dev)
            x = synth.activations(self.T, self.H, seed=seed + 11, device=dev, dtype=torch.bfloat16)
            out = torch.empty((self.T, self.H), dtype=torch.bfloat16, device=dev)
            self.layers.append(L)
            self.routes.append((ids, w))
            self.xs.append(x)
            self.outs.append(out)
            self.ubytes.append(L.unique_bytes(ids) + self.T * self.H * 2 * 2)
            self.uniq.append(int(torch.unique(ids).numel()))
            self._argv.append((x.data_ptr(), _lib.DT_BF16, out.data_ptr(), _lib.DT_BF16, self.T, self.H, self.I,
                               *[t.data_ptr() for t in L.table_list()], self.E, L.ktab.data_ptr(), 3, 3,
                               synth.CB_MCG, ids.data_ptr(), w.data_ptr(), self.topk, 10.0,
                               self.scratch.data_ptr(), self.scratch.numel()))
        self.h_x = [x.cpu().pin_memory() for x in self.xs]
        self.h_ids = [r[0].cpu().pin_memory() for r in self.routes]
        self.h_w = [r[1].cpu().pin_memory() for r in self.routes]
        self.h_out = [torch.empty((self.T, self.H), dtype=torch.bfloat16).pin_memory() for _ in self.layers]
        self.d_ids = [torch.empty_like(r[0]) for r in self.routes]
        self.d_w = [torch.empty_like(r[1]) for r in self.routes]
        self.h2d = self.T * self.H * 2 + self.T * self.topk * 8
        self.d2h = self.T * self.H * 2

    def launch(self, i, stream_handle):
        rc = self.lib.exl3_moe_prefill(*self._argv[i % len(self.layers)], stream_handle)
        if rc:
            raise RuntimeError(self.lib.exl3_last_error().decode())

    def allreduce(self, out):
        if self.world > 1:
            self.torch.distributed.all_reduce(out)

    def step(self, i, stream_handle):
        self.launch(i, stream_handle)
        self.allreduce(self.outs[i % len(self.layers)])

    def check(self, li, snap, stream_handle):
        """Status word; a fresh run equals the timed region's output bit for
        bit; the decode kernel (precise arithmetic, the same fp16-rounded
        weights) on the chunk's first 32 tokens agrees within 2e-3."""
        torch = self.torch
        again = torch.empty_like(self.outs[li])
        a = list(self._argv[li])
        a[2] = again.data_ptr()
        rc = self.lib.exl3_moe_prefill(*a, stream_handle)
        if rc:
            raise RuntimeError(self.lib.exl3_last_error().decode())
        self.allreduce(again)
        L = self.layers[li]
        ids, w = self.routes[li]
        n = min(32, self.T)
        dec = torch.empty((n, self.H), dtype=torch.bfloat16, device=self.dev)
        dscr = torch.zeros(self.ext.lna2_moe_scratch_bytes(n, self.topk, self.H, self.I), dtype=torch.uint8,
                           device=self.dev)
        self.ext.lna2_moe_decode(self.xs[li][:n].contiguous(), dec, *L.table_list(), ids[:n].contiguous(),
                                 w[:n].contiguous(), 3, 10.0, dscr, intermediate=self.I, k_table=L.ktab,
                                 codebook=L.cb, precise=True)
        self.allreduce(dec)
        torch.cuda.synchronize(self.dev)
        status = self.ext.lna2_moe_status(self.scratch) | self.ext.lna2_moe_status(dscr)
        err = float((snap[:n].float() - dec.float()).abs().max().item())
        scale = max(1.0, float(dec.float().abs().max().item()))
        # bf16 outputs: each rank's partial and the all-reduced sum are rounded to
        # bf16 (8 significant bits), once per rank and once for the sum
        tol = max(2e-3, (self.world + 1) * 2.0 ** -8) * scale
        return status, bool(torch.equal(again, snap)), err, tol

    e2e_api = "vllm_exl3_c.lna2_moe_prefill"

    def e2e_step(self, i, stream_handle):
        li = i % len(self.layers)
        L = self.layers[li]
        x = self.xs[li]
        x.copy_(self.h_x[li], non_blocking=True)
        self.d_ids[li].copy_(self.h_ids[li], non_blocking=True)
        self.d_w[li].copy_(self.h_w[li], non_blocking=True)
        out = self.outs[li]
        self.ext.lna2_moe_prefill(x, out, *L.table_list(), self.d_ids[li], self.d_w[li], 3, 10.0, self.scratch,
                                  intermediate=self.I, k_table=L.ktab, codebook=L.cb)
        self.allreduce(out)
        self.h_out[li].copy_(out, non_blocking=True)

    def bytes_per_step(self, i):
        return self.ubytes[i % len(self.layers)]

    def describe(self):
        return {"workload": "config4b_prefill_moe_layer", "tokens": self.T, "topk": 8, "experts": self.E,
                "hidden": 4096, "intermediate": 2048, "intermediate_per_gpu": self.I, "route": "uniform",
                "activations": "bf16", "layers_cycled": len(self.layers), "unique_experts_per_layer": self.uniq,
                "parallelism": (f"tp{self.world}" if self.world > 1 else
                                f"rank 0 shard of tp{self.shards} on one GPU (no collective)" if self.shards > 1
                                else "single"),
                "l2": "inputs larger than L2 (packed weights per layer > 126 MB; layers cycled)",
                "path": "tcgen05 dequant-then-MMA", "precise": True}


class DenseWorkload:
    """Config 1: the dense EXL3 6-bit linears of attention / shared experts,
    [4096 -> 4096], [4096 -> 1536], [1536 -> 4096], K = 6, 3INST, R rows of
    fp16 N(0,1).  A step applies the three linears to one batch; sets of the
    three matrices are cycled so that steps stream from HBM (8 sets = 176 MB).
    TP: the two 4096-input matrices are column-sharded in whole 128-column
    blocks, [1536 -> 4096] is row-sharded and its partial output all-reduced.

    With --config single (config 0): one [4096 -> 4096] K4 3INST linear per
    step, R = --rows (1 in the config), 16 matrices cycled (134 MB > L2); with
    N > 1 it is replicated (every rank runs its own copy, no collective)."""

    launches_per_step = 3
    kernel_name = "exl3::linear_kernel"
    metric = "dense EXL3 K6 linear set (config 1: [4096->4096], [4096->1536], [1536->4096]): packed-weight HBM GB/s"

    def __init__(self, args, rank, world, dev):
        if args.config == "single":
            return self._init_single(args, rank, world, dev)
        import torch

        from dsv4_carve_b200 import _lib, synth
        from dsv4_carve_b200 import vllm_exl3_c as ext

        self.torch, self.ext, self.args, self.world, self.dev = torch, ext, args, world, dev
        self.R = args.rows
        self.lib = _lib.load()
        self.sets, self.xs, self.ys, self.argv, self.nbytes = [], [], [], [], []
        shapes = [(4096, 4096, "col"), (4096, 1536, "col"), (1536, 4096, "row")]
        nsets = max(1, args.layers * 2)
        for si in range(nsets):
            mats = []
            for mi, (k, n, mode) in enumerate(shapes):
                w = synth.make_dense(k, n, 6, seed=5000 + 10 * si + mi, device=dev, cb=synth.CB_3INST)
                if world > 1:
                    w = synth.shard_col_blocks(w, rank, world) if mode == "col" else synth.shard_row_blocks(w, rank, world)
                mats.append(w)
            self.sets.append(mats)
        scratch_need = max(self.lib.exl3_linear_scratch_bytes(self.R, m.in_features, m.out_features, 6)
                           for mats in self.sets for m in mats)
        self.scratch = torch.zeros(scratch_need, dtype=torch.uint8, device=dev)
        self._keep = []
        if args.group:
            import ctypes

            m0 = self.sets[0]
            gneed = self.lib.exl3_linear_group_scratch_bytes(
                self.R, 4096, 2, (ctypes.c_int64 * 2)(m0[0].out_features, m0[1].out_features), 6)
            self.gscratch = torch.zeros(gneed, dtype=torch.uint8, device=dev)
            self.launches_per_step = 2
        x = synth.activations(self.R, 4096, seed=77, device=dev)
        for mats in self.sets:
            a, b, c = mats
            xin_c = synth.activations(self.R, c.in_features, seed=78, device=dev)
            outs = [torch.empty((self.R, m.out_features), dtype=torch.float16, device=dev) for m in mats]
            ins = [x, x, xin_c]
            argv = []
            for m, xi, yo in zip(mats, ins, outs):
                argv.append((xi.data_ptr(), _lib.DT_F16, self.R, m.in_features, m.out_features, m.trellis.data_ptr(),
                             6, synth.CB_3INST, m.suh.data_ptr(), m.svh.data_ptr(), yo.data_ptr(), _lib.DT_F16,
                             self.scratch.data_ptr(), self.scratch.numel(), 1))
            if args.group:
                # [4096 -> 4096] and [4096 -> 1536] share x: one grouped launch
                import ctypes

                gn = (ctypes.c_int64 * 2)(a.out_features, b.out_features)
                vp = lambda ts: (ctypes.c_void_p * 2)(*[t.data_ptr() for t in ts])   # noqa: E731
                garr = (gn, vp([a.trellis, b.trellis]), vp([a.suh, b.suh]), vp([a.svh, b.svh]), vp(outs[:2]))
                self._keep.append(garr)
                argv = [("group", (x.data_ptr(), _lib.DT_F16, self.R, 4096, 2, garr[0], garr[1], 6, synth.CB_3INST,
                                   garr[2], garr[3], garr[4], _lib.DT_F16, self.gscratch.data_ptr(),
                                   self.gscratch.numel(), 1)), ("single", argv[2])]
            else:
                argv = [("single", a_) for a_ in argv]
            self.argv.append(argv)
            self.xs.append(ins)
            self.ys.append(outs)
            self.nbytes.append(sum(m.nbytes() + self.R * 2 * (m.in_features + m.out_features) for m in mats))
        self.h_x = [t.cpu().pin_memory() for t in (x,)]
        self.h_y = torch.empty((self.R, 4096), dtype=torch.float16).pin_memory()
        self.h2d = self.R * 4096 * 2
        self.d2h = self.R * 4096 * 2
        self.uniq = []

    def _init_single(self, args, rank, world, dev):
        import torch

        from dsv4_carve_b200 import _lib, synth
        from dsv4_carve_b200 import vllm_exl3_c as ext

        self.torch, self.ext, self.args, self.world, self.dev = torch, ext, args, world, dev
        self.R = args.rows
        self.lib = _lib.load()
        self.single = True
        self.launches_per_step = 1
        self.metric = "single EXL3 linear (config 0: [4096->4096], K4, 3INST): packed-weight HBM GB/s"
        self.sets, self.xs, self.ys, self.argv, self.nbytes = [], [], [], [], []
        for si in range(16):
            w = synth.make_dense(4096, 4096, 4, seed=7000 + si, device=dev, cb=synth.CB_3INST)
            self.sets.append([w])
        self.scratch = torch.zeros(self.lib.exl3_linear_scratch_bytes(self.R, 4096, 4096, 4), dtype=torch.uint8,
                                   device=dev)
        x = synth.activations(self.R, 4096, seed=79, device=dev)
        for (w,) in self.sets:
            y = torch.empty((self.R, 4096), dtype=torch.float16, device=dev)
            self.argv.append([("single", (x.data_ptr(), _lib.DT_F16, self.R, 4096, 4096, w.trellis.data_ptr(), 4,
                                          synth.CB_3INST, w.suh.data_ptr(), w.svh.data_ptr(), y.data_ptr(),
                                          _lib.DT_F16, self.scratch.data_ptr(), self.scratch.numel(), 1))])
            self.xs.append([x, x, x])
            self.ys.append([y, y, y])
            self.nbytes.append(w.nbytes() + self.R * 2 * (4096 + 4096))
        self.h_x = [x.cpu().pin_memory()]
        self.h_y = torch.empty((self.R, 4096), dtype=torch.float16).pin_memory()
        self.h2d = self.R * 4096 * 2
        self.d2h = self.R * 4096 * 2
        self.uniq = []

    def launch(self, i, stream_handle):
        for kind, a in self.argv[i % len(self.argv)]:
            fn = self.lib.exl3_linear_group if kind == "group" else self.lib.exl3_linear
            rc = fn(*a, stream_handle)
            if rc:
                raise RuntimeError(self.lib.exl3_last_error().decode())

    def allreduce(self, out):
        if self.world > 1 and not getattr(self, "single", False):
            self.torch.distributed.all_reduce(out)

    @property
    def outs(self):
        return [ys[2] for ys in self.ys]

    @property
    def layers(self):
        return self.sets

    def step(self, i, stream_handle):
        self.launch(i, stream_handle)
        self.allreduce(self.outs[i % len(self.sets)])

    def check(self, li, snap, stream_handle):
        """Status word of the linear scratch; a fresh run of set li equals the
        timed region's output bit for bit; the fast arithmetic (unrounded
        weights, a second computation) agrees within 2e-3."""
        torch = self.torch
        c = self.sets[li][-1]
        xin = self.xs[li][2]
        again = self.ext.linear_forward(xin, c.trellis, c.suh, c.svh, c.K, 0, torch.float16, True)
        fast = self.ext.linear_forward(xin, c.trellis, c.suh, c.svh, c.K, 0, torch.float16, False)
        self.allreduce(again)
        self.allreduce(fast)
        torch.cuda.synchronize(self.dev)
        import ctypes

        word = ctypes.c_uint32(0)
        from dsv4_carve_b200 import _lib

        _lib.check(self.lib.exl3_scratch_status(self.scratch.data_ptr(), 0, 0, ctypes.addressof(word), stream_handle))
        err = float((snap.float() - fast.float()).abs().max().item())
        scale = max(1.0, float(fast.float().abs().max().item()))
        return int(word.value), bool(torch.equal(again, snap)), err, 2e-3 * scale

    e2e_api = "vllm_exl3_c.linear_forward"

    def e2e_step(self, i, stream_handle):
        """x from pinned host memory, the three linears through the public
        linear_forward call, the last output back to pinned host memory."""
        torch = self.torch
        si = i % len(self.sets)
        x = self.xs[si][0]
        x.copy_(self.h_x[0], non_blocking=True)
        if getattr(self, "single", False):
            (w,) = self.sets[si]
            y = self.ext.linear_forward(x, w.trellis, w.suh, w.svh, 4, 0, torch.float16, True)
            self.h_y.copy_(y, non_blocking=True)
            return (y,)
        a, b, c = self.sets[si]
        ya = self.ext.linear_forward(x, a.trellis, a.suh, a.svh, 6, 0, torch.float16, True)
        yb = self.ext.linear_forward(x, b.trellis, b.suh, b.svh, 6, 0, torch.float16, True)
        yc = self.ext.linear_forward(self.xs[si][2], c.trellis, c.suh, c.svh, 6, 0, torch.float16, True)
        self.allreduce(yc)
        self.h_y.copy_(yc, non_blocking=True)
        return ya, yb

    def bytes_per_step(self, i):
        return self.nbytes[i % len(self.sets)]

    def describe(self):
        if getattr(self, "single", False):
            return {"workload": "config0_single_linear", "rows": self.R, "K": 4, "codebook": "3INST",
                    "matrices": ["4096x4096"], "sets_cycled": len(self.sets),
                    "parallelism": f"{self.world} replicas" if self.world > 1 else "single",
                    "l2": "16 matrices cycled: 16 x 8.4 MB > 126 MB L2", "precise": True}
        return {"workload": "config1_dense_k6_linear_set", "rows": self.R, "K": 6, "codebook": "3INST",
                "matrices": ["4096x4096", "4096x1536", "1536x4096"], "sets_cycled": len(self.sets),
                "parallelism": f"tp{self.world}" if self.world > 1 else "single",
                "l2": "sets cycled: 8 x 22 MB > 126 MB L2", "precise": True,
                "grouped": bool(self.args.group)}


# ----------------------------------------------------------------------------- CPU baseline
_CPU_CACHE: dict = {}


def _cpu_units(args):
    """(expert, projection) units of layer 0 of the workload, in routed order,
    with the rows each expert serves (config 2 routing, CPU generators)."""
    from dsv4_carve_b200 import synth

    key = (args.experts, args.tokens, args.route)
    if key not in _CPU_CACHE:
        E, T, topk, seed = args.experts, args.tokens, 8, 1000
        kbits = synth.expert_bits(E, seed)
        if args.route == "zipf":
            ids, _ = synth.route_zipf(T, E, topk, seed=seed + 7)
        else:
            ids, _ = synth.route_uniform(T, E, topk, seed=seed + 7)
        x = synth.activations(T, 4096, seed=seed + 11)
        order = sorted(set(int(e) for e in ids.flatten().tolist()))
        units = [(e, p, kbits[e], [r for r in range(T) if e in ids[r].tolist()])
                 for e in order for p in ("gate", "up", "down")]
        _CPU_CACHE[key] = (units, x)
    return _CPU_CACHE[key]


def cpu_reference_sample(args, seconds: float, start_unit: int = 0):
    """The reference's CPU linear (recipe-lna/lna2/bindings.cpp:135-148:
    dequant_cpu + at::mm) over 512-column slices of the routed experts'
    gate/up/down matrices of config 2, until `seconds` of reference time have
    been spent.  Weight generation is outside the timed calls.  Returns
    (GB/s of packed bytes, sample description, cores, kind, seconds, units used)."""
    import torch

    from dsv4_carve_b200 import synth
    from oracle import oracle as O

    ref = O.ref_ext()
    kind = "reference" if ref is not None else "port"
    units, x = _cpu_units(args)
    H, I, cols = 4096, 2048, 512
    done_bytes, spent, n = 0, 0.0, 0
    u = start_unit
    while spent < seconds and n < 10000:
        e, proj, K, rows = units[u % len(units)]
        k = H if proj != "down" else I
        g = synth._gen("cpu", 7919 * u + 1)
        tr = synth.random_trellis(k // 16, cols // 16, K, g, "cpu")
        su, sv = synth.random_signs(k, g, "cpu"), synth.random_svh(cols, g, "cpu")
        xe = x[rows].contiguous() if proj != "down" else x[rows][:, :I].contiguous()
        t0 = time.perf_counter()
        if ref is not None:
            ref.exl3_gemv(xe, tr, su, sv, K, True, 1)
        else:
            O.gemv(xe.numpy(), tr.numpy(), su.numpy(), sv.numpy(), K, 1)
        spent += time.perf_counter() - t0
        done_bytes += tr.numel() * 2 + su.numel() * 2 + sv.numel() * 2
        n += 1
        u += 1
    sample = (f"{n} slices of {cols} output columns (MCG, K2/K3) from the gate/up/down matrices of the "
              f"routed experts of a config-2 layer, each over the rows routed to its expert")
    return done_bytes / spent / 1e9, sample, torch.get_num_threads(), kind, spent, n


# ----------------------------------------------------------------------------- main
def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    # each step: a bounded sample, sized so that the whole run stays near 2 minutes
    per = max(0.3, min(20.0, 120.0 / max(1, args.steps + args.warmup)))
    vals = []
    desc = kind = None
    cores = 1
    unit = 0
    for s in range(args.warmup + args.steps):
        v, desc, cores, kind, _, used = cpu_reference_sample(args, per, unit)
        unit += used
        if s >= args.warmup:
            vals.append(v)
    value = statistics.median(vals) if vals else None
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "u16 trellis -> fp32",
        "data": "synthetic", "config": {"workload": "config2_moe_decode_layer", "tokens": args.tokens, "topk": 8,
                                        "experts": args.experts, "hidden": 4096, "intermediate": 2048},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": f"per step: {desc}; {per:.1f} s per step"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def decode_roof(weights_by_k: dict, kernel_us: float, dev) -> dict:
    """Decode-issue roof of the launch: the layer's weights (per bit width)
    over the rate of exl3_decode_roof -- the GEMV engine's decode loop on
    shared-memory tiles, no HBM traffic -- timed here with CUDA events."""
    import ctypes

    import torch

    from dsv4_carve_b200 import _lib

    lib = _lib.load()
    words = torch.randint(-2**31, 2**31 - 1, (32 * 8 * 8,), dtype=torch.int32, device=dev)
    out = torch.empty(int(lib.exl3_decode_roof_out_floats()), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    rates = {}
    for K in sorted(weights_by_k):
        n = ctypes.c_int64(0)
        args = (K, 1, 600, ctypes.c_void_p(words.data_ptr()), words.numel(), ctypes.c_void_p(out.data_ptr()),
                out.numel(), ctypes.byref(n), ctypes.c_void_p(stream.cuda_stream))
        _lib.check(lib.exl3_decode_roof(*args))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            _lib.check(lib.exl3_decode_roof(*args))
        e1.record(stream)
        torch.cuda.synchronize(dev)
        rates[K] = 5 * n.value / (e0.elapsed_time(e1) / 1e3)
    roof_us = sum(w / rates[k] for k, w in weights_by_k.items()) * 1e6
    return {"weights_per_launch": sum(weights_by_k.values()),
            "weights_per_s": {str(k): v for k, v in rates.items()},
            "layer_us": roof_us, "frac": roof_us / kernel_us, "codebook": "MCG",
            "how": "exl3_decode_roof: the GEMV engine's decode loop on shared-memory tiles, 2 CTAs x 8 warps per SM"}


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import datetime

    import torch

    rank, world, local = dist_env()
    assert world == args.gpus or world == 1, "launch with torchrun for --gpus > 1"
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier(device_ids=[local])

    wl = {"dense": DenseWorkload, "single": DenseWorkload, "prefill": PrefillWorkload}.get(args.config, MoeWorkload)(
        args, rank, world, dev)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    for i in range(args.warmup):
        wl.step(i, sh)
    torch.cuda.synchronize(dev)

    bus = None
    try:
        pr = torch.cuda.get_device_properties(dev)
        bus = f"{int(pr.pci_bus_id):02x}:{int(pr.pci_device_id):02x}.0"
    except Exception:
        bus = None
    clocks = None
    if rank == 0 and not args.no_clocks:
        try:
            clocks = NvmlClockSampler(bus)
        except Exception:
            clocks = ClockSampler(bus)
    if clocks:
        clocks.start()
        time.sleep(0.6)

    # ---- device-resident timed region
    K = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    barrier()
    torch.cuda.synchronize(dev)
    t_wall0 = time.time()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # Only the region's own start / end events: an event recorded between two
    # launches would stand between them in the stream and keep the next layer's
    # launch from overlapping this one's tail (programmatic dependent launch).
    start.record(stream)
    for i in range(K):
        wl.launch(i, sh)
        wl.allreduce(wl.outs[i % len(wl.layers)])
    end.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    t_wall1 = time.time()
    ms = start.elapsed_time(end)
    # the last layer the timed region ran, and the output it left, for the check
    last_li = (K - 1) % len(wl.layers)
    snap = wl.outs[last_li].clone()
    # per-launch kernel durations (roofline.achieved): a second pass with
    # events around each launch
    for i in range(K):
        ev[i][0].record(stream)
        wl.launch(i, sh)
        ev[i][1].record(stream)
        wl.allreduce(wl.outs[i % len(wl.layers)])
    torch.cuda.synchronize(dev)
    barrier()
    kern_ms = [a.elapsed_time(b) for a, b in ev]
    my_bytes = sum(wl.bytes_per_step(i) for i in range(K))
    t = torch.tensor([ms, float(my_bytes)], dtype=torch.float64, device=dev)
    if world > 1:
        tm = t[:1].clone()
        torch.distributed.all_reduce(tm, op=torch.distributed.ReduceOp.MAX)
        tb = t[1:].clone()
        torch.distributed.all_reduce(tb)
        ms_max, all_bytes = float(tm.item()), float(tb.item())
    else:
        ms_max, all_bytes = ms, float(my_bytes)

    # ---- end-to-end through the public call with host buffers
    e2e = None
    if not args.no_e2e:
        for i in range(min(3, args.warmup) or 1):
            wl.e2e_step(i, sh)
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(stream)
        for i in range(K):
            wl.e2e_step(i, sh)
        e2.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        ms2 = torch.tensor([s2.elapsed_time(e2)], dtype=torch.float64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(ms2, op=torch.distributed.ReduceOp.MAX)
        e2e = {"value": all_bytes / (float(ms2.item()) / 1e3) / 1e9, "unit": UNIT,
               "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h,
               "ms_per_step": float(ms2.item()) / K, "api": wl.e2e_api}

    # ---- validation: status words and a second computation of one layer
    status, same, err, tol = wl.check(last_li, snap, sh)
    chk = torch.tensor([float(status), 0.0 if same else 1.0, err / tol], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(chk, op=torch.distributed.ReduceOp.MAX)
    status_all, differs, err_ratio = int(chk[0].item()), bool(chk[1].item()), float(chk[2].item())
    check = {"status_word": status_all, "rerun_bitwise_equal": not differs,
             "second_computation_max_abs_over_tol": err_ratio,
             "ok": status_all == 0 and not differs and err_ratio <= 1.0,
             "how": ("device status word of every rank after the timed and e2e loops; a fresh run of the last "
                     "timed layer must equal the output the timed region left bit for bit; a second "
                     "computation in the other arithmetic must agree within 2e-3 of the output scale (bf16 "
                     "outputs: one bf16 rounding per rank and one for the sum), max over ranks")}

    clock_info = None
    if clocks:
        clocks.stop()
        clock_info = clocks.summary(t_wall0, t_wall1)
    if hasattr(wl, "close"):
        wl.close()       # every rank, before any rank leaves the group

    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    peak, peak_kind = measured_peak()
    kern_avg_ms = statistics.mean(kern_ms)
    bytes_per_launch = my_bytes / K
    achieved = bytes_per_launch / (kern_avg_ms / 1e3) / 1e9
    traffic = None
    if NCU_TRAFFIC_FILE.exists() and world == 1 and args.config == "moe":
        try:
            tr = json.loads(NCU_TRAFFIC_FILE.read_text())
            # captured launch's DRAM bytes, scaled to this run's algorithmic bytes per launch
            traffic = tr["dram_bytes_per_launch"] / tr["algorithmic_bytes_per_launch"] * (my_bytes / K)
        except Exception:
            traffic = None
    rows = args.rows if args.config in ("dense", "single") else getattr(wl, "rows", args.tokens)
    line = {
        "metric": wl.metric or METRIC, "value": all_bytes / (ms_max / 1e3) / 1e9, "unit": UNIT, "n_gpus": world,
        "steps": K, "warmup": args.warmup, "ms_per_step": ms_max / K, "us_per_layer": ms_max / K * 1e3,
        "tokens_per_s_per_layer": rows * K / (ms_max / 1e3),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "u16 trellis -> fp16 MMA, fp32 accumulate", "data": "synthetic",
        "config": wl.describe(),
        "roofline": {"bound": "hbm", "kernel": wl.kernel_name, "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic,
                     "traffic_source": ("ncu capture in profiles/, scaled from the captured launch's algorithmic "
                                        "bytes to this run's" if traffic is not None else None),
                     "algorithmic_bytes_per_launch": bytes_per_launch,
                     "kernel_us_avg": kern_avg_ms * 1e3,
                     "kernel_us_source": ("second, serialised pass with CUDA events around each launch (the events "
                                          "stop the launch overlap, so this is slower than ms_per_step)")},
        "gpu_launches": K * wl.launches_per_step,
        "e2e": e2e,
        "check": check,
        "clocks": clock_info,
    }
    if args.config == "moe" and args.stack:
        # every layer of the stack is cycled through the timed steps; one
        # decode step runs all of them once
        step_us = ms_max / K * 1e3 * args.layers
        line["stack"] = {"layers": args.layers, "us_per_decode_step": step_us,
                         "tokens_per_s": args.tokens / (step_us / 1e6)}
    if args.config == "moe" and hasattr(wl, "weights_by_k"):
        try:
            line["roofline"]["decode_roof"] = decode_roof(wl.weights_by_k(), kern_avg_ms * 1e3, dev)
        except Exception as exc:   # the measurement aid must not void the bench line
            line["roofline"]["decode_roof"] = {"error": repr(exc)}
    if world == 1 and not args.no_cpu and args.config == "moe":
        v, desc, cores, kind, dt, _ = cpu_reference_sample(args, args.cpu_seconds)
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": kind, "sample": desc,
                                "seconds": dt}
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    if not check["ok"]:
        sys.exit("bench: the validation check failed (see the line's `check`); the numbers are not valid")


if __name__ == "__main__":
    main()
