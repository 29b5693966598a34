"""Fused tensor-parallel sum of the MoE decode layer on 2, 4 and 8 GPUs.

N ranks (spawned processes, one GPU each, NCCL process group on 127.0.0.1
for the handle exchange and the comparison) hold the TP=N shards of one
layer (recipe-lna/vllm_exl3_exl3.py.lna:855-871 slicing).  Each call of
exl3_moe_decode_tp must give, on every rank, the NCCL all-reduce of the
ranks' plain partial outputs (fp32 sums in a different order: max-abs 1e-5),
and rank 0's result must match the oracle's unsharded layer at the MoE
tolerance (max-abs 2e-3); every rank ends with the same bits.  Several calls
in a row exercise both epoch parities of the exchange buffers; the last one
goes through the routed entry (int64 global ids and an expert map, the
plugin's inputs).  Each world size is skipped when fewer GPUs are present.
"""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

E, H, I_FULL, T, TOPK, CALLS = 16, 1024, 1024, 4, 4, 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from dsv4_carve_b200 import synth
    from dsv4_carve_b200 import vllm_exl3_c as ext
    from dsv4_carve_b200.tp import MoeTpExchange

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    out = {"rank": rank, "diff": [], "status": [], "fused": [], "error": None}
    try:
        # generated on the CPU (the oracle's generator), then moved
        cpu = synth.make_moe_layer(E, H, I_FULL, synth.expert_bits(E, 3), 3, device="cpu", cb=1, rank=rank,
                                   world=world)
        L = synth.MoeLayer(E=cpu.E, H=cpu.H, I=cpu.I, kbits=cpu.kbits, cb=cpu.cb)
        L.experts = [{k: v.to(dev) for k, v in ex_.items()} for ex_ in cpu.experts]
        L.build_tables()
        ex = MoeTpExchange(None, dev, max_rows=8, hidden=H)
        emap = torch.arange(E, dtype=torch.long, device=dev)   # every expert on every rank (TP, not EP)
        for it in range(CALLS):
            ids, w = synth.route_uniform(T, E, TOPK, seed=70 + it, device=dev)
            x = synth.activations(T, H, seed=80 + it).to(dev)
            scratch = torch.zeros(ext.lna2_moe_scratch_bytes(T, TOPK, H, L.I), dtype=torch.uint8, device=dev)
            fused = torch.empty((T, H), dtype=torch.float32, device=dev)
            if it == CALLS - 1:
                ext.lna2_moe_decode_routed(x, fused, *L.table_list(), ids.long(), w, 3, 10.0, scratch,
                                           intermediate=L.I, k_table=L.ktab, codebook=L.cb, expert_map=emap,
                                           tp_exchange=ex)
            else:
                ext.lna2_moe_decode(x, fused, *L.table_list(), ids, w, 3, 10.0, scratch, intermediate=L.I,
                                    k_table=L.ktab, codebook=L.cb, tp_exchange=ex)
            plain = torch.empty_like(fused)
            ext.lna2_moe_decode(x, plain, *L.table_list(), ids, w, 3, 10.0, scratch, intermediate=L.I,
                                k_table=L.ktab, codebook=L.cb)
            dist.all_reduce(plain)
            torch.cuda.synchronize(dev)
            out["diff"].append(float((fused - plain).abs().max().item()))
            out["status"].append(ext.lna2_moe_status(scratch))
            out["fused"].append(fused.cpu().numpy())
        dist.barrier()
        torch.cuda.synchronize(dev)
        ex.close()
    except Exception as exc:   # reported to the parent, which fails the test
        out["error"] = repr(exc)
    finally:
        dist.destroy_process_group()
    q.put(out)


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_tp_sum(oracle, world):
    import torch.multiprocessing as mp

    from dsv4_carve_b200 import synth
    from tests.helpers import max_abs, moe_np, oracle_x

    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r = q.get(timeout=240)
            results[r["rank"]] = r
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert set(results) == set(range(world))
    for r in results.values():
        assert r["error"] is None, r["error"]
        assert all(s == 0 for s in r["status"]), r["status"]
        assert max(r["diff"]) <= 1e-5, r["diff"]
    full = synth.make_moe_layer(E, H, I_FULL, synth.expert_bits(E, 3), 3, device="cpu", cb=1)
    for it in range(CALLS):
        ids, w = synth.route_uniform(T, E, TOPK, seed=70 + it)
        x = synth.activations(T, H, seed=80 + it)
        xa, code = oracle_x(x)
        want, _ = oracle.moe(xa, moe_np(full), full.kbits, ids.numpy(), w.numpy(), 10.0, cb=1, dtype_code=code,
                             exact=True)
        got0 = results[0]["fused"][it]
        assert max_abs(got0, want) <= 2e-3
        for r in range(1, world):
            assert (got0 == results[r]["fused"][it]).all()
