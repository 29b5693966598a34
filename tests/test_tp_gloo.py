"""Tensor-parallel sharding maths on CPU ranks (gloo, world size 2).

Each rank keeps intermediate columns [r*I/W, (r+1)*I/W) of every expert's
gate/up and the same rows of down (recipe-lna/vllm_exl3_exl3.py.lna:855-871,
restated by dsv4_carve_b200.synth.shard_col / shard_row), computes its
partial layer output with the oracle, and one all-reduce(sum) must give the
unsharded layer.  The same holds for a row-parallel dense linear.  This is
the exchange step the multi-GPU bench performs with NCCL.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsv4_carve_b200 import synth


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _experts_np(layer):
    return [{p: (ex[p].trellis.numpy(), ex[p].suh.numpy(), ex[p].svh.numpy()) for p in ex} for ex in layer.experts]


def _worker(rank: int, world: int, port: int, q):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        E, H, I, T, topk = 6, 256, 256, 3, 2
        kbits = [2, 3, 2, 3, 2, 3]
        shard = synth.make_moe_layer(E, H, I, kbits, seed=5, rank=rank, world=world)
        ids, w = synth.route_uniform(T, E, topk, seed=6)
        x = synth.activations(T, H, seed=7)
        part, _ = O.moe(x.numpy(), _experts_np(shard), kbits, ids.numpy(), w.numpy(), 10.0)
        t = torch.from_numpy(part)
        dist.all_reduce(t)
        full = synth.make_moe_layer(E, H, I, kbits, seed=5)
        want, _ = O.moe(x.numpy(), _experts_np(full), kbits, ids.numpy(), w.numpy(), 10.0)
        moe_err = float(np.abs(t.numpy() - want).max())

        d = synth.make_dense(512, 256, 6, seed=9)
        xd = synth.activations(2, 512, seed=10)
        ds = synth.shard_row(d, rank, world)
        k0 = rank * (512 // world)
        xs = xd[:, k0:k0 + 512 // world].contiguous()
        yp = torch.from_numpy(O.gemv(xs.numpy(), ds.trellis.numpy(), ds.suh.numpy(), ds.svh.numpy(), 6, 1))
        dist.all_reduce(yp)
        yw = O.gemv(xd.numpy(), d.trellis.numpy(), d.suh.numpy(), d.svh.numpy(), 6, 1)
        lin_err = float(np.abs(yp.numpy() - yw).max())
        q.put((rank, moe_err, lin_err))
    finally:
        dist.destroy_process_group()


def test_tp2_shards_sum_to_full_layer():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, moe_err, lin_err in res:
        # the only difference is where the fp16 roundings of the activations
        # fall; the sharded sum is otherwise the same fp64 arithmetic
        assert moe_err <= 1e-3, (rank, moe_err)
        assert lin_err <= 1e-3, (rank, lin_err)
