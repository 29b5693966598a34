"""Fused tensor-parallel sum for the routed-MoE decode layer.

The reference shards every expert's intermediate dim over the TP ranks
(recipe-lna/vllm_exl3_exl3.py.lna:855-871) and runs one NCCL all-reduce of
the [m, hidden] layer output after its kernel.  MoeTpExchange sets up what
exl3_moe_decode_tp needs to do that sum inside the kernel over NVLink: one
exchange buffer per rank (cudaMalloc'ed by the library), its CUDA IPC
handle shared with the other ranks over the process group, the peers'
buffers mapped into this process, and a device table of all ranks' buffer
addresses.  torch.distributed carries only the 64-byte handles.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


class MoeTpExchange:
    """Exchange buffers of one TP group for layers of up to `max_rows` rows."""

    def __init__(self, group, device: torch.device, max_rows: int, hidden: int, *, single: bool = False):
        import torch.distributed as dist

        self.rank = 0 if single else dist.get_rank(group)
        self.world = 1 if single else dist.get_world_size(group)
        self.max_rows, self.hidden, self.device = int(max_rows), int(hidden), device
        lib = _lib.load()
        ptr = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.call("exl3_tp_buffer_alloc", self.world, self.max_rows, self.hidden, ctypes.addressof(ptr))
            self.local = int(ptr.value)
            handle = (ctypes.c_uint8 * 64)()
            _lib.call("exl3_tp_ipc_handle", self.local, ctypes.addressof(handle))
            handles = [bytes(handle)]
            if not single:
                handles = [None] * self.world
                dist.all_gather_object(handles, bytes(handle), group=group)
            self.mapped = []
            addrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    addrs.append(self.local)
                    continue
                hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
                out = ctypes.c_void_p()
                _lib.call("exl3_tp_ipc_open", ctypes.addressof(hb), ctypes.addressof(out))
                self.mapped.append(int(out.value))
                addrs.append(int(out.value))
        self.table = torch.tensor(addrs, dtype=torch.int64, device=device)
        self._lib = lib

    @classmethod
    def single(cls, device: torch.device, max_rows: int, hidden: int) -> "MoeTpExchange":
        """A world of one (no process group): the in-kernel exchange runs
        against this rank's own buffer only."""
        return cls(None, device, max_rows, hidden, single=True)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank's
        last exchange has completed: call after a barrier)."""
        with torch.cuda.device(self.device):
            for p in self.mapped:
                _lib.call("exl3_tp_ipc_close", p)
            self.mapped = []
            if self.local:
                _lib.call("exl3_tp_buffer_free", self.local)
                self.local = 0
