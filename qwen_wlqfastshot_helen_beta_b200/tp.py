"""Tensor-parallel communication buffers for the fused row-parallel all-reduce.

vLLM shards row-parallel linears (o_proj, down_proj) along K and sums the
ranks' outputs with an NCCL all-reduce after the layer
(vllm: model_executor/layers/linear.py:1558-1559).  ``wlq_gemv_allreduce``
does that sum inside the decode GEMV over NVLink peer memory; ``TPComm`` sets
up the memory it needs: one buffer per rank (``wlq_tp_buffer_alloc``), its
CUDA IPC handle shared with the other ranks through the process group, and
the other ranks' buffers mapped into this process (``wlq_tp_buffer_open``).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from ._lib import check, lib


class TPComm:
    """Buffers of one tensor-parallel group (all ranks on this node)."""

    def __init__(self, max_N: int, group=None, device: Optional[torch.device] = None):
        import torch.distributed as dist
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= 8:
            raise ValueError(f"TPComm: 2..8 ranks supported, got {self.world}")
        self.max_N = int(max_N)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        nbytes = int(lib.wlq_tp_buffer_bytes(self.world, self.max_N))
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            check(lib.wlq_tp_buffer_alloc(nbytes, ctypes.byref(ptr), handle), "wlq_tp_buffer_alloc")
        self._local = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        ptrs, self._peers = [], []
        with torch.cuda.device(self.device):
            for q in range(self.world):
                if q == self.rank:
                    ptrs.append(self._local)
                    continue
                pq = ctypes.c_void_p()
                check(lib.wlq_tp_buffer_open(handles[q], ctypes.byref(pq)), "wlq_tp_buffer_open")
                ptrs.append(pq.value)
                self._peers.append(pq.value)
        self.bufs = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=group)  # every rank's buffer is mapped everywhere before first use

    def error(self, clear: bool = True) -> int:
        """Error word (bit 0: a fused all-reduce gave up waiting for a rank)."""
        v = ctypes.c_uint(0)
        with torch.cuda.device(self.device):
            check(lib.wlq_tp_error(ctypes.c_void_p(self._local), ctypes.byref(v), 1 if clear else 0), "wlq_tp_error")
        return int(v.value)

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (after all ranks
        are done with them: call from every rank after a barrier)."""
        with torch.cuda.device(self.device):
            for pq in self._peers:
                lib.wlq_tp_buffer_close(ctypes.c_void_p(pq))
            if self._local:
                lib.wlq_tp_buffer_free(ctypes.c_void_p(self._local))
        self._peers, self._local = [], None
