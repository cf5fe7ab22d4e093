"""Tensor-parallel communicators.

The reference runs TP over a ``(1, N)`` Blackhole mesh with TT_CCL all-gather / reduce-scatter /
all-reduce (``scripts/ci/fixtures/qwen36_model.py:31-38``, ``graft/gdn/tp.py:24``).  Here one
process drives one GPU and ``torch.distributed`` provides the process group (``nccl`` on GPUs,
``gloo`` on CPU).  ``TorchComm`` is the library baseline; ``qwen38_b200.parallel.symm`` adds the
in-kernel NVLink path on top of the same group.

Every rank issues the same collectives in the same order (warm-up, timing and error paths).
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


class NullComm:
    """Single-rank communicator (TP1)."""
    rank, world = 0, 1
    group = None

    def all_reduce_(self, t):
        return t

    def all_gather_cat(self, t, dim=0):
        return t

    def argmax_reduce(self, val, idx):
        return idx

    def barrier(self):
        pass

    def broadcast_(self, t, src=0):
        return t


class TorchComm:
    """torch.distributed collectives over a TP group."""

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def all_reduce_(self, t):
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t

    def all_gather_cat(self, t, dim=0):
        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t.contiguous(), group=self.group)
        return torch.cat(parts, dim)

    def argmax_reduce(self, val, idx):
        """Cross-rank argmax of per-rank (value, global index) pairs [T]; ties -> lowest index."""
        v = self.all_gather_cat(val.float()[None], 0)                # [W, T]
        i = self.all_gather_cat(idx.to(torch.int64)[None], 0)        # [W, T]
        best = v.max(0, keepdim=True).values
        cand = torch.where(v == best, i, torch.full_like(i, torch.iinfo(torch.int64).max))
        return cand.min(0).values

    def barrier(self):
        dist.barrier(group=self.group)

    def broadcast_(self, t, src=0):
        dist.broadcast(t, src=src, group=self.group)
        return t


def init_distributed(backend: str | None = None, timeout_s: float = 120.0):
    """Initialise the default process group from torchrun's environment (RANK, WORLD_SIZE,
    LOCAL_RANK, MASTER_ADDR/PORT).  Returns (rank, world, local_rank)."""
    if not dist.is_available():
        return 0, 1, 0
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1 and not dist.is_initialized():
        return 0, 1, 0
    if not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        local = int(os.environ.get("LOCAL_RANK", "0"))
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist.get_rank(), dist.get_world_size(), int(os.environ.get("LOCAL_RANK", "0"))


def make_comm(world: int, *, device=None, hidden: int = 0, peer: bool = False, fused: bool = True,
              prefill_rows: int = 0):
    """TP communicator: NullComm at one rank, the peer-memory kernels (``SymmComm``; with
    ``fused`` the row-parallel GEMMs carry the all-reduce themselves; ``prefill_rows`` sizes the
    fused prefill all-reduce's buffers for chunks of up to that many rows) when ``peer`` is set on
    GPUs, otherwise torch.distributed collectives."""
    if world == 1:
        return NullComm()
    if peer:
        from .symm import SymmComm
        return SymmComm(device, hidden, fused=fused, prefill_rows=prefill_rows)
    return TorchComm()
