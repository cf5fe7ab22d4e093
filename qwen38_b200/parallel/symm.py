"""Peer-memory tensor-parallel collectives (the in-kernel NVLink path).

``SymmComm`` extends the ``torch.distributed`` communicator: it allocates one peer buffer per
rank, exchanges CUDA IPC handles over the process group once, and serves the decode / verify
collectives with the kernels in ``csrc/comm.cu``:

* ``reduce_slot_add(slot, residual)`` - the row-parallel GEMM already wrote this rank's fp32
  partial into ``slot`` (``slot_out``); one kernel barriers the ranks, sums the partials in rank
  order and adds into the residual.  No NCCL call, no copy.
* ``argmax_reduce(val, idx)`` - cross-rank (value, index) argmax for the vocab-parallel LM head.
* ``markov_ptrs`` - every rank's receive words of the fused Markov selector (``csrc/markov.cu``),
  which exchanges each step's winner inside its one launch.

* pushed all-reduce (``NativeOps.linear_push`` + ``NativeOps.rms_norm_ar``): the out-projection
  GEMM pushes each finished fp32 tile into every rank's receive area as {value, epoch} 8-byte
  words; the next RMSNorm of the residual spins on the words of its row until this use's epoch
  appears, adds the rank-ordered sum and normalises (receive blocks [slot][source rank]).  When
  the NVSwitch offers multicast (``torch.distributed._symmetric_memory`` with a multicast
  pointer), the receive areas live in that symmetric memory and each word leaves the GPU once,
  through the multicast address (``recv_mc``), instead of once per rank (opt in: ``Q38_NVLS=1``;
  measured at TP8 on B200 it shortened the GEMMs but not the verify, 5.75 vs 5.65 ms per block).

Prefill chunks (more than ``slot_rows`` rows) take the fused prefill all-reduce when NVSwitch
multicast is available (``prefill_push``: a reduce-scatter GEMM epilogue, an owner-side reduce and a
multicast broadcast of the finished residual rows, see csrc/prefill_ar.cu); otherwise NCCL (the
base class).

Slot reuse is safe when two uses of one slot are separated by another collective: a rank writes a
slot again only after the barrier of a later call, which every peer reaches only after finishing
its reads of the earlier one.  Each graph capture therefore numbers its collectives from slot 0
(graphs run one at a time and each holds many collectives, so two uses of a slot always have
other barriers between them), and eager calls rotate through a separate range.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops.build import load
from .comm import TorchComm

MAX_RANKS = 8
AR_CTAS = 32
PUSH_ROWS = 64            # rows of a pushed all-reduce (csrc: AR_MAX_ROWS): a packed verify of 4 x 16
MARKOV_STEPS = 32         # Markov selector steps per launch (csrc/markov.cu MAX_STEPS)


class SymmComm(TorchComm):
    def __init__(self, device, hidden: int, group=None, slot_rows: int = 32, graph_slots: int = 768,
                 eager_slots: int = 64, fused_graph_slots: int = 160, fused_eager_slots: int = 32,
                 fused: bool = True, nvls: bool | None = None, prefill_rows: int = 0):
        super().__init__(group)
        self.fused = fused          # row-parallel GEMMs push their tiles; the next norm reduces
        if self.world > MAX_RANKS:
            raise ValueError("peer-memory collectives serve at most 8 ranks")
        self.C = load()
        self.device = torch.device(device)
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.slot_rows, self.hidden = slot_rows, hidden
        self.slot_floats = -(-(slot_rows * hidden) // 64) * 64
        self.n_slots = graph_slots + eager_slots
        self.graph_slots, self.eager_slots = graph_slots, eager_slots
        data_bytes = self.n_slots * self.slot_floats * 4
        flag_bytes = self.n_slots * AR_CTAS * MAX_RANKS * 4
        # pushed all-reduce: receive blocks [slot][source rank][32 rows][hidden] of {value, epoch}
        # 8-byte words, and this rank's per-(slot, row) epochs
        self.block_words = PUSH_ROWS * hidden
        self.fused_graph_slots, self.fused_eager_slots = fused_graph_slots, fused_eager_slots
        n_fused = fused_graph_slots + fused_eager_slots
        recv_bytes = n_fused * self.world * self.block_words * 8
        # fused Markov selector: one 64-bit word per (step, source rank)
        markov_bytes = MARKOV_STEPS * MAX_RANKS * 8
        # the pushed all-reduce's receive areas in NVLS-capable symmetric memory when the switch
        # supports multicast: a GEMM then stores each word once through the multicast address
        self.recv_mc, self._recv_sym = 0, None
        if nvls is None:           # opt in (Q38_NVLS=1): no gain measured at TP8 on B200
            nvls = os.environ.get("Q38_NVLS", "0") == "1"
        if nvls:
            self._recv_sym = self._nvls_recv(recv_bytes)
            agree = torch.tensor([1 if self._recv_sym is not None else 0], dtype=torch.int32, device=self.device)
            dist.all_reduce(agree, op=dist.ReduceOp.MIN, group=self.group)
            if int(agree.item()) == 0:              # every rank takes the same path
                self._recv_sym = None
        if self._recv_sym is not None:
            recv_bytes_local = 0
        else:
            recv_bytes_local = recv_bytes
        self.buf = self.C.peer_alloc(data_bytes + flag_bytes + recv_bytes_local + markov_bytes, dev)
        handle = self.C.ipc_handle(self.buf).to(self.device)
        handles = [torch.empty_like(handle) for _ in range(self.world)]
        dist.all_gather(handles, handle, group=self.group)
        base = self.buf.data_ptr()
        self._opened = []
        ptrs = []
        for p, h in enumerate(handles):
            if p == self.rank:
                ptrs.append(base)
            else:
                ptr = self.C.ipc_open(h.cpu(), dev)
                self._opened.append(ptr)
                ptrs.append(ptr)
        self.data_ptrs = ptrs
        self.flag_ptrs = [p + data_bytes for p in ptrs]
        if self._recv_sym is not None:
            self.recv_ptrs = list(self._recv_sym[1].buffer_ptrs)
            self.recv_mc = int(self._recv_sym[1].multicast_ptr)
        else:
            self.recv_ptrs = [p + data_bytes + flag_bytes for p in ptrs]
        self.markov_ptrs = [p + data_bytes + flag_bytes + recv_bytes_local for p in ptrs]
        self.fepochs = torch.zeros(n_fused * PUSH_ROWS, dtype=torch.int32, device=self.device)
        self._next_fgraph = 0
        self._next_feager = 0
        self.local = self.buf[:data_bytes].view(torch.float32).view(self.n_slots, self.slot_floats)
        self.epochs = torch.zeros(self.n_slots * AR_CTAS, dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._next_graph = 0
        self._next_eager = 0
        self._pf = None
        # opt in (Q38_PREFILL_AR=1): measured slower than NCCL's all-reduce at TP2 on B200
        if prefill_rows > PUSH_ROWS and self._recv_sym is not None and os.environ.get("Q38_PREFILL_AR", "0") == "1":
            self._init_prefill(prefill_rows)
        dist.barrier(group=self.group)

    # ------------------------------------------------------------------ prefill all-reduce
    def _init_prefill(self, rows: int):
        """Symmetric buffers of the fused prefill all-reduce (csrc/prefill_ar.cu): the replicated
        fp32 residual of a chunk (every rank's copy written through the multicast address), the
        reduce-scatter areas [source][local rows][hidden], the arrival counter and the completion
        flag."""
        import torch.distributed._symmetric_memory as symm_mem
        H, W = self.hidden, self.world
        tiles = -(-rows // 128)
        cap = -(-tiles // W) * 128
        x_bytes = -(-rows * H * 4 // 256) * 256
        rs_bytes = W * cap * H * 4
        total = x_bytes + rs_bytes + 256
        t = symm_mem.empty(total, dtype=torch.uint8, device=self.device)
        h = symm_mem.rendezvous(t, (self.group or dist.group.WORLD).group_name)
        t.zero_()
        torch.cuda.synchronize(self.device)
        ptrs = list(h.buffer_ptrs)
        mc = int(h.multicast_ptr)
        self._pf = dict(
            tensor=t, handle=h, rows=rows, cap=cap,
            x=t[:rows * H * 4].view(torch.float32).view(rows, H),
            recv_ptrs=[p + x_bytes for p in ptrs], count_ptrs=[p + x_bytes + rs_bytes for p in ptrs],
            flag_local=ptrs[self.rank] + x_bytes + rs_bytes + 8, x_mc=mc, flag_mc=mc + x_bytes + rs_bytes + 8,
            count_target=0, flag_target=0)

    def prefill_fits(self, x) -> bool:
        """True when ``x`` is this communicator's prefill residual buffer (fused path available)."""
        pf = self._pf
        return (pf is not None and x.shape[0] > PUSH_ROWS and x.shape[1] == self.hidden
                and x.data_ptr() == pf["x"].data_ptr())

    def prefill_x(self, rows: int):
        """The [rows, hidden] fp32 residual view in symmetric memory, or None when the fused prefill
        all-reduce is off or the chunk does not fit."""
        pf = self._pf
        if pf is None or rows <= PUSH_ROWS or rows > pf["rows"]:
            return None
        return pf["x"][:rows]

    def prefill_push(self, ops, h, w, x) -> int:
        """x += h @ w^T summed over ranks, launched: the reduce-scatter GEMM and this rank's
        reduce + broadcast kernel.  Returns the completion-flag target the next reader waits for."""
        pf = self._pf
        T, W = x.shape[0], self.world
        tiles = -(-T // 128)
        slots = -(-tiles // W) * 128
        owned = len(range(self.rank, tiles, W))
        pf["count_target"] += W * owned * -(-w.N // 256)
        ops.C.linear_rs(h.contiguous(), w.t, w.N, ops.ws, ops.counters, ops.err, pf["recv_ptrs"], pf["count_ptrs"],
                        self.rank, pf["cap"])
        ops.C.rs_reduce_bcast(pf["recv_ptrs"][self.rank], pf["count_ptrs"][self.rank], pf["count_target"], x,
                              pf["x_mc"], pf["flag_mc"], self.rank, W, pf["cap"], slots, ops.err)
        pf["flag_target"] += W * slots
        ops.launches += 2
        return pf["flag_target"]

    def prefill_norm(self, ops, x, w, eps, target):
        out = torch.empty(x.shape[0], x.shape[1], dtype=torch.bfloat16, device=x.device)
        ops.C.rms_norm_wait(x, w, float(eps), out, self._pf["flag_local"], int(target), ops.err)
        ops.launches += 1
        return out

    def prefill_wait(self, ops, target):
        ops.C.rs_wait(self._pf["flag_local"], int(target), ops.err)
        ops.launches += 1

    def _nvls_recv(self, nbytes: int):
        """(tensor, handle) of a zeroed symmetric-memory buffer bound to an NVSwitch multicast object,
        or None when this system or torch build offers none."""
        try:
            import torch.distributed._symmetric_memory as symm_mem
            name = (self.group or dist.group.WORLD).group_name
            t = symm_mem.empty(nbytes, dtype=torch.uint8, device=self.device)
            h = symm_mem.rendezvous(t, name)
            if not int(getattr(h, "multicast_ptr", 0) or 0):
                return None
            t.zero_()
            torch.cuda.synchronize(self.device)
            return t, h
        except Exception:                     # no symmetric memory / multicast: per-rank stores
            return None

    # ------------------------------------------------------------------ slots
    def begin_capture(self):
        """Called before capturing a graph: its collectives take slots 0, 1, 2, ..."""
        self._next_graph = 0
        self._next_fgraph = 0

    def fused_slot(self) -> int:
        """Slot of the fused GEMM + all-reduce areas (same reuse rule as ``_slot``)."""
        if torch.cuda.is_current_stream_capturing():
            if self._next_fgraph >= self.fused_graph_slots:
                raise RuntimeError("out of fused collective slots; raise fused_graph_slots")
            s = self._next_fgraph
            self._next_fgraph += 1
            return s
        s = self.fused_graph_slots + self._next_feager
        self._next_feager = (self._next_feager + 1) % self.fused_eager_slots
        return s

    def fused_fits(self, rows: int, cols: int) -> bool:
        return rows <= PUSH_ROWS and cols == self.hidden

    def _slot(self) -> int:
        if torch.cuda.is_current_stream_capturing():
            if self._next_graph >= self.graph_slots:
                raise RuntimeError("out of graph collective slots; raise graph_slots")
            s = self._next_graph
            self._next_graph += 1
            return s
        s = self.graph_slots + self._next_eager
        self._next_eager = (self._next_eager + 1) % self.eager_slots
        return s

    def fits(self, rows: int, cols: int) -> bool:
        return rows * cols <= self.slot_floats and rows <= self.slot_rows

    def slot_out(self, rows: int, cols: int):
        """A fresh slot and the [rows, cols] fp32 view of this rank's part of it."""
        s = self._slot()
        return s, self.local[s, :rows * cols].view(rows, cols)

    # ------------------------------------------------------------------ collectives
    def reduce_slot_add(self, slot: int, residual: torch.Tensor):
        self.C.allreduce_residual(self.data_ptrs, self.flag_ptrs, self.rank, slot, self.slot_floats, residual,
                                  self.epochs, self.err)
        return residual

    def all_reduce_(self, t):
        """Sum in place.  Small fp32 tensors go through a slot (copy in, reduce into zeros)."""
        if t.dtype == torch.float32 and t.is_cuda and t.dim() == 2 and self.fits(*t.shape):
            s, view = self.slot_out(*t.shape)
            view.copy_(t)
            t.zero_()
            return self.reduce_slot_add(s, t)
        return super().all_reduce_(t)

    def argmax_reduce(self, val, idx):
        rows = val.numel()
        if 2 * rows > self.slot_floats or not val.is_cuda:
            return super().argmax_reduce(val, idx)
        out = torch.empty(rows, dtype=torch.int64, device=val.device)
        s = self._slot()
        self.C.argmax_allreduce(self.data_ptrs, self.flag_ptrs, self.rank, s, self.slot_floats,
                                val.float().contiguous(), idx.to(torch.int64).contiguous(), out, self.epochs,
                                self.err)
        return out

    def check(self):
        e = int(self.err.item())
        if e:
            self.err.zero_()
            raise RuntimeError(f"peer collective timed out (device error word {e})")

    def close(self):
        for p in self._opened:
            self.C.ipc_close(p)
        self._opened = []
