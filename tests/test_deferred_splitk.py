"""Deferred split-K reduction on one rank: the out-projections leave their K slices for the next
norm of the residual (``HybridTarget.local_row_parallel``).  These CPU tests drive the bookkeeping
with an ops class whose ``linear_split`` keeps the product as slice 0 of two slices, so every raw
read of the residual that is not settled first (a tap, the head, the drafter's residual) would
see a stale value and change the result."""
import torch

from qwen38_b200.config import RuntimeConfig
from qwen38_b200.models.drafter import BlockDrafter
from qwen38_b200.models.target import HybridTarget
from qwen38_b200.ops import TorchOps
from qwen38_b200.spec.engine import SpecRuntime, greedy_reference

RT = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)


class DeferredOps(TorchOps):
    """TorchOps whose <= 64-row residual GEMMs leave two slices (the product and zeros)."""

    max_pack_rows = 64

    def __init__(self):
        super().__init__()
        self.parts = None
        self.completed = 0

    def linear_split(self, x, w, residual):
        if self.parts is not None:
            raise AssertionError("a second split GEMM before the previous one was completed")
        p = (x.float() @ w.float().t()) if x.device.type == "cpu" else (x @ w.t()).float()
        self.parts = [p, torch.zeros_like(p)]
        return 2

    def rms_norm_split(self, x, w, eps, out_dtype, S):
        acc = torch.zeros_like(x)
        for p in self.parts[:S]:
            acc = acc + p
        x += acc
        self.parts = None
        self.completed += 1
        return None if w is None else self.rms_norm(x, w, eps, out_dtype)


def _pair(tiny):
    plain = HybridTarget(tiny["cfg"], tiny["src"], RT)
    ops = DeferredOps()
    deferred = HybridTarget(tiny["cfg"], tiny["src"], RT, ops=ops)
    assert deferred.defer_splits and not plain.defer_splits
    return plain, deferred, ops


def test_deferred_verify_matches_in_gemm_fixup(tiny):
    plain, deferred, ops = _pair(tiny)
    toks = torch.tensor(tiny["prompt"][:100])
    block = torch.tensor(tiny["prompt"][100:108])
    outs = []
    for tgt in (plain, deferred):
        seq = tgt.new_sequence()
        tgt.prefill(seq, toks)
        pred, feats = tgt.verify([(seq, block)], taps=(0, 2))
        tgt.commit(seq, 5)
        outs.append((pred, feats, tgt.snapshot(seq)["rec"]))
    assert ops.completed > 0 and ops.parts is None
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])        # taps read the settled residual
    assert torch.equal(outs[0][2], outs[1][2])


def test_deferred_speculative_equals_greedy(tiny):
    plain, deferred, ops = _pair(tiny)
    gold = greedy_reference(plain, tiny["prompt"], 32)
    dr = BlockDrafter(tiny["dcfg"], tiny["dsrc"], deferred)
    res = SpecRuntime(deferred, dr, verifier_rows=4).generate(tiny["prompt"], 32, gold_check=gold)
    assert res["tokens"] == gold
    assert ops.parts is None
