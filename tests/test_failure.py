"""Failure detection on the host (CPU, gloo): a rank that dies before a collective turns into an
error on its peer within the process-group timeout instead of a hang; a verifier failure poisons
the session and releases the request's resources; corrupted proposals cannot change the output and
out-of-vocabulary ones fail the request cleanly; publication failures are covered in
test_spec_protocol.py and request quarantine in test_serving.py."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qwen38_b200.config import RuntimeConfig
from qwen38_b200.models.target import HybridTarget
from qwen38_b200.spec.engine import SpecRuntime


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(0)                     # dies between steps, before the next collective
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put("no error")
    except Exception as e:             # noqa: BLE001 - any collective error is the expected outcome
        q.put("error: " + type(e).__name__)


def test_dead_rank_becomes_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
    assert res.startswith("error")


def test_verifier_failure_poisons_session_and_releases(tiny):
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16))
    free0, slots0 = tgt.allocator.num_free, len(tgt.free_slots)
    real_verify = tgt.verify
    calls = {"n": 0}

    def flaky(batch, taps=()):
        calls["n"] += 1
        if calls["n"] == 3:
            raise RuntimeError("injected verifier failure")
        return real_verify(batch, taps)

    tgt.verify = flaky
    sr = SpecRuntime(tgt, None, verifier_rows=4, lookup=True)
    with pytest.raises(RuntimeError, match="injected"):
        sr.generate(tiny["prompt"], 16)
    assert sr.last_session.phase == "failed"
    assert tgt.allocator.num_free == free0 and len(tgt.free_slots) == slots0


def _drafter_with(tiny, tgt, corrupt):
    """The tiny DSpark drafter with its proposals replaced by ``corrupt(proposals)``."""
    from qwen38_b200.models.drafter import BlockDrafter
    dr = BlockDrafter(tiny["dcfg"], tiny["dsrc"], tgt)
    real = dr.propose
    dr.propose = lambda anchor, slot=0: corrupt(real(anchor, slot))
    return dr


def test_corrupted_proposals_cannot_change_the_output(tiny):
    """Wrong but valid proposals (shuffled, constant, reversed) are rejected by verification: the
    output stays the greedy output."""
    from qwen38_b200.spec.engine import greedy_reference
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16))
    gold = greedy_reference(tgt, tiny["prompt"], 16)
    g = torch.Generator().manual_seed(5)
    V = tiny["cfg"].vocab_size
    for corrupt in (lambda p: torch.randint(0, V, p.shape, generator=g),
                    lambda p: torch.full_like(p, 7),
                    lambda p: p.flip(0)):
        dr = _drafter_with(tiny, tgt, corrupt)
        res = SpecRuntime(tgt, dr, verifier_rows=tiny["dcfg"].block_rows).generate(tiny["prompt"], 16)
        assert res["tokens"] == gold


def test_out_of_vocab_proposals_fail_the_request_cleanly(tiny):
    """Proposals outside the vocabulary are refused before any verify; the request fails and its
    sequence, state slot and KV blocks are released."""
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16))
    free0, slots0 = tgt.allocator.num_free, len(tgt.free_slots)
    V = tiny["cfg"].vocab_size
    dr = _drafter_with(tiny, tgt, lambda p: p + V)
    sr = SpecRuntime(tgt, dr, verifier_rows=tiny["dcfg"].block_rows)
    with pytest.raises(ValueError):
        sr.generate(tiny["prompt"], 16)
    assert tgt.allocator.num_free == free0 and len(tgt.free_slots) == slots0
