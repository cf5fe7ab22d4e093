"""Run-report helpers: token / source digests and the itemised device-memory ledger with its
budget check (CPU: the ledger itemises the same tensors it would on a GPU)."""
import pytest
import torch

from qwen38_b200.config import RuntimeConfig
from qwen38_b200.models.drafter import BlockDrafter
from qwen38_b200.models.target import HybridTarget
from qwen38_b200.spec.engine import SpecRuntime, greedy_reference
from qwen38_b200.utils.trace import MemoryBudgetExceeded, memory_ledger, nvtx, source_digests, token_digest


def test_digests_are_stable():
    assert token_digest([1, 2, 3]) == token_digest(torch.tensor([1, 2, 3]))
    assert token_digest([1, 2, 3]) != token_digest([1, 2, 4])
    d = source_digests()
    assert any(k.endswith("gemm_kernel.cuh") for k in d) and all(len(v) == 64 for v in d.values())
    with nvtx("noop"):
        pass


def test_memory_ledger_itemises_and_checks_budget(tiny):
    rt = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)
    tgt = HybridTarget(tiny["cfg"], tiny["src"], rt)
    dr = BlockDrafter(tiny["dcfg"], tiny["dsrc"], tgt)
    led = memory_ledger(tgt, dr)
    assert led["kv_cache"] == 2 * tgt.kcache.numel() * tgt.kcache.element_size()
    assert led["gdn_state"] == tgt.rec.numel() * 4
    assert led["weights.mlp"] > 0 and led["drafter.history"] > 0
    assert led["total_itemised"] == sum(v for k, v in led.items() if k != "total_itemised")
    with pytest.raises(MemoryBudgetExceeded):
        memory_ledger(tgt, dr, budget_bytes=1024)


def test_generate_reports_digests(tiny):
    rt = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)
    tgt = HybridTarget(tiny["cfg"], tiny["src"], rt)
    gold = greedy_reference(tgt, tiny["prompt"], 8)
    res = SpecRuntime(tgt, None, verifier_rows=4).generate(tiny["prompt"], 8, gold_check=gold)
    assert res["output_sha256"] == token_digest(gold) and res["prompt_sha256"] == token_digest(tiny["prompt"])
