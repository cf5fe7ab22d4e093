"""Offline lookup-acceptance scoring over a native tape and the block latency budget."""
import pytest

from qwen38_b200.config import RuntimeConfig
from qwen38_b200.models.target import HybridTarget
from qwen38_b200.spec.analysis import latency_budget, score_lookup, sweep_lookup
from qwen38_b200.spec.engine import PinnedAcceptance, SpecRuntime, greedy_reference


def test_lookup_scoring_on_a_periodic_tape():
    prompt = [1, 2, 3, 4, 5, 6, 7, 8] * 4
    emitted = ([1, 2, 3, 4, 5, 6, 7, 8] * 8)[:40]
    r = score_lookup(prompt, emitted, vocab_size=16, max_new_tokens=40, max_rows=16)
    assert r["committed"] == 39                         # every decode token after the prefill seed
    assert r["mean_committed_per_block"] > 4            # nearest earlier period: 7-token proposals
    assert [b["accepted"] for b in r["blocks"][:4]] == [7, 7, 7, 7]   # every proposal accepted
    one = score_lookup(prompt, emitted, vocab_size=16, max_new_tokens=40, max_rows=1)
    assert one["mean_committed_per_block"] == 1 and len(one["blocks"]) == 39
    arms = sweep_lookup(prompt, emitted, vocab_size=16, max_new_tokens=40)
    assert len(arms) == 6 * 4 * 2
    assert max(a["mean_committed_per_block"] for a in arms) >= r["mean_committed_per_block"]


def test_lookup_scoring_rejects_bad_tapes():
    with pytest.raises(ValueError):
        score_lookup([1, 2], [3, 4], vocab_size=16, max_new_tokens=4)            # incomplete tape
    with pytest.raises(ValueError):
        score_lookup([1, 2], [3, 9, 4], vocab_size=16, max_new_tokens=3, eos_ids=(9,))   # EOS mid-tape
    with pytest.raises(ValueError):
        score_lookup([1, 2], [3], vocab_size=16, max_new_tokens=1, max_rows=3)   # not a bucket


def test_latency_budget():
    blocks = [dict(rows=16, committed=8, draft_ms=2.0, verify_ms=12.0, commit_ms=1.0, cycle_ms=15.0)] * 4
    b = latency_budget(blocks, target_tg=800)
    assert b["observed_tg"] == pytest.approx(1000 * 8 / 15)
    assert b["cycle_needed_ms"] == pytest.approx(10.0)
    assert b["cycle_cut_needed_pct"] == pytest.approx(100 * (1 - 10 / 15))
    assert b["tokens_per_block_needed"] == pytest.approx(800 * 15 / 1000)
    assert b["tg_if_free"]["draft"] == pytest.approx(1000 * 8 / 13)
    assert b["tg_if_free"]["verify"] == pytest.approx(1000 * 8 / 3)
    with pytest.raises(ValueError):
        latency_budget(blocks + [dict(blocks[0], rows=8)])
    with pytest.raises(ValueError):
        latency_budget([dict(blocks[0], verify_ms=16.0)])          # a phase longer than the cycle


def test_generate_block_records_feed_the_budget(tiny):
    rt = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)
    tgt = HybridTarget(tiny["cfg"], tiny["src"], rt)
    gold = greedy_reference(tgt, tiny["prompt"], 12)
    res = SpecRuntime(tgt, None, verifier_rows=4).generate(tiny["prompt"], 12, gold_check=gold)
    recs = res["block_records"]
    assert len(recs) == res["blocks"] and sum(r["committed"] for r in recs) == res["committed"]
    assert latency_budget(recs)["profile"]["blocks"] == len(recs)


def test_acceptance_report_statistics():
    from qwen38_b200.spec.analysis import acceptance_report
    blocks = [dict(rows=4, accepted=a, committed=a + 1) for a in (3, 1, 0, 2, 3)] + [dict(rows=4, accepted=1,
                                                                                            committed=1)]
    r = acceptance_report(blocks)
    assert r["full_draft_blocks"] == 5 and r["histogram"] == [1, 1, 1, 2]
    assert r["mean_accepted"] == 9 / 5
    assert r["unconditional"] == [4 / 5, 3 / 5, 2 / 5]
    assert r["conditional"] == [4 / 5, 3 / 4, 2 / 3]
    assert abs(r["mean_committed_per_block"] - 15 / 6) < 1e-12
    with pytest.raises(ValueError):
        acceptance_report([dict(rows=4, accepted=4, committed=4)])
    with pytest.raises(ValueError):
        acceptance_report([])


def test_acceptance_report_of_a_pinned_run(tiny):
    """Pinned acceptance with mean m cuts each block at a uniform position in [0, 2m]: the report
    of a real run sees a mean accepted near m and a decreasing unconditional curve."""
    from qwen38_b200.spec.analysis import acceptance_report
    from qwen38_b200.models.drafter import BlockDrafter
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16))
    dr = BlockDrafter(tiny["dcfg"], tiny["dsrc"], tgt)
    gold = greedy_reference(tgt, tiny["prompt"], 120)
    res = SpecRuntime(tgt, dr, verifier_rows=4).generate(
        tiny["prompt"], 120, pinned=PinnedAcceptance(gold, seed=1, mean_accepted=1), gold_check=gold)
    r = acceptance_report(res["block_records"])
    assert r["rows"] == 4 and r["full_draft_blocks"] >= 10
    assert 0.5 <= r["mean_accepted"] <= 1.6
    u = [x for x in r["unconditional"] if x is not None]
    assert all(a >= b for a, b in zip(u, u[1:]))
