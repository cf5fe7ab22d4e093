"""The runtime (packed weights, paged KV, chunked prefill, verify + commit replay) against the
reference model, and speculative decoding against plain greedy decode."""
import torch

from qwen38_b200.config import RuntimeConfig
from qwen38_b200.models.drafter import BlockDrafter
from qwen38_b200.models.reference import ReferenceModel
from qwen38_b200.models.target import HybridTarget
from qwen38_b200.spec.engine import PinnedAcceptance, SpecRuntime, greedy_reference

RT = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)


def _target(tiny, **kw):
    return HybridTarget(tiny["cfg"], tiny["src"], RT, **kw)


def test_runtime_greedy_matches_reference(tiny):
    ref = ReferenceModel(tiny["cfg"], tiny["sd"])
    toks = torch.tensor(tiny["prompt"])
    assert _target(tiny).greedy(toks, 32) == ref.greedy(toks, 32)


def test_verify_rows_match_sequential_decode(tiny):
    tgt = _target(tiny)
    toks = torch.tensor(tiny["prompt"][:100])
    block = torch.tensor(tiny["prompt"][100:108])
    seq = tgt.new_sequence()
    tgt.prefill(seq, toks)
    snap = tgt.snapshot(seq)
    pred, _ = tgt.verify([(seq, block)])
    tgt.commit(seq, 5)
    after_commit = tgt.snapshot(seq)
    tgt.restore(seq, snap)
    seq_preds = []
    for t in block[:5]:
        p, _ = tgt.decode(seq, t.reshape(1))
        seq_preds.append(int(p))
    assert pred[:5].tolist() == seq_preds
    assert torch.allclose(tgt.rec[seq.slot], after_commit["rec"], atol=1e-6)
    assert seq.pos == after_commit["pos"]


def test_speculative_equals_greedy(tiny):
    tgt = _target(tiny)
    dr = BlockDrafter(tiny["dcfg"], tiny["dsrc"], tgt)
    gold = greedy_reference(tgt, tiny["prompt"], 32)
    for pinned in (None, PinnedAcceptance(gold, seed=0, mean_accepted=1)):
        res = SpecRuntime(tgt, dr, verifier_rows=4).generate(tiny["prompt"], 32, gold_check=gold, pinned=pinned)
        assert res["tokens"] == gold
        assert res["committed"] == 31
    res = SpecRuntime(tgt, dr, verifier_rows=4, lookup=True).generate(tiny["prompt"], 32, gold_check=gold)
    assert res["tokens"] == gold


def test_pinned_acceptance_mean():
    pa = PinnedAcceptance(list(range(1000)), seed=5, mean_accepted=6)
    cuts = []
    for _ in range(400):
        props = pa.apply(10, 15, 2000)
        gold = list(range(10, 25))
        cuts.append(next((i for i, (a, b) in enumerate(zip(props, gold)) if a != b), 15))
    assert abs(sum(cuts) / len(cuts) - 6) < 0.7


def test_sampled_generate_speculates_exactly(tiny):
    """``SpecRuntime.generate`` with a temperature reproduces the target's own one-token-per-step
    sample while committing several tokens per block."""
    from qwen38_b200.models.drafter import BlockDrafter
    from qwen38_b200.spec.engine import PinnedAcceptance, SpecRuntime
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16))
    dr = BlockDrafter(tiny["dcfg"], tiny["dsrc"], tgt)
    ref = tgt.sample(torch.tensor(tiny["prompt"]), 24, temperature=0.7, seed=3)
    res = SpecRuntime(tgt, dr, verifier_rows=4).generate(
        tiny["prompt"], 24, temperature=0.7, seed=3, pinned=PinnedAcceptance(ref, seed=1, mean_accepted=2))
    assert res["tokens"] == ref and res["tokens_per_block"] > 1
    greedy = SpecRuntime(tgt, dr, verifier_rows=4).generate(tiny["prompt"], 24)["tokens"]
    assert greedy == tgt.greedy(torch.tensor(tiny["prompt"]), 24)
