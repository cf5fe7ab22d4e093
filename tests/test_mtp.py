"""MTP head as a drafter: speculative output with MTP proposals equals plain greedy decode, and
the MTP history follows the committed rows (successor tokens + last-layer hidden states)."""
import torch

from qwen38_b200.config import RuntimeConfig
from qwen38_b200.models.mtp import MTPDrafter, random_mtp_source
from qwen38_b200.models.target import HybridTarget
from qwen38_b200.spec.engine import PinnedAcceptance, SpecRuntime, greedy_reference


def test_mtp_drafter_speculative_equals_greedy(tiny):
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16))
    mtp = MTPDrafter(random_mtp_source(tiny["cfg"]), tgt, steps=3)
    assert mtp.dcfg.taps == [tiny["cfg"].num_hidden_layers - 1] and mtp.dcfg.block_rows == 4
    gold = greedy_reference(tgt, tiny["prompt"], 24)
    sr = SpecRuntime(tgt, mtp, verifier_rows=4)
    res = sr.generate(tiny["prompt"], 24, gold_check=gold)
    assert res["tokens"] == gold
    assert mtp.positions[0] >= len(tiny["prompt"])
    res = sr.generate(tiny["prompt"], 24, gold_check=gold, pinned=PinnedAcceptance(gold, seed=2, mean_accepted=1))
    assert res["tokens"] == gold


def test_mtp_history_rows_match_recomputation(tiny):
    """Row p written incrementally (prompt, then committed blocks) equals row p written in one
    publication of the whole committed sequence."""
    rt = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)
    tgt = HybridTarget(tiny["cfg"], tiny["src"], rt)
    src = random_mtp_source(tiny["cfg"])
    mtp = MTPDrafter(src, tgt, steps=3)
    gold = greedy_reference(tgt, tiny["prompt"], 12)
    SpecRuntime(tgt, mtp, verifier_rows=4).generate(tiny["prompt"], 12, gold_check=gold)
    n = mtp.positions[0]
    k_inc = mtp.kctx_all[0, 0, :n].clone()
    # one-shot: prefill prompt + emitted tokens, publish every row at once
    full = tiny["prompt"] + gold[:-1]
    seq = tgt.new_sequence()
    nxt, feats = tgt.prefill(seq, torch.tensor(full), taps=mtp.dcfg.taps)
    tgt.release(seq)
    mtp2 = MTPDrafter(src, tgt, steps=3)
    mtp2.append(feats, 0, next_tokens=full[1:] + [gold[-1]])
    assert mtp2.positions[0] == n
    assert torch.allclose(mtp2.kctx_all[0, 0, :n], k_inc, atol=2e-3)
