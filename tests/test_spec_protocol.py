"""Greedy block protocol: prefix selection, session state machine, lookup and hybrid routing
(behaviours of speculative-decoding/harness/test_greedy_*.py and test_lookup_draft.py)."""
import pytest

from qwen38_b200.spec.greedy import GreedySession, select_prefix
from qwen38_b200.spec.lookup import HybridDraft, LookupDraft

V = 100


def test_every_forced_rejection_prefix():
    props = (5, 6, 7)
    for cut in range(4):
        preds = list(props[:cut]) + [50] * (4 - cut)
        d = select_prefix(props, preds, vocab_size=V, max_proposals=3)
        assert d.accepted == cut and d.state_rows == cut + 1
        assert d.emitted == props[:cut] + (50,)


def test_all_accepted_bonus_and_target_only():
    d = select_prefix((1, 2, 3), (1, 2, 3, 9), vocab_size=V, max_proposals=3)
    assert d.emitted == (1, 2, 3, 9) and d.next_input == 9
    d = select_prefix((), (4,), vocab_size=V)
    assert d.emitted == (4,) and d.state_rows == 1


def test_eos_handling():
    d = select_prefix((1, 2, 3), (1, 2, 3, 4), vocab_size=V, eos_ids=(2,), max_proposals=3)
    assert d.emitted == (1, 2) and d.finished and d.state_rows == 2
    d = select_prefix((1, 5), (1, 2, 0), vocab_size=V, eos_ids=(2,), max_proposals=3)
    assert d.emitted == (1, 2) and d.finished and d.next_input is None
    d = select_prefix((2,), (3, 4), vocab_size=V, eos_ids=(2,), max_proposals=3)
    assert not d.finished and d.emitted == (3,)


def test_invalid_shapes_and_tokens():
    with pytest.raises(ValueError):
        select_prefix((1,), (1,), vocab_size=V)
    with pytest.raises(ValueError):
        select_prefix((1,), (1, V), vocab_size=V)
    with pytest.raises(ValueError):
        select_prefix((1,) * 16, (1,) * 17, vocab_size=V, max_proposals=15)


class _Drafter:
    def __init__(self, props):
        self.props, self.history, self.closed = list(props), [], False

    def propose(self, rid, count, selected=None):
        from qwen38_b200.spec.lookup import Proposal
        return Proposal("fake", tuple(self.props[:count]))

    def commit_verified(self, rid, toks):
        self.history.extend(toks)

    def close(self, rid):
        self.closed = True


def test_session_accounting_and_budget():
    dr = _Drafter([1, 2, 3])
    s = GreedySession("r", [9, 9], 7, vocab_size=V, max_new_tokens=6, drafter=dr, verifier_rows=4)
    t = s.propose("r")
    assert t.tokens == (7, 1, 2, 3) and t.position == 2
    d = s.commit("r", t, (1, 2, 30, 31), lambda rows: None)
    assert d.emitted == (1, 2, 30) and s.position == 5 and s.seed == 30
    assert s.committed_decode_tokens == 3 and s.emitted == [7, 1, 2, 30]
    t = s.propose("r")                                      # 2 tokens left -> bucket of 2 rows
    assert len(t.tokens) == 2
    s.commit("r", t, (1, 40), lambda rows: None)
    assert s.finished and len(s.emitted) == 6


def test_publication_failure_poisons():
    s = GreedySession("r", [1], 2, vocab_size=V, max_new_tokens=8, drafter=_Drafter([3]), verifier_rows=4)
    t = s.propose("r")

    def bad(rows):
        raise RuntimeError("device")

    with pytest.raises(RuntimeError):
        s.commit("r", t, (3, 4), bad)
    assert s.phase == "failed"
    with pytest.raises(ValueError):
        s.propose("r")


def test_abort_and_stale_ticket():
    s = GreedySession("r", [1], 2, vocab_size=V, max_new_tokens=8, drafter=_Drafter([3, 4, 5]), verifier_rows=4)
    t = s.propose("r")
    s.abort("r", t, lambda rows: None)
    assert s.aborted_blocks == 1 and s.phase == "idle"
    with pytest.raises(ValueError):
        s.commit("r", t, (3, 4, 5, 6), lambda rows: None)
    t2 = s.propose("r")
    assert t2.epoch == t.epoch + 1


def test_narrow_and_owner_guards():
    s = GreedySession("r", [1], 2, vocab_size=V, max_new_tokens=20, drafter=_Drafter([3, 4, 5]), verifier_rows=4)
    t = s.propose("r")
    with pytest.raises(ValueError):
        s.propose("other")
    n = s.narrow("r", t, 2)
    assert n.tokens == (2, 3) and n.epoch == t.epoch + 1
    with pytest.raises(ValueError):
        s.commit("r", t, (3, 4, 5, 6), lambda rows: None)
    s.commit("r", n, (3, 9), lambda rows: None)


def test_lookup_longest_suffix_and_recency():
    lk = LookupDraft("r", [1, 2, 3, 9, 1, 2, 3, 8, 5, 2, 3])
    toks, m = lk.propose_with_match("r", 2)
    assert toks == [8, 5] and m == 2
    lk2 = LookupDraft("r", [4, 1, 5, 1, 6, 1])
    assert lk2.propose("r", 1) == [6]                     # most recent equal-length match


def test_lookup_bounds_and_isolation():
    lk = LookupDraft("r", list(range(10)), history_limit=4)
    assert lk.history == [6, 7, 8, 9]
    assert lk.propose("r", 3) == []
    with pytest.raises(ValueError):
        lk.propose("x", 1)
    lk.close("r")
    with pytest.raises(ValueError):
        lk.commit("r", [1])


def test_hybrid_routing():
    calls = []

    def neural(rid, hist, count):
        calls.append(count)
        return (1,) * count

    h = HybridDraft("r", [5, 6, 5], vocab_size=V, neural={"n": neural}, max_proposals=3)
    p = h.propose("r", 2)
    assert p.source == "lookup" and not calls
    h2 = HybridDraft("r", [5, 6, 7], vocab_size=V, neural={"n": neural}, max_proposals=3)
    p = h2.propose("r", 2, selected="n")
    assert p.source == "n" and p.tokens == (1, 1)
    h3 = HybridDraft("r", [5, 6, 7], vocab_size=V, neural={"n": lambda *a: (V,)}, max_proposals=3)
    with pytest.raises(ValueError):
        h3.propose("r", 1, selected="n")
    assert h2.propose("r", 1, selected="missing").source == "target"


def test_bucket_widths():
    from qwen38_b200.spec.greedy import bucket_at_most
    assert [bucket_at_most(n) for n in (1, 2, 3, 5, 8, 15, 16, 31, 40)] == [1, 2, 2, 4, 8, 8, 16, 16, 32]


def test_device_selection_matches_host_rule():
    """``device_accept`` (tensor ops, no read-back) publishes the rows and next seed that the host
    rule ``select_prefix`` gives, for every cut of a 16-row block."""
    import random

    import torch

    from qwen38_b200.spec.greedy import accepted_length, device_accept
    rng = random.Random(3)
    for cut in range(17):
        drafts = [rng.randrange(V) for _ in range(15)]
        preds = list(drafts) + [rng.randrange(V)]
        if cut < 15:
            preds[cut] = (drafts[cut] + 1) % V
        d = select_prefix(drafts, preds, vocab_size=V)
        block = torch.tensor([7] + drafts)
        rows, nxt = device_accept(block, torch.tensor(preds))
        assert int(rows) == d.state_rows and int(nxt) == d.next_input
        assert int(accepted_length(block[1:], torch.tensor(preds))) == accepted_length(drafts, preds) == d.accepted


def _lookup_spec(hist, count, match_limit, prefer_full):
    """Specification of the lookup policy: among earlier occurrences of the last token, the one
    with the longest backwards match (capped), then (optionally) the most continuation tokens,
    then the most recent."""
    n = len(hist)
    if n < 2:
        return [], 0
    limit = min(match_limit, n - 1)
    best = None
    for end in range(n - 1):
        if hist[end] != hist[-1]:
            continue
        k = 1
        while k < min(limit, end + 1) and hist[end - k] == hist[n - 1 - k]:
            k += 1
        key = (k, min(count, n - 1 - end) if prefer_full else 0, end)
        best = key if best is None or key > best else best
    if best is None:
        return [], 0
    return hist[best[2] + 1:best[2] + 1 + count], best[0]


def test_lookup_matches_its_specification_on_random_histories():
    import random
    rng = random.Random(11)
    for trial in range(300):
        alphabet = rng.choice([2, 3, 5, 20])
        hist = [rng.randrange(alphabet) for _ in range(rng.randrange(1, 80))]
        limit = rng.choice([1, 2, 4, 128])
        window = rng.choice([4, 16, 1000])
        pf = rng.random() < 0.5
        lk = LookupDraft("r", hist[:5], history_limit=window, match_limit=limit, prefer_full_suffix=pf)
        for i in range(5, len(hist), 7):                 # commits in pieces (window trimming, compaction)
            lk.commit("r", hist[i:i + 7])
        visible = hist[-window:]
        assert lk.history == visible
        for count in (1, 3, 15):
            assert tuple(lk.propose_with_match("r", count)) == tuple(_lookup_spec(visible, count, limit, pf))
