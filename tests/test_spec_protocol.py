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
