"""Host-side proposal sources: n-gram lookup and lookup-first hybrid routing.

``LookupDraft`` proposes the continuation of the longest earlier occurrence of the history's
suffix (``speculative-decoding/harness/lookup_draft.py:4-65``); ``HybridDraft`` tries lookup
first, then a named neural adapter, else proposes nothing (target-only block,
``hybrid_draft.py:15-61``).  Proposals are never emitted without target verification.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Proposal:
    source: str
    tokens: tuple
    match_length: int = 0


class LookupDraft:
    def __init__(self, request_id, prompt, *, history_limit=32768, match_limit=128, max_proposals=15,
                 prefer_full_suffix=False):
        if not isinstance(request_id, str) or not request_id:
            raise ValueError("a request identity is required")
        if history_limit < 2 or match_limit < 1 or max_proposals < 1:
            raise ValueError("history_limit >= 2, match_limit >= 1 and max_proposals >= 1 required")
        self.request_id, self.history_limit, self.match_limit = request_id, history_limit, match_limit
        self.max_proposals, self.prefer_full_suffix = max_proposals, bool(prefer_full_suffix)
        self.closed = False
        self.history = []
        self.commit(request_id, prompt)

    def check_owner(self, request_id):
        if self.closed or request_id != self.request_id:
            raise ValueError("closed or mismatched request identity")

    def commit(self, request_id, tokens):
        self.check_owner(request_id)
        tokens = list(tokens)
        if any(type(t) is not int or t < 0 for t in tokens):
            raise ValueError("non-negative integer token ids expected")
        self.history = (self.history + tokens)[-self.history_limit:]

    def propose_with_match(self, request_id, count):
        """Continuation of the most recent earlier occurrence with the longest suffix match.
        Scans candidate ends from newest to oldest; stops early at a full-length match."""
        self.check_owner(request_id)
        if not 1 <= count <= self.max_proposals:
            raise ValueError("proposal count exceeds the verifier capacity")
        h = self.history
        n = len(h)
        if n < 2:
            return [], 0
        last = h[-1]
        limit = min(self.match_limit, n - 1)
        best_len, best_end = 0, None
        for end in range(n - 2, -1, -1):
            if h[end] != last:
                continue
            length = 1
            cap = min(limit, end + 1)
            while length < cap and h[end - length] == h[n - 1 - length]:
                length += 1
            better = length > best_len
            if (not better and self.prefer_full_suffix and length == best_len and best_end is not None
                    and min(count, n - end - 1) > min(count, n - best_end - 1)):
                better = True
            if better:
                best_len, best_end = length, end
                if length == limit and (not self.prefer_full_suffix or n - end - 1 >= count):
                    break
        if best_end is None:
            return [], 0
        return h[best_end + 1:best_end + 1 + count], best_len

    def propose(self, request_id, count):
        return self.propose_with_match(request_id, count)[0]

    def close(self, request_id):
        self.check_owner(request_id)
        self.history.clear()
        self.closed = True


class HybridDraft:
    """Lookup first, then the selected neural adapter ``adapter(request_id, history, count)``."""

    def __init__(self, request_id, prompt, *, vocab_size, neural=None, lookup_enabled=True, max_proposals=15,
                 **lookup_options):
        if type(lookup_enabled) is not bool:
            raise ValueError("explicit lookup routing selection required")
        if vocab_size < 1:
            raise ValueError("vocab_size must be positive")
        self.vocab_size, self.lookup_enabled = vocab_size, lookup_enabled
        self.neural = dict(neural or {})
        for name, adapter in self.neural.items():
            if not isinstance(name, str) or not name or name in ("lookup", "target") or not callable(adapter):
                raise ValueError("named callable neural adapters expected")
        self.lookup = LookupDraft(request_id, self.validate(prompt), max_proposals=max_proposals, **lookup_options)

    def validate(self, tokens):
        tokens = tuple(tokens)
        if any(type(t) is not int or not 0 <= t < self.vocab_size for t in tokens):
            raise ValueError("token outside the target vocabulary")
        return tokens

    def propose(self, request_id, count, *, selected=None):
        self.lookup.check_owner(request_id)
        if not 1 <= count <= self.lookup.max_proposals:
            raise ValueError("proposal count exceeds the verifier capacity")
        if self.lookup_enabled:
            tokens, m = self.lookup.propose_with_match(request_id, count)
            if tokens:
                return Proposal("lookup", tuple(tokens), m)
        if selected is None and len(self.neural) == 1:
            selected = next(iter(self.neural))
        adapter = self.neural.get(selected)
        if adapter is None:
            return Proposal("target", ())
        tokens = self.validate(adapter(request_id, tuple(self.lookup.history), count))
        if len(tokens) > count:
            raise ValueError("neural proposal exceeds the requested count")
        return Proposal(selected, tokens) if tokens else Proposal("target", ())

    def commit_verified(self, request_id, tokens):
        self.lookup.commit(request_id, self.validate(tokens))

    def close(self, request_id):
        self.lookup.close(request_id)
        self.neural.clear()
