"""Host-side proposal sources: n-gram lookup over the request's own history, and routing between
lookup, neural drafters and target-only blocks.

``LookupDraft`` proposes the continuation of the earlier occurrence whose context matches the end
of the history best: the longest backwards match of the suffix, the most recent occurrence among
equally long matches, optionally preferring an occurrence that can supply the full requested
continuation (the reference's proposal policy, ``speculative-decoding/harness/lookup_draft.py:4-65``,
which the offline acceptance scorer's policy grid is defined over).  Here the history keeps an
inverted index from token id to its positions, so a proposal visits only the occurrences of the
last token instead of scanning the whole history.

``HybridDraft`` asks an ordered chain of sources - lookup (when enabled), then the selected neural
adapter - and falls back to a target-only block when none proposes anything (the reference's
routing, ``hybrid_draft.py:15-61``).  Proposals are never emitted without target verification.
"""
from __future__ import annotations

from bisect import bisect_left
from dataclasses import dataclass


@dataclass(frozen=True)
class Proposal:
    source: str
    tokens: tuple
    match_length: int = 0


def _require_ids(tokens, vocab_size=None):
    out = tuple(tokens)
    for t in out:
        if type(t) is not int or t < 0 or (vocab_size is not None and t >= vocab_size):
            bound = f" below {vocab_size}" if vocab_size is not None else ""
            raise ValueError(f"token id {t!r} is not a non-negative int{bound}")
    return out


class LookupDraft:
    """N-gram lookup over the last ``history_limit`` committed tokens of one request.  Matches are
    compared over at most ``match_limit`` tokens."""

    def __init__(self, request_id, prompt, *, history_limit=32768, match_limit=128, max_proposals=15,
                 prefer_full_suffix=False):
        if not isinstance(request_id, str) or not request_id:
            raise ValueError("LookupDraft needs a non-empty request id")
        if history_limit < 2 or match_limit < 1 or max_proposals < 1:
            raise ValueError("history_limit >= 2, match_limit >= 1 and max_proposals >= 1 are required")
        self.request_id = request_id
        self.history_limit, self.match_limit, self.max_proposals = history_limit, match_limit, max_proposals
        self.prefer_full_suffix = bool(prefer_full_suffix)
        self.closed = False
        self._tokens = []        # committed tokens; positions below _base have left the window
        self._base = 0
        self._where = {}         # token id -> ascending absolute positions
        self.commit(request_id, prompt)

    # ------------------------------------------------------------------ history
    @property
    def history(self):
        return self._tokens[self._base:]

    def check_owner(self, request_id):
        if self.closed:
            raise ValueError(f"lookup history of {self.request_id} is closed")
        if request_id != self.request_id:
            raise ValueError(f"lookup history of {self.request_id} asked for {request_id!r}")

    def commit(self, request_id, tokens):
        """Append committed tokens (the window keeps the last ``history_limit``)."""
        self.check_owner(request_id)
        for t in _require_ids(tokens):
            self._where.setdefault(t, []).append(len(self._tokens))
            self._tokens.append(t)
        self._base = max(self._base, len(self._tokens) - self.history_limit)
        if self._base > self.history_limit:          # compact: drop what left the window, re-index
            keep = self._tokens[self._base:]
            self._tokens, self._base, self._where = [], 0, {}
            for t in keep:
                self._where.setdefault(t, []).append(len(self._tokens))
                self._tokens.append(t)

    def _match_length(self, end: int, cap: int) -> int:
        """Tokens matching backwards from absolute positions ``end`` and the history's last one."""
        toks, last = self._tokens, len(self._tokens) - 1
        k = 1
        while k < cap and toks[end - k] == toks[last - k]:
            k += 1
        return k

    def propose_with_match(self, request_id, count):
        """(continuation tokens, match length) of the best earlier occurrence of the history's
        suffix; ([], 0) when the last token never occurred before."""
        self.check_owner(request_id)
        if not 1 <= count <= self.max_proposals:
            raise ValueError(f"{count} proposals requested; the verifier takes 1..{self.max_proposals}")
        n = len(self._tokens) - self._base
        if n < 2:
            return [], 0
        last = len(self._tokens) - 1
        limit = min(self.match_limit, n - 1)
        spots = self._where[self._tokens[last]]
        first = bisect_left(spots, self._base)
        best_len, best_end, best_room = 0, -1, -1
        for i in range(len(spots) - 1, first - 1, -1):     # newest occurrence first
            end = spots[i]
            if end == last:
                continue
            length = self._match_length(end, min(limit, end - self._base + 1))
            room = min(count, last - end)                  # continuation tokens this occurrence has
            if length > best_len or (self.prefer_full_suffix and length == best_len and room > best_room):
                best_len, best_end, best_room = length, end, room
            if length == limit and (not self.prefer_full_suffix or last - end >= count):
                break                                      # nothing older can do better
        if best_end < 0:
            return [], 0
        return self._tokens[best_end + 1:best_end + 1 + count], best_len

    def propose(self, request_id, count):
        return self.propose_with_match(request_id, count)[0]

    def close(self, request_id):
        self.check_owner(request_id)
        self._tokens, self._where, self._base = [], {}, 0
        self.closed = True


class HybridDraft:
    """Proposal routing for one request: lookup first (when ``lookup_enabled``), then the neural
    adapter named by ``selected`` (the only one when there is exactly one), else a target-only
    block.  A neural adapter is called as ``adapter(request_id, history, count)``."""

    RESERVED = ("lookup", "target")

    def __init__(self, request_id, prompt, *, vocab_size, neural=None, lookup_enabled=True, max_proposals=15,
                 **lookup_options):
        if type(lookup_enabled) is not bool:
            raise ValueError("lookup_enabled must be True or False")
        if vocab_size < 1:
            raise ValueError("vocab_size must be positive")
        self.vocab_size, self.lookup_enabled = vocab_size, lookup_enabled
        self.neural = dict(neural or {})
        for name, adapter in self.neural.items():
            if not isinstance(name, str) or not name or name in self.RESERVED or not callable(adapter):
                raise ValueError(f"neural adapter {name!r}: a callable under a free, non-empty name is required")
        self.lookup = LookupDraft(request_id, self.validate(prompt), max_proposals=max_proposals, **lookup_options)

    def validate(self, tokens):
        return _require_ids(tokens, self.vocab_size)

    def _from_lookup(self, request_id, count, selected):
        if not self.lookup_enabled:
            return None
        tokens, m = self.lookup.propose_with_match(request_id, count)
        return Proposal("lookup", tuple(tokens), m) if tokens else None

    def _from_neural(self, request_id, count, selected):
        name = selected if selected is not None else (next(iter(self.neural)) if len(self.neural) == 1 else None)
        adapter = self.neural.get(name)
        if adapter is None:
            return None
        tokens = self.validate(adapter(request_id, tuple(self.lookup.history), count))
        if len(tokens) > count:
            raise ValueError(f"adapter {name!r} proposed {len(tokens)} tokens, {count} were requested")
        return Proposal(name, tokens) if tokens else None

    def propose(self, request_id, count, *, selected=None):
        self.lookup.check_owner(request_id)
        if not 1 <= count <= self.lookup.max_proposals:
            raise ValueError(f"{count} proposals requested; the verifier takes 1..{self.lookup.max_proposals}")
        for source in (self._from_lookup, self._from_neural):
            p = source(request_id, count, selected)
            if p is not None:
                return p
        return Proposal("target", ())

    def commit_verified(self, request_id, tokens):
        self.lookup.commit(request_id, self.validate(tokens))

    def close(self, request_id):
        self.lookup.close(request_id)
        self.neural.clear()
