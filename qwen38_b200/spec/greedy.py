"""Greedy block-verification protocol: prefix selection and the request-scoped session.

Semantics match the reference harness (``speculative-decoding/harness/greedy_verify.py:15-37``,
``greedy_session.py:19-173``): a block ticket carries ``[seed, *proposals]`` at the committed
position; the target's argmax for row i predicts the token after row i; proposals are accepted
while they equal those predictions; the first disagreement contributes the target's correction;
``state_rows = accepted + 1`` rows are published.  The session moves
``idle -> drafting -> pending -> committing -> idle`` and is poisoned (``failed``) by any error
inside drafting or publication.

Verifier widths are the bucket set (1, 2, 4, 8, 16, 32) capped by the session's
``verifier_rows``; the reference pins 16/32, the tiny CPU configuration uses 4.
"""
from __future__ import annotations

from dataclasses import dataclass

BUCKETS = (1, 2, 4, 8, 16, 32)


@dataclass(frozen=True)
class Decision:
    emitted: tuple
    accepted: int
    state_rows: int
    next_input: int | None
    finished: bool


def select_prefix(proposals, target_argmax, *, vocab_size, eos_ids=(), max_proposals=15) -> Decision:
    """Rows consume ``[seed, *proposals]``; ``target_argmax[i]`` is the target's next token after
    row i.  Returns the emitted tokens (accepted proposals then the correction)."""
    if type(vocab_size) is not int or vocab_size < 1:
        raise ValueError("positive vocabulary size required")
    if type(max_proposals) is not int or max_proposals + 1 not in BUCKETS[1:]:
        raise ValueError("proposal capacity must be a verifier bucket minus one")
    proposals, target_argmax, eos_ids = tuple(proposals), tuple(target_argmax), tuple(eos_ids)
    if len(proposals) > max_proposals or len(target_argmax) != len(proposals) + 1:
        raise ValueError("expected at most max_proposals proposals and one more prediction row")
    for tok in (*proposals, *target_argmax, *eos_ids):
        if type(tok) is not int or not 0 <= tok < vocab_size:
            raise ValueError("token outside the target vocabulary")
    accepted = 0
    for prop, pred in zip(proposals, target_argmax):
        if prop != pred:
            break
        accepted += 1
        if prop in eos_ids:
            return Decision(proposals[:accepted], accepted, accepted, None, True)
    correction = target_argmax[accepted]
    finished = correction in eos_ids
    return Decision(proposals[:accepted] + (correction,), accepted, accepted + 1,
                    None if finished else correction, finished)


@dataclass(frozen=True)
class BlockTicket:
    request_id: str
    epoch: int
    position: int
    tokens: tuple
    source: str
    match_length: int = 0


class GreedySession:
    """Host coordinator of one request's blocks.  Device work is done by callbacks:
    ``commit(..., publish)`` calls ``publish(state_rows)`` which must synchronise the target and
    drafter state and return None; ``abort(..., restore)`` calls ``restore(0)``."""

    def __init__(self, request_id, prompt, seed, *, vocab_size, max_new_tokens, eos_ids=(), drafter=None,
                 verifier_rows=16):
        if type(max_new_tokens) is not int or max_new_tokens < 1:
            raise ValueError("positive generation budget required")
        if verifier_rows not in BUCKETS[1:]:
            raise ValueError("verifier_rows must be a bucket of at least 2")
        prompt, eos_ids = tuple(prompt), tuple(eos_ids)
        select_prefix((), (seed,), vocab_size=vocab_size, eos_ids=eos_ids, max_proposals=verifier_rows - 1)
        self.request_id, self.vocab_size = request_id, vocab_size
        self.max_new_tokens, self.eos_ids, self.verifier_rows = max_new_tokens, eos_ids, verifier_rows
        self.drafter = drafter
        if drafter is not None:
            drafter.commit_verified(request_id, (seed,))
        self.position, self.seed = len(prompt), seed
        self.emitted = [seed]
        self.finished = seed in eos_ids or max_new_tokens == 1
        self.phase, self.epoch, self.pending = "idle", 0, None
        self.committed_block_proposals = self.accepted_proposals = self.committed_blocks = 0
        self.committed_decode_tokens = self.aborted_blocks = 0

    def check_owner(self, request_id):
        if request_id != self.request_id or self.phase in ("failed", "closed"):
            raise ValueError("closed, failed or mismatched request")

    def propose(self, request_id, *, max_rows=None, selected=None):
        self.check_owner(request_id)
        if self.phase != "idle" or self.finished:
            raise ValueError("an unfinished idle request is required")
        max_rows = self.verifier_rows if max_rows is None else max_rows
        if max_rows not in BUCKETS or max_rows > self.verifier_rows:
            raise ValueError("supported verifier bucket required")
        remaining = self.max_new_tokens - len(self.emitted)
        limit = min(max_rows, remaining)
        self.phase = "drafting"
        try:
            if limit > 1 and self.drafter is not None:
                proposal = self.drafter.propose(request_id, limit - 1, selected=selected)
            else:
                proposal = None
        except BaseException:
            self.phase = "failed"
            raise
        tokens = () if proposal is None else tuple(proposal.tokens)
        rows = max(w for w in BUCKETS if w <= min(limit, len(tokens) + 1))
        self.epoch += 1
        ticket = BlockTicket(request_id, self.epoch, self.position, (self.seed, *tokens[:rows - 1]),
                             proposal.source if rows > 1 else "target",
                             proposal.match_length if rows > 1 else 0)
        self.pending, self.phase = ticket, "pending"
        return ticket

    def check_ticket(self, request_id, ticket):
        self.check_owner(request_id)
        if self.phase != "pending" or ticket is not self.pending:
            raise ValueError("the current live block ticket is required")

    def narrow(self, request_id, ticket, rows):
        """Replace the live ticket by its first ``rows`` tokens (a smaller bucket) under a new
        epoch; nothing was verified for it, so this is host-only."""
        self.check_ticket(request_id, ticket)
        if rows not in BUCKETS or rows > len(ticket.tokens):
            raise ValueError("a bucket no wider than the live ticket is required")
        self.epoch += 1
        t = BlockTicket(request_id, self.epoch, ticket.position, tuple(ticket.tokens[:rows]),
                        ticket.source if rows > 1 else "target", min(ticket.match_length, rows - 1) if rows > 1 else 0)
        self.pending = t
        return t

    def commit(self, request_id, ticket, predictions, publish, *, max_rows=None) -> Decision:
        self.check_ticket(request_id, ticket)
        if not callable(publish):
            raise ValueError("state publication callback required")
        proposals, targets = ticket.tokens[1:], tuple(predictions)
        if max_rows is not None:
            if type(max_rows) is not int or not 1 <= max_rows <= len(ticket.tokens):
                raise ValueError("commit cap outside the ticket")
            proposals, targets = ticket.tokens[1:max_rows], targets[:max_rows]
        decision = select_prefix(proposals, targets, vocab_size=self.vocab_size, eos_ids=self.eos_ids,
                                 max_proposals=self.verifier_rows - 1)
        self.phase = "committing"
        try:
            if publish(decision.state_rows) is not None:
                raise RuntimeError("publication must return None after synchronising")
            if self.drafter is not None:
                self.drafter.commit_verified(request_id, decision.emitted)
        except BaseException:
            self.phase = "failed"
            raise
        self.position += decision.state_rows
        self.seed = decision.next_input
        self.emitted.extend(decision.emitted)
        self.committed_block_proposals += len(ticket.tokens) - 1
        self.accepted_proposals += decision.accepted
        self.committed_blocks += 1
        self.committed_decode_tokens += len(decision.emitted)
        self.finished = decision.finished or len(self.emitted) >= self.max_new_tokens
        self.pending, self.phase = None, "idle"
        return decision

    def abort(self, request_id, ticket, restore):
        self.check_ticket(request_id, ticket)
        if not callable(restore):
            raise ValueError("entry-state restore callback required")
        self.phase = "committing"
        try:
            if restore(0) is not None:
                raise RuntimeError("abort must return None after synchronising")
        except BaseException:
            self.phase = "failed"
            raise
        self.aborted_blocks += 1
        self.pending, self.phase = None, "idle"

    def fail_verification(self, request_id, ticket):
        self.check_ticket(request_id, ticket)
        self.phase = "failed"

    def close(self, request_id):
        if request_id != self.request_id or self.phase not in ("idle", "failed"):
            raise ValueError("finish or abort the block before closing")
        if self.drafter is not None:
            self.drafter.close(request_id)
        self.seed, self.pending, self.phase = None, None, "closed"
