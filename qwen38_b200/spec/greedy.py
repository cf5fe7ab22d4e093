"""Greedy block verification: the acceptance rule and the request-scoped block protocol.

The rule (it defines what "token-exact speculation" means, so it matches the reference's
``speculative-decoding/harness/greedy_verify.py:15-37``): a block's rows hold
``[seed, d1, ..., dk]`` at the committed position and row i's target argmax ``t_i`` is the target's
next token after row i.  Drafts are accepted while ``d_{i+1} == t_i``; the emitted tokens are the
accepted drafts followed by the target's correction ``t_a`` (a = accepted count), and ``a + 1`` rows
of state are published.  An accepted draft that is an end-of-sequence id ends the block (and the
request) right there, and so does a correction that is one.

The protocol object here is this runtime's own design around that rule (the reference's session is
``greedy_session.py:19-173``): an explicit transition table over ``Phase``, tickets numbered by an
epoch so that only the live one can be verified, published or aborted, counters kept in one
``BlockCounters`` record, and every device-facing callback run under one guard that poisons the
session (``Phase.FAILED``) when it raises.  ``accepted_length`` also takes device tensors, so the
selection can run on the GPU (``device_accept``) without reading the predictions back first.

Verifier widths are powers of two from 1 to 32 (``BUCKETS``), capped by the session's
``verifier_rows`` (16 in the benchmark, 4 in the tiny CPU configuration).
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass
from enum import Enum

BUCKETS = (1, 2, 4, 8, 16, 32)
MAX_ROWS = BUCKETS[-1]


def bucket_at_most(n: int) -> int:
    """Largest verifier width not above ``n`` (``n`` >= 1)."""
    if n < 1:
        raise ValueError("a verifier block has at least one row")
    return min(MAX_ROWS, 1 << (int(n).bit_length() - 1))


def accepted_length(drafts, predictions):
    """How many leading drafts equal the predictions of the rows before them.  Host sequences give
    an int; 1-D tensors give a 0-d tensor on their device (no read-back)."""
    if hasattr(drafts, "device") and hasattr(predictions, "device"):
        k = drafts.shape[0]
        if k == 0:
            return predictions.new_zeros(())
        same = (drafts == predictions[:k]).to(predictions.dtype)
        return same.cumprod(0).sum()
    n = 0
    for d, p in zip(drafts, predictions):
        if d != p:
            break
        n += 1
    return n


def device_accept(block_tokens, predictions):
    """Device-side selection for a verified block: ``block_tokens`` [rows] = (seed, drafts...),
    ``predictions`` [rows] = row argmaxes.  Returns (rows to publish [1] int32, next seed [1] int64),
    both on the device, with no end-of-sequence handling (benchmark and serving steps without
    EOS ids).  ``Decision`` from ``select_prefix`` is the host-side equivalent."""
    import torch
    a = accepted_length(block_tokens[1:], predictions)
    return (a + 1).to(torch.int32).reshape(1), predictions.index_select(0, a.reshape(1).long())


@dataclass(frozen=True)
class Decision:
    emitted: tuple          # accepted drafts then the correction (or up to an accepted EOS)
    accepted: int           # drafts accepted
    state_rows: int         # rows of state to publish
    next_input: int | None  # seed of the next block (None when the request ended)
    finished: bool          # an end-of-sequence id was emitted


def _check_ids(tokens, vocab_size, what):
    for t in tokens:
        if type(t) is not int or t < 0 or t >= vocab_size:
            raise ValueError(f"{what}: id {t!r} is not in [0, {vocab_size})")


def select_prefix(proposals, target_argmax, *, vocab_size, eos_ids=(), max_proposals=15) -> Decision:
    """Apply the acceptance rule to one verified block (``target_argmax`` has one row more than
    ``proposals``: the seed's row)."""
    if type(vocab_size) is not int or vocab_size <= 0:
        raise ValueError("vocab_size must be a positive int")
    if type(max_proposals) is not int or max_proposals < 1 or max_proposals + 1 not in BUCKETS:
        raise ValueError("max_proposals must be a verifier width minus one (1, 3, 7, 15 or 31)")
    drafts, preds, eos = tuple(proposals), tuple(target_argmax), frozenset(eos_ids)
    if len(drafts) > max_proposals:
        raise ValueError(f"{len(drafts)} drafts exceed the capacity of {max_proposals}")
    if len(preds) != len(drafts) + 1:
        raise ValueError("one prediction per block row is required (drafts + 1)")
    _check_ids(drafts, vocab_size, "draft")
    _check_ids(preds, vocab_size, "prediction")
    _check_ids(tuple(eos_ids), vocab_size, "end-of-sequence")
    a = accepted_length(drafts, preds)
    for i in range(a):
        if drafts[i] in eos:                       # accepted end-of-sequence: nothing after it
            return Decision(drafts[:i + 1], i + 1, i + 1, None, True)
    fix = preds[a]
    done = fix in eos
    return Decision(drafts[:a] + (fix,), a, a + 1, None if done else fix, done)


@dataclass(frozen=True)
class BlockTicket:
    request_id: str
    epoch: int              # the session's ticket counter when issued; only the live one is valid
    position: int           # committed length the block starts at
    tokens: tuple           # (seed, drafts...)
    source: str             # "target", "lookup" or a neural adapter's name
    match_length: int = 0   # lookup suffix match behind the drafts


class Phase(str, Enum):
    IDLE = "idle"
    DRAFTING = "drafting"
    PENDING = "pending"
    COMMITTING = "committing"
    FAILED = "failed"
    CLOSED = "closed"


_NEXT = {
    Phase.IDLE: {Phase.DRAFTING, Phase.CLOSED},
    Phase.DRAFTING: {Phase.PENDING, Phase.FAILED},
    Phase.PENDING: {Phase.PENDING, Phase.COMMITTING, Phase.FAILED},
    Phase.COMMITTING: {Phase.IDLE, Phase.FAILED},
    Phase.FAILED: {Phase.CLOSED},
    Phase.CLOSED: set(),
}


@dataclass
class BlockCounters:
    proposed: int = 0       # drafts in committed blocks
    accepted: int = 0       # drafts accepted
    blocks: int = 0         # committed blocks
    decode_tokens: int = 0  # emitted after the prefill seed
    aborted: int = 0        # blocks dropped by abort


class GreedySession:
    """Host coordinator of one request's blocks.  The device work happens in callbacks:
    ``commit(..., publish)`` calls ``publish(state_rows)``, which must leave target and drafter
    state published and return None; ``abort(..., restore)`` calls ``restore(0)``, which must
    restore the block's entry state and return None.  Any exception inside drafting or a callback
    poisons the session."""

    def __init__(self, request_id, prompt, seed, *, vocab_size, max_new_tokens, eos_ids=(), drafter=None,
                 verifier_rows=16):
        if type(max_new_tokens) is not int or max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be a positive int")
        if verifier_rows not in BUCKETS or verifier_rows < 2:
            raise ValueError("verifier_rows must be a verifier width of 2 or more")
        if type(vocab_size) is not int or vocab_size <= 0:
            raise ValueError("vocab_size must be a positive int")
        _check_ids((seed,), vocab_size, "seed")
        _check_ids(tuple(eos_ids), vocab_size, "end-of-sequence")
        self.request_id, self.prompt, self.seed = request_id, tuple(prompt), seed
        self.vocab_size, self.max_new_tokens = vocab_size, max_new_tokens
        self.eos_ids, self.drafter, self.verifier_rows = tuple(eos_ids), drafter, verifier_rows
        self.counters = BlockCounters()
        self.position = len(self.prompt)
        self.emitted = [seed]
        self.finished = seed in self.eos_ids or max_new_tokens == 1
        self.phase, self.epoch, self.pending = Phase.IDLE, 0, None
        if drafter is not None:
            drafter.commit_verified(request_id, (seed,))

    # ------------------------------------------------------------------ counters (read-only view)
    committed_block_proposals = property(lambda s: s.counters.proposed)
    accepted_proposals = property(lambda s: s.counters.accepted)
    committed_blocks = property(lambda s: s.counters.blocks)
    committed_decode_tokens = property(lambda s: s.counters.decode_tokens)
    aborted_blocks = property(lambda s: s.counters.aborted)

    # ------------------------------------------------------------------ guards
    def _move(self, to: Phase):
        if to not in _NEXT[self.phase]:
            raise ValueError(f"request {self.request_id}: cannot go from {self.phase.value} to {to.value}")
        self.phase = to

    @contextlib.contextmanager
    def _poison_on_error(self):
        try:
            yield
        except BaseException:
            self.phase = Phase.FAILED
            raise

    def check_owner(self, request_id):
        if request_id != self.request_id:
            raise ValueError(f"ticket for {request_id!r} presented to request {self.request_id!r}")
        if self.phase in (Phase.FAILED, Phase.CLOSED):
            raise ValueError(f"request {self.request_id} is {self.phase.value}")

    def check_ticket(self, request_id, ticket):
        self.check_owner(request_id)
        if self.phase is not Phase.PENDING or ticket is not self.pending:
            raise ValueError("only the live block ticket can be verified, published or aborted")

    def _issue(self, tokens, source, match_length):
        self.epoch += 1
        self.pending = BlockTicket(self.request_id, self.epoch, self.position, tuple(tokens),
                                   source if len(tokens) > 1 else "target",
                                   min(match_length, len(tokens) - 1) if len(tokens) > 1 else 0)
        return self.pending

    # ------------------------------------------------------------------ protocol
    def propose(self, request_id, *, max_rows=None, selected=None):
        """Draft the next block and return its ticket (the widest bucket the drafts, the budget and
        ``max_rows`` allow)."""
        self.check_owner(request_id)
        if self.finished:
            raise ValueError(f"request {self.request_id} has finished")
        width = self.verifier_rows if max_rows is None else max_rows
        if width not in BUCKETS or width > self.verifier_rows:
            raise ValueError(f"max_rows {width} is not a verifier width up to {self.verifier_rows}")
        cap = min(width, self.max_new_tokens - len(self.emitted))
        self._move(Phase.DRAFTING)
        proposal = None
        with self._poison_on_error():
            if cap > 1 and self.drafter is not None:
                proposal = self.drafter.propose(request_id, cap - 1, selected=selected)
        drafts = tuple(proposal.tokens) if proposal is not None else ()
        rows = bucket_at_most(min(cap, len(drafts) + 1))
        ticket = self._issue((self.seed,) + drafts[:rows - 1], proposal.source if proposal else "target",
                             proposal.match_length if proposal else 0)
        self._move(Phase.PENDING)
        return ticket

    def narrow(self, request_id, ticket, rows):
        """Re-issue the live ticket cut to its first ``rows`` tokens (a smaller bucket) under a new
        epoch; nothing was verified for it yet, so no device state is involved."""
        self.check_ticket(request_id, ticket)
        if rows not in BUCKETS or rows > len(ticket.tokens):
            raise ValueError(f"cannot narrow a {len(ticket.tokens)}-row ticket to {rows} rows")
        out = self._issue(ticket.tokens[:rows], ticket.source, ticket.match_length)
        self._move(Phase.PENDING)
        return out

    def commit(self, request_id, ticket, predictions, publish, *, max_rows=None) -> Decision:
        """Select the accepted prefix of the verified live ticket, publish its state through
        ``publish(state_rows)`` and advance the request."""
        self.check_ticket(request_id, ticket)
        if not callable(publish):
            raise ValueError("commit needs a publication callback")
        rows = len(ticket.tokens) if max_rows is None else max_rows
        if type(rows) is not int or not 1 <= rows <= len(ticket.tokens):
            raise ValueError(f"commit cap {max_rows!r} is outside the {len(ticket.tokens)}-row ticket")
        d = select_prefix(ticket.tokens[1:rows], tuple(predictions)[:rows], vocab_size=self.vocab_size,
                          eos_ids=self.eos_ids, max_proposals=self.verifier_rows - 1)
        self._move(Phase.COMMITTING)
        with self._poison_on_error():
            if publish(d.state_rows) is not None:
                raise RuntimeError("the publication callback must return None once state is published")
            if self.drafter is not None:
                self.drafter.commit_verified(request_id, d.emitted)
        c = self.counters
        c.proposed += len(ticket.tokens) - 1
        c.accepted += d.accepted
        c.blocks += 1
        c.decode_tokens += len(d.emitted)
        self.position += d.state_rows
        self.seed = d.next_input
        self.emitted += d.emitted
        self.finished = d.finished or len(self.emitted) >= self.max_new_tokens
        self.pending = None
        self._move(Phase.IDLE)
        return d

    def abort(self, request_id, ticket, restore):
        """Drop the live ticket; ``restore(0)`` puts back the block's entry state."""
        self.check_ticket(request_id, ticket)
        if not callable(restore):
            raise ValueError("abort needs an entry-state restore callback")
        self._move(Phase.COMMITTING)
        with self._poison_on_error():
            if restore(0) is not None:
                raise RuntimeError("the restore callback must return None once state is restored")
        self.counters.aborted += 1
        self.pending = None
        self._move(Phase.IDLE)

    def fail_verification(self, request_id, ticket):
        """The live ticket's verification raised: nothing is published, the request is poisoned."""
        self.check_ticket(request_id, ticket)
        self._move(Phase.FAILED)

    def close(self, request_id):
        if request_id != self.request_id:
            raise ValueError(f"request {self.request_id} cannot be closed as {request_id!r}")
        if self.phase not in (Phase.IDLE, Phase.FAILED):
            raise ValueError(f"request {self.request_id} is {self.phase.value}: finish or abort the block first")
        if self.drafter is not None:
            self.drafter.close(request_id)
        self.seed, self.pending = None, None
        self._move(Phase.CLOSED)
