"""Step scheduler for the serving engine.

Policy of the reference's TT scheduler (``scripts/ci/fixtures/plugin_scheduler.py:4-180``,
``platform_chunked_prefill_policy.py``): a step is either prefill work or decode work, never both
(no mixed batches); a request whose prompt is longer than one chunk continues its prefill on the
following steps; prefill goes first while a request waits and a slot is free, otherwise every
running request takes one speculative block in a single packed verify
(``scripts/ci/packed_verifier.py:1-12``).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field


WAITING, PREFILL, RUNNING, FINISHED, ABORTED = "waiting", "prefill", "running", "finished", "aborted"


@dataclass
class Request:
    request_id: str
    prompt: list
    max_new_tokens: int
    eos_ids: tuple = ()
    arrival: float = 0.0
    pinned: object = None               # PinnedAcceptance or None
    state: str = WAITING
    prefilled: int = 0                  # prompt tokens already prefilled
    seq: object = None                  # target SeqState
    dslot: int = -1                     # drafter history slot
    session: object = None              # GreedySession
    ticket: object = None
    error: str | None = None
    t_first: float | None = None        # first output token (host time)
    t_done: float | None = None
    decode_time: float = 0.0            # generation-loop time attributed to this request
    reused_prefix: int = 0
    temperature: float = 0.0            # > 0: sampled (Gumbel-max keyed by seed and position)
    seed: int = 0                       # sampling noise seed
    blocks: list = field(default_factory=list)   # per verified block: {rows, accepted, committed}

    @property
    def output(self):
        return list(self.session.emitted) if self.session is not None else []


@dataclass
class PrefillStep:
    request: Request
    start: int
    end: int


@dataclass
class DecodeStep:
    requests: list


class Scheduler:
    def __init__(self, max_running: int, prefill_chunk: int, max_step_rows: int, verifier_rows: int):
        if max_running < 1 or prefill_chunk < 1 or max_step_rows < verifier_rows:
            raise ValueError("bad scheduler limits")
        self.max_running, self.prefill_chunk = max_running, prefill_chunk
        self.max_step_rows, self.verifier_rows = max_step_rows, verifier_rows
        self.waiting: deque = deque()
        self.running: list = []
        self.prefilling: Request | None = None

    def add(self, req: Request):
        self.waiting.append(req)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running or self.prefilling)

    def schedule(self, can_admit) -> PrefillStep | DecodeStep | None:
        """``can_admit(req)`` says whether resources (slots, KV blocks) exist for a new request."""
        if self.prefilling is not None:
            r = self.prefilling
            return PrefillStep(r, r.prefilled, min(len(r.prompt), r.prefilled + self.prefill_chunk))
        if self.waiting and len(self.running) < self.max_running and can_admit(self.waiting[0]):
            r = self.waiting.popleft()
            r.state = PREFILL
            self.prefilling = r
            return PrefillStep(r, r.prefilled, min(len(r.prompt), r.prefilled + self.prefill_chunk))
        if self.running:
            per = self.verifier_rows
            n = max(1, min(len(self.running), self.max_step_rows // per))
            batch = self.running[:n]
            # rotate so every request is served when the row budget is smaller than the set
            self.running = self.running[n:] + batch
            return DecodeStep(batch)
        return None

    def prefill_done(self, req: Request):
        self.prefilling = None
        req.state = RUNNING
        self.running.append(req)

    def finish(self, req: Request, state: str = FINISHED):
        req.state = state
        if self.prefilling is req:
            self.prefilling = None
        if req in self.running:
            self.running.remove(req)
        try:
            self.waiting.remove(req)
        except ValueError:
            pass
