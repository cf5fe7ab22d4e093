"""Multi-request serving engine: continuous batching of speculative blocks.

Each admitted request owns a target sequence (paged KV blocks + a GDN state slot), a drafter
history slot and a ``GreedySession``.  One ``step()`` either prefills (a chunk of) one request or
runs one speculative block for every running request: each drafter proposes, the target
verifies all requests' rows in one packed forward (weights read once), and every session commits
its own accepted prefix (``scripts/ci/serving_packed_step.py:1-15``).

Failures are quarantined per request (``scripts/ci/serving_request_quarantine.py:1-60``): an
exception while serving one request aborts that request (state ``aborted``, resources released)
and the engine keeps serving the others.
"""
from __future__ import annotations

import itertools
import time

import torch

from ..spec.greedy import GreedySession
from ..spec.lookup import HybridDraft
from .scheduler import ABORTED, FINISHED, DecodeStep, PrefillStep, Request, Scheduler


class ServingEngine:
    def __init__(self, target, drafter=None, *, verifier_rows: int = 16, max_running: int | None = None,
                 prefill_chunk: int | None = None, max_step_rows: int | None = None, prefix=None,
                 lookup: bool = False, clock=time.perf_counter, speculate_sampled: bool = True):
        self.target, self.drafter, self.prefix = target, drafter, prefix
        # Sampled requests speculate too: the Gumbel noise of a position depends only on (seed,
        # position), so the sampled token of every verified row is a fixed function of its prefix and
        # the greedy acceptance rule applied to sampled tokens reproduces one-token-per-step sampling
        # exactly.  False: sampled requests decode one token per step.
        self.speculate_sampled = speculate_sampled
        self.verifier_rows, self.lookup, self.clock = verifier_rows, lookup, clock
        slots = target.max_slots if drafter is None else min(target.max_slots, drafter.slots)
        self.max_running = max_running or slots
        if self.max_running > slots:
            raise ValueError("more running requests than target/drafter slots")
        # a packed verify stays within the rows the target's kernels keep batch-invariant; more
        # running requests than that are served in rotation
        step_rows = max_step_rows or self.max_running * verifier_rows
        pack = getattr(target, "max_pack_rows", None)
        if pack:
            step_rows = min(step_rows, max(pack, verifier_rows))
        self.sched = Scheduler(self.max_running, prefill_chunk or target.rt.prefill_chunk, step_rows, verifier_rows)
        self.taps = tuple(drafter.dcfg.taps) if drafter is not None else ()
        self.free_dslots = list(range(slots - 1, -1, -1))
        self.requests: dict = {}
        self._ids = itertools.count()
        self._anchor = torch.zeros(1, dtype=torch.long, device=target.device)
        self.steps = {"prefill": 0, "decode": 0}
        self.quarantined = 0

    # ------------------------------------------------------------------ API
    def add_request(self, prompt, max_new_tokens: int, *, eos_ids=(), request_id=None, pinned=None,
                    temperature: float = 0.0, seed: int = 0) -> Request:
        prompt = [int(t) for t in prompt]
        if not prompt:
            raise ValueError("empty prompt")
        if any(not 0 <= t < self.target.cfg.vocab_size for t in prompt):
            raise ValueError("token outside the vocabulary")
        if int(max_new_tokens) < 1:
            raise ValueError("max_new_tokens must be >= 1")
        if len(prompt) + max_new_tokens + self.verifier_rows > self.target.rt.max_context:
            raise ValueError("prompt + budget exceed max_context")
        rid = request_id or f"req-{next(self._ids)}"
        if rid in self.requests and self.requests[rid].state not in (FINISHED, ABORTED):
            raise ValueError(f"request id {rid!r} is already in flight")
        if temperature < 0:
            raise ValueError("temperature must be >= 0")
        req = Request(rid, prompt, max_new_tokens, tuple(eos_ids), self.clock(), pinned,
                      temperature=float(temperature), seed=int(seed))
        self.requests[rid] = req
        self.sched.add(req)
        return req

    def complete(self, request_id: str):
        """End a request now as finished (a stop string appeared in its output): its sequence and
        drafter slot are released, its output is kept."""
        req = self.requests[request_id]
        if req.state in (FINISHED, ABORTED):
            return
        req.t_done = self.clock()
        self._release(req)
        self.sched.finish(req, FINISHED)

    def abort(self, request_id: str, reason: str = "aborted by caller"):
        req = self.requests[request_id]
        self._quarantine(req, reason)

    def has_work(self) -> bool:
        return self.sched.has_work()

    def step(self):
        """One scheduler step.  Returns the requests that finished or aborted in it."""
        step = self.sched.schedule(self._can_admit)
        if step is None:
            return []
        if isinstance(step, PrefillStep):
            self.steps["prefill"] += 1
            return self._prefill(step)
        self.steps["decode"] += 1
        return self._decode(step)

    def run(self, max_steps: int = 1 << 30):
        done = []
        for _ in range(max_steps):
            if not self.has_work():
                break
            done.extend(self.step())
        return done

    # ------------------------------------------------------------------ internals
    def _can_admit(self, req) -> bool:
        if not self.free_dslots and self.drafter is not None:
            return False
        if not self.target.free_slots:
            return False
        need = -(-(len(req.prompt) + req.max_new_tokens + self.verifier_rows) // self.target.block_size)
        return self.target.allocator.num_free >= need

    def _release(self, req):
        if req.seq is not None:
            self.target.release(req.seq)
            req.seq = None
        if req.dslot >= 0:
            self.free_dslots.append(req.dslot)
            req.dslot = -1

    def _quarantine(self, req, err):
        req.error = str(err)
        req.t_done = self.clock()
        self.quarantined += 1
        self._release(req)
        self.sched.finish(req, ABORTED)

    def _prefill(self, st: PrefillStep):
        req = st.request
        tgt, dr = self.target, self.drafter
        try:
            if req.seq is None:
                ck = self.prefix.lookup(req.prompt) if self.prefix is not None else None
                if dr is not None:
                    req.dslot = self.free_dslots.pop()
                    dr.reset(req.dslot)
                if ck is not None:
                    self.prefix.pin(ck)
                    try:
                        req.seq = self.prefix.restore(ck, dr, req.dslot)
                    finally:
                        self.prefix.unpin(ck)
                    req.prefilled = req.reused_prefix = ck.pos
                    return []          # the next step continues the prefill from the checkpoint
                req.seq = tgt.new_sequence()
            end = st.end
            if self.prefix is not None:       # stop at checkpoint boundaries
                b = self.prefix.boundary
                nb = (req.prefilled // b + 1) * b
                if nb < end:
                    end = nb
            toks = torch.tensor(req.prompt[req.prefilled:end], dtype=torch.long, device=tgt.device)
            samp = (tgt.sampling_args(req.temperature, req.seed, [len(req.prompt)])
                    if req.temperature > 0 and end == len(req.prompt) else None)
            nxt, feats = tgt.prefill(req.seq, toks, taps=self.taps, sampling=samp)
            if dr is not None:
                succ = (req.prompt[req.prefilled + 1:end + 1] if end < len(req.prompt)
                        else req.prompt[req.prefilled + 1:] + [int(nxt.item())])
                dr.append(feats, req.prefilled, req.dslot, next_tokens=succ)
            req.prefilled = end
            if self.prefix is not None and end % self.prefix.boundary == 0 and end < len(req.prompt):
                self.prefix.capture(req.seq, req.prompt, dr, req.dslot)
            if end < len(req.prompt):
                return []
            seed = int(nxt.item())
            req.t_first = self.clock()
            neural = {"dspark": self._adapter(req)} if dr is not None else None
            hd = HybridDraft(req.request_id, req.prompt, vocab_size=tgt.cfg.vocab_size, neural=neural,
                             lookup_enabled=self.lookup, max_proposals=self.verifier_rows - 1)
            req.session = GreedySession(req.request_id, req.prompt, seed, vocab_size=tgt.cfg.vocab_size,
                                        max_new_tokens=req.max_new_tokens, eos_ids=req.eos_ids, drafter=hd,
                                        verifier_rows=self.verifier_rows)
            if req.session.finished:
                req.t_done = self.clock()
                self._release(req)
                self.sched.prefilling = None
                self.sched.finish(req, FINISHED)
                return [req]
            self.sched.prefill_done(req)
            return []
        except Exception as e:          # quarantine this request only
            self._quarantine(req, e)
            return [req]

    def _adapter(self, req):
        def adapter(request_id, history, count):
            self._anchor.fill_(history[-1])
            props = self.drafter.propose(self._anchor, req.dslot)
            if req.pinned is not None:
                return tuple(req.pinned.apply(len(req.session.emitted), count, self.target.cfg.vocab_size))
            return tuple(int(t) for t in props[:count].tolist())
        return adapter

    def _decode(self, st: DecodeStep):
        tgt, dr = self.target, self.drafter
        t0 = self.clock()
        live, finished = [], []
        for req in st.requests:
            try:
                one = req.temperature > 0 and not self.speculate_sampled
                req.ticket = (req.session.propose(req.request_id, max_rows=1) if one
                              else req.session.propose(req.request_id))
                live.append(req)
            except Exception as e:
                self._quarantine(req, e)
                finished.append(req)
        if not live:
            return finished
        batch = [(r.seq, torch.tensor(r.ticket.tokens, dtype=torch.long, device=tgt.device)) for r in live]
        sampling = None
        if any(r.temperature > 0 for r in live):
            scales, keys = [], []
            for r in live:
                n = len(r.ticket.tokens)
                sc, ky = tgt.sampling_args(r.temperature, r.seed, range(r.seq.pos + 1, r.seq.pos + 1 + n))
                scales.append(sc)
                keys.append(ky)
            sampling = (torch.cat(scales), torch.cat(keys))
        try:
            pred, feats = tgt.verify(batch, taps=self.taps, sampling=sampling)
            preds = pred.tolist()
        except Exception as e:          # a failed packed verify poisons every member's block
            for r in live:
                r.session.fail_verification(r.request_id, r.ticket)
                self._quarantine(r, e)
            return finished + live
        for r in live:
            o0, n = r.seq.verify_rows
            rows = feats[o0:o0 + n] if feats is not None else None
            pos = r.seq.pos

            def publish(k, r=r, rows=rows, pos=pos, pr=preds[o0:o0 + n]):
                tgt.commit(r.seq, k)
                if dr is not None:
                    nxt = list(r.ticket.tokens[1:k]) + [pr[k - 1]]
                    dr.append(rows[:k], pos, r.dslot, next_tokens=nxt)

            try:
                d = r.session.commit(r.request_id, r.ticket, preds[o0:o0 + n], publish)
            except Exception as e:
                self._quarantine(r, e)
                finished.append(r)
                continue
            r.blocks.append({"rows": n, "accepted": int(d.accepted), "committed": len(d.emitted)})
            if r.session.finished:
                r.t_done = self.clock()
                self._release(r)
                self.sched.finish(r, FINISHED)
                finished.append(r)
        dt = self.clock() - t0
        for r in live:
            r.decode_time += dt
        return finished
