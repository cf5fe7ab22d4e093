"""Speculative request runtime: drafter + target + greedy session, and the request driver.

One request = prefill (PP timer) then blocks of propose -> verify -> select -> commit/publish
(TG timer) until the budget or EOS, as in the reference's ``measure_request``
(``scripts/ci/full_request.py:36-241``): PP = prompt tokens / prefill seconds; TG = committed
decode tokens (the prefill seed excluded) / generation-loop seconds; the loop includes drafting,
verification, selection, commit and read-back.

Pinned acceptance (benchmark configuration): the drafter runs its full forward every block, then
its proposals are overwritten with the target's own greedy continuation corrupted at a seeded
per-block point, so every build does identical verify work.  The greedy gold continuation comes
from plain single-row decode of the same engine (untimed), and the speculative output is checked
token-exact against it.
"""
from __future__ import annotations

import random
import time
from dataclasses import dataclass, field

import torch

from ..utils.trace import nvtx, token_digest
from .greedy import GreedySession
from .lookup import HybridDraft, Proposal


@dataclass
class PinnedAcceptance:
    """Overwrites proposals with ``gold`` continued from the block's seed, corrupted at an offset
    drawn uniformly from ``[0, 2*mean_accepted]`` (mean ``mean_accepted``)."""
    gold: list
    seed: int = 0
    mean_accepted: int = 6
    rng: random.Random = field(init=False)

    def __post_init__(self):
        self.rng = random.Random(self.seed)

    def apply(self, emitted_len: int, count: int, vocab: int):
        start = emitted_len          # gold[emitted_len - 1] is the seed; proposals follow it
        props = list(self.gold[start:start + count])
        while len(props) < count:
            props.append(0)
        cut = self.rng.randint(0, 2 * self.mean_accepted)
        if cut < count:
            props[cut] = (props[cut] + 1) % vocab
        return props


class NeuralAdapter:
    """Callable adapter the session's HybridDraft invokes: runs the drafter on the device and
    (optionally) applies pinned acceptance."""

    def __init__(self, runtime: "SpecRuntime"):
        self.rt = runtime

    def __call__(self, request_id, history, count):
        rt = self.rt
        anchor = rt._anchor_dev
        anchor.fill_(history[-1])
        props = rt.drafter.propose(anchor)                 # device work, every block
        if rt.pinned is not None:
            rt.d2h_bytes += 0
            return tuple(rt.pinned.apply(len(rt.session.emitted), count, rt.target.cfg.vocab_size))
        host = props[:count].tolist()
        rt.d2h_bytes += 8 * len(host)
        return tuple(int(t) for t in host)


class SpecRuntime:
    def __init__(self, target, drafter=None, *, verifier_rows: int = 16, lookup: bool = False, prefix=None):
        self.target, self.drafter = target, drafter
        self.prefix = prefix                       # optional PrefixRegistry
        self.verifier_rows = verifier_rows
        self.lookup = lookup
        self.taps = tuple(drafter.dcfg.taps) if drafter is not None else ()
        self._anchor_dev = torch.zeros(1, dtype=torch.long, device=target.device)
        self.pinned = None
        self._sampling = None
        self.session = self.last_session = None
        self.h2d_bytes = self.d2h_bytes = 0

    # ------------------------------------------------------------------------------ timing
    def _event(self):
        if self.target.device.type == "cuda":
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            return e
        return time.perf_counter()

    def _elapsed_ms(self, a, b):
        if self.target.device.type == "cuda":
            b.synchronize()
            return a.elapsed_time(b)
        return (b - a) * 1e3

    # ------------------------------------------------------------------------------ request
    @torch.no_grad()
    def generate(self, prompt, max_new_tokens: int, *, request_id="req", eos_ids=(), pinned=None,
                 gold_check=None, prompt_host=None, temperature: float = 0.0, seed: int = 0):
        """Runs one request.  ``prompt``: list/1-D tensor of ids.  Returns a result dict with the
        emitted tokens and PP/TG figures.  ``temperature`` > 0 samples (Gumbel-max keyed by seed
        and position, so block speculation reproduces ``HybridTarget.sample`` exactly)."""
        tgt = self.target
        self._sampling = (float(temperature), int(seed)) if temperature > 0 else None
        self.pinned = pinned
        if prompt_host is None:
            prompt_host = torch.as_tensor(list(prompt) if not torch.is_tensor(prompt) else prompt.cpu(),
                                          dtype=torch.long)
            if tgt.device.type == "cuda":
                prompt_host = prompt_host.pin_memory()
        seq = None
        ck = None
        try:
            t0 = self._event()
            prompt_dev = prompt_host.to(tgt.device, non_blocking=True)
            self.h2d_bytes += prompt_host.numel() * 8
            with nvtx("prefill"):
                seq, nxt, ck = self._prefill(prompt_host, prompt_dev)
            seed = int(nxt.item())
            self.d2h_bytes += 8
            t1 = self._event()
            pp_ms = self._elapsed_ms(t0, t1)
            neural = {"dspark": NeuralAdapter(self)} if self.drafter is not None else None
            drafter = HybridDraft(request_id, [int(t) for t in prompt_host.tolist()],
                                  vocab_size=tgt.cfg.vocab_size, neural=neural, lookup_enabled=self.lookup,
                                  max_proposals=self.verifier_rows - 1)
            s = GreedySession(request_id, prompt_host.tolist(), seed, vocab_size=tgt.cfg.vocab_size,
                              max_new_tokens=max_new_tokens, eos_ids=eos_ids, drafter=drafter,
                              verifier_rows=self.verifier_rows)
            self.session = self.last_session = s
            blocks = []
            tok_host = torch.zeros(self.verifier_rows, dtype=torch.long)
            if tgt.device.type == "cuda":
                tok_host = tok_host.pin_memory()
            t2 = self._event()
            marks = []                       # per block: (start, drafted, verified, committed) events
            while not s.finished:
                e0 = self._event()
                with nvtx("draft"):
                    ticket = s.propose(request_id)
                e1 = self._event()
                n = len(ticket.tokens)
                tok_host[:n] = torch.tensor(ticket.tokens, dtype=torch.long)
                toks = tok_host[:n].to(tgt.device, non_blocking=True)
                self.h2d_bytes += 8 * n
                try:
                    with nvtx("verify"):
                        if self._sampling is None:
                            pred, vfeats = tgt.verify([(seq, toks)], taps=self.taps)
                        else:
                            samp = tgt.sampling_args(*self._sampling, range(seq.pos + 1, seq.pos + 1 + n))
                            pred, vfeats = tgt.verify([(seq, toks)], taps=self.taps, sampling=samp)
                except BaseException:
                    s.fail_verification(request_id, ticket)     # poison: the block never publishes
                    tgt.abort(seq)
                    raise
                e2 = self._event()
                predictions = [int(x) for x in pred.tolist()]
                self.d2h_bytes += 8 * n
                pos = seq.pos

                def publish(rows, vfeats=vfeats, pos=pos, ticket=ticket, predictions=predictions):
                    # successor of committed row i: the ticket's next token, or the target's
                    # correction after the last accepted row
                    nxt = list(ticket.tokens[1:rows]) + [predictions[rows - 1]]
                    self._publish(seq, rows, vfeats, pos, nxt)

                with nvtx("commit"):
                    d = s.commit(request_id, ticket, predictions, publish)
                marks.append((e0, e1, e2, self._event()))
                blocks.append((n, d.accepted, len(d.emitted)))
                if gold_check is not None and s.emitted != gold_check[:len(s.emitted)]:
                    raise AssertionError(f"speculative output diverged from greedy at block {len(blocks)}")
            t3 = self._event()
            tg_ms = self._elapsed_ms(t2, t3)
            committed = s.committed_decode_tokens
            phase = [0.0, 0.0, 0.0]
            records = []
            for (a0, a1, a2, a3), (rows, acc, emitted_n) in zip(marks, blocks):
                # draft, verify (+ read-back), select + commit + publish
                d_ms, v_ms, c_ms = self._elapsed_ms(a0, a1), self._elapsed_ms(a1, a2), self._elapsed_ms(a2, a3)
                phase[0] += d_ms
                phase[1] += v_ms
                phase[2] += c_ms
                records.append(dict(rows=rows, accepted=acc, committed=emitted_n, draft_ms=d_ms, verify_ms=v_ms,
                                    commit_ms=c_ms, cycle_ms=d_ms + v_ms + c_ms))
            nb = max(1, len(marks))
            return dict(
                tokens=list(s.emitted), prompt_tokens=int(prompt_host.numel()), pp_ms=pp_ms, tg_ms=tg_ms,
                pp_tok_s=prompt_host.numel() / (pp_ms / 1e3), committed=committed,
                tg_tok_s=committed / (tg_ms / 1e3) if tg_ms > 0 else float("nan"), blocks=len(blocks),
                mean_accepted=sum(b[1] for b in blocks) / max(1, len(blocks)),
                tokens_per_block=committed / max(1, len(blocks)), reused_prefix=ck.pos if ck else 0,
                draft_ms_per_block=phase[0] / nb, verify_ms_per_block=phase[1] / nb,
                commit_ms_per_block=phase[2] / nb,
                prompt_sha256=token_digest(prompt_host), output_sha256=token_digest(s.emitted),
                block_records=records)
        finally:
            if ck is not None:
                self.prefix.unpin(ck)
            if seq is not None:
                tgt.release(seq)
            self.session = None

    def _publish(self, seq, rows, vfeats, pos, nxt):
        """Commit ``rows`` verified rows and append their features to the drafter history."""
        self.target.commit(seq, rows)
        if self.drafter is not None:
            self.drafter.append(vfeats[:rows], pos, next_tokens=nxt)

    def _prefill(self, prompt_host, prompt_dev):
        """Prefill through the prefix registry when attached: restore the longest exact checkpoint,
        prefill the rest in boundary-aligned segments and capture a checkpoint at each boundary."""
        tgt, dr = self.target, self.drafter
        n = int(prompt_host.numel())
        toks = None
        ck = None
        if self.prefix is not None:
            toks = prompt_host.tolist()
            ck = self.prefix.lookup(toks)
        if ck is not None:
            self.prefix.pin(ck)
            seq = self.prefix.restore(ck, dr)
            start = ck.pos
        else:
            seq = tgt.new_sequence()
            start = 0
            if dr is not None:
                dr.reset()
        try:
            cuts = [n]
            if self.prefix is not None:
                b = self.prefix.boundary
                cuts = [p for p in range((start // b + 1) * b, n, b)] + [n]
            nxt, cur = None, start
            plist = prompt_host.tolist() if dr is not None else None
            for end in cuts:
                samp = None
                if getattr(self, "_sampling", None) is not None and end == n:
                    samp = tgt.sampling_args(*self._sampling, [n])
                nxt, feats = tgt.prefill(seq, prompt_dev[cur:end], taps=self.taps, sampling=samp)
                if dr is not None:
                    succ = plist[cur + 1:end + 1] if end < n else plist[cur + 1:n] + [int(nxt.item())]
                    dr.append(feats, cur, next_tokens=succ)
                if self.prefix is not None and end < n:
                    self.prefix.capture(seq, toks, dr)
                cur = end
            return seq, nxt, ck
        except BaseException:
            if ck is not None:
                self.prefix.unpin(ck)
            tgt.release(seq)
            raise


def greedy_reference(target, prompt, max_new_tokens, eos=None):
    """Plain single-row greedy decode through the same engine (the token-exact oracle)."""
    p = torch.as_tensor(prompt, dtype=torch.long, device=target.device)
    return target.greedy(p, max_new_tokens, eos=eos)
