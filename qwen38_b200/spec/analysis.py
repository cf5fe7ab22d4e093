"""Offline acceptance scoring and block latency budgets.

``score_lookup`` answers "how much would n-gram lookup accept on this request?" without a device:
it walks a native greedy tape (the target's own output after the prompt) block by block.  Each
block asks ``LookupDraft`` for drafts over the history so far, keeps them only when the suffix
match is at least ``minimum_match`` tokens, sizes the block to a verifier width, and applies the
acceptance rule against the tape itself - the tape's next tokens are exactly the target's
predictions for the rows up to the first rejected draft, which is all the rule consumes.
``sweep_lookup`` runs that over a policy grid (verifier width x minimum match x full-suffix
preference), the grid the reference's offline scorer reports
(``speculative-decoding/harness/lookup_acceptance.py:17-100``).

``cycle_profile`` / ``latency_budget`` turn measured per-block phase times (``block_records`` from
``SpecRuntime.generate``) into what a TG target asks of the block cycle, and the TG ceiling with each
phase made free (the reference's 200-TG budget calculation,
``scripts/ci/speculative_latency_budget.py``).  ``acceptance_report`` summarises acceptance per
draft position.
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass

from .greedy import BUCKETS, bucket_at_most, select_prefix
from .lookup import LookupDraft


def _native_tape(prompt, emitted, vocab_size, max_new_tokens, eos_ids):
    """Validated (prompt, tape, eos set): the tape is complete (it fills the budget or ends at its
    first end-of-sequence id) and every id is in the vocabulary."""
    if vocab_size < 1 or max_new_tokens < 1:
        raise ValueError("positive vocabulary size and token budget required")
    prompt, tape, eos = list(prompt), list(emitted), set(eos_ids)
    if not 1 <= len(tape) <= max_new_tokens:
        raise ValueError(f"the tape must hold 1..{max_new_tokens} tokens, it holds {len(tape)}")
    bad = [t for t in prompt + tape + sorted(eos) if not 0 <= int(t) < vocab_size]
    if bad:
        raise ValueError(f"ids outside the vocabulary: {bad[:4]}")
    first_eos = next((i for i, t in enumerate(tape) if t in eos), None)
    if first_eos is not None and first_eos != len(tape) - 1:
        raise ValueError(f"the tape continues after its end-of-sequence id at {first_eos}")
    if first_eos is None and len(tape) != max_new_tokens:
        raise ValueError("the tape stops before the budget without an end-of-sequence id")
    return prompt, tape, eos


def score_lookup(prompt, emitted, *, vocab_size: int, max_new_tokens: int, eos_ids=(), max_rows: int = 32,
                 minimum_match: int = 1, prefer_full_suffix: bool = False) -> dict:
    """Lookup-only speculation replayed over a native tape (``emitted[0]`` is the prefill's token,
    emitted before the first block).  Returns per-block records and totals."""
    if max_rows not in BUCKETS:
        raise ValueError(f"max_rows {max_rows} is not a verifier width {BUCKETS}")
    if minimum_match < 1:
        raise ValueError("minimum_match must be at least 1")
    prompt, tape, eos = _native_tape(prompt, emitted, vocab_size, max_new_tokens, eos_ids)
    rid = "offline-lookup"
    lookup = LookupDraft(rid, prompt + tape[:1], max_proposals=BUCKETS[-1] - 1,
                         prefer_full_suffix=prefer_full_suffix)
    done, pos = tape[0] in eos, 1                 # tape[:pos] has been emitted
    blocks = []
    while not done and pos < max_new_tokens:
        cap = min(max_rows, max_new_tokens - pos)
        drafts, match = lookup.propose_with_match(rid, cap - 1) if cap > 1 else ([], 0)
        if match < minimum_match:
            drafts = []
        rows = bucket_at_most(min(cap, len(drafts) + 1))
        drafts = list(drafts[:rows - 1])
        preds = tape[pos:pos + rows]
        preds += [0] * (rows - len(preds))         # rows past the tape's end are never consumed
        d = select_prefix(drafts, preds, vocab_size=vocab_size, eos_ids=tuple(eos), max_proposals=BUCKETS[-1] - 1)
        if list(d.emitted) != tape[pos:pos + len(d.emitted)]:
            raise AssertionError(f"block at {pos} emitted beyond the tape")
        blocks.append(dict(position=len(prompt) + pos - 1, rows=rows, source="lookup" if drafts else "target",
                           match_length=match if drafts else 0, accepted=d.accepted, committed=len(d.emitted)))
        lookup.commit(rid, list(d.emitted))
        pos += len(d.emitted)
        done = d.finished
    if pos != len(tape):
        raise AssertionError(f"the replay emitted {pos} of the tape's {len(tape)} tokens")
    committed = sum(b["committed"] for b in blocks)
    return dict(max_rows=max_rows, minimum_match=minimum_match, prefer_full_suffix=prefer_full_suffix,
                blocks=blocks, committed=committed, accepted=sum(b["accepted"] for b in blocks),
                proposed=sum(b["rows"] - 1 for b in blocks),
                mean_committed_per_block=committed / len(blocks) if blocks else None)


def sweep_lookup(prompt, emitted, *, vocab_size: int, max_new_tokens: int, eos_ids=(),
                 buckets=BUCKETS, minimum_matches=(1, 2, 4, 8)) -> list:
    """``score_lookup`` over every (width, minimum match, full-suffix preference) policy."""
    return [score_lookup(prompt, emitted, vocab_size=vocab_size, max_new_tokens=max_new_tokens, eos_ids=eos_ids,
                         max_rows=b, minimum_match=m, prefer_full_suffix=pf)
            for b in buckets for m in minimum_matches for pf in (False, True)]


PHASES = ("draft_ms", "verify_ms", "commit_ms")


@dataclass(frozen=True)
class CycleProfile:
    """Mean block cycle of one verifier width: phase times (ms) and committed tokens per block."""
    rows: int
    blocks: int
    committed: int
    draft_ms: float
    verify_ms: float
    commit_ms: float
    cycle_ms: float

    @property
    def tokens_per_block(self) -> float:
        return self.committed / self.blocks

    @property
    def tg(self) -> float:
        """Committed tokens per second at this cycle."""
        return 1000.0 * self.tokens_per_block / self.cycle_ms

    def cycle_for(self, tg: float) -> float:
        """Cycle (ms) that reaches ``tg`` at this acceptance."""
        return 1000.0 * self.tokens_per_block / tg

    def tg_without(self, phase: str):
        """TG if ``phase`` cost nothing (None when it is the whole cycle)."""
        rest = self.cycle_ms - getattr(self, phase)
        return 1000.0 * self.tokens_per_block / rest if rest > 0 else None


def cycle_profile(blocks) -> CycleProfile:
    """Mean cycle of timed block records (``rows``, ``committed``, the three phase times and
    ``cycle_ms``); all blocks must share one verifier width."""
    if not blocks:
        raise ValueError("no timed blocks")
    widths = {b.get("rows") for b in blocks}
    if len(widths) != 1:
        raise ValueError(f"blocks of several verifier widths {sorted(map(str, widths))}: profile them apart")
    sums = dict.fromkeys(PHASES + ("cycle_ms",), 0.0)
    committed = 0
    for i, b in enumerate(blocks):
        if not (isinstance(b["rows"], int) and b["rows"] >= 1 and 1 <= b.get("committed", 0) <= b["rows"]):
            raise ValueError(f"block {i}: committed must be in 1..rows")
        for k in sums:
            v = b.get(k)
            if not isinstance(v, (int, float)) or not math.isfinite(v) or v < 0:
                raise ValueError(f"block {i}: {k} must be a finite non-negative time")
            sums[k] += v
        if b["cycle_ms"] <= 0 or max(b[k] for k in PHASES) > b["cycle_ms"] * (1 + 1e-6):
            raise ValueError(f"block {i}: the cycle must be positive and cover each phase")
        committed += b["committed"]
    n = len(blocks)
    return CycleProfile(rows=widths.pop(), blocks=n, committed=committed,
                        **{k: v / n for k, v in sums.items()})


def latency_budget(blocks, target_tg: float = 200.0) -> dict:
    """What ``target_tg`` asks of the measured cycle: the cycle it needs at the observed acceptance
    (and the cut from today's), the tokens per block it needs at today's cycle, and the TG with each
    phase made free."""
    if not (isinstance(target_tg, (int, float)) and math.isfinite(target_tg) and target_tg > 0):
        raise ValueError("target_tg must be a positive finite rate")
    p = cycle_profile(blocks)
    need = p.cycle_for(target_tg)
    return dict(profile=asdict(p), tokens_per_block=p.tokens_per_block, observed_tg=p.tg, target_tg=target_tg,
                cycle_needed_ms=need, cycle_cut_needed_pct=100.0 * (1.0 - need / p.cycle_ms),
                tokens_per_block_needed=target_tg * p.cycle_ms / 1000.0,
                tg_if_free={k[:-3]: p.tg_without(k) for k in PHASES})


def acceptance_report(blocks) -> dict:
    """Acceptance statistics of one request's blocks (``SpecRuntime.generate``'s ``block_records``:
    rows, accepted, committed per block), as the reference's acceptance report computes them
    (``scripts/ci/acceptance_report.py``, ``block_stats`` / ``per_position``):

    * ``full_draft``: blocks that verified the widest row count seen, excluding the request's last
      block (cut by EOS or the budget, not by a rejection); their mean accepted drafts is the
      acceptance measurement;
    * per draft position i = 1..rows-1 over the full-draft blocks: ``unconditional`` = share of
      blocks accepting at least i drafts, ``conditional`` = share accepting i among those that
      accepted i - 1 (None once no block got that far);
    * histogram of accepted drafts and the mean committed tokens per block over all blocks."""
    return acceptance_report_requests([blocks])


def acceptance_report_requests(requests) -> dict:
    """``acceptance_report`` over several requests' block lists (each request's last block is left
    out of the full-draft set; every block counts toward the committed mean)."""
    blocks = [b for r in requests for b in r]
    if not blocks:
        raise ValueError("no blocks")
    for b in blocks:
        if not (isinstance(b.get("rows"), int) and b["rows"] >= 1 and 0 <= b.get("accepted", -1) < b["rows"]
                and 1 <= b.get("committed", 0) <= b["rows"]):
            raise ValueError("blocks with rows, accepted < rows and committed in 1..rows required")
    width = max(b["rows"] for b in blocks)
    full = [b for r in requests for b in r[:-1] if b["rows"] == width]
    hist = [0] * width
    for b in full:
        hist[b["accepted"]] += 1
    uncond, cond = [], []
    for i in range(1, width):
        at_least = sum(1 for b in full if b["accepted"] >= i)
        prev = sum(1 for b in full if b["accepted"] >= i - 1)
        uncond.append(at_least / len(full) if full else None)
        cond.append(at_least / prev if prev else None)
    return dict(rows=width, blocks=len(blocks), full_draft_blocks=len(full),
                mean_accepted=(sum(b["accepted"] for b in full) / len(full)) if full else None,
                mean_committed_per_block=sum(b["committed"] for b in blocks) / len(blocks),
                histogram=hist, unconditional=uncond, conditional=cond)


def main(argv=None):
    """Acceptance report of a server's phase log (``serving.phase_log``: one JSON line per finished
    request with its block records)."""
    import argparse
    import json
    ap = argparse.ArgumentParser(description="acceptance report from a serving phase log")
    ap.add_argument("log")
    a = ap.parse_args(argv)
    reqs = []
    with open(a.log) as f:
        for line in f:
            line = line.strip()
            if line.startswith("{"):
                rec = json.loads(line)
                if rec.get("stage") == "request_phases" and rec.get("blocks"):
                    reqs.append(rec["blocks"])
    print(json.dumps(dict(requests=len(reqs), **acceptance_report_requests(reqs))))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
