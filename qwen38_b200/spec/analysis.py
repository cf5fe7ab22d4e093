"""Offline acceptance scoring and block latency budgets.

``score_lookup`` replays a native greedy tape (prompt + the target's own greedy output) through
the request protocol with the lookup drafter only, and counts what each block would accept: the
target's predictions for a block are the tape's next tokens, which are valid up to the first
mismatching proposal (what the selection rule consumes).  ``sweep_lookup`` runs the policy grid
(verifier bucket x minimum match length x full-suffix preference), as the reference's offline
scorer does (``speculative-decoding/harness/lookup_acceptance.py:17-100``).  Nothing here runs a
device or measures time.

``acceptance_report`` summarises one request's blocks (full-draft mean acceptance, per-position
acceptance rates, histogram).  ``latency_budget`` turns measured per-block phase times (``SpecRuntime.generate`` returns them in
``block_records``) into the cycle time a target TG needs at the observed acceptance, and the
TG ceiling if drafting were free (``speculative-decoding/harness/speculative_latency_budget.py``).
"""
from __future__ import annotations

import math

from .greedy import BUCKETS, GreedySession
from .lookup import HybridDraft


def score_lookup(prompt, emitted, *, vocab_size: int, max_new_tokens: int, eos_ids=(), max_rows: int = 32,
                 minimum_match: int = 1, prefer_full_suffix: bool = False) -> dict:
    prompt, emitted, eos_ids = list(prompt), list(emitted), tuple(eos_ids)
    if max_rows not in BUCKETS:
        raise ValueError("max_rows must be a verifier bucket")
    if minimum_match < 1 or vocab_size < 1 or max_new_tokens < 1:
        raise ValueError("positive minimum match, vocabulary and budget required")
    if not emitted or len(emitted) > max_new_tokens:
        raise ValueError("a nonempty native output within the budget is required")
    if any(not 0 <= int(t) < vocab_size for t in (*prompt, *emitted, *eos_ids)):
        raise ValueError("token outside the vocabulary")
    if any(t in eos_ids for t in emitted[:-1]):
        raise ValueError("the native output must stop at its first terminal token")
    if len(emitted) != max_new_tokens and emitted[-1] not in eos_ids:
        raise ValueError("incomplete native tape: neither budget exhaustion nor EOS")
    rid = "offline-lookup"
    drafter = HybridDraft(rid, prompt, vocab_size=vocab_size, lookup_enabled=True, max_proposals=31,
                          prefer_full_suffix=prefer_full_suffix)
    s = GreedySession(rid, prompt, emitted[0], vocab_size=vocab_size, max_new_tokens=max_new_tokens,
                      eos_ids=eos_ids, drafter=drafter, verifier_rows=32)
    blocks = []
    try:
        while not s.finished:
            cursor = len(s.emitted)
            limit = min(max_rows, max_new_tokens - cursor)
            match = drafter.lookup.propose_with_match(rid, limit - 1)[1] if limit > 1 else 0
            ticket = s.propose(rid, max_rows=max_rows if match >= minimum_match else 1)
            preds = emitted[cursor:cursor + len(ticket.tokens)]
            preds += [0] * (len(ticket.tokens) - len(preds))
            d = s.commit(rid, ticket, preds, lambda rows: None)
            if s.emitted != emitted[:len(s.emitted)]:
                raise AssertionError("offline scoring consumed beyond the native tape")
            blocks.append(dict(rows=len(ticket.tokens), match_length=match, source=ticket.source,
                               accepted=d.accepted, committed=len(d.emitted), position=ticket.position))
        if s.emitted != emitted:
            raise AssertionError("offline scoring did not consume the whole native tape")
        return dict(max_rows=max_rows, minimum_match=minimum_match, prefer_full_suffix=prefer_full_suffix,
                    accepted=s.accepted_proposals, proposed=s.committed_block_proposals,
                    committed=s.committed_decode_tokens, blocks=blocks,
                    mean_committed_per_block=s.committed_decode_tokens / len(blocks) if blocks else None)
    finally:
        s.close(rid)


def sweep_lookup(prompt, emitted, *, vocab_size: int, max_new_tokens: int, eos_ids=(),
                 buckets=(1, 2, 4, 8, 16, 32), minimum_matches=(1, 2, 4, 8)) -> list:
    return [score_lookup(prompt, emitted, vocab_size=vocab_size, max_new_tokens=max_new_tokens, eos_ids=eos_ids,
                         max_rows=b, minimum_match=m, prefer_full_suffix=pf)
            for b in buckets for m in minimum_matches for pf in (False, True)]


def latency_budget(blocks, target_tg: float = 200.0) -> dict:
    """``blocks``: dicts with rows, committed, draft_ms, verify_ms, commit_ms, cycle_ms."""
    if not blocks or not (isinstance(target_tg, (int, float)) and math.isfinite(target_tg) and target_tg > 0):
        raise ValueError("timed blocks and a positive finite target required")
    fields = ("draft_ms", "verify_ms", "commit_ms", "cycle_ms")
    tot = dict.fromkeys(fields, 0.0)
    widths, committed = set(), 0
    for b in blocks:
        if not (isinstance(b.get("rows"), int) and b["rows"] >= 1 and 1 <= b.get("committed", 0) <= b["rows"]):
            raise ValueError("blocks with valid committed counts required")
        for f in fields:
            v = b.get(f)
            if not isinstance(v, (int, float)) or not math.isfinite(v) or v < 0:
                raise ValueError(f"finite non-negative {f} required")
            tot[f] += v
        if b["cycle_ms"] <= 0 or any(b[f] > b["cycle_ms"] * (1 + 1e-6) for f in fields[:-1]):
            raise ValueError("the cycle must cover each phase")
        widths.add(b["rows"])
        committed += b["committed"]
    if len(widths) != 1:
        raise ValueError("separate verifier widths before computing a budget")
    n = len(blocks)
    mean = {f: v / n for f, v in tot.items()}
    per_block = committed / n
    need_ms = 1000.0 * per_block / target_tg
    return dict(rows=widths.pop(), blocks=n, committed=committed, mean_committed_per_block=per_block,
                mean_ms=mean, observed_block_tg=1000.0 * committed / tot["cycle_ms"], target_tg=target_tg,
                required_cycle_ms=need_ms, required_cycle_reduction_percent=100.0 * (1 - need_ms / mean["cycle_ms"]),
                required_committed_at_current_latency=target_tg * mean["cycle_ms"] / 1000.0,
                zero_draft_ceiling_tg=(1000.0 * per_block / (mean["cycle_ms"] - mean["draft_ms"])
                                       if mean["cycle_ms"] > mean["draft_ms"] else None))


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
