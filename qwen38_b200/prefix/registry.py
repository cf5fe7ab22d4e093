"""Prefix reuse: checkpoints of KV + GDN state at chunk boundaries, in a byte-budgeted LRU.

Reference behaviour (``scripts/ci/qwen_prefix_registry.py:136-565``, ``prefill_gdn_checkpoint.py``,
``prefill_prefix_resume.py``, ``docs/combined-prefix-cache.md``):

* A checkpoint exists only at a ``boundary`` (2,048-token) multiple, where chunked prefill has
  exactly consumed that many tokens: the GDN recurrent state and conv window are then exact.
* Keyed by the exact token prefix; a hit is verified token by token (a hash match alone never
  vouches for reuse).
* Bounded by bytes; pinned (in-use) entries are never evicted; least recently used goes first.
* A kill switch (flag file, polled, latching) disables lookups and captures at run time.
* Stats are exported for observability.

Here a checkpoint holds copies of the per-slot GDN state and conv windows, the KV blocks below
the boundary (shared with the sequence that produced them through the allocator's reference
counts, never copied) and the drafter's projected K/V history rows for those positions.
"""
from __future__ import annotations

import hashlib
import os
import time
from array import array
from collections import OrderedDict
from dataclasses import dataclass, field

STAT_NAMES = ("lookups", "hits", "misses", "token_mismatch", "captures", "capture_replaced",
              "capture_skipped_budget", "capture_disabled", "evicted_lru", "reused_tokens")


def prefix_key(tokens) -> str:
    return hashlib.sha256(array("q", [int(t) for t in tokens]).tobytes()).hexdigest()


@dataclass
class Checkpoint:
    key: str
    pos: int
    token_ids: array
    target: dict                   # HybridTarget.prefix_snapshot
    drafter: dict | None           # {"lo": first row, "k": [L, pos - lo, kv, D], "v": ...}
    nbytes: int
    pins: int = 0
    serial: int = 0

    def matches(self, tokens) -> bool:
        return len(tokens) >= self.pos and self.token_ids == array("q", [int(t) for t in tokens[:self.pos]])


class KillSwitch:
    """Latching flag-file switch, polled at most every ``poll_s`` seconds."""

    def __init__(self, path: str | None, poll_s: float = 1.0, clock=time.monotonic, exists=os.path.exists):
        self.path, self.poll_s, self.clock, self.exists = path, float(poll_s), clock, exists
        self.engaged = False
        self._last = None

    def poll(self) -> bool:
        if self.engaged or not self.path:
            return self.engaged
        now = self.clock()
        if self._last is not None and now - self._last < self.poll_s:
            return False
        self._last = now
        try:
            self.engaged = bool(self.exists(self.path))
        except OSError:
            self.engaged = False
        return self.engaged


class PrefixRegistry:
    def __init__(self, target, budget_bytes: int, *, boundary: int = 2048, kill_switch: KillSwitch | None = None):
        if boundary % target.block_size:
            raise ValueError("the checkpoint boundary must be a multiple of the KV block size")
        if target.rt.prefill_chunk % boundary and boundary % target.rt.prefill_chunk:
            raise ValueError("prefill chunks must align with checkpoint boundaries")
        self.target = target
        self.budget = int(budget_bytes)
        self.boundary = boundary
        self.entries: "OrderedDict[str, Checkpoint]" = OrderedDict()
        self.bytes = 0
        self.kill = kill_switch or KillSwitch(None)
        self.stats = dict.fromkeys(STAT_NAMES, 0)
        self._serial = 0

    @property
    def disabled(self) -> bool:
        return self.kill.poll()

    # ---------------------------------------------------------------- lookup
    def lookup(self, tokens) -> Checkpoint | None:
        """Longest checkpoint that is an exact prefix of ``tokens`` and leaves at least one token
        to prefill (the last prompt row must run to produce the first output)."""
        if self.disabled:
            return None
        self.stats["lookups"] += 1
        n = len(tokens)
        best = None
        pos = ((n - 1) // self.boundary) * self.boundary
        while pos > 0:
            ck = self.entries.get(prefix_key(tokens[:pos]))
            if ck is not None:
                if ck.matches(tokens):
                    best = ck
                    break
                self.stats["token_mismatch"] += 1
            pos -= self.boundary
        if best is None:
            self.stats["misses"] += 1
            return None
        self.entries.move_to_end(best.key)
        self.stats["hits"] += 1
        self.stats["reused_tokens"] += best.pos
        return best

    def pin(self, ck: Checkpoint):
        ck.pins += 1

    def unpin(self, ck: Checkpoint):
        ck.pins = max(0, ck.pins - 1)
        self._enforce_budget()

    # ---------------------------------------------------------------- capture
    def capture(self, seq, tokens, drafter=None, dslot: int = 0) -> Checkpoint | None:
        """Checkpoint ``seq`` at its committed length (a boundary multiple)."""
        pos = seq.pos
        if pos <= 0 or pos % self.boundary:
            raise ValueError(f"checkpoints are exact only at {self.boundary}-token boundaries, not {pos}")
        if self.disabled:
            self.stats["capture_disabled"] += 1
            return None
        key = prefix_key(tokens[:pos])
        old = self.entries.get(key)
        if old is not None:
            self.entries.move_to_end(key)
            if old.pins:
                return old
            self._remove(key)
            self.stats["capture_replaced"] += 1
        snap = self.target.prefix_snapshot(seq, pos)
        dsnap = None
        nbytes = snap["nbytes"]
        if drafter is not None:
            if drafter.positions[dslot] < pos:
                raise ValueError("drafter history behind the target at capture")
            # rows below the drafter's floor are never read again (a windowed drafter's older rows)
            lo = drafter.history_floor(pos) if hasattr(drafter, "history_floor") else 0
            dsnap = {"lo": lo, "k": drafter.kctx_all[dslot, :, lo:pos].clone(),
                     "v": drafter.vctx_all[dslot, :, lo:pos].clone()}
            nbytes += 2 * dsnap["k"].numel() * dsnap["k"].element_size()
        if nbytes > self.budget:
            self.target.release_prefix(snap)
            self.stats["capture_skipped_budget"] += 1
            return None
        self._serial += 1
        ck = Checkpoint(key, pos, array("q", [int(t) for t in tokens[:pos]]), snap, dsnap, nbytes,
                        serial=self._serial)
        self.entries[key] = ck
        self.bytes += nbytes
        self.stats["captures"] += 1
        self._enforce_budget()
        return ck

    def restore(self, ck: Checkpoint, drafter=None, dslot: int = 0):
        """New target sequence at ``ck.pos`` (and the drafter history rewound to the same rows)."""
        seq = self.target.sequence_from_prefix(ck.target)
        if drafter is not None and ck.drafter is not None:
            lo = ck.drafter.get("lo", 0)
            drafter.kctx_all[dslot, :, lo:ck.pos].copy_(ck.drafter["k"])
            drafter.vctx_all[dslot, :, lo:ck.pos].copy_(ck.drafter["v"])
            drafter.positions[dslot] = ck.pos
        return seq

    # ---------------------------------------------------------------- eviction
    def _remove(self, key):
        ck = self.entries.pop(key, None)
        if ck is not None:
            self.bytes -= ck.nbytes
            self.target.release_prefix(ck.target)
        return ck

    def _enforce_budget(self):
        for key in list(self.entries):
            if self.bytes <= self.budget:
                break
            if self.entries[key].pins:
                continue
            self._remove(key)
            self.stats["evicted_lru"] += 1

    def clear(self):
        for key in list(self.entries):
            self._remove(key)

    def export_stats(self) -> dict:
        return dict(self.stats, entries=len(self.entries), bytes=self.bytes, budget=self.budget,
                    disabled=self.kill.engaged)
