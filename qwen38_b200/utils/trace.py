"""Tracing, digests and the device-memory ledger.

* ``nvtx(name)``: an NVTX range around a host phase (prefill, draft, verify, commit), visible in
  any CUDA timeline tool; a no-op without CUDA.  The reference brackets the same phases with its
  device profiler signposts and host phase logs (``graft/layer.py:18-90``,
  ``scripts/ci/serving_worker_hook.py:9-15``).
* ``token_digest`` / ``source_digests``: sha256 of token ids and of every source file, for run
  reports that pin exactly what produced a number (``scripts/ci/full_request.py:212-232``).
* ``memory_ledger(target, drafter)``: bytes per category (weights per kind, KV cache, GDN state,
  verify stash, drafter history) from the tensors themselves, plus the allocator's view, with a
  budget check (``scripts/ci/memory_ledger.py``).
"""
from __future__ import annotations

import contextlib
import hashlib
import os

import torch

_NVTX = os.environ.get("Q38_NVTX", "1") != "0"


@contextlib.contextmanager
def nvtx(name: str):
    if _NVTX and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


def token_digest(ids) -> str:
    t = torch.as_tensor(list(ids) if not torch.is_tensor(ids) else ids.cpu(), dtype=torch.int64)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def source_digests(root: str | None = None) -> dict:
    root = root or os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = {}
    for d, _, files in os.walk(root):
        if "_build" in d or "__pycache__" in d:
            continue
        for f in sorted(files):
            if f.endswith((".py", ".cu", ".cuh", ".cpp")):
                p = os.path.join(d, f)
                with open(p, "rb") as fh:
                    out[os.path.relpath(p, root)] = hashlib.sha256(fh.read()).hexdigest()
    return dict(sorted(out.items()))


def _nbytes(t) -> int:
    if t is None:
        return 0
    if hasattr(t, "t") and hasattr(t, "N"):          # tile-contiguous weight wrapper
        t = t.t
    if isinstance(t, torch.Tensor):
        return t.numel() * t.element_size()
    return 0


class MemoryBudgetExceeded(RuntimeError):
    pass


def memory_ledger(target, drafter=None, budget_bytes: int | None = None) -> dict:
    """Itemised device bytes of a ``HybridTarget`` (and drafter); raises ``MemoryBudgetExceeded``
    when the itemised total passes ``budget_bytes``."""
    items = {}

    def add(k, n):
        items[k] = items.get(k, 0) + int(n)

    add("weights.embed", _nbytes(target.embed))
    if target.lm_head is not target.embed:
        add("weights.lm_head", _nbytes(target.lm_head))
    for L in target.layers:
        kind = "gdn" if "conv_w" in L else "attn"
        for key in ("w_in", "w_out"):
            add(f"weights.{kind}_proj", _nbytes(L.get(key)))
        for key in ("w_gu", "w_down"):
            add("weights.mlp", _nbytes(L.get(key)))
    for name, key in (("kv_cache", "kcache"), ("kv_cache", "vcache"), ("gdn_state", "rec"), ("gdn_conv", "conv"),
                      ("verify_stash", "gdn_stash")):
        add(name, _nbytes(getattr(target, key, None)))
    if drafter is not None:
        for key in ("kctx_all", "vctx_all"):
            add("drafter.history", _nbytes(getattr(drafter, key, None)))
        for key in ("fc", "pred", "succ"):
            add("drafter.weights", _nbytes(getattr(drafter, key, None)))
        for L in getattr(drafter, "layers", []) or []:
            for v in L.values():
                add("drafter.weights", _nbytes(v))
    items["total_itemised"] = sum(v for k, v in items.items())
    if torch.cuda.is_available() and getattr(target, "device", torch.device("cpu")).type == "cuda":
        st = torch.cuda.memory_stats(target.device)
        items["allocator.allocated"] = int(st.get("allocated_bytes.all.current", 0))
        items["allocator.reserved"] = int(st.get("reserved_bytes.all.current", 0))
    if budget_bytes is not None and items["total_itemised"] > budget_bytes:
        raise MemoryBudgetExceeded(f"itemised {items['total_itemised']} B > budget {budget_bytes} B")
    return items
