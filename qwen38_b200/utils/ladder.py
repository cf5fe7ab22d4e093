"""Context ladder: committed TG and PP of one stream at several prompt lengths on one model.

The model is built once with room for the longest context; each rung prefills a fresh seeded
prompt of that length, computes its greedy gold continuation through the same engine (untimed),
then runs ``SpecRuntime.generate`` with pinned acceptance and checks the output token-exact.
Decode cost grows only through the 16 attention layers (the 48 GDN layers carry constant-size
state), which is what the ladder shows (the reference's long-context sweep:
``scripts/ci/longctx_cycle_bench.py``; 131,072 tokens is its longest passing context).

    python -m qwen38_b200.utils.ladder --ctx 4096 32768 131072 --new-tokens 128
    python -m qwen38_b200.utils.ladder --model tiny --ctx 256 1024            # CPU plumbing
"""
from __future__ import annotations

import argparse
import json

import torch


def main():
    from ..checkpoint import random_drafter_source, random_target_source
    from ..config import RuntimeConfig, full_drafter_config, full_model_config, tiny_drafter_config, tiny_model_config
    from ..models.drafter import BlockDrafter
    from ..models.target import HybridTarget
    from ..spec.analysis import acceptance_report
    from ..spec.engine import PinnedAcceptance, SpecRuntime, greedy_reference

    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="full", choices=["full", "tiny"])
    ap.add_argument("--ctx", type=int, nargs="+", default=[4096, 32768, 131072])
    ap.add_argument("--new-tokens", type=int, default=128)
    ap.add_argument("--mean-accepted", type=int, default=6)
    ap.add_argument("--repeats", type=int, default=1)
    a = ap.parse_args()
    cuda = torch.cuda.is_available()
    cfg, dcfg = (full_model_config(), full_drafter_config()) if a.model == "full" else \
        (tiny_model_config(), tiny_drafter_config())
    max_ctx = max(a.ctx) + a.new_tokens + 64
    chunk = 2048 if a.model == "full" else 64
    rt = RuntimeConfig(max_context=max_ctx, prefill_chunk=chunk, gdn_chunk=64 if a.model == "full" else 16)
    ops = None
    if cuda:
        from ..ops.native import NativeOps
        ops = NativeOps(max_keys=max_ctx + 64)
    dev, dt = ("cuda", torch.bfloat16) if cuda else ("cpu", torch.float32)
    tgt = HybridTarget(cfg, random_target_source(cfg, 0), rt, device=dev, dtype=dt, ops=ops)
    dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, 1), tgt, max_context=max_ctx)
    sr = SpecRuntime(tgt, dr, verifier_rows=dcfg.block_rows)
    for ctx in a.ctx:
        g = torch.Generator().manual_seed(ctx)
        prompt = torch.randint(0, cfg.vocab_size, (ctx,), generator=g)
        gold = greedy_reference(tgt, prompt.tolist(), a.new_tokens + 1)
        rows = []
        for r in range(a.repeats + 1):                   # the first pass warms graphs and caches
            res = sr.generate(prompt.tolist(), a.new_tokens + 1, gold_check=gold,
                              pinned=PinnedAcceptance(gold, seed=r, mean_accepted=a.mean_accepted))
            if r:
                rows.append(res)
        out = {"ctx": ctx, "new_tokens": a.new_tokens, "exact": True,
               "tg_tok_s": round(sum(x["tg_tok_s"] for x in rows) / len(rows), 2),
               "pp_tok_s": round(sum(x["pp_tok_s"] for x in rows) / len(rows), 1),
               "verify_ms_per_block": round(sum(x["verify_ms_per_block"] for x in rows) / len(rows), 3),
               "draft_ms_per_block": round(sum(x["draft_ms_per_block"] for x in rows) / len(rows), 3),
               "acceptance": acceptance_report(rows[-1]["block_records"]),
               "model": a.model, "device": dev}
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
