"""Context ladder: committed TG and PP of one stream at several prompt lengths on one model.

The model is built once with room for the longest context; each rung prefills a fresh seeded
prompt of that length, computes its greedy gold continuation through the same engine (untimed),
then runs ``SpecRuntime.generate`` with pinned acceptance and checks the output token-exact.
Decode cost grows only through the 16 attention layers (the 48 GDN layers carry constant-size
state), which is what the ladder shows (the reference's long-context sweep:
``scripts/ci/longctx_cycle_bench.py``; 131,072 tokens is its longest passing context).

    python -m qwen38_b200.utils.ladder --ctx 4096 32768 131072 --new-tokens 128
    python -m qwen38_b200.utils.ladder --model tiny --ctx 256 1024            # CPU plumbing
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m qwen38_b200.utils.ladder --ctx 8192 131072

Under torchrun every rank runs the ladder tensor-parallel (peer-memory collectives with the pushed
all-reduce on GPUs, gloo collectives on CPU); rank 0 prints, with per-rung times taken as the max
over ranks.
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
    ap.add_argument("--comm", default="fused", choices=["fused", "peer", "nccl"])
    a = ap.parse_args()
    from ..parallel.comm import init_distributed, make_comm
    rank, world, local = init_distributed()
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.set_device(local)
    cfg, dcfg = (full_model_config(), full_drafter_config()) if a.model == "full" else \
        (tiny_model_config(), tiny_drafter_config())
    max_ctx = max(a.ctx) + a.new_tokens + 64
    chunk = 2048 if a.model == "full" else 64
    rt = RuntimeConfig(max_context=max_ctx, prefill_chunk=chunk, gdn_chunk=64 if a.model == "full" else 16)
    ops = None
    if cuda:
        from ..ops.native import NativeOps
        ops = NativeOps(max_keys=max_ctx + 64)
    dev, dt = (torch.device("cuda", local), torch.bfloat16) if cuda else (torch.device("cpu"), torch.float32)
    comm = make_comm(world, device=dev, hidden=cfg.hidden_size, peer=cuda and a.comm != "nccl",
                     fused=a.comm == "fused", prefill_rows=chunk if a.comm == "fused" else 0)
    tgt = HybridTarget(cfg, random_target_source(cfg, 0), rt, device=dev, dtype=dt, ops=ops, comm=comm)
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
        # max over ranks of the per-rank times (every rank runs the same rungs in the same order)
        t = torch.tensor([[x["tg_ms"], x["pp_ms"], x["verify_ms_per_block"], x["draft_ms_per_block"]]
                          for x in rows], dtype=torch.float64)
        if world > 1:
            import torch.distributed as dist
            tt = t.to(dev) if cuda else t
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = tt.cpu()
        committed = rows[0]["committed"]
        out = {"ctx": ctx, "new_tokens": a.new_tokens, "exact": True, "tp": world,
               "tg_tok_s": round(sum(committed / (float(r[0]) / 1e3) for r in t) / len(rows), 2),
               "pp_tok_s": round(sum(ctx / (float(r[1]) / 1e3) for r in t) / len(rows), 1),
               "verify_ms_per_block": round(float(t[:, 2].mean()), 3),
               "draft_ms_per_block": round(float(t[:, 3].mean()), 3),
               "acceptance": acceptance_report(rows[-1]["block_records"]),
               "model": a.model, "device": dev.type}
        if rank == 0:
            print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
