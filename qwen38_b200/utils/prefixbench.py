"""Prefix-reuse benchmark: a prompt whose first ``--reuse`` tokens match an earlier request.

The workload of the reference's prefix-reuse measurement (README.md:78-80: a 4,096-token prompt whose
first 2,048 tokens were served before, 0.684 s with reuse against 1.239 s cold on its hardware).
Request A (``--ctx`` seeded random ids) is served once through a ``PrefixRegistry`` with a
``--reuse``-token boundary, which captures the checkpoint at that boundary: the KV blocks below it
(shared, reference-counted) and a copy of the GDN recurrent and conv state.  Request B shares A's
first ``--reuse`` ids and continues with new ones.  B is then served twice: cold, without the
registry, and with it, where the prefill restores the checkpoint and computes only the new suffix.
Both decode ``--new-tokens`` committed tokens with pinned acceptance, and both must equal the
single-row greedy decode of B (token-exact).  Prefill and decode times are CUDA-event times, the
maximum over ranks.  Tensor parallelism: launch under torchrun with ``--gpus N`` (one rank per GPU).

    python -m qwen38_b200.utils.prefixbench                      # full shape, one GPU
    torchrun --nnodes 1 --nproc-per-node 2 --master-addr 127.0.0.1 -m qwen38_b200.utils.prefixbench --gpus 2
    python -m qwen38_b200.utils.prefixbench --model tiny --ctx 512 --reuse 256 --new-tokens 32   # CPU
"""
from __future__ import annotations

import argparse
import json


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="full", choices=["full", "tiny"])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--reuse", type=int, default=2048)
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--mean-accepted", type=int, default=6)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--budget-mb", type=int, default=4096)
    return ap.parse_args(argv)


def run(a) -> dict:
    import torch
    import torch.distributed as dist

    from ..checkpoint import random_drafter_source, random_target_source
    from ..config import RuntimeConfig, full_drafter_config, full_model_config, tiny_drafter_config, tiny_model_config
    from ..models.drafter import BlockDrafter
    from ..models.target import HybridTarget
    from ..ops import TorchOps
    from ..parallel.comm import init_distributed, make_comm
    from ..prefix.registry import PrefixRegistry
    from ..spec.engine import PinnedAcceptance, SpecRuntime, greedy_reference

    if a.ctx <= a.reuse or a.reuse <= 0:
        raise SystemExit("--reuse must be a positive prefix shorter than --ctx")
    cuda = torch.cuda.is_available()
    rank, world, local = init_distributed()
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    if cuda:
        torch.cuda.set_device(local)
    device = torch.device("cuda", local) if cuda else torch.device("cpu")
    cfg, dcfg = (full_model_config(), full_drafter_config()) if a.model == "full" else \
        (tiny_model_config(), tiny_drafter_config())
    dtype = torch.bfloat16 if cuda else torch.float32
    rt = RuntimeConfig(max_context=a.ctx + a.new_tokens + 64, prefill_chunk=a.reuse)
    comm = make_comm(world, device=device, hidden=cfg.hidden_size, peer=cuda, fused=cuda) if world > 1 else None
    if cuda:
        from ..ops.native import NativeOps
        ops = NativeOps(device=device, max_keys=rt.max_context + 64)
    else:
        ops = TorchOps()
    tgt = HybridTarget(cfg, random_target_source(cfg, a.seed), rt, device=device, dtype=dtype, ops=ops, comm=comm,
                       max_slots=2)
    dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, a.seed + 1), tgt)
    g = torch.Generator().manual_seed(a.seed)
    prompt_a = torch.randint(0, cfg.vocab_size, (a.ctx,), generator=g).tolist()
    suffix = torch.randint(0, cfg.vocab_size, (a.ctx - a.reuse,), generator=torch.Generator().manual_seed(a.seed + 7))
    prompt_b = prompt_a[:a.reuse] + suffix.tolist()
    n_out = a.new_tokens + 1
    gold = greedy_reference(tgt, prompt_b, n_out)
    reg = PrefixRegistry(tgt, a.budget_mb << 20, boundary=a.reuse)
    cold_rt = SpecRuntime(tgt, dr, verifier_rows=dcfg.block_rows)
    reuse_rt = SpecRuntime(tgt, dr, verifier_rows=dcfg.block_rows, prefix=reg)

    def serve(sr, prompt, step):
        res = sr.generate(prompt, n_out, gold_check=gold if prompt is prompt_b else None,
                          pinned=PinnedAcceptance(gold, seed=100 + step, mean_accepted=a.mean_accepted)
                          if prompt is prompt_b else None)
        if hasattr(ops, "check"):
            ops.check()
        return res

    serve(cold_rt, prompt_b, 0)                      # warm-up: graphs, caches
    cold = serve(cold_rt, prompt_b, 1)
    serve(reuse_rt, prompt_a, 2)                     # request A: captures the boundary checkpoint
    reused = serve(reuse_rt, prompt_b, 1)            # same pinned schedule as the cold run
    t = torch.tensor([cold["pp_ms"], cold["tg_ms"], reused["pp_ms"], reused["tg_ms"]], dtype=torch.float64,
                     device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    cpp, ctg, rpp, rtg = t.tolist()
    out = {
        "metric": "prefix reuse: prefill ms and committed TG, cold vs reused prefix",
        "n_gpus": world, "ctx": a.ctx, "reused_prefix": reused["reused_prefix"], "new_tokens": a.new_tokens,
        "cold": {"prefill_ms": round(cpp, 2), "tg_tok_s": round(cold["committed"] / (ctg / 1e3), 1),
                 "total_s": round((cpp + ctg) / 1e3, 4)},
        "reused": {"prefill_ms": round(rpp, 2), "tg_tok_s": round(reused["committed"] / (rtg / 1e3), 1),
                   "total_s": round((rpp + rtg) / 1e3, 4)},
        "prefill_speedup": round(cpp / rpp, 2),
        "token_exact": reused["tokens"] == gold and cold["tokens"] == gold,
        "registry": reg.export_stats(),
        "data": "synthetic (seeded uniform-random ids, random-init weights of the named shape)",
        "config": {"model": a.model, "parallelism": f"tp{world}", "dtype": str(dtype).replace("torch.", "")},
    }
    tgt.release_graphs()
    dr.release_graphs()
    return out if rank == 0 else {}


def main(argv=None):
    out = run(parse(argv))
    if out:
        print(json.dumps(out))


if __name__ == "__main__":
    main()
