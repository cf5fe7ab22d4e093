"""Multi-user continuous-batching load generator (BASELINE config 5 workload).

Streams arrive at seeded Poisson times (rate ``rate`` req/s), each with a seeded uniform-random
prompt of ``prompt_len`` tokens and ``new_tokens`` output tokens; optional pinned acceptance per
stream (the stream's own greedy continuation, corrupted at a seeded point per block).  The engine
is stepped in real time; reported: aggregate committed tok/s over the run and per-stream TG
(committed tokens / time from first token to completion) p50 / p90, as the reference's serving
bench reports them (``scripts/ci/longctx_cycle_bench.py``, ``docs/baseline-2026-09-05.md``).

    python -m qwen38_b200.serving.loadgen --model full --streams 8 --rate 2 --prompt-len 4096 --new-tokens 256
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m qwen38_b200.serving.loadgen --model full \
        --streams 32 --rate 2 --prompt-len 32768 --new-tokens 512 --weights mxfp8

Under torchrun every rank runs the engine tensor-parallel; rank 0's clock decides which arrivals are
due before each step and the others follow it, so every rank admits the same requests in lockstep.
"""
from __future__ import annotations

import argparse
import json
import random
import statistics
import time

import torch

from ..spec.engine import PinnedAcceptance


def poisson_arrivals(n: int, rate: float, seed: int):
    rng = random.Random(seed)
    t, out = 0.0, []
    for _ in range(n):
        out.append(t)
        t += rng.expovariate(rate)
    return out


def run(engine, prompts, new_tokens: int, arrivals, *, golds=None, mean_accepted: int = 6, seed: int = 0,
        clock=time.perf_counter, sync=None, agree=None):
    """Feeds requests at their arrival times and steps until all finish; returns the report.

    ``agree(n)``: under tensor parallelism every rank must admit the same requests before the same
    step, so the number of arrivals due is decided by one rank's clock and shared (rank 0's value,
    one small broadcast per step); None on one rank."""
    order = sorted(range(len(prompts)), key=lambda i: arrivals[i])
    t0 = clock()
    nxt = 0
    reqs = [None] * len(prompts)
    while nxt < len(order) or engine.has_work():
        now = clock() - t0
        due = nxt
        while due < len(order) and arrivals[order[due]] <= now:
            due += 1
        if agree is not None:
            due = agree(due)
        while nxt < due:
            i = order[nxt]
            pinned = PinnedAcceptance(golds[i], seed=seed + i, mean_accepted=mean_accepted) if golds else None
            reqs[i] = engine.add_request(prompts[i], new_tokens, pinned=pinned, request_id=f"s{i}")
            nxt += 1
        if engine.has_work():
            engine.step()
        elif nxt < len(order):
            time.sleep(max(0.0, min(0.01, arrivals[order[nxt]] - (clock() - t0))))
    if sync is not None:
        sync()
    t1 = clock()
    done = [r for r in reqs if r is not None and r.state == "finished"]
    per_stream = [(len(r.output) - 1) / max(1e-9, r.t_done - r.t_first) for r in done if len(r.output) > 1]
    committed = sum(len(r.output) - 1 for r in done)
    firsts = [r.t_first for r in done if r.t_first is not None]
    gen_window = (max(r.t_done for r in done) - min(firsts)) if done and firsts else float("nan")
    out = dict(streams=len(prompts), finished=len(done), aborted=sum(1 for r in reqs if r and r.state == "aborted"),
               committed_tokens=committed, wall_s=t1 - t0,
               aggregate_tok_s=committed / gen_window if gen_window == gen_window and gen_window > 0 else 0.0,
               p50_stream_tg=statistics.median(per_stream) if per_stream else 0.0,
               p90_stream_tg=sorted(per_stream)[int(0.9 * (len(per_stream) - 1))] if per_stream else 0.0,
               prefill_steps=engine.steps["prefill"], decode_steps=engine.steps["decode"])
    ttft = sorted(r.t_first - r.arrival for r in done if r.t_first is not None)
    if ttft:
        out.update(p50_ttft_s=statistics.median(ttft), p90_ttft_s=ttft[int(0.9 * (len(ttft) - 1))])
    if golds:
        out["exact"] = all(r.output == golds[i][:len(r.output)] for i, r in enumerate(reqs) if r is not None)
    return out


def main():
    from ..checkpoint import random_drafter_source, random_target_source
    from ..config import RuntimeConfig, full_drafter_config, full_model_config, tiny_drafter_config, tiny_model_config
    from ..models.drafter import BlockDrafter
    from ..models.target import HybridTarget
    from ..spec.engine import greedy_reference
    from .engine import ServingEngine

    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny", choices=["tiny", "full"])
    ap.add_argument("--streams", type=int, default=8)
    ap.add_argument("--rate", type=float, default=2.0)
    ap.add_argument("--prompt-len", type=int, default=4096)
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--mean-accepted", type=int, default=6)
    ap.add_argument("--no-pinned", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--weights", default="bf16", choices=["bf16", "mxfp8"])
    ap.add_argument("--comm", default="fused", choices=["fused", "peer", "nccl"])
    a = ap.parse_args()
    from ..parallel.comm import init_distributed, make_comm
    rank, world, local = init_distributed()
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.set_device(local)
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    cfg, dcfg = (full_model_config(), full_drafter_config()) if a.model == "full" else \
        (tiny_model_config(), tiny_drafter_config())
    ops = None
    max_ctx = a.prompt_len + a.new_tokens + 64
    if cuda:
        from ..ops.native import NativeOps
        ops = NativeOps(device=dev, max_keys=max_ctx + 64, weight_format=a.weights)
    rt = RuntimeConfig(max_context=max_ctx, weight_format=a.weights)
    comm = make_comm(world, device=dev, hidden=cfg.hidden_size, peer=cuda and a.comm != "nccl",
                     fused=a.comm == "fused", prefill_rows=rt.prefill_chunk if a.comm == "fused" else 0)
    tsrc = random_target_source(cfg, a.seed)
    if a.weights == "mxfp8":
        from ..checkpoint import MXFP8Source
        tsrc = MXFP8Source(tsrc)
    tgt = HybridTarget(cfg, tsrc, rt, device=dev, dtype=torch.bfloat16 if cuda else torch.float32, ops=ops,
                       comm=comm, max_slots=a.streams + 1, max_verify_rows=a.streams * dcfg.block_rows)
    dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, a.seed + 1), tgt, slots=a.streams)
    g = torch.Generator().manual_seed(a.seed)
    prompts = [torch.randint(0, cfg.vocab_size, (a.prompt_len,), generator=g).tolist() for _ in range(a.streams)]
    golds = None if a.no_pinned else [greedy_reference(tgt, p, a.new_tokens) for p in prompts]
    eng = ServingEngine(tgt, dr, verifier_rows=dcfg.block_rows)
    agree = None
    if world > 1:
        import torch.distributed as dist

        def agree(n):
            t = torch.tensor([n], dtype=torch.int64, device=dev if dist.get_backend() == "nccl" else "cpu")
            dist.broadcast(t, 0)
            return int(t.item())
    rep = run(eng, prompts, a.new_tokens, poisson_arrivals(a.streams, a.rate, a.seed), golds=golds,
              mean_accepted=a.mean_accepted, seed=a.seed, sync=torch.cuda.synchronize if cuda else None,
              agree=agree)
    rep.update(model=a.model, prompt_len=a.prompt_len, new_tokens=a.new_tokens, rate=a.rate,
               weights=a.weights, tp=world, device=dev.type)
    if rank == 0:
        print(json.dumps(rep))


if __name__ == "__main__":
    main()
