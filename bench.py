#!/usr/bin/env python
"""Headline benchmark: committed TG tok/s (and PP tok/s), one stream, CTX 4,096, on N GPUs (TP=N).

Workload: full-size random-init hybrid (vocab 151,936, hidden 5,120, 64 layers
3 GDN : 1 gated attention, SwiGLU 17,408), bf16, a seeded 4,096-token uniform-random prompt, 256
committed output tokens, 16-row blocks from a 5-layer DSpark-style drafter with pinned acceptance
(proposals overwritten by the target's own greedy continuation corrupted at a seeded point; mean
accepted 6 of 15).  One step = one complete request (prefill + generation loop).

PP = prompt tokens / prefill seconds; TG = committed decode tokens / generation-loop seconds
(drafting, verification, selection, commit and read-back included), as the reference defines them
(README.md:28-31).  Device times are CUDA events on the launching stream, max over ranks.
``value`` is TG (the whole job serves one stream, so the aggregate equals that stream's TG).

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
For N > 1 launch with torchrun (one rank per GPU).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

BASELINE_TG = 128.65      # committed TG tok/s, README.md:21 (2 x Blackhole P150A, TP2)
BASELINE_PP = 3320.13


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ops", default="native", choices=["native", "torch"])
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--model", default="full", choices=["full", "tiny"])
    ap.add_argument("--layers", type=int, default=0, help="debug only: truncate the target (invalid as a bench)")
    ap.add_argument("--mean-accepted", type=int, default=6)
    ap.add_argument("--temperature", type=float, default=0.0,
                    help="> 0: sampled decoding (speculative, exact against the target's own sampler)")
    ap.add_argument("--weights", default="bf16", choices=["bf16", "mxfp8"],
                    help="mxfp8: target linear weights are MXFP8 (streamed as e4m3 + E8M0 scales by the "
                         "verify / decode GEMMs, expanded exactly to bf16 in shared memory)")
    ap.add_argument("--drafter", default="dspark", choices=["dspark", "dflash2"],
                    help="dspark: the headline drafter; dflash2: the windowed drafter (same block rows)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--prefill-chunk", type=int, default=4096,
                    help="prefill chunk rows (multiple of 64); 4096 prefills the CTX 4,096 prompt in one chunk")
    ap.add_argument("--comm", default="fused", choices=["fused", "peer", "nccl"],
                    help="TP collectives: all-reduce pushed by the out-projection GEMMs and completed by the "
                         "next RMSNorm (default), separate peer-memory all-reduce kernels, or NCCL")
    return ap.parse_args()


REFERENCE_UNAVAILABLE = (
    "reference is a Tenstorrent TT-NN/tt-metal programme for Blackhole P150A cards with no installable "
    "package (pip: 'Neither setup.py nor pyproject.toml found') and no CUDA code path; it cannot run on B200")


def _provenance():
    try:
        from qwen38_b200.utils.provenance import manifest
        return manifest()
    except Exception as e:          # provenance never blocks the measurement
        return {"error": repr(e)}


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons, power = [], [], set(), []
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [s for s, p in zip(sm, power) if p > 200] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power)}


def main():
    args = parse()
    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": REFERENCE_UNAVAILABLE}))
        return 0

    import torch
    import torch.distributed as dist

    from qwen38_b200.checkpoint import random_drafter_source, random_target_source
    from qwen38_b200.config import (RuntimeConfig, full_drafter_config, full_model_config, tiny_drafter_config,
                                    tiny_model_config)
    from qwen38_b200.models.drafter import BlockDrafter
    from qwen38_b200.models.target import HybridTarget
    from qwen38_b200.ops import TorchOps
    from qwen38_b200.parallel.comm import init_distributed, make_comm
    from qwen38_b200.spec.engine import PinnedAcceptance, SpecRuntime, greedy_reference

    rank, world, local = init_distributed()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    comm = None

    if args.model == "full":
        cfg, dcfg = full_model_config(), full_drafter_config()
    else:
        cfg, dcfg = tiny_model_config(), tiny_drafter_config()
        dcfg.block_rows = 16
    if args.layers:
        from qwen38_b200.config import ModelConfig
        cfg = ModelConfig(**{**cfg.__dict__, "num_hidden_layers": args.layers,
                             "layer_types": cfg.layer_types[:args.layers]})
        dcfg.taps = [t for t in dcfg.taps if t < args.layers] or [args.layers - 1]
    from qwen38_b200.parallel.plan import check_tp_plan
    bad = check_tp_plan(cfg, dcfg, world)
    if bad:
        raise SystemExit(f"TP={world} cannot run this shape: " + "; ".join(bad))
    topo = None
    if world > 1:
        from qwen38_b200.parallel.topology import check_topology
        topo = check_topology(world, comm=args.comm if args.ops == "native" else "nccl")
    comm = make_comm(world, device=device, hidden=cfg.hidden_size, peer=(args.comm != "nccl" and args.ops == "native"),
                     fused=(args.comm == "fused"), prefill_rows=args.prefill_chunk if args.comm == "fused" else 0)
    # the library op set reads positions on the host inside attention, which a CUDA graph cannot
    # capture: it runs eagerly
    rt = RuntimeConfig(max_context=args.ctx + args.new_tokens + 64, prefill_chunk=args.prefill_chunk,
                       use_cuda_graphs=not args.no_graphs and args.ops == "native")
    if args.ops == "native":
        from qwen38_b200.ops.native import NativeOps
        ops = NativeOps(device=device, max_keys=rt.max_context + 64, weight_format=args.weights)
    else:
        ops = TorchOps()
    t_load = time.time()
    tsrc = random_target_source(cfg, args.seed)
    if args.weights == "mxfp8":
        from qwen38_b200.checkpoint import MXFP8Source
        tsrc = MXFP8Source(tsrc)
    tgt = HybridTarget(cfg, tsrc, rt, device=device, dtype=torch.bfloat16, ops=ops, comm=comm)
    if args.drafter == "dflash2":
        import dataclasses
        from qwen38_b200.checkpoint import random_window_drafter_source
        from qwen38_b200.config import WindowDrafterConfig, tiny_window_drafter_config
        from qwen38_b200.models.window_drafter import WindowDrafter
        wcfg = WindowDrafterConfig() if args.model == "full" else tiny_window_drafter_config()
        dcfg = dataclasses.replace(wcfg, block_rows=dcfg.block_rows, taps=dcfg.taps)
        dr = WindowDrafter(dcfg, random_window_drafter_source(dcfg, cfg.vocab_size, args.seed + 3), tgt)
    else:
        dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, args.seed + 1), tgt)
    torch.cuda.synchronize()
    t_load = time.time() - t_load

    g = torch.Generator().manual_seed(args.seed)
    prompt = torch.randint(0, cfg.vocab_size, (args.ctx,), generator=g)
    prompt_host = prompt.pin_memory()
    n_out = args.new_tokens + 1                      # the prefill seed + committed decode tokens
    t_gold = time.time()
    if args.temperature > 0:
        gold = tgt.sample(prompt.to(device), n_out, temperature=args.temperature, seed=args.seed)
    else:
        gold = greedy_reference(tgt, prompt.tolist(), n_out)
    torch.cuda.synchronize()
    t_gold = time.time() - t_gold
    sr = SpecRuntime(tgt, dr, verifier_rows=dcfg.block_rows)
    # token-exactness against greedy decode rests on batch-invariant kernels; the library op set
    # (cuBLAS) is not batch-invariant, so its speculative output is not checked against greedy
    exact = args.ops == "native"

    def one(step, timed):
        sr.h2d_bytes = sr.d2h_bytes = 0
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        res = sr.generate(prompt_host, n_out, pinned=PinnedAcceptance(gold, seed=1000 + step,
                                                                     mean_accepted=args.mean_accepted),
                          gold_check=gold if exact else None, prompt_host=prompt_host,
                          **({"temperature": args.temperature, "seed": args.seed} if args.temperature > 0 else {}))
        torch.cuda.synchronize()
        wall = time.perf_counter() - w0
        if hasattr(ops, "check"):
            ops.check()
        if hasattr(comm, "check"):
            comm.check()
        if world > 1:
            dist.barrier()
        res["wall_s"] = wall
        res["h2d"], res["d2h"] = sr.h2d_bytes, sr.d2h_bytes
        return res

    for i in range(args.warmup):
        one(i, False)
    sampler = ClockSampler(local)
    if rank == 0:
        sampler.start()
    launches0 = getattr(ops, "launches", 0)
    results = [one(args.warmup + i, True) for i in range(args.steps)]
    launches = getattr(ops, "launches", 0) - launches0
    clocks = sampler.stop() if rank == 0 else None

    pp_ms = sum(r["pp_ms"] for r in results)
    tg_ms = sum(r["tg_ms"] for r in results)
    wall_s = sum(r["wall_s"] for r in results)
    times = torch.tensor([pp_ms, tg_ms, wall_s], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    pp_ms, tg_ms, wall_s = times.tolist()
    # per-step spread (each step's TG time is the max over ranks, like the totals)
    step_tg = torch.tensor([r["tg_ms"] for r in results], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(step_tg, op=dist.ReduceOp.MAX)
    step_tok_s = sorted(r["committed"] / (ms / 1e3) for r, ms in zip(results, step_tg.tolist()))
    step_verify = sorted(r["verify_ms_per_block"] for r in results)
    committed = sum(r["committed"] for r in results)
    prompt_toks = sum(r["prompt_tokens"] for r in results)
    tg = committed / (tg_ms / 1e3)
    pp = prompt_toks / (pp_ms / 1e3)
    e2e_tg = committed / max(1e-9, wall_s - pp_ms / 1e3)
    if rank == 0:
        line = {
            "metric": "committed TG tok/s (1 stream, CTX 4096, pinned acceptance; PP tok/s in pp_tok_s)",
            "value": round(tg, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round((pp_ms + tg_ms) / args.steps, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": round(tg / BASELINE_TG, 3), "dtype": "bf16",
            "data": "synthetic (seeded uniform-random prompt ids, random-init weights of the named shape)",
            "pp_tok_s": round(pp, 2), "pp_vs_baseline": round(pp / BASELINE_PP, 3),
            "config": {"model": f"{args.model}-hybrid-27B-class" if args.model == "full" else "tiny",
                       "layers": cfg.num_hidden_layers, "global_batch": 1, "seq_len": args.ctx,
                       "new_tokens": args.new_tokens, "block_rows": dcfg.block_rows, "prefill_chunk": args.prefill_chunk,
                       "drafter": args.drafter, "drafter_layers": dcfg.num_hidden_layers, "weights": args.weights, "temperature": args.temperature,
                       "parallelism": f"tp{world}",
                       "ops": args.ops, "comm": args.comm if world > 1 else None,
                       "cuda_graphs": tgt.use_graphs, "gold_checked": exact,
                       "deferred_splitk": bool(getattr(tgt, "defer_splits", False)) and world == 1,
                       "nvlinks": (topo or {}).get("nvlink_active_links"),
                       "nvls_push": bool(getattr(comm, "recv_mc", 0)),
                       "prefill_allreduce": "fused (reduce-scatter GEMM + multicast broadcast)"
                       if getattr(comm, "_pf", None) is not None else ("nccl" if world > 1 else None),
                       "mean_accepted_target": args.mean_accepted,
                       "l2": "inputs larger than L2: every step streams all weights (54 GB at TP1)"},
            "mean_accepted": round(statistics.mean(r["mean_accepted"] for r in results), 3),
            "block_ms": {k: round(statistics.mean(r[k + "_ms_per_block"] for r in results), 3)
                         for k in ("draft", "verify", "commit")},
            "tokens_per_block": round(statistics.mean(r["tokens_per_block"] for r in results), 3),
            "step_spread": {"tg_tok_s": [round(step_tok_s[0], 1), round(statistics.median(step_tok_s), 1),
                                         round(step_tok_s[-1], 1)],
                            "verify_ms_per_block": [round(step_verify[0], 3), round(statistics.median(step_verify), 3),
                                                    round(step_verify[-1], 3)],
                            "order": "min, median, max over the timed steps"},
            "clocks": clocks,
            "provenance": {k: v for k, v in _provenance().items() if k in ("sources_sha256", "extension_sha256",
                                                                                 "device", "driver", "torch")},
            "e2e": {"value": round(e2e_tg, 3), "unit": "tok/s (committed TG, host wall clock via "
                    "SpecRuntime.generate)", "h2d_bytes_per_step": results[-1]["h2d"],
                    "d2h_bytes_per_step": results[-1]["d2h"]},
            "gpu_launches": launches,
            "load_s": round(t_load, 1), "gold_s": round(t_gold, 1),
        }
        if args.layers:
            line["invalid"] = "truncated model (--layers); debug only"
        print(json.dumps(line), flush=True)
    # graphs may hold NCCL work: release them before the process group goes away
    sr = None
    dr.release_graphs()
    tgt.release_graphs()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
