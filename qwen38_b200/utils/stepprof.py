"""Per-kernel breakdown of one speculative block (draft, verify, commit) at TP=N.

Builds the benchmark's model (full-size random-init hybrid + 5-layer block drafter, bf16, or the
tiny shape), prefills a seeded prompt, then times each phase of a block on its own:

* ``verify``  - the captured 16-row verify graph replayed ``--iters`` times at one position;
* ``draft``   - the captured propose graph (drafter forward + Markov selector);
* ``commit``  - GDN commit replay of ``--accept`` rows + drafter publication of their features;
* ``prefill`` - a committed prefill of the whole prompt (opt in: ``--phases prefill,...``).

For every phase it reports the CUDA-event time per iteration (max over ranks) and, from a
``torch.profiler`` CUDA activity trace of the same loop, the device time per iteration of every
kernel class on every rank.  With programmatic dependent launch on (the default) a kernel's span
includes the time its CTAs sat at ``griddepcontrol.wait`` for the previous kernel, so class sums
overlap; ``Q38_PDL=0`` gives disjoint spans whose sum plus the idle gaps is the phase time.  A
pushed all-reduce's wait for the slowest rank shows up in ``rms_norm_ar_kernel``'s span.

The profiler's numbers explain shares; the phase times are plain CUDA-event timings taken outside
the profiler.  The reference breaks its block down the same way (draft / verify / select ms per
block, ``docs/200tg-latency-budget.md:9-11``) with the Tracy device profiler per op
(``docs/trace-op-attribution.md``).

    python -m qwen38_b200.utils.stepprof --iters 20 --out gpurun_out/prof_tp1.json
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m qwen38_b200.utils.stepprof --iters 20
"""
from __future__ import annotations

import argparse
import json
import re
from collections import defaultdict

import torch

_EPI = {"0": "bf16", "1": "f32", "2": "add", "3": "swiglu", "4": "argmax", "5": "push"}


def kernel_class(name: str) -> str:
    """Short class name of a demangled kernel name (template arguments kept where they pick the
    role, e.g. the GEMM's epilogue and swap/prefill mode)."""
    n = name.replace("void ", "").replace("q38::", "").replace("(anonymous namespace)::", "")
    n = n.split("(")[0].strip()
    m = re.match(r"gemm_tn_kernel<(\d+), (\d+), (\d+), (true|false)>", n)
    if m:
        mode = "swap" if m.group(4) == "true" else "tile"
        return f"gemm[{mode},{_EPI.get(m.group(3), m.group(3))}]"
    m = re.match(r"([A-Za-z_0-9:]+)<", n)
    if m:
        return m.group(1)
    return n[:80]


def profile_loop(fn, iters: int):
    """(ms per iteration by CUDA events, {class: [count, device us]} per iteration, span stats)."""
    fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / iters
    classes = defaultdict(lambda: [0, 0.0])
    busy = None
    try:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(iters):
                fn()
            torch.cuda.synchronize()
        spans = []
        for ev in prof.events():
            if getattr(ev, "device_type", None) != torch.autograd.DeviceType.CUDA:
                continue
            nm = ev.name
            if nm.startswith(("Memcpy", "Memset", "cudaGraph")):
                cls = nm.split(" ")[0]
            else:
                cls = kernel_class(nm)
            t0, t1 = ev.time_range.start, ev.time_range.end
            classes[cls][0] += 1
            classes[cls][1] += (t1 - t0)
            spans.append((t0, t1))
        if spans:
            spans.sort()
            union, cur0, cur1 = 0.0, spans[0][0], spans[0][1]
            for a, b in spans[1:]:
                if a > cur1:
                    union += cur1 - cur0
                    cur0, cur1 = a, b
                else:
                    cur1 = max(cur1, b)
            union += cur1 - cur0
            busy = union / iters
    except Exception as ex:          # a profiler problem never hides the event timings
        classes["profiler_error: " + repr(ex)[:120]] = [0, 0.0]
    per_iter = {k: [v[0] / iters, v[1] / iters] for k, v in classes.items()}
    return ms, per_iter, busy


def main():
    from ..checkpoint import random_drafter_source, random_target_source
    from ..config import RuntimeConfig, full_drafter_config, full_model_config, tiny_drafter_config, tiny_model_config
    from ..models.drafter import BlockDrafter
    from ..models.target import HybridTarget
    from ..parallel.comm import init_distributed, make_comm

    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="full", choices=["full", "tiny"])
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--rows", type=int, default=16)
    ap.add_argument("--accept", type=int, default=7, help="rows committed per block in the commit phase")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--comm", default="fused", choices=["fused", "peer", "nccl"])
    ap.add_argument("--phases", default="verify,draft,commit")
    ap.add_argument("--out", default="")
    a = ap.parse_args()

    rank, world, local = init_distributed()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg, dcfg = (full_model_config(), full_drafter_config()) if a.model == "full" else \
        (tiny_model_config(), tiny_drafter_config())
    dcfg.block_rows = a.rows
    from ..ops.native import NativeOps
    max_ctx = a.ctx + a.iters * a.accept * 4 + 256
    rt = RuntimeConfig(max_context=max_ctx, prefill_chunk=min(4096, a.ctx))
    ops = NativeOps(device=dev, max_keys=max_ctx + 64)
    comm = make_comm(world, device=dev, hidden=cfg.hidden_size, peer=a.comm != "nccl", fused=a.comm == "fused",
                     prefill_rows=rt.prefill_chunk if a.comm == "fused" else 0)
    tgt = HybridTarget(cfg, random_target_source(cfg, 0), rt, device=dev, dtype=torch.bfloat16, ops=ops, comm=comm,
                       max_slots=2)
    dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, 1), tgt, max_context=max_ctx)
    taps = tuple(dcfg.taps)

    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (a.ctx,), generator=g).to(dev)
    seq = tgt.new_sequence()
    nxt, feats = tgt.prefill(seq, prompt, taps=taps)
    dr.append(feats, 0)
    anchor = nxt.reshape(1).clone()
    block = torch.randint(0, cfg.vocab_size, (a.rows,), generator=g).to(dev)
    torch.cuda.synchronize()

    out = {"tp": world, "rank": rank, "ctx": a.ctx, "rows": a.rows, "iters": a.iters, "phases": {}}
    phases = a.phases.split(",")
    state = {}

    def verify():
        state["pred"], state["feats"] = tgt.verify([(seq, block)], taps=taps)

    def draft():
        dr.propose(anchor)

    def commit():
        tgt.commit(seq, a.accept)
        dr.append(state["feats"][:a.accept], dr.position)
        seq.verify_rows = (0, a.rows)                   # the next iteration commits the same stash

    if "prefill" in phases:
        # one committed prefill of the whole prompt on a second slot-free sequence each time
        def prefill():
            sq = tgt.new_sequence()
            try:
                tgt.prefill(sq, prompt, taps=taps)
            finally:
                tgt.release(sq)
        out["phases"]["prefill"] = profile_loop(prefill, max(1, a.iters // 10))
    if "verify" in phases:
        out["phases"]["verify"] = profile_loop(verify, a.iters)
    if "draft" in phases:
        out["phases"]["draft"] = profile_loop(draft, a.iters)
    if "commit" in phases:
        verify()
        torch.cuda.synchronize()
        out["phases"]["commit"] = profile_loop(commit, a.iters)
    if hasattr(ops, "check"):
        ops.check()
    if hasattr(comm, "check"):
        comm.check()

    allr = [out]
    if world > 1:
        import torch.distributed as dist
        allr = [None] * world
        dist.all_gather_object(allr, out)
    if rank == 0:
        summary = {"tp": world, "ctx": a.ctx, "rows": a.rows, "iters": a.iters,
                   "nvls_push": bool(getattr(comm, "recv_mc", 0)), "phases": {}}
        for ph in out["phases"]:
            ms = max(r["phases"][ph][0] for r in allr)
            busy = [r["phases"][ph][2] for r in allr]
            classes = sorted({c for r in allr for c in r["phases"][ph][1]})
            rows = {}
            for c in classes:
                per = [r["phases"][ph][1].get(c, [0, 0.0]) for r in allr]
                rows[c] = {"count": round(per[0][0], 2), "us_max": round(max(p[1] for p in per), 1),
                           "us_min": round(min(p[1] for p in per), 1)}
            rows = dict(sorted(rows.items(), key=lambda kv: -kv[1]["us_max"]))
            summary["phases"][ph] = {"ms_per_iter": round(ms, 3),
                                     "busy_us_per_iter": [round(b, 1) if b else None for b in busy],
                                     "kernels": rows}
        print(json.dumps(summary), flush=True)
        if a.out:
            with open(a.out, "w") as f:
                json.dump(summary, f, indent=1)
    dr.release_graphs()
    tgt.release_graphs()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
