"""Collective micro-benchmark: time per message size, bus bandwidth, and the fixed cost per call.

The reference measured its fabric this way (all-gather 83.74 GB/s at 42 MB and a ~10 us fixed
cost per collective from a linear fit, ``docs/fabric-bandwidth-2026-09-19.md:18-21``; ABBA-ordered
A/B comparisons, ``optimisation/fabric-relay/README.md:41-46``).  Here the same figures come from
the process group's own collectives (``dist``: NCCL over NVLink / NVSwitch on B200, gloo on CPU)
and, on GPUs, from the peer-memory all-reduce kernel the runtime uses for decode-sized messages
(``peer``: ``SymmComm.all_reduce_`` on fp32 ``[rows <= 32, hidden]``).

* Every (op, size) is timed for each implementation in ABBA order (A B B A A B B A ...) so a slow
  drift of clocks or of a neighbour's load lands on both arms equally.
* A time is the max over ranks of the per-rank time (CUDA events on the launching stream on GPUs,
  a host clock on CPU), after warm-up; the median over repetitions is reported.
* ``bus_gbs`` follows the usual convention: all-reduce moves 2 (n-1)/n of the message per rank,
  all-gather (n-1)/n of the gathered output.
* ``fit`` regresses time = t0 + bytes / bandwidth over the sizes of one (op, impl): t0 is the fixed
  cost of a call, bandwidth the asymptote.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m qwen38_b200.utils.commbench \\
        --ops all_reduce all_gather --impls dist peer --out comm.json
"""
from __future__ import annotations

import argparse
import json
import statistics
import time

import torch
import torch.distributed as dist


def abba(reps: int, arms: list) -> list:
    """Order of arm runs: A B B A A B B A ... (for two arms); more arms rotate the same way."""
    order = []
    for r in range(reps):
        order.extend(arms if r % 2 == 0 else list(reversed(arms)))
    return order


def fit_line(points) -> dict:
    """Least squares time_s = t0 + bytes / bw over ``points`` [(bytes, seconds)]."""
    n = len(points)
    if n < 2:
        raise ValueError("two or more sizes are needed for a fit")
    xs = [float(b) for b, _ in points]
    ys = [float(t) for _, t in points]
    mx, my = sum(xs) / n, sum(ys) / n
    sxx = sum((x - mx) ** 2 for x in xs)
    if sxx == 0:
        raise ValueError("sizes must differ")
    slope = sum((x - mx) * (y - my) for x, y in zip(xs, ys)) / sxx
    t0 = my - slope * mx
    return {"t0_us": t0 * 1e6, "bw_gbs": (1.0 / slope / 1e9) if slope > 0 else None}


def bus_factor(op: str, world: int) -> float:
    if op == "all_reduce":
        return 2.0 * (world - 1) / world
    if op == "all_gather":
        return (world - 1) / world
    raise ValueError(op)


class _Timer:
    def __init__(self, device):
        self.cuda = device.type == "cuda"

    def start(self):
        if self.cuda:
            self.a = torch.cuda.Event(enable_timing=True)
            self.b = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            self.a.record()
        else:
            self.t = time.perf_counter()

    def stop(self) -> float:
        if self.cuda:
            self.b.record()
            self.b.synchronize()
            return self.a.elapsed_time(self.b) / 1e3
        return time.perf_counter() - self.t


def _make_call(op, impl, numel, device, world, comm=None, hidden=0):
    if impl == "peer":
        rows = numel // hidden
        t = torch.ones(rows, hidden, dtype=torch.float32, device=device)
        return (lambda: comm.all_reduce_(t)), rows * hidden * 4
    t = torch.ones(numel, dtype=torch.float32, device=device)
    if op == "all_reduce":
        return (lambda: dist.all_reduce(t)), numel * 4
    out = [torch.empty_like(t) for _ in range(world)]
    return (lambda: dist.all_gather(out, t)), numel * 4 * world


def run(ops, impls, sizes, *, reps=10, warmup=3, calls=10, device=None, comm=None, hidden=0):
    """Returns {"results": [...], "fits": [...]} (identical on every rank)."""
    world = dist.get_world_size()
    device = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    timer = _Timer(device)
    sync_dev = device if dist.get_backend() == "nccl" else torch.device("cpu")
    results = []
    for op in ops:
        for numel in sizes:
            arms = [i for i in impls if i != "peer" or (op == "all_reduce" and comm is not None and hidden
                                                         and numel % hidden == 0 and comm.fits(numel // hidden, hidden))]
            fns = {i: _make_call(op, i, numel, device, world, comm, hidden) for i in arms}
            for i in arms:
                for _ in range(warmup):
                    fns[i][0]()
            times = {i: [] for i in arms}
            for i in abba(reps, arms):
                dist.barrier()
                timer.start()
                for _ in range(calls):
                    fns[i][0]()
                dt = torch.tensor([timer.stop() / calls], dtype=torch.float64, device=sync_dev)
                dist.all_reduce(dt, op=dist.ReduceOp.MAX)       # max over ranks
                times[i].append(float(dt.item()))
            for i in arms:
                med = statistics.median(times[i])
                nbytes = fns[i][1]
                results.append({"op": op, "impl": i, "bytes": nbytes, "median_us": med * 1e6,
                                "alg_gbs": nbytes / med / 1e9, "bus_gbs": nbytes / med / 1e9 * bus_factor(op, world)})
    fits = []
    for op in ops:
        for i in impls:
            pts = [(r["bytes"], r["median_us"] / 1e6) for r in results if r["op"] == op and r["impl"] == i]
            if len(pts) >= 2 and len({b for b, _ in pts}) >= 2:
                fits.append({"op": op, "impl": i, **fit_line(pts)})
    return {"world": world, "backend": dist.get_backend(), "device": device.type, "reps": reps,
            "calls_per_rep": calls, "results": results, "fits": fits}


def main(argv=None):
    from ..parallel.comm import init_distributed
    ap = argparse.ArgumentParser(description="collective micro-benchmark (ABBA-ordered, max over ranks)")
    ap.add_argument("--ops", nargs="+", default=["all_reduce", "all_gather"], choices=["all_reduce", "all_gather"])
    ap.add_argument("--impls", nargs="+", default=["dist"], choices=["dist", "peer"],
                    help="dist: the process group's collective (NCCL on GPUs); peer: the peer-memory all-reduce")
    ap.add_argument("--sizes", nargs="+", type=int,
                    default=[5120, 16 * 5120, 32 * 5120, 1 << 20, 1 << 24, 1 << 26], help="fp32 elements per rank")
    ap.add_argument("--hidden", type=int, default=5120, help="row width of the peer all-reduce")
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    rank, world, local = init_distributed()
    if world < 2:
        raise SystemExit("run under torchrun with two or more ranks")
    comm = None
    if "peer" in a.impls and torch.cuda.is_available():
        from ..parallel.symm import SymmComm
        comm = SymmComm(torch.device("cuda", local), a.hidden, fused=False)
    rep = run(a.ops, a.impls, a.sizes, reps=a.reps, comm=comm, hidden=a.hidden)
    if rank == 0:
        print(json.dumps(rep))
        if a.out:
            with open(a.out, "w") as f:
                json.dump(rep, f, indent=1)
    if comm is not None:
        comm.close()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
