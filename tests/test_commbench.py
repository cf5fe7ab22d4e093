"""Collective micro-benchmark harness on gloo ranks: ABBA ordering, the fixed-cost / bandwidth fit,
and a two-rank run whose report is the same on every rank."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from qwen38_b200.utils.commbench import abba, bus_factor, fit_line


def test_abba_order_and_bus_factors():
    assert abba(4, ["A", "B"]) == list("ABBAABBA")
    assert abba(1, ["A"]) == ["A"]
    assert bus_factor("all_reduce", 8) == 1.75 and bus_factor("all_gather", 4) == 0.75
    with pytest.raises(ValueError):
        bus_factor("broadcast", 2)


def test_fit_recovers_fixed_cost_and_bandwidth():
    pts = [(b, 10e-6 + b / 700e9) for b in (1 << 10, 1 << 20, 1 << 26, 1 << 28)]
    f = fit_line(pts)
    assert abs(f["t0_us"] - 10.0) < 1e-6 and abs(f["bw_gbs"] - 700.0) < 1e-6
    with pytest.raises(ValueError):
        fit_line([(1, 1.0)])


def _rank(rank, port, q):
    import torch.distributed as dist
    from qwen38_b200.utils.commbench import run
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        q.put((rank, run(["all_reduce", "all_gather"], ["dist", "peer"], [256, 4096], reps=2, warmup=1, calls=2,
                         device="cpu")))
    except BaseException as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_two_rank_run():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted((q.get(timeout=120) for _ in procs), key=lambda x: x[0])
    for p in procs:
        p.join(timeout=30)
    reps = [r for _, r in out]
    assert all(isinstance(r, dict) for r in reps), reps
    r0 = reps[0]
    assert r0["world"] == 2 and r0["backend"] == "gloo"
    assert {(x["op"], x["impl"]) for x in r0["results"]} == {("all_reduce", "dist"), ("all_gather", "dist")}
    assert {x["op"] for x in r0["fits"]} == {"all_reduce", "all_gather"}
    ag = [x for x in r0["results"] if x["op"] == "all_gather"]
    assert sorted(x["bytes"] for x in ag) == [256 * 4 * 2, 4096 * 4 * 2]
    # the timings are maxima over ranks, so both ranks report the same numbers
    assert [x["median_us"] for x in reps[0]["results"]] == [x["median_us"] for x in reps[1]["results"]]
