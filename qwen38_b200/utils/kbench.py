"""Kernel micro-benchmarks with roofline fractions.

Times one native kernel in isolation with CUDA events on the launching stream (warm-up, an L2
flush of 256 MB between timed iterations, synchronise on both sides) and reports the achieved
bandwidth / throughput against the measured peaks (``MEASURED_PEAKS.json`` at the repo root;
6.65 TB/s and 1.59 PFLOP/s as fallback).

    python -m qwen38_b200.utils.kbench gemm --T 16 --N 5120 --K 17408
    python -m qwen38_b200.utils.kbench gemm --T 4096 --N 34816 --K 5120 --epi swiglu
    python -m qwen38_b200.utils.kbench gdn --T 16 --nv 48
    python -m qwen38_b200.utils.kbench gdnpf --T 2048 --nv 48
    python -m qwen38_b200.utils.kbench attn --T 16 --ctx 4096
    python -m qwen38_b200.utils.kbench markov --V 151936 --R 256 --P 15
"""
from __future__ import annotations

import argparse
import json
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def time_kernel(fn, iters=20, warmup=3, flush=True):
    flush_buf = torch.empty(64 << 20, dtype=torch.float32, device="cuda") if flush else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush_buf is not None:
            flush_buf.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def bench_gemm(a):
    from ..ops.native import EPI_ADD_F32, EPI_BF16, EPI_SWIGLU, MXWeight, NativeOps
    ops = NativeOps(weight_format="mxfp8" if a.mx else "bf16")
    x = torch.randn(a.T, a.K, device="cuda").to(torch.bfloat16)
    w_plain = (torch.randn(a.N, a.K, device="cuda") * 0.02).to(torch.bfloat16)
    if a.mx:                                     # an MXFP8 weight: its exact bf16 expansion
        from ..checkpoint import dequant_mxfp8, quant_mxfp8
        w_plain = dequant_mxfp8(*quant_mxfp8(w_plain.float())).to(torch.bfloat16)
    w = ops.prepare_weight(w_plain)              # tile-contiguous storage, done once at load time
    if a.mx and not isinstance(w, MXWeight):
        raise SystemExit("weight did not convert to MXFP8")
    if a.epi == "swiglu":
        fn = lambda: ops.linear_swiglu(x, w, 64)
    elif a.epi == "add":
        res = torch.zeros(a.T, a.N, device="cuda")
        fn = lambda: ops.linear_residual(x, w, res)
    else:
        fn = lambda: ops.linear(x, w)
    if a.iters == 0:            # single launch (profiler captures)
        fn()
        torch.cuda.synchronize()
        ops.check()
        return {}
    ms = time_kernel(fn, a.iters)
    ops.check()
    hbm, tf, src = peaks()
    flops = 2.0 * a.T * a.N * a.K
    wb = a.N * a.K * (1 + 1 / 32) if a.mx else a.N * a.K * 2
    bytes_ = wb + a.T * a.K * 2 + a.T * a.N * (2 if a.epi != "add" else 8)
    out = {"kernel": "gemm_mx" if a.mx else "gemm", "T": a.T, "N": a.N, "K": a.K, "epi": a.epi, "ms": round(ms, 4),
           "tflops": round(flops / ms / 1e9, 1), "gbs": round(bytes_ / ms / 1e6, 1)}
    out[f"frac_bw_of_{src}"] = round(bytes_ / ms / 1e6 / hbm, 3)
    out[f"frac_tc_of_{src}"] = round(flops / ms / 1e9 / tf, 3)
    if a.graph:
        out.update(gemm_graph(ops, x, w_plain, a))
    if a.trace:
        out["trace"] = gemm_trace(ops, x, w, a.epi)
    if a.compare:
        ref = lambda: x @ w_plain.t()
        out["cublas_ms"] = round(time_kernel(ref, a.iters), 4)
    if a.mx:                                     # the same GEMM over the bf16 weight: same bits
        bops = NativeOps()
        wb16 = bops.prepare_weight(w_plain)
        y_mx = ops.linear(x, w, out_dtype=torch.float32)
        y_bf = bops.linear(x, wb16, out_dtype=torch.float32)
        out["bits_equal_bf16_weight"] = bool(torch.equal(y_mx, y_bf))
        out["bf16_weight_ms"] = round(time_kernel(lambda: bops.linear(x, wb16), a.iters), 4)
    return out


def gemm_graph(ops, x, w_plain, a):
    """Per-GEMM time when ``a.graph`` launches run back to back inside one CUDA graph (the verify
    setting: no host launch gaps), cycling over enough weight copies that no launch reads a
    weight another left in L2."""
    wbytes = int(w_plain.numel() * ((1 + 1 / 32) if a.mx else 2))
    copies = max(1, -(-3 * 126 * 2 ** 20 // wbytes))
    ws = [ops.prepare_weight(w_plain.clone()) for _ in range(copies)]
    if a.epi == "swiglu":
        calls = [lambda w=w: ops.linear_swiglu(x, w, 64) for w in ws]
    elif a.epi == "add":
        res = torch.zeros(a.T, a.N, device="cuda")
        calls = [lambda w=w: ops.linear_residual(x, w, res) for w in ws]
    else:
        out = torch.empty(a.T, a.N, dtype=torch.bfloat16, device="cuda")
        calls = [lambda w=w: ops.linear(x, w, out=out) for w in ws]
    for f in calls:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(a.graph):
            calls[i % copies]()
    g.replay()
    torch.cuda.synchronize()
    ms = []
    for _ in range(5):
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        g.replay()
        e0.record()
        torch.cuda.synchronize()
        ms.append(s0.elapsed_time(e0) / a.graph)
    ms.sort()
    hbm, _, src = peaks()
    per = ms[len(ms) // 2]
    return {"graph_launches": a.graph, "weight_copies": copies, "graph_ms_per_call": round(per, 4),
            f"graph_frac_bw_of_{src}": round(wbytes / per / 1e6 / hbm, 3)}


def gemm_trace(ops, x, w, epi):
    """One launch with per-CTA %globaltimer stamps: where a GEMM's time goes (launch skew, setup,
    first TMA round trip, streaming, epilogue, split-K fix-up) in microseconds."""
    from ..ops.native import EPI_ADD_F32, EPI_BF16, EPI_SWIGLU, MXWeight
    T = x.shape[0]
    mx = isinstance(w, MXWeight)
    code = {"bf16": EPI_BF16, "add": EPI_ADD_F32, "swiglu": EPI_SWIGLU}[epi]
    N = w.N
    if epi == "swiglu":
        out = torch.empty(T, N // 2, dtype=torch.bfloat16, device="cuda")
    elif epi == "add":
        out = torch.zeros(T, N, device="cuda")
    else:
        out = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
    kb = -(-x.shape[1] // 64)
    tiles = -(-N // 128) * -(-T // 32) if T <= 64 else -(-T // 128) * -(-N // 256)
    tr = torch.zeros(tiles * kb * (12 if mx else 8), dtype=torch.int64, device="cuda")
    torch.empty(64 << 20, dtype=torch.float32, device="cuda").zero_()     # cold L2
    torch.cuda.synchronize()
    grid = ops.C.linear_trace(x, w.q if mx else w.t, N, out, code, ops.ws, ops.counters, ops.err, tr,
                              w.s if mx else None)
    torch.cuda.synchronize()
    t8 = tr.cpu()
    ctas = grid * ops.C.swap_splits(N, x.shape[1]) if T <= 64 else grid
    extra = {}
    if mx:
        # per CTA cycle totals after the stamps: converter waiting (load, free slot) / converting /
        # publishing (proxy fence, barrier, arrivals), MMA thread waiting for tiles (medians)
        c = t8[ctas * 8:ctas * 12].view(-1, 4).double()
        med = lambda v: int(float(v.median()))
        extra = {"mx_cycles_med": {"conv_wait": med(c[:, 0]), "conv_convert": med(c[:, 1]),
                                   "conv_publish": med(c[:, 2]), "mma_wait_tile": med(c[:, 3])}}
    t = t8[:ctas * 8].view(-1, 8)
    t = t[t[:, 0] > 0].double()
    t0 = t[:, 0].min()
    q = lambda v: [round(float(v.quantile(p)) / 1e3, 2) for p in (0.0, 0.5, 1.0)]
    return {"ctas": int(t.shape[0]), "span_us": round(float(t[:, 7].max() - t0) / 1e3, 2),
            "start_skew_us[min,med,max]": q(t[:, 0] - t0), "setup_us": q(t[:, 1] - t[:, 0]),
            "first_stage_us": q(t[:, 2] - t[:, 1]), "stream_us": q(t[:, 3] - t[:, 2]),
            "mma_drain_us": q(t[:, 4] - t[:, 3]), "epilogue_us": q(t[:, 6] - t[:, 4]),
            "teardown_us": q(t[:, 7] - t[:, 6]), "last_stream_end_us": round(float(t[:, 3].max() - t0) / 1e3, 2),
            **extra}


def bench_gdn(a):
    from ..ops.native import NativeOps
    ops = NativeOps()
    nk, nv, D = a.nv // 3, a.nv, 128
    C = 2 * nk * D + nv * D
    width = -(-(C + nv * D + 2 * nv) // 8) * 8          # the runtime's packed width (16-byte rows)
    proj = torch.randn(a.T, width, device="cuda").to(torch.bfloat16)
    window = torch.randn(3, C, device="cuda").to(torch.bfloat16)
    state = torch.randn(nv, D, D, device="cuda") * 0.1
    conv_w = torch.rand(C, 4, device="cuda") - 0.5
    A_log = torch.rand(nv, device="cuda")
    dt = torch.ones(nv, device="cuda")
    nw = torch.ones(D, device="cuda")
    fn = lambda: ops.gdn_verify(proj, window, state, conv_w, A_log, dt, nw, 1e-6, (nk, nv, D, D), torch.bfloat16)
    if a.iters == 0:
        fn()
        torch.cuda.synchronize()
        return {}
    ms = time_kernel(fn, a.iters)
    bytes_ = state.numel() * 4 + proj.numel() * 2
    hbm, tf, src = peaks()
    out = {"kernel": "gdn_verify", "T": a.T, "nv": nv, "ms": round(ms, 4), "gbs": round(bytes_ / ms / 1e6, 1),
           f"frac_bw_of_{src}": round(bytes_ / ms / 1e6 / hbm, 3)}
    if a.trace:
        # one launch with per-CTA stamps; phases in us from the earliest entry, median / max over CTAs
        tr = torch.zeros(nv * 4 * 8, dtype=torch.int64, device="cuda")
        ops.C.gdn_set_trace(tr)
        torch.cuda.synchronize()
        fn()
        torch.cuda.synchronize()
        ops.C.gdn_set_trace(None)
        t = tr.view(-1, 8).cpu().double()
        t0 = t[:, 0].min()
        names = ["entry", "pdl_wait", "staged", "conv_norms", "recurrence", "cluster_sync", "written", "exit"]
        out["trace_us"] = {n: {"median": round(float((t[:, k] - t0).median()) / 1e3, 2),
                               "max": round(float((t[:, k] - t0).max()) / 1e3, 2)}
                           for k, n in enumerate(names) if bool((t[:, k] > 0).all())}
    return out


def bench_gdn_prefill(a):
    """Chunked GDN prefill of one layer (prep + scan + gated norm) on T rows."""
    from ..ops.native import NativeOps
    ops = NativeOps()
    nk, nv, D = a.nv // 3, a.nv, 128
    C = 2 * nk * D + nv * D
    proj = torch.randn(a.T, C + nv * D + 2 * nv, device="cuda").to(torch.bfloat16)
    window = torch.randn(3, C, device="cuda").to(torch.bfloat16)
    state = torch.randn(nv, D, D, device="cuda") * 0.1
    conv_w = torch.rand(C, 4, device="cuda") - 0.5
    A_log = torch.rand(nv, device="cuda")
    dt = torch.ones(nv, device="cuda")
    nw = torch.ones(D, device="cuda")
    fn = lambda: ops.gdn_prefill(proj, window, state, conv_w, A_log, dt, nw, 1e-6, (nk, nv, D, D), 64,
                                 torch.bfloat16)
    if a.iters == 0:
        fn()
        torch.cuda.synchronize()
        return {}
    ms = time_kernel(fn, a.iters)
    nch = -(-a.T // 64)
    flops = 2.0 * nv * nch * (64 * 64 * D * 2 + 64 * 64 * D * 2 + 64 * D * D * 4 + 64 * 64 * D)
    hbm, tf, src = peaks()
    return {"kernel": "gdn_chunk_prefill", "T": a.T, "nv": nv, "ms": round(ms, 4),
            "tflops": round(flops / ms / 1e9, 1), "us_per_row": round(ms * 1e3 / a.T, 3)}


def bench_markov(a):
    """The drafter's Markov selector over a vocabulary shard of ``--V`` rows, ``--P`` sequential
    steps of rank ``--R``: the one-launch kernel against the per-step two-launch kernels."""
    from ..ops.native import NativeOps
    ops = NativeOps()
    g = torch.Generator(device="cuda").manual_seed(0)
    logits = torch.randn(a.P, a.V, generator=g, device="cuda")
    pred = (torch.randn(a.V, a.R, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    succ = (torch.randn(a.V, a.R, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    anchor = torch.tensor([7], device="cuda")
    fused = lambda: ops.markov_select(logits, anchor, pred, succ)
    if a.iters == 0:
        fused()
        torch.cuda.synchronize()
        ops.check()
        return {}
    prev = anchor.clone()
    steps = torch.empty(a.P, dtype=torch.int64, device="cuda")
    val = torch.empty(1, device="cuda")

    def per_step():
        prev.copy_(anchor)
        for i in range(a.P):
            ops.C.markov_step(logits[i], pred, succ, prev, steps[i:i + 1], val, ops.amax_val, ops.amax_idx, 0, True)
    ms_f = time_kernel(fused, a.iters)
    ms_s = time_kernel(per_step, a.iters)
    ops.check()
    hbm, _, src = peaks()
    bytes_step = a.V * a.R * 2 + a.V * 4
    return {"kernel": "markov_select", "V": a.V, "R": a.R, "P": a.P, "fused_ms": round(ms_f, 4),
            "per_step_kernels_ms": round(ms_s, 4), "fused_us_per_step": round(ms_f * 1e3 / a.P, 2),
            f"fused_frac_bw_of_{src}": round(bytes_step * a.P / ms_f / 1e6 / hbm, 3)}


def bench_attn(a):
    from ..ops.native import NativeOps
    ops = NativeOps(max_keys=a.ctx + 64)
    H, Hkv, D, bs = a.heads, a.kv_heads, 256, 16
    nb = (a.ctx + a.T) // bs + 2
    kc = torch.randn(nb, bs, Hkv, D, device="cuda").to(torch.bfloat16)
    vc = torch.randn(nb, bs, Hkv, D, device="cuda").to(torch.bfloat16)
    bt = torch.arange(nb, dtype=torch.int32, device="cuda")
    q = torch.randn(a.T, H, D, device="cuda").to(torch.bfloat16)
    gate = torch.randn(a.T, H * D, device="cuda").to(torch.bfloat16)
    pos = torch.arange(a.ctx, a.ctx + a.T, dtype=torch.int32, device="cuda")
    fn = lambda: ops.attn_decode(q, gate, kc, vc, bt, pos, bs, torch.bfloat16)
    if a.iters == 0:
        fn()
        torch.cuda.synchronize()
        return {}
    ms = time_kernel(fn, a.iters)
    bytes_ = 2 * (a.ctx + a.T) * Hkv * D * 2
    flops = 4.0 * a.T * H * (a.ctx + a.T) * D
    hbm, tf, src = peaks()
    return {"kernel": "attn_decode", "T": a.T, "ctx": a.ctx, "ms": round(ms, 4), "gbs": round(bytes_ / ms / 1e6, 1),
            "tflops": round(flops / ms / 1e9, 2), f"frac_bw_of_{src}": round(bytes_ / ms / 1e6 / hbm, 3)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kind", choices=["gemm", "gdn", "gdnpf", "attn", "markov"])
    ap.add_argument("--V", type=int, default=151936)
    ap.add_argument("--R", type=int, default=256)
    ap.add_argument("--P", type=int, default=15)
    ap.add_argument("--T", type=int, default=16)
    ap.add_argument("--N", type=int, default=5120)
    ap.add_argument("--K", type=int, default=17408)
    ap.add_argument("--epi", default="bf16", choices=["bf16", "add", "swiglu"])
    ap.add_argument("--nv", type=int, default=48)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--heads", type=int, default=24)
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--compare", action="store_true", help="also time torch/cuBLAS for the same GEMM")
    ap.add_argument("--trace", action="store_true", help="GEMM: per-CTA phase stamps of one launch")
    ap.add_argument("--mx", action="store_true", help="GEMM: MXFP8 weight (e4m3 + E8M0 scales) streamed by the MX kernel")
    ap.add_argument("--graph", type=int, default=0, help="GEMM: time N back-to-back launches in one CUDA graph")
    a = ap.parse_args()
    out = {"gemm": bench_gemm, "gdn": bench_gdn, "gdnpf": bench_gdn_prefill, "attn": bench_attn,
           "markov": bench_markov}[a.kind](a)
    if out:
        print(json.dumps(out))


if __name__ == "__main__":
    main()
