"""Endpoint isolation gate: greedy outputs streamed through the OpenAI endpoint are the same whether
a request runs alone or next to others, and the server interleaves a long prefill with running
decodes.

Parity with the reference's rig gate (``optimisation/rig/interleave_bench.py:80-117``): every
prompt is first streamed alone (the baseline); then B decoders stream concurrently, a long prompt A
is injected once every decoder is streaming, and a short prompt C follows after ``short_delay``.
Checks: each prompt's streamed token ids equal its baseline; every decoder is still streaming after
A's first token (the long prefill did not stall the decoders until they finished); C was submitted
before A's first token (it waited behind a prefill in progress).  Timing (TTFT, decode tok/s, event
gaps) is client-observed; an event can carry several tokens (a speculative block), so event gaps are
not per-token latency.

Prompts are token ids below 256 (valid for every vocabulary here; no tokenizer download).

    python -m qwen38_b200.serving.isolation --base-url http://127.0.0.1:8000 --output gate.json
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import threading
import time
import urllib.request
from concurrent.futures import ThreadPoolExecutor


def quantile(values, fraction):
    ordered = sorted(values)
    return ordered[max(0, math.ceil(len(ordered) * fraction) - 1)] if ordered else None


def stream(base_url, model, prompt, count, ready=None, timeout=1800.0):
    """Stream one greedy completion of ``count`` tokens; returns token ids, text and event times."""
    payload = dict(model=model, prompt=list(prompt), max_tokens=count, temperature=0.0, stream=True,
                   stream_options={"include_usage": True}, seed=123)
    req = urllib.request.Request(base_url.rstrip("/") + "/v1/completions", json.dumps(payload).encode(),
                                 {"Content-Type": "application/json"})
    started = time.perf_counter()
    events, tokens, text, usage, done = [], [], [], None, False
    with urllib.request.urlopen(req, timeout=timeout) as resp:
        for raw in resp:
            line = raw.decode("utf-8").strip()
            if not line.startswith("data:"):
                continue
            data = line[5:].strip()
            if data == "[DONE]":
                done = True
                break
            msg = json.loads(data)
            if "error" in msg:
                raise RuntimeError(msg["error"])
            usage = msg.get("usage") or usage
            for choice in msg.get("choices", []):
                if choice.get("index", 0) != 0:
                    raise RuntimeError("expected exactly one completion")
                ids = choice.get("token_ids") or []
                if any(type(t) is not int or t < 0 for t in ids):
                    raise ValueError("invalid streamed token ids")
                text.append(choice.get("text", ""))
                if ids:
                    events.append((time.perf_counter(), len(ids)))
                    tokens.extend(ids)
                    if ready is not None:
                        ready.set()
    if (not done or len(tokens) != count or not events or usage is None
            or usage.get("completion_tokens") != count or usage.get("prompt_tokens") != len(prompt)):
        raise RuntimeError(f"incomplete stream or token accounting: done={done} tokens={len(tokens)} "
                           f"expected={count} usage={usage}")
    gaps = [b[0] - a[0] for a, b in zip(events, events[1:])]
    span = events[-1][0] - events[0][0]
    joined = "".join(text)
    return dict(tokens=tokens, text_sha256=hashlib.sha256(joined.encode()).hexdigest(), started=started,
                first=events[0][0], last=events[-1][0], events=len(events), ttft_s=events[0][0] - started,
                decode_tok_s=(len(tokens) - events[0][1]) / span if span > 0 else None,
                event_gap_p99_s=quantile(gaps, 0.99), event_gap_max_s=max(gaps) if gaps else None,
                coalesced_events=sum(n > 1 for _, n in events))


def _wait_ready(futures, flags, timeout):
    deadline = time.monotonic() + timeout
    while not all(f.is_set() for f in flags):
        for fut in futures:
            if fut.done():
                fut.result()
                raise RuntimeError("a decoder ended before every decoder was streaming")
        if time.monotonic() >= deadline:
            raise TimeoutError("decoders did not start streaming")
        time.sleep(0.01)


def make_prompts(prompt_length: int, decoders: int):
    unit = [(7 * i + 3) % 250 + 3 for i in range(37)]
    prompts = {f"B{i}": [(11 * i + 5 * j + 1) % 250 + 3 for j in range(24 + 3 * i)] for i in range(decoders)}
    prompts["A"] = (unit * math.ceil(prompt_length / len(unit)))[:prompt_length]
    prompts["C"] = [(13 * j + 9) % 250 + 3 for j in range(16)]
    return prompts


def measure(base_url, model="qwen38-hybrid", prompt_length=2049, decoders=1, decode_tokens=512, short_delay=0.1,
            ready_timeout=1800.0, short_tokens=32):
    prompts = make_prompts(prompt_length, decoders)
    counts = {name: decode_tokens if name.startswith("B") else short_tokens for name in prompts}
    stream(base_url, model, prompts["C"], 8)                  # warm-up
    baseline = {name: stream(base_url, model, p, counts[name]) for name, p in prompts.items()}
    concurrent = {}
    with ThreadPoolExecutor(max_workers=decoders + 2) as pool:
        flags = [threading.Event() for _ in range(decoders)]
        futs = [pool.submit(stream, base_url, model, prompts[f"B{i}"], counts[f"B{i}"], flags[i])
                for i in range(decoders)]
        _wait_ready(futs, flags, ready_timeout)
        if any(f.done() for f in futs):
            raise RuntimeError("a decoder finished before the long prompt was injected")
        injected = time.perf_counter()
        long_req = pool.submit(stream, base_url, model, prompts["A"], counts["A"])
        time.sleep(short_delay)
        short_req = pool.submit(stream, base_url, model, prompts["C"], counts["C"])
        for i, fut in enumerate(futs):
            concurrent[f"B{i}"] = fut.result()
        concurrent["A"], concurrent["C"] = long_req.result(), short_req.result()
    checks = {f"greedy_equal_{n}": baseline[n]["tokens"] == concurrent[n]["tokens"]
              and baseline[n]["text_sha256"] == concurrent[n]["text_sha256"] for n in prompts}
    checks["decoders_overlap_long_prefill"] = all(
        r["last"] > concurrent["A"]["first"] for n, r in concurrent.items() if n.startswith("B"))
    checks["short_arrives_before_long_first_token"] = concurrent["C"]["started"] < concurrent["A"]["first"]
    return dict(passed=all(checks.values()), checks=checks, prompt_length=prompt_length, decoders=decoders,
                injected=injected, baseline=baseline, concurrent=concurrent,
                timing_scope="client-observed; one event can carry a whole speculative block")


def main(argv=None):
    ap = argparse.ArgumentParser(description="OpenAI endpoint isolation / interleaving gate")
    ap.add_argument("--base-url", default="http://127.0.0.1:8000")
    ap.add_argument("--model", default="qwen38-hybrid")
    ap.add_argument("--prompt-length", type=int, default=2049)
    ap.add_argument("--decoders", type=int, default=1)
    ap.add_argument("--decode-tokens", type=int, default=512)
    ap.add_argument("--short-delay", type=float, default=0.1)
    ap.add_argument("--ready-timeout", type=float, default=1800.0)
    ap.add_argument("--output", required=True)
    a = ap.parse_args(argv)
    if a.prompt_length < 1 or a.decode_tokens < 2 or a.short_delay < 0 or a.decoders < 1:
        ap.error("positive prompt length and decoders, at least two decode tokens, non-negative delay")
    report = dict(passed=False)
    try:
        report = measure(a.base_url, a.model, a.prompt_length, a.decoders, a.decode_tokens, a.short_delay,
                         a.ready_timeout)
    except Exception as e:
        report["error"] = f"{type(e).__name__}: {e}"
        raise
    finally:
        with open(a.output, "w") as f:
            json.dump(report, f, indent=1)
    print(json.dumps({k: v for k, v in report.items() if k not in ("baseline", "concurrent")}, indent=1))
    return 0 if report["passed"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
