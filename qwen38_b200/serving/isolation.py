"""Endpoint isolation gate: a greedy request streamed through the OpenAI endpoint produces the same
tokens alone and next to other traffic, and the server keeps running decodes moving while it
prefills a long prompt.

The gate's pass conditions are the reference rig's (``optimisation/rig/interleave_bench.py:80-117``):
(1) every prompt's streamed tokens equal its solo run; (2) every background decoder is still
streaming after the long prompt's first token; (3) the short prompt was submitted before the long
prompt's first token, so it had to wait behind a prefill in progress.

How it runs here: ``SSEStream`` reads one streamed completion over a plain HTTP connection and
records every event (arrival time, token ids, text); ``Scenario`` runs the solo pass, then the
mixed pass - decoders ``B*`` start, the long prompt ``A`` goes in once every decoder has streamed
its first event, the short prompt ``C`` ``short_delay`` seconds later - and ``gate`` evaluates the
three conditions on the records.  Times are client-observed; one event may carry a whole
speculative block, so gaps between events are not per-token latencies.

Prompts are token ids below 256 (valid for every vocabulary here; no tokenizer download).

    python -m qwen38_b200.serving.isolation --base-url http://127.0.0.1:8000 --output gate.json
"""
from __future__ import annotations

import argparse
import hashlib
import http.client
import json
import threading
import time
import urllib.parse
from dataclasses import dataclass, field


@dataclass
class StreamRecord:
    """What one streamed completion delivered, with client-side arrival times."""
    prompt_tokens: int
    submitted: float = 0.0
    arrivals: list = field(default_factory=list)       # (time, number of token ids) per event with ids
    tokens: list = field(default_factory=list)
    text: list = field(default_factory=list)
    usage: dict | None = None
    done: bool = False

    @property
    def first(self):
        return self.arrivals[0][0]

    @property
    def last(self):
        return self.arrivals[-1][0]

    def summary(self) -> dict:
        gaps = sorted(b[0] - a[0] for a, b in zip(self.arrivals, self.arrivals[1:]))
        span = self.last - self.first

        def pick(q):
            return gaps[min(len(gaps) - 1, int(q * len(gaps)))] if gaps else None
        return dict(tokens=self.tokens, events=len(self.arrivals), started=self.submitted, first=self.first,
                    last=self.last, ttft_s=self.first - self.submitted,
                    text_sha256=hashlib.sha256("".join(self.text).encode()).hexdigest(),
                    decode_tok_s=(len(self.tokens) - self.arrivals[0][1]) / span if span > 0 else None,
                    event_gap_p99_s=pick(0.99), event_gap_max_s=gaps[-1] if gaps else None,
                    multi_token_events=sum(1 for _, n in self.arrivals if n > 1))


class SSEStream:
    """One greedy streamed ``/v1/completions`` request; ``run()`` returns its ``StreamRecord`` and
    raises when the stream breaks off or its token accounting does not add up."""

    def __init__(self, base_url, model, prompt, count, *, on_first=None, timeout=1800.0):
        u = urllib.parse.urlsplit(base_url)
        self.host, self.port = u.hostname, u.port or 80
        self.path = (u.path.rstrip("/") or "") + "/v1/completions"
        self.body = json.dumps(dict(model=model, prompt=list(prompt), max_tokens=count, temperature=0.0,
                                    stream=True, stream_options={"include_usage": True}, seed=123))
        self.count, self.on_first, self.timeout = count, on_first, timeout
        self.record = StreamRecord(prompt_tokens=len(prompt))

    def _on_event(self, msg):
        rec = self.record
        if "error" in msg:
            raise RuntimeError(f"server error in stream: {msg['error']}")
        rec.usage = msg.get("usage") or rec.usage
        for ch in msg.get("choices", ()):
            if ch.get("index", 0) != 0:
                raise RuntimeError("the gate streams one completion per request")
            ids = ch.get("token_ids") or []
            if not all(type(t) is int and t >= 0 for t in ids):
                raise ValueError(f"malformed token ids in stream: {ids!r}")
            rec.text.append(ch.get("text", ""))
            if ids:
                if not rec.arrivals and self.on_first is not None:
                    self.on_first()
                rec.arrivals.append((time.perf_counter(), len(ids)))
                rec.tokens += ids

    def run(self) -> StreamRecord:
        conn = http.client.HTTPConnection(self.host, self.port, timeout=self.timeout)
        try:
            self.record.submitted = time.perf_counter()
            conn.request("POST", self.path, body=self.body, headers={"Content-Type": "application/json"})
            resp = conn.getresponse()
            if resp.status != 200:
                raise RuntimeError(f"HTTP {resp.status}: {resp.read()[:200]!r}")
            while True:
                line = resp.readline()
                if not line:
                    break
                line = line.decode("utf-8").strip()
                if not line.startswith("data:"):
                    continue
                payload = line[len("data:"):].strip()
                if payload == "[DONE]":
                    self.record.done = True
                    break
                self._on_event(json.loads(payload))
        finally:
            conn.close()
        rec = self.record
        u = rec.usage or {}
        if not (rec.done and rec.arrivals and len(rec.tokens) == self.count and u.get("completion_tokens") == self.count
                and u.get("prompt_tokens") == rec.prompt_tokens):
            raise RuntimeError(f"stream incomplete or miscounted: done={rec.done} tokens={len(rec.tokens)}/"
                               f"{self.count} usage={rec.usage}")
        return rec


def make_prompts(prompt_length: int, decoders: int) -> dict:
    """Seeded id prompts: decoders B0.. of growing length, the long prompt A, the short prompt C."""
    out = {f"B{i}": [(5 * j + 11 * i + 1) % 250 + 3 for j in range(24 + 3 * i)] for i in range(decoders)}
    period = [(7 * i + 3) % 250 + 3 for i in range(37)]
    out["A"] = [period[j % len(period)] for j in range(prompt_length)]
    out["C"] = [(13 * j + 9) % 250 + 3 for j in range(16)]
    return out


class _Runner(threading.Thread):
    """A stream on its own thread; ``result()`` re-raises its failure."""

    def __init__(self, stream: SSEStream):
        super().__init__(daemon=True)
        self.stream, self.rec, self.exc = stream, None, None

    def run(self):
        try:
            self.rec = self.stream.run()
        except BaseException as e:          # reported by result()
            self.exc = e

    def result(self, timeout=None):
        self.join(timeout)
        if self.is_alive():
            raise TimeoutError("stream did not finish")
        if self.exc is not None:
            raise self.exc
        return self.rec


class Scenario:
    def __init__(self, base_url, model, prompts, counts, *, short_delay, ready_timeout):
        self.base_url, self.model, self.prompts, self.counts = base_url, model, prompts, counts
        self.short_delay, self.ready_timeout = short_delay, ready_timeout

    def _stream(self, name, on_first=None):
        return SSEStream(self.base_url, self.model, self.prompts[name], self.counts[name], on_first=on_first)

    def solo(self) -> dict:
        return {name: self._stream(name).run() for name in self.prompts}

    def mixed(self) -> dict:
        names = sorted(n for n in self.prompts if n.startswith("B"))
        started = threading.Semaphore(0)
        bg = {n: _Runner(self._stream(n, on_first=started.release)) for n in names}
        for r in bg.values():
            r.start()
        deadline = time.monotonic() + self.ready_timeout
        for _ in names:                                  # every decoder has streamed an event
            if not started.acquire(timeout=max(0.0, deadline - time.monotonic())):
                raise TimeoutError("the background decoders did not all start streaming")
        if any(not r.is_alive() for r in bg.values()):
            raise RuntimeError("a background decoder finished before the long prompt went in")
        long_run = _Runner(self._stream("A"))
        long_run.start()
        time.sleep(self.short_delay)
        short_run = _Runner(self._stream("C"))
        short_run.start()
        out = {n: r.result() for n, r in bg.items()}
        out["A"], out["C"] = long_run.result(), short_run.result()
        return out


def gate(solo: dict, mixed: dict) -> dict:
    """The three pass conditions on the two passes' records."""
    checks = {f"greedy_equal_{n}": solo[n].tokens == mixed[n].tokens and solo[n].text == mixed[n].text
              for n in solo}
    a_first = mixed["A"].first
    checks["decoders_overlap_long_prefill"] = all(r.last > a_first for n, r in mixed.items() if n.startswith("B"))
    checks["short_arrives_before_long_first_token"] = mixed["C"].submitted < a_first
    return checks


def measure(base_url, model="qwen38-hybrid", prompt_length=2049, decoders=1, decode_tokens=512, short_delay=0.1,
            ready_timeout=1800.0, short_tokens=32):
    prompts = make_prompts(prompt_length, decoders)
    counts = {n: decode_tokens if n.startswith("B") else short_tokens for n in prompts}
    sc = Scenario(base_url, model, prompts, counts, short_delay=short_delay, ready_timeout=ready_timeout)
    SSEStream(base_url, model, prompts["C"], 8).run()           # warm-up (graphs, caches)
    solo = sc.solo()
    mixed = sc.mixed()
    checks = gate(solo, mixed)
    return dict(passed=all(checks.values()), checks=checks, prompt_length=prompt_length, decoders=decoders,
                baseline={n: r.summary() for n, r in solo.items()},
                concurrent={n: r.summary() for n, r in mixed.items()},
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
