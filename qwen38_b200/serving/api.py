"""OpenAI-compatible HTTP front end over ``ServingEngine``.

The reference serves through vLLM's OpenAI server with a TT platform plugin
(``scripts/ci/fixtures/qwen36_vllm.py``, ``fixtures/plugin_scheduler.py``).  Here a single engine
loop thread owns the GPU and steps the scheduler; HTTP handlers only enqueue requests and wait for
their completion, so requests arriving concurrently are continuously batched into packed verifies.

Endpoints: ``POST /v1/completions`` (``prompt`` as a list of token ids, or a string encoded with
the byte-level fallback tokenizer below - checkpoints' own tokenizers need network access to
fetch), ``POST /v1/chat/completions`` (``messages`` rendered with a plain role template),
``GET /v1/models``, ``GET /health``, ``GET /metrics`` (Prometheus text).  ``"logprobs": k`` on a
non-streaming completion returns each output token's log-probability and the top k, scored on the
engine thread(s) by the model's own final norm and LM head; ``"stop"`` strings end a request at
the step they appear in and cut the text before them (streams hold back a possible partial match).  With ``"stream": true``
both generation endpoints answer with server-sent events, one event per engine step that emitted
tokens (a speculative block commits several tokens at once), then ``data: [DONE]``.

Run:  python -m qwen38_b200.serving.api --profile single-stream-4k --set serving.port=8000
      python -m qwen38_b200.serving.api --profile tiny-cpu            (CPU, tiny shape)
      torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m qwen38_b200.serving.api \
          --profile single-stream-4k --set parallel.tp=2              (TP2: rank 0 serves HTTP)
"""
from __future__ import annotations

import argparse
import collections
import json
import queue
import threading
import time
import uuid

import torch
from pydantic import BaseModel

from .scheduler import ABORTED, FINISHED


class StreamOptions(BaseModel):
    include_usage: bool = False       # a last event carrying the token accounting


class CompletionRequest(BaseModel):
    model: str | None = None
    prompt: list[int] | str | list[str] | list[list[int]]     # one prompt, or a batch of them
    n: int = 1                        # completions per prompt (seeds seed, seed+1, ... when sampled)
    max_tokens: int = 16
    stop_token_ids: list[int] | None = None
    temperature: float = 0.0          # 0: greedy; > 0: sampled (both run block speculation)
    seed: int | None = None
    stream: bool = False
    stream_options: StreamOptions | None = None
    logprobs: int | None = None       # > 0: log-probability of each output token and the top-k
    stop: str | list[str] | None = None   # text ends before the first stop string
    echo: bool = False                # the prompt's text is prepended to the completion's text


class ChatMessage(BaseModel):
    role: str
    content: str


class ChatRequest(BaseModel):
    model: str | None = None
    messages: list[ChatMessage]
    max_tokens: int = 16
    stop_token_ids: list[int] | None = None
    temperature: float = 0.0
    seed: int | None = None
    stream: bool = False
    stream_options: StreamOptions | None = None
    stop: str | list[str] | None = None
    n: int = 1
    logprobs: bool = False            # per-token log-probabilities of the answer ...
    top_logprobs: int = 0             # ... with this many alternatives each (0..20)


def render_chat(messages) -> str:
    """Plain role template (the checkpoint's own chat template needs its tokenizer files)."""
    return "".join(f"<|{m.role}|>\n{m.content}\n" for m in messages) + "<|assistant|>\n"


class ByteTokenizer:
    """Fallback tokenizer: UTF-8 bytes are ids 0..255 (no network access to fetch a real one)."""

    def encode(self, text: str):
        return list(text.encode("utf-8"))

    def decode(self, ids):
        return bytes(int(i) for i in ids if 0 <= int(i) < 256).decode("utf-8", errors="replace")


def _score_op(engine, ids, out, k):
    from ..utils.tp_agreement import score
    return score(engine.target, ids, out, top_k=k)


SHARED_OPS = {"score": _score_op}        # engine operations every tensor-parallel rank runs together


class Histogram:
    """Prometheus-style cumulative histogram (seconds)."""

    BUCKETS = (0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0, 30.0, 60.0)

    def __init__(self):
        self.counts = [0] * len(self.BUCKETS)
        self.n, self.total = 0, 0.0

    def observe(self, v: float):
        self.n += 1
        self.total += v
        for i, b in enumerate(self.BUCKETS):
            if v <= b:
                self.counts[i] += 1

    def lines(self, name: str):
        out = [f"# TYPE {name} histogram"]
        out += [f'{name}_bucket{{le="{b}"}} {c}' for b, c in zip(self.BUCKETS, self.counts)]
        out += [f'{name}_bucket{{le="+Inf"}} {self.n}', f"{name}_sum {self.total}", f"{name}_count {self.n}"]
        return out


class EngineLoop:
    """Owns the engine: a background thread admits queued requests and steps the scheduler.

    Tensor parallel (one process per GPU): rank 0 runs this loop and the HTTP server; before each
    iteration it hands ``sync`` the requests it admitted and whether it steps, and the other ranks,
    running ``follow``, admit the same requests under the same ids and take the same step, so every
    rank's engine runs in lockstep.  While idle, rank 0 still syncs every ``heartbeat_s`` so the
    followers' waiting collective never runs into the process-group timeout."""

    def __init__(self, engine, idle_sleep: float = 0.001, sync=None, heartbeat_s: float = 1.0, decode=None,
                 phase_log: str | None = None):
        self.engine = engine
        self.phase_log = phase_log          # one JSON line per finished request (blocks, timings)
        self.recent_blocks = collections.deque(maxlen=256)     # block records of the last requests
        self.sync, self.heartbeat_s = sync, heartbeat_s
        self.decode = decode or ByteTokenizer().decode
        self._completes = []                # stop-string completions the followers still have to apply
        self._aborts_pending = []           # fault aborts the followers still have to apply
        self.faults = 0
        self.inbox: "queue.Queue" = queue.Queue()
        self.waiters: dict = {}
        self.idle_sleep = idle_sleep
        self.stop_event = threading.Event()
        self.completed = self.aborted = self.tokens = 0
        self.ttft, self.tpot = Histogram(), Histogram()      # time to first token, time per output token
        self.calls: "queue.Queue" = queue.Queue()
        self.cancels: "queue.Queue" = queue.Queue()
        self.shared: "queue.Queue" = queue.Queue()
        self.thread = threading.Thread(target=self._run, name="q38-engine", daemon=True)
        self.thread.start()

    def call(self, fn, timeout: float = 600.0):
        """Run ``fn()`` on the engine thread between two steps (the model is not thread-safe)."""
        done, box = threading.Event(), {}
        self.calls.put((fn, done, box))
        if not done.wait(timeout):
            raise TimeoutError("engine call timed out")
        if "error" in box:
            raise box["error"]
        return box["value"]

    def call_shared(self, name: str, *args, timeout: float = 600.0):
        """Run ``SHARED_OPS[name](engine, *args)`` on the engine thread of every tensor-parallel rank
        (an operation with collectives inside, such as scoring with the vocabulary-sharded head)."""
        done, box = threading.Event(), {}
        self.shared.put((name, args, done, box))
        if not done.wait(timeout):
            raise TimeoutError("engine call timed out")
        if "error" in box:
            raise box["error"]
        return box["value"]

    def cancel(self, request_id: str):
        """Abort a request (its client went away); applied on the engine thread before the next step,
        on every tensor-parallel rank."""
        self.cancels.put(request_id)

    def submit(self, prompt, max_new_tokens, eos_ids=(), temperature=0.0, seed=0, stream=False, stop=()):
        """Queue a request.  Returns (done event, result box); with ``stream`` the box's "stream"
        queue receives each step's newly emitted token ids, then None when the request ends.  With
        ``stop`` strings the request ends early once one appears in its decoded output."""
        done = threading.Event()
        box = {"stream": queue.Queue()} if stream else {}
        if stop:
            box["stop"] = list(stop)
        self.inbox.put((prompt, max_new_tokens, tuple(eos_ids), done, box, float(temperature), int(seed)))
        return done, box

    def _run(self):
        dev = getattr(self.engine.target, "device", None)
        if dev is not None and torch.device(dev).type == "cuda" and torch.device(dev).index is not None:
            torch.cuda.set_device(torch.device(dev))     # the current device is per thread
        last_sync = time.monotonic()
        while True:
            stop = self.stop_event.is_set()
            while not self.calls.empty():
                fn, done, box = self.calls.get_nowait()
                try:
                    box["value"] = fn()
                except Exception as e:          # handed back to the caller's thread
                    box["error"] = e
                done.set()
            adds = []
            try:
                while not stop:
                    prompt, n, eos, done, box, temp, seed = self.inbox.get_nowait()
                    try:
                        req = self.engine.add_request(prompt, n, eos_ids=eos, temperature=temp, seed=seed)
                        box["sent"] = 0
                        box["rid"] = req.request_id
                        self.waiters[req.request_id] = (done, box, req)
                        adds.append((req.request_id, list(req.prompt), n, eos, temp, seed))
                    except Exception as e:          # invalid request: answer at once
                        box["error"] = str(e)
                        if "stream" in box:
                            box["stream"].put(None)
                        done.set()
            except queue.Empty:
                pass
            aborted = []
            while not self.cancels.empty():
                rid = self.cancels.get_nowait()
                req = self.engine.requests.get(rid)
                if req is not None and req.state not in (FINISHED, ABORTED):
                    self.engine.abort(rid, "cancelled by the client")
                    aborted.append(rid)
                    self._settle(req)
            aborted += self._aborts_pending
            self._aborts_pending = []
            shared = []
            while not stop and not self.shared.empty():
                shared.append(self.shared.get_nowait())
            step = not stop and self.engine.has_work()
            if self.sync is not None and (adds or step or stop or self._completes or aborted or shared
                                          or time.monotonic() - last_sync >= self.heartbeat_s):
                self.sync({"add": adds, "complete": self._completes, "abort": aborted,
                           "shared": [(name, args) for name, args, _, _ in shared], "step": step, "stop": stop})
                self._completes = []
                last_sync = time.monotonic()
            for name, args, done, box in shared:        # every rank runs these at this point
                try:
                    box["value"] = SHARED_OPS[name](self.engine, *args)
                except Exception as e:
                    box["error"] = e
                done.set()
            if stop:
                break
            if not step:
                time.sleep(self.idle_sleep)
                continue
            try:
                finished = self.engine.step()
            except Exception as e:              # an engine fault: fail the requests, keep serving
                self.faults += 1
                finished = []
                for rid, req in list(self.engine.requests.items()):
                    if req.state not in (FINISHED, ABORTED):
                        self.engine.abort(rid, f"engine fault: {e}")
                        self._aborts_pending.append(rid)
                        finished.append(req)
            for rid, (done, box, req) in list(self.waiters.items()):    # stop strings end a request early
                if "stop" in box and req.state not in (FINISHED, ABORTED) and req not in finished:
                    text = self.decode(req.output)
                    if any(st in text for st in box["stop"]):
                        self.engine.complete(rid)
                        self._completes.append(rid)
                        finished.append(req)
            for done, box, req in list(self.waiters.values()):     # stream what each step emitted
                if "stream" in box:
                    out = req.output
                    if len(out) > box["sent"]:
                        box["stream"].put(out[box["sent"]:])
                        box["sent"] = len(out)
            for req in finished:
                self._settle(req)

    def _settle(self, req):
        """Hand a finished or aborted request to its waiter."""
        entry = self.waiters.pop(req.request_id, None)
        if entry is None:
            return
        done, box, _ = entry
        box["request"] = req
        if "stream" in box:
            box["stream"].put(None)
        if req.state == FINISHED:
            self.completed += 1
            self.tokens += max(0, len(req.output) - 1)
            if req.blocks:
                self.recent_blocks.append(list(req.blocks))
            if self.phase_log:
                rec = {"stage": "request_phases", "request_id": req.request_id, "prompt_tokens": len(req.prompt),
                       "output_tokens": len(req.output), "blocks": req.blocks,
                       "ttft_s": None if req.t_first is None else req.t_first - req.arrival,
                       "decode_s": None if req.t_first is None or req.t_done is None else req.t_done - req.t_first}
                with open(self.phase_log, "a") as f:
                    f.write(json.dumps(rec) + "\n")
            if req.t_first is not None:
                self.ttft.observe(max(0.0, req.t_first - req.arrival))
                if req.t_done is not None and len(req.output) > 1:
                    self.tpot.observe(max(0.0, req.t_done - req.t_first) / (len(req.output) - 1))
        elif req.state == ABORTED:
            self.aborted += 1
        done.set()

    def close(self):
        self.stop_event.set()
        self.thread.join(timeout=10)


def broadcast_sync(group=None):
    """``sync`` for ``EngineLoop`` / ``follow``: rank 0's command object, broadcast to every rank."""
    import torch.distributed as dist

    def sync(cmd):
        box = [cmd]
        dist.broadcast_object_list(box, src=0, group=group)
        return box[0]
    return sync


def follow(engine, sync):
    """Rank > 0 of a tensor-parallel server: admit what rank 0 admitted, step when it steps, return
    when it stops."""
    while True:
        cmd = sync(None)
        for rid in cmd.get("complete", ()):
            engine.complete(rid)
        for rid in cmd.get("abort", ()):
            engine.abort(rid, "cancelled by the client")
        for rid, prompt, n, eos, temp, seed in cmd["add"]:
            engine.add_request(prompt, n, eos_ids=eos, temperature=temp, seed=seed, request_id=rid)
        for name, args in cmd.get("shared", ()):
            try:
                SHARED_OPS[name](engine, *args)
            except Exception:                   # rank 0 reports the error; stay in step
                pass
        if cmd["stop"]:
            return
        if cmd["step"]:
            engine.step()


class TextStream:
    """Incremental text of a streamed completion.  Every step decodes the whole output so far and
    returns only the part no later token can change:

    * a multi-byte character whose bytes arrive over several steps decodes as trailing replacement
      characters until its last byte lands, so up to three trailing U+FFFD are held back (the
      character then goes out once, whole);
    * with stop strings, text that could still be the start of one is held back; when a stop
      string appears, the text before it is returned with ``stopped`` set.

    ``finish()`` returns whatever is still held when generation ends."""

    def __init__(self, tok, stops=()):
        self.tok, self.stops = tok, list(stops)
        self.hold = max((len(x) for x in self.stops), default=1) - 1
        self.ids, self.sent = [], 0

    @staticmethod
    def settled(text: str) -> int:
        n, k = len(text), 0
        while k < 3 and n - k > 0 and text[n - k - 1] == "\ufffd":
            k += 1
        return n - k

    def _stop_at(self, text):
        cuts = [text.find(x) for x in self.stops if x in text]
        return min(cuts) if cuts else None

    def push(self, new):
        """(new text, stopped) after the step's tokens ``new``."""
        self.ids += list(new)
        text = self.tok.decode(self.ids)
        cut = self._stop_at(text)
        if cut is not None:
            out, self.sent = text[self.sent:cut], cut
            return out, True
        safe = max(self.sent, self.settled(text) - self.hold)
        out, self.sent = text[self.sent:safe], safe
        return out, False

    def finish(self):
        """(remaining text, stopped) at the end of generation."""
        text = self.tok.decode(self.ids)
        cut = self._stop_at(text)
        end = len(text) if cut is None else cut
        out, self.sent = text[self.sent:end], max(self.sent, end)
        return out, cut is not None


def build_app(engine, model_name: str = "qwen38-hybrid", tokenizer=None, timeout_s: float = 600.0,
              output_budget_multiple: int = 0, sync=None, phase_log: str | None = None):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse, StreamingResponse

    tok = tokenizer or ByteTokenizer()
    loop = EngineLoop(engine, sync=sync, decode=tok.decode, phase_log=phase_log)
    app = FastAPI(title="qwen38_b200")
    app.state.loop = loop

    @app.get("/health")
    def health():
        return {"status": "ok" if loop.thread.is_alive() else "engine loop stopped",
                "running": len(engine.sched.running), "waiting": len(engine.sched.waiting),
                "tp": engine.target.tp, "engine_faults": loop.faults}

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "qwen38_b200",
                                            "max_model_len": engine.target.rt.max_context}]}

    def _start(ids, body, seed=None):
        if not ids:
            raise HTTPException(400, "empty prompt")
        if output_budget_multiple and body.max_tokens % output_budget_multiple:
            raise HTTPException(400, f"max_tokens must be a multiple of {output_budget_multiple}")
        # the first output token comes from the prefill; max_tokens counts output tokens
        if seed is None:
            seed = body.seed if body.seed is not None else uuid.uuid4().int & 0x7FFFFFFF
        stops = _stops(body)
        return loop.submit(ids, body.max_tokens, body.stop_token_ids or (), body.temperature, seed, body.stream,
                           stop=stops)

    def _stops(body):
        st = body.stop
        stops = [st] if isinstance(st, str) else list(st or [])
        if any(not x for x in stops) or len(stops) > 4:
            raise HTTPException(400, "stop: up to 4 non-empty strings")
        return stops

    def _text(out, body):
        """(text, finish reason): the text ends before the first stop string, if one appears."""
        text = tok.decode(out)
        cuts = [text.find(x) for x in _stops(body) if x in text]
        if cuts:
            return text[:min(cuts)], "stop"
        return text, _finish_reason(out, body)

    def _finished(done, box):
        if not done.wait(timeout_s):
            raise HTTPException(504, "generation timed out")
        if "error" in box:
            raise HTTPException(400, box["error"])
        req = box["request"]
        if req.state != FINISHED:
            raise HTTPException(500, f"request aborted: {req.error}")
        return req.output

    def _finish_reason(out, body):
        return "stop" if out and out[-1] in (body.stop_token_ids or ()) else "length"

    def _events(box, body, chunk, n_prompt, echo_text=""):
        """Server-sent events: the echoed prompt (completions with ``echo``), one event per engine
        step that emitted tokens, the finish event (with the token accounting when
        ``stream_options.include_usage``), then [DONE]."""
        emitted, ended = [], False
        try:
            yield from _event_lines(box, body, chunk, n_prompt, emitted, echo_text)
            ended = True
        finally:
            if not ended and "rid" in box:          # the client went away mid-stream
                loop.cancel(box["rid"])

    def _event_lines(box, body, chunk, n_prompt, emitted, echo_text=""):
        """Each event carries the new part of the decoded output text (``TextStream``); at a stop
        string the stream ends with finish_reason "stop" (the engine ends the request at the same
        step)."""
        ts = TextStream(tok, _stops(body))

        def event(obj):
            return "data: " + json.dumps(obj) + "\n\n"

        def usage(last):
            if body.stream_options is not None and body.stream_options.include_usage:
                last["usage"] = {"prompt_tokens": n_prompt, "completion_tokens": len(emitted),
                                 "total_tokens": n_prompt + len(emitted)}
            return last

        if echo_text:
            yield event(chunk([], None, text=echo_text))
        while True:
            try:
                new = box["stream"].get(timeout=timeout_s)
            except queue.Empty:
                yield event({"error": "generation timed out"})
                break
            if new is None:
                req = box.get("request")
                if "error" in box or req is None or req.state != FINISHED:
                    reason = box.get("error") or getattr(req, "error", "aborted")
                    yield event({"error": str(reason)})
                else:
                    text, stopped = ts.finish()
                    yield event(usage(chunk([], "stop" if stopped else _finish_reason(emitted, body), text=text)))
                break
            emitted += new
            text, stopped = ts.push(new)
            if stopped:
                yield event(usage(chunk(new, "stop", text=text)))
                break
            yield event(chunk(new, None, text=text))
        yield "data: [DONE]\n\n"

    def _logprobs(ids, out, k):
        """OpenAI completions ``logprobs`` object: each output token's log-probability and the top
        k, scored by the engine's own final norm and LM head on the engine thread."""
        try:
            chosen, ti, tv = loop.call_shared("score", list(ids), list(out), int(k))
        except MemoryError:
            raise HTTPException(503, "no free sequence slot to score the output")
        return {"tokens": [tok.decode([t]) for t in out], "token_ids": out,
                "token_logprobs": [float(v) for v in chosen],
                "top_logprobs": [{tok.decode([int(i)]): float(v) for i, v in zip(ir, vr)}
                                 for ir, vr in zip(ti.tolist(), tv.tolist())],
                "top_token_ids": ti.tolist(), "top_token_logprobs": tv.tolist()}

    def _completion_logprobs(ids, out, body):
        """``logprobs`` of a completion; with ``echo`` they cover the prompt tokens too (the first
        prompt token has no context, so its entries are null, as in the OpenAI API)."""
        if body.logprobs is None:
            return None
        k = max(1, body.logprobs)
        if not body.echo or len(ids) < 1:
            return _logprobs(ids, out, k)
        lp = _logprobs(ids[:1], list(ids[1:]) + list(out), k)
        return {"tokens": [tok.decode([ids[0]])] + lp["tokens"], "token_ids": [ids[0]] + lp["token_ids"],
                "token_logprobs": [None] + lp["token_logprobs"], "top_logprobs": [None] + lp["top_logprobs"],
                "top_token_ids": [None] + lp["top_token_ids"],
                "top_token_logprobs": [None] + lp["top_token_logprobs"]}

    def _prompt_list(p):
        if isinstance(p, str):
            return [tok.encode(p)]
        if p and all(isinstance(x, str) for x in p):
            return [tok.encode(x) for x in p]
        if p and all(isinstance(x, list) for x in p):
            return [list(x) for x in p]
        return [list(p)]

    @app.post("/v1/completions")
    def completions(body: CompletionRequest):
        prompts = _prompt_list(body.prompt)
        if body.logprobs is not None and (body.logprobs < 0 or body.logprobs > 20 or body.stream):
            raise HTTPException(400, "logprobs: 0..20, non-streaming requests")
        if not 1 <= body.n <= 16 or len(prompts) > 64:
            raise HTTPException(400, "n: 1..16 completions per prompt, up to 64 prompts")
        if len(prompts) * body.n > 1:
            if body.stream:
                raise HTTPException(400, "streaming serves one completion per request")
            return _batch(prompts, body)
        ids = prompts[0]
        done, box = _start(ids, body)
        cid, created, model = "cmpl-" + uuid.uuid4().hex[:16], int(time.time()), body.model or model_name
        if body.stream:
            def chunk(new, reason, text=None):
                return {"id": cid, "object": "text_completion", "created": created, "model": model,
                        "choices": [{"index": 0, "text": tok.decode(new) if text is None else text,
                                     "token_ids": new, "finish_reason": reason}]}
            return StreamingResponse(_events(box, body, chunk, len(ids), tok.decode(ids) if body.echo else ""),
                                     media_type="text/event-stream")
        out = _finished(done, box)
        lp = _completion_logprobs(ids, out, body)
        text, reason = _text(out, body)
        if body.echo:
            text = tok.decode(ids) + text
        return {
            "id": cid, "object": "text_completion", "created": created, "model": model,
            "choices": [{"index": 0, "text": text, "token_ids": out, "logprobs": lp, "finish_reason": reason}],
            "usage": {"prompt_tokens": len(ids), "completion_tokens": len(out),
                      "total_tokens": len(ids) + len(out)},
        }

    def _batch(prompts, body):
        """Several prompts and / or ``n`` completions each: all are queued at once (continuous
        batching packs them), choice ``i * n + j`` is completion j of prompt i."""
        base = body.seed if body.seed is not None else uuid.uuid4().int & 0x7FFFFFFF
        jobs = [(ids, _start(ids, body, seed=base + j)) for ids in prompts for j in range(body.n)]
        choices, n_out = [], 0
        for i, (ids, (done, box)) in enumerate(jobs):
            out = _finished(done, box)
            lp = _completion_logprobs(ids, out, body)
            text, reason = _text(out, body)
            if body.echo:
                text = tok.decode(ids) + text
            choices.append({"index": i, "text": text, "token_ids": out, "logprobs": lp, "finish_reason": reason})
            n_out += len(out)
        n_in = sum(len(p) for p in prompts)
        return {"id": "cmpl-" + uuid.uuid4().hex[:16], "object": "text_completion", "created": int(time.time()),
                "model": body.model or model_name, "choices": choices,
                "usage": {"prompt_tokens": n_in, "completion_tokens": n_out, "total_tokens": n_in + n_out}}

    @app.post("/v1/chat/completions")
    def chat(body: ChatRequest):
        if not body.messages:
            raise HTTPException(400, "no messages")
        ids = tok.encode(render_chat(body.messages))
        if not 1 <= body.n <= 16 or not 0 <= body.top_logprobs <= 20:
            raise HTTPException(400, "n: 1..16, top_logprobs: 0..20")
        if body.stream and (body.n > 1 or body.logprobs):
            raise HTTPException(400, "streaming serves one completion without logprobs")
        cid, created, model = "chatcmpl-" + uuid.uuid4().hex[:16], int(time.time()), body.model or model_name
        if body.n > 1 or body.logprobs:
            base = body.seed if body.seed is not None else uuid.uuid4().int & 0x7FFFFFFF
            jobs = [_start(ids, body, seed=base + j) for j in range(body.n)]
            choices, n_out = [], 0
            for j, (done, box) in enumerate(jobs):
                out = _finished(done, box)
                text, reason = _text(out, body)
                c = {"index": j, "message": {"role": "assistant", "content": text}, "token_ids": out,
                     "finish_reason": reason, "logprobs": None}
                if body.logprobs:
                    lp = _logprobs(ids, out, max(1, body.top_logprobs))
                    c["logprobs"] = {"content": [
                        {"token": t, "token_id": i, "logprob": v,
                         "top_logprobs": [{"token": tok.decode([a]), "token_id": a, "logprob": b}
                                          for a, b in zip(ti, tv)][:body.top_logprobs]}
                        for t, i, v, ti, tv in zip(lp["tokens"], lp["token_ids"], lp["token_logprobs"],
                                                   lp["top_token_ids"], lp["top_token_logprobs"])]}
                choices.append(c)
                n_out += len(out)
            return {"id": cid, "object": "chat.completion", "created": created, "model": model, "choices": choices,
                    "usage": {"prompt_tokens": len(ids), "completion_tokens": n_out,
                              "total_tokens": len(ids) + n_out}}
        done, box = _start(ids, body)
        if body.stream:
            def chunk(new, reason, text=None):
                content = tok.decode(new) if text is None else text
                delta = {"role": "assistant", "content": content} if (new or content) else {}
                return {"id": cid, "object": "chat.completion.chunk", "created": created, "model": model,
                        "choices": [{"index": 0, "delta": delta, "finish_reason": reason}]}
            return StreamingResponse(_events(box, body, chunk, len(ids)), media_type="text/event-stream")
        out = _finished(done, box)
        text, reason = _text(out, body)
        return {
            "id": cid, "object": "chat.completion", "created": created, "model": model,
            "choices": [{"index": 0, "message": {"role": "assistant", "content": text},
                         "token_ids": out, "finish_reason": reason}],
            "usage": {"prompt_tokens": len(ids), "completion_tokens": len(out),
                      "total_tokens": len(ids) + len(out)},
        }

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        lines = [
            "# TYPE q38_requests_completed counter", f"q38_requests_completed {loop.completed}",
            "# TYPE q38_requests_aborted counter", f"q38_requests_aborted {loop.aborted}",
            "# TYPE q38_engine_faults counter", f"q38_engine_faults {loop.faults}",
            "# TYPE q38_tokens_generated counter", f"q38_tokens_generated {loop.tokens}",
            "# TYPE q38_steps counter",
            f"q38_steps{{kind=\"prefill\"}} {engine.steps['prefill']}",
            f"q38_steps{{kind=\"decode\"}} {engine.steps['decode']}",
            "# TYPE q38_running gauge", f"q38_running {len(engine.sched.running)}",
            "# TYPE q38_waiting gauge", f"q38_waiting {len(engine.sched.waiting)}",
            "# TYPE q38_kv_free_blocks gauge", f"q38_kv_free_blocks {engine.target.allocator.num_free}",
            *loop.ttft.lines("q38_time_to_first_token_seconds"),
            *loop.tpot.lines("q38_time_per_output_token_seconds"),
        ]
        if loop.recent_blocks:
            from ..spec.analysis import acceptance_report_requests
            rep = acceptance_report_requests(list(loop.recent_blocks))
            lines += ["# TYPE q38_committed_tokens_per_block gauge",
                      f"q38_committed_tokens_per_block {rep['mean_committed_per_block']}"]
            if rep["mean_accepted"] is not None:
                lines += ["# TYPE q38_mean_accepted_drafts gauge", f"q38_mean_accepted_drafts {rep['mean_accepted']}"]
        if engine.prefix is not None:
            for k, v in engine.prefix.export_stats().items():
                if isinstance(v, (int, float)):
                    lines.append(f"q38_prefix_{k} {int(v)}")
        return "\n".join(lines) + "\n"

    @app.on_event("shutdown")
    def _shutdown():
        loop.close()

    return app


def main():
    import uvicorn

    from ..runconfig import load_run_config
    from .factory import build_engine

    ap = argparse.ArgumentParser(description="OpenAI-compatible completions server")
    ap.add_argument("--profile", default=None, help="named profile from serving/profiles.yaml")
    ap.add_argument("--config", default=None, help="YAML run configuration")
    ap.add_argument("--set", action="append", default=[], metavar="SECTION.FIELD=VALUE")
    a = ap.parse_args()
    rc = load_run_config(a.config, profile=a.profile, overrides=a.set)
    from ..parallel.comm import init_distributed
    rank, world, local = init_distributed()
    if world != rc.parallel.tp:
        raise SystemExit(f"parallel.tp={rc.parallel.tp} but {world} processes: launch one per GPU with torchrun")
    device = None
    if torch.cuda.is_available() and rc.kernels.ops == "native":
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
    eng = build_engine(rc, device=device)
    sync = broadcast_sync() if world > 1 else None
    if rank > 0:
        follow(eng, sync)                       # rank 0 serves HTTP; the others follow its steps
        return
    app = build_app(eng, timeout_s=rc.serving.request_timeout_s,
                    output_budget_multiple=rc.serving.output_budget_multiple, sync=sync,
                    phase_log=rc.serving.phase_log or None)
    uvicorn.run(app, host=rc.serving.host, port=rc.serving.port)


if __name__ == "__main__":
    main()
