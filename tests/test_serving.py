"""Serving engine on CPU: continuous batching of several requests through packed verifies matches
each request's single-stream greedy output; a failing request is quarantined while the others
finish; prefix reuse inside the engine; scheduler policy (prefill first, no mixed steps)."""
import torch

from qwen38_b200.config import RuntimeConfig
from qwen38_b200.models.drafter import BlockDrafter
from qwen38_b200.models.target import HybridTarget
from qwen38_b200.prefix.registry import PrefixRegistry
from qwen38_b200.serving.engine import ServingEngine
from qwen38_b200.serving.scheduler import ABORTED, FINISHED, DecodeStep, PrefillStep, Request, Scheduler
from qwen38_b200.spec.engine import PinnedAcceptance, greedy_reference

RT = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)


def _setup(tiny, slots=3):
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RT, max_slots=slots + 1, max_verify_rows=4 * slots)
    dr = BlockDrafter(tiny["dcfg"], tiny["dsrc"], tgt, slots=slots)
    return tgt, dr


def _prompt(seed, n):
    return torch.randint(0, 4096, (n,), generator=torch.Generator().manual_seed(seed)).tolist()


def test_continuous_batching_matches_single_stream(tiny):
    tgt, dr = _setup(tiny)
    prompts = [_prompt(1, 100), _prompt(2, 70), _prompt(3, 130)]
    golds = [greedy_reference(tgt, p, 20) for p in prompts]
    eng = ServingEngine(tgt, dr, verifier_rows=4)
    reqs = [eng.add_request(p, 20, pinned=PinnedAcceptance(g, seed=i, mean_accepted=1))
            for i, (p, g) in enumerate(zip(prompts, golds))]
    eng.run()
    for r, g in zip(reqs, golds):
        assert r.state == FINISHED, r.error
        assert r.output == g
    assert eng.steps["decode"] < sum(len(g) for g in golds)      # blocks were packed
    assert tgt.allocator.num_free == tgt.allocator.num_blocks


def test_quarantine_isolates_a_failing_request(tiny):
    tgt, dr = _setup(tiny)

    class Boom:
        def apply(self, *a):
            raise RuntimeError("injected drafter failure")

    good = _prompt(4, 60)
    gold = greedy_reference(tgt, good, 12)
    eng = ServingEngine(tgt, dr, verifier_rows=4)
    bad = eng.add_request(_prompt(5, 60), 12, pinned=Boom())
    ok = eng.add_request(good, 12)
    eng.run()
    assert bad.state == ABORTED and "injected" in bad.error
    assert ok.state == FINISHED and ok.output == gold
    assert eng.quarantined == 1


def test_engine_prefix_reuse(tiny):
    tgt, dr = _setup(tiny, slots=2)
    reg = PrefixRegistry(tgt, 1 << 30, boundary=64)
    shared = _prompt(6, 128)
    a, b = shared + _prompt(7, 40), shared + _prompt(8, 30)
    gold_b = greedy_reference(tgt, b, 10)
    eng = ServingEngine(tgt, dr, verifier_rows=4, prefix=reg)
    eng.add_request(a, 10)
    eng.run()
    rb = eng.add_request(b, 10)
    eng.run()
    assert rb.reused_prefix == 128 and rb.output == gold_b


def test_scheduler_policy():
    s = Scheduler(max_running=2, prefill_chunk=64, max_step_rows=32, verifier_rows=16)
    r1 = Request("a", list(range(100)), 8)
    r2 = Request("b", list(range(10)), 8)
    s.add(r1)
    s.add(r2)
    st = s.schedule(lambda r: True)
    assert isinstance(st, PrefillStep) and (st.start, st.end) == (0, 64)
    r1.prefilled = 64
    st = s.schedule(lambda r: True)                  # continuation, not a new request
    assert isinstance(st, PrefillStep) and st.request is r1 and st.end == 100
    s.prefill_done(r1)
    st = s.schedule(lambda r: True)                  # prefill first while r2 waits
    assert isinstance(st, PrefillStep) and st.request is r2
    s.prefill_done(r2)
    st = s.schedule(lambda r: True)
    assert isinstance(st, DecodeStep) and len(st.requests) == 2
    s.finish(r1)
    assert s.running == [r2]


def test_openai_http_front_end(tiny):
    from fastapi.testclient import TestClient

    from qwen38_b200.serving.api import build_app
    tgt, dr = _setup(tiny, slots=2)
    p1, p2 = _prompt(11, 50), _prompt(12, 40)
    g1 = greedy_reference(tgt, p1, 8)
    eng = ServingEngine(tgt, dr, verifier_rows=4)
    app = build_app(eng, model_name="tiny")
    with TestClient(app) as client:
        assert client.get("/health").json()["status"] == "ok"
        assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
        assert client.get("/v1/models").json()["data"][0]["max_model_len"] == eng.target.rt.max_context
        r = client.post("/v1/completions", json={"prompt": p1, "max_tokens": 8})
        assert r.status_code == 200
        body = r.json()
        assert body["choices"][0]["token_ids"] == g1
        assert body["usage"]["completion_tokens"] == 8
        r2 = client.post("/v1/completions", json={"prompt": "hello", "max_tokens": 4})
        assert r2.status_code == 200 and len(r2.json()["choices"][0]["token_ids"]) == 4
        assert client.post("/v1/completions", json={"prompt": [999999], "max_tokens": 4}).status_code == 400
        m = client.get("/metrics").text
        assert "q38_requests_completed 2" in m
        assert "q38_time_to_first_token_seconds_count 2" in m
        assert 'q38_time_per_output_token_seconds_bucket{le="+Inf"} 2' in m
    app.state.loop.close()


def test_poisson_loadgen_report(tiny):
    from qwen38_b200.serving.loadgen import poisson_arrivals, run
    tgt, dr = _setup(tiny, slots=3)
    prompts = [_prompt(20 + i, 40 + 10 * i) for i in range(3)]
    golds = [greedy_reference(tgt, p, 12) for p in prompts]
    eng = ServingEngine(tgt, dr, verifier_rows=4)
    arr = poisson_arrivals(3, 50.0, seed=1)
    assert arr[0] == 0.0 and arr == sorted(arr)
    rep = run(eng, prompts, 12, arr, golds=golds, mean_accepted=1)
    assert rep["finished"] == 3 and rep["exact"]
    assert rep["committed_tokens"] == 3 * 11 and rep["aggregate_tok_s"] > 0
    assert 0 <= rep["p50_ttft_s"] <= rep["p90_ttft_s"]


def test_factory_builds_engines_from_profiles():
    """``tiny-cpu`` profile -> engine; the MTP drafter serves packed requests token-exact; the
    output budget multiple is enforced at the HTTP boundary."""
    from fastapi.testclient import TestClient

    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.api import build_app
    from qwen38_b200.serving.factory import build_engine
    rc = load_run_config(profile="tiny-cpu", overrides=["serving.slots=2"])
    eng = build_engine(rc)
    assert eng.drafter is not None and eng.verifier_rows == 4
    p = _prompt(31, 48)
    gold = greedy_reference(eng.target, p, 8)
    eng.add_request(p, 8, request_id="a")
    eng.add_request(_prompt(32, 40), 8, request_id="b")
    done = eng.run()
    assert {r.request_id: r.output for r in done}["a"] == gold
    rc = load_run_config(profile="tiny-cpu", overrides=["spec.drafter=mtp", "spec.block_rows=4", "serving.slots=2"])
    eng = build_engine(rc)
    gold = greedy_reference(eng.target, p, 10)
    eng.add_request(p, 10, request_id="m1")
    eng.add_request(_prompt(33, 30), 10, request_id="m2")
    done = {r.request_id: r for r in eng.run()}
    assert done["m1"].output == gold and done["m2"].state == FINISHED
    app = build_app(eng, output_budget_multiple=4)
    with TestClient(app) as client:
        assert client.post("/v1/completions", json={"prompt": p, "max_tokens": 6}).status_code == 400
        assert client.post("/v1/completions", json={"prompt": p, "max_tokens": 8}).status_code == 200
    app.state.loop.close()


def test_sampled_requests_next_to_greedy_ones(tiny):
    """A sampled request (temperature > 0, one token per step) runs packed with greedy speculative
    ones; its tokens equal the target's own sampled decoding for the same seed, and the greedy
    request stays token-exact."""
    tgt, dr = _setup(tiny, slots=2)
    p1, p2 = _prompt(41, 48), _prompt(42, 40)
    gold = greedy_reference(tgt, p1, 10)
    ref = tgt.sample(torch.tensor(p2), 10, temperature=0.9, seed=5)
    eng = ServingEngine(tgt, dr, verifier_rows=4)
    eng.add_request(p1, 10, request_id="g")
    eng.add_request(p2, 10, request_id="s", temperature=0.9, seed=5)
    done = {r.request_id: r for r in eng.run()}
    assert done["g"].output == gold
    assert done["s"].output == ref


def test_streaming_and_chat_endpoints(tiny):
    """Server-sent events deliver each step's tokens (their concatenation is the whole greedy
    output) and end with [DONE]; chat completions render messages and answer in both modes."""
    import json as _json

    from fastapi.testclient import TestClient

    from qwen38_b200.serving.api import ByteTokenizer, build_app, render_chat
    tgt, dr = _setup(tiny, slots=2)
    p1 = _prompt(51, 40)
    gold = greedy_reference(tgt, p1, 12)
    eng = ServingEngine(tgt, dr, verifier_rows=4)
    app = build_app(eng, model_name="tiny")
    with TestClient(app) as client:
        r = client.post("/v1/completions", json={"prompt": p1, "max_tokens": 12, "stream": True})
        assert r.status_code == 200 and r.headers["content-type"].startswith("text/event-stream")
        events = [ln[len("data: "):] for ln in r.text.splitlines() if ln.startswith("data: ")]
        assert events[-1] == "[DONE]"
        chunks = [_json.loads(e) for e in events[:-1]]
        toks = [t for c in chunks for t in c["choices"][0]["token_ids"]]
        assert toks == gold
        assert chunks[-1]["choices"][0]["finish_reason"] == "length"
        assert len(chunks) > 2                              # several steps, several events
        msgs = [{"role": "user", "content": "hi"}]
        r = client.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 6})
        assert r.status_code == 200
        body = r.json()
        ids = ByteTokenizer().encode(render_chat([type("M", (), m) for m in msgs]))
        assert body["choices"][0]["token_ids"] == greedy_reference(tgt, ids, 6)
        assert body["usage"]["prompt_tokens"] == len(ids)
        r = client.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 6, "stream": True})
        events = [ln[len("data: "):] for ln in r.text.splitlines() if ln.startswith("data: ")]
        assert events[-1] == "[DONE]" and _json.loads(events[0])["object"] == "chat.completion.chunk"
        bad = client.post("/v1/completions", json={"prompt": [999999], "max_tokens": 4, "stream": True})
        assert "error" in bad.text
    app.state.loop.close()


def test_endpoint_isolation_gate():
    """The isolation gate against a live server (uvicorn on 127.0.0.1): streamed greedy outputs are
    the same alone and concurrent, the decoders keep streaming through a long prefill, and the
    token accounting of every stream adds up."""
    import socket
    import threading
    import time

    import uvicorn

    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.api import build_app
    from qwen38_b200.serving.factory import build_engine
    from qwen38_b200.serving.isolation import measure
    eng = build_engine(load_run_config(profile="tiny-cpu", overrides=["serving.slots=4"]))
    app = build_app(eng)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    try:
        for _ in range(500):
            if server.started:
                break
            time.sleep(0.01)
        rep = measure(f"http://127.0.0.1:{port}", prompt_length=600, decoders=2, decode_tokens=40,
                      short_delay=0.0, ready_timeout=120.0, short_tokens=8)
        assert rep["passed"], rep["checks"]
        assert set(rep["concurrent"]) == {"A", "B0", "B1", "C"}
        assert all(r["tokens"] == rep["baseline"][n]["tokens"] for n, r in rep["concurrent"].items())
    finally:
        server.should_exit = True
        th.join(timeout=30)
        app.state.loop.close()


def test_real_text_concurrent_equals_sequential():
    """Repository text as prompts: every answer is byte-identical alone and packed with the others."""
    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.factory import build_engine
    from qwen38_b200.serving.realtext import compare, text_prompts
    eng = build_engine(load_run_config(profile="tiny-cpu", overrides=["serving.slots=4"]))
    prompts = text_prompts(chars=300)
    assert len(prompts) == 4
    rep = compare(eng, prompts, max_tokens=16)
    assert rep["passed"], rep
    assert all(r["tokens"] == 16 for r in rep["prompts"])


def _loadgen_rank(rank, port, q):
    import os

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        from qwen38_b200.checkpoint import MXFP8Source, random_drafter_source, random_target_source
        from qwen38_b200.config import tiny_drafter_config, tiny_model_config
        from qwen38_b200.parallel.comm import TorchComm
        from qwen38_b200.serving.loadgen import poisson_arrivals, run
        cfg, dcfg = tiny_model_config(), tiny_drafter_config()
        tgt = HybridTarget(cfg, MXFP8Source(random_target_source(cfg, 0)), RuntimeConfig(max_context=512),
                           comm=TorchComm(), max_slots=4, max_verify_rows=3 * dcfg.block_rows)
        dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, 1), tgt, slots=3)
        g = torch.Generator().manual_seed(0)
        prompts = [torch.randint(0, cfg.vocab_size, (80,), generator=g).tolist() for _ in range(3)]
        golds = [greedy_reference(tgt, p, 12) for p in prompts]

        def agree(n):
            t = torch.tensor([n])
            dist.broadcast(t, 0)
            return int(t.item())
        rep = run(ServingEngine(tgt, dr, verifier_rows=dcfg.block_rows), prompts, 12,
                  poisson_arrivals(3, 50.0, 0), golds=golds, mean_accepted=1, agree=agree)
        q.put((rank, rep["finished"], rep["exact"], rep["decode_steps"]))
    except BaseException as e:
        q.put((rank, repr(e), False, -1))
    finally:
        dist.destroy_process_group()


def test_loadgen_tp2_ranks_admit_in_lockstep():
    """Two gloo ranks with MXFP8 weights: rank 0's clock decides the arrivals, both ranks run the
    same steps, every stream finishes token-exact."""
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_loadgen_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert out[0][1:] == out[1][1:], out
    assert out[0][1] == 3 and out[0][2] is True


def test_completion_logprobs():
    """``logprobs`` on a greedy completion: every output token is its own row's top-1, with a
    non-positive log-probability; streaming requests refuse the option."""
    from fastapi.testclient import TestClient

    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.api import build_app
    from qwen38_b200.serving.factory import build_engine
    eng = build_engine(load_run_config(profile="tiny-cpu", overrides=["serving.slots=2"]))
    app = build_app(eng)
    with TestClient(app) as client:
        r = client.post("/v1/completions", json={"prompt": list(range(20, 60)), "max_tokens": 10, "logprobs": 3})
        assert r.status_code == 200, r.text
        ch = r.json()["choices"][0]
        lp = ch["logprobs"]
        assert lp["token_ids"] == ch["token_ids"] and len(lp["token_logprobs"]) == 10
        assert all(v <= 0 for v in lp["token_logprobs"])
        assert all(top[0] == t for top, t in zip(lp["top_token_ids"], ch["token_ids"]))
        assert all(len(d) <= 3 for d in lp["top_logprobs"])
        assert client.post("/v1/completions", json={"prompt": [5, 6], "max_tokens": 2}).json()["choices"][0][
            "logprobs"] is None
        bad = client.post("/v1/completions", json={"prompt": [5, 6], "max_tokens": 2, "logprobs": 2, "stream": True})
        assert bad.status_code == 400
    app.state.loop.close()


def test_request_validation(tiny):
    """Bad budgets and a request id already in flight are refused at admission."""
    import pytest
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16),
                       max_slots=3)
    eng = ServingEngine(tgt, None, verifier_rows=4)
    with pytest.raises(ValueError):
        eng.add_request([1, 2, 3], 0)
    with pytest.raises(ValueError):
        eng.add_request([1, 2, 3], 600)
    eng.add_request([1, 2, 3], 4, request_id="x")
    with pytest.raises(ValueError):
        eng.add_request([4, 5], 4, request_id="x")
    done = {r.request_id for r in eng.run()}
    assert "x" in done
    eng.add_request([4, 5], 4, request_id="x")          # finished ids may be reused
    assert {r.request_id for r in eng.run()} == {"x"}


def _serve_rank(rank, port, q):
    import os
    import time

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        from qwen38_b200.parallel.comm import TorchComm
        from qwen38_b200.runconfig import load_run_config
        from qwen38_b200.serving.api import EngineLoop, broadcast_sync, follow
        from qwen38_b200.serving.factory import build_engine
        rc = load_run_config(profile="tiny-cpu", overrides=["parallel.tp=2", "serving.slots=3"])
        eng = build_engine(rc, comm=TorchComm())
        sync = broadcast_sync()
        if rank > 0:
            follow(eng, sync)
            q.put((rank, "followed"))
            return
        # decode stand-in: a request's text contains "STOP" once it has 5 tokens
        loop = EngineLoop(eng, sync=sync, heartbeat_s=0.05, decode=lambda ids: "STOP" if len(ids) >= 5 else "")
        prompts = [list(range(10 + i, 50 + 3 * i)) for i in range(3)]
        boxes = [loop.submit(p, 8) for p in prompts]
        stopped = loop.submit(list(range(60, 100)), 30, stop=["STOP"])     # ends early on every rank
        gone = loop.submit(list(range(61, 90)), 200)                        # cancelled once admitted
        for _ in range(3000):
            if "rid" in gone[1]:
                break
            time.sleep(0.01)
        loop.cancel(gone[1]["rid"])
        bad = loop.submit([10 ** 6], 4)                  # refused on rank 0, never sent to the others
        time.sleep(0.3)                                  # idle heartbeats in between
        late = loop.submit(list(range(7, 30)), 8)
        outs = []
        for done, box in boxes + [late]:
            assert done.wait(300)
            outs.append(box["request"].output)
        assert bad[0].wait(10) and "error" in bad[1]
        assert stopped[0].wait(300) and 5 <= len(stopped[1]["request"].output) < 30
        assert gone[0].wait(300) and gone[1]["request"].state == "aborted"
        chosen, top_ids, _ = loop.call_shared("score", prompts[0], outs[0], 3)    # collectives on both ranks
        loop.close()
        q.put((rank, (outs, chosen.tolist(), top_ids.tolist())))
    except BaseException as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_server_ranks_follow_rank0(tiny):
    """A TP2 server on gloo ranks: rank 0 admits and steps, rank 1 follows its commands; outputs
    equal single-rank greedy decode, idle heartbeats and a refused request keep the ranks in step."""
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_serve_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert out[1] == "followed", out
    assert isinstance(out[0], tuple), out[0]
    outs, chosen, top_ids = out[0]
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=2048, prefill_chunk=256, gdn_chunk=16))
    prompts = [list(range(10 + i, 50 + 3 * i)) for i in range(3)] + [list(range(7, 30))]
    for p, o in zip(prompts, outs):
        assert o == greedy_reference(tgt, p, len(o))
    from qwen38_b200.utils.tp_agreement import score
    c1, t1, _ = score(tgt, prompts[0], outs[0], 3)
    assert t1.tolist() == top_ids and max(abs(a - b) for a, b in zip(c1.tolist(), chosen)) < 1e-4


def test_stop_strings_end_requests_early():
    """A stop string cuts the text before it, reports finish_reason "stop" and ends generation at
    the step it appears in (fewer tokens than the budget), streamed or not."""
    from fastapi.testclient import TestClient

    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.api import ByteTokenizer, build_app
    from qwen38_b200.serving.factory import build_engine
    eng = build_engine(load_run_config(profile="tiny-cpu", overrides=["serving.slots=2"]))
    tok = ByteTokenizer()
    app = build_app(eng)
    with TestClient(app) as client:
        prompt = list(range(40, 90))
        full = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 80}).json()["choices"][0]
        ids = full["token_ids"]
        text = tok.decode(ids)
        # a printable character the greedy output emits early on serves as the stop string
        k = next(i for i in range(3, 70) if 32 <= ids[i] < 127)
        stop = chr(ids[k])
        r = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 80, "stop": [stop]}).json()
        ch = r["choices"][0]
        assert ch["finish_reason"] == "stop" and ch["text"] == text[:text.find(stop)]
        assert len(ch["token_ids"]) < 80 and ch["token_ids"] == ids[:len(ch["token_ids"])]
        # streamed: the text before the stop string arrives in pieces, then finish_reason "stop"
        import json as _json
        sr = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 80, "stop": [stop, "zzz"],
                                                  "stream": True})
        events = [_json.loads(l[6:]) for l in sr.text.splitlines() if l.startswith("data: {")]
        assert "".join(e["choices"][0]["text"] for e in events) == text[:text.find(stop)]
        assert events[-1]["choices"][0]["finish_reason"] == "stop"
    app.state.loop.close()


def test_batched_prompts_and_n_choices():
    """A batch of prompts with n completions each: greedy choices of one prompt are identical and
    equal single-request greedy decode; sampled choices use seeds seed, seed+1, ..."""
    from fastapi.testclient import TestClient

    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.api import build_app
    from qwen38_b200.serving.factory import build_engine
    eng = build_engine(load_run_config(profile="tiny-cpu", overrides=["serving.slots=4"]))
    app = build_app(eng)
    pa, pb = list(range(30, 70)), list(range(100, 130))
    with TestClient(app) as client:
        r = client.post("/v1/completions", json={"prompt": [pa, pb], "max_tokens": 6, "n": 2}).json()
        ch = r["choices"]
        assert [c["index"] for c in ch] == [0, 1, 2, 3]
        assert ch[0]["token_ids"] == ch[1]["token_ids"] == greedy_reference(eng.target, pa, 6)
        assert ch[2]["token_ids"] == ch[3]["token_ids"] == greedy_reference(eng.target, pb, 6)
        assert r["usage"]["prompt_tokens"] == len(pa) + len(pb) and r["usage"]["completion_tokens"] == 24
        s = client.post("/v1/completions", json={"prompt": pa, "max_tokens": 6, "n": 2, "temperature": 1.0,
                                                  "seed": 11}).json()["choices"]
        one = [client.post("/v1/completions", json={"prompt": pa, "max_tokens": 6, "temperature": 1.0,
                                                     "seed": 11 + j}).json()["choices"][0]["token_ids"]
               for j in range(2)]
        assert [c["token_ids"] for c in s] == one
        assert client.post("/v1/completions", json={"prompt": [pa, pb], "max_tokens": 2,
                                                    "stream": True}).status_code == 400
        assert client.post("/v1/completions", json={"prompt": pa, "max_tokens": 2, "n": 0}).status_code == 400
    app.state.loop.close()


def test_chat_n_and_logprobs():
    """Chat with n answers and per-token log-probabilities (OpenAI chat layout)."""
    from fastapi.testclient import TestClient

    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.api import build_app
    from qwen38_b200.serving.factory import build_engine
    eng = build_engine(load_run_config(profile="tiny-cpu", overrides=["serving.slots=3"]))
    app = build_app(eng)
    msgs = [{"role": "user", "content": "hello there"}]
    with TestClient(app) as client:
        r = client.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 5, "n": 2, "logprobs": True,
                                                       "top_logprobs": 2})
        assert r.status_code == 200, r.text
        ch = r.json()["choices"]
        assert len(ch) == 2 and ch[0]["token_ids"] == ch[1]["token_ids"]        # greedy: the same answer
        content = ch[0]["logprobs"]["content"]
        assert [c["token_id"] for c in content] == ch[0]["token_ids"]
        assert all(c["logprob"] <= 0 and len(c["top_logprobs"]) == 2 for c in content)
        assert all(c["top_logprobs"][0]["token_id"] == c["token_id"] for c in content)
        assert client.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 2, "n": 2,
                                                         "stream": True}).status_code == 400
    app.state.loop.close()


def test_cancel_aborts_a_running_request(tiny):
    """A cancelled request (its client went away) is aborted before its budget and frees its slot."""
    import time as _t

    from qwen38_b200.serving.api import EngineLoop
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=1024, prefill_chunk=64, gdn_chunk=16),
                       max_slots=2)
    eng = ServingEngine(tgt, None, verifier_rows=4)
    free0 = tgt.allocator.num_free
    loop = EngineLoop(eng)
    done, box = loop.submit(list(range(10, 40)), 500)
    for _ in range(3000):
        if box.get("rid") and len(eng.requests[box["rid"]].output) > 2:
            break
        _t.sleep(0.01)
    loop.cancel(box["rid"])
    assert done.wait(60)
    req = box["request"]
    assert req.state == ABORTED and len(req.output) < 500 and "cancelled" in req.error
    assert tgt.allocator.num_free == free0 and loop.aborted == 1
    loop.close()


def test_phase_log_and_acceptance_metrics(tmp_path):
    """Finished requests land in the phase log with their block records; the acceptance report of
    the log and the /metrics gauges agree with the engine's blocks."""
    import json
    import subprocess
    import sys

    from fastapi.testclient import TestClient

    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.api import build_app
    from qwen38_b200.serving.factory import build_engine
    from qwen38_b200.spec.analysis import acceptance_report_requests
    log = str(tmp_path / "phases.jsonl")
    eng = build_engine(load_run_config(profile="tiny-cpu", overrides=["serving.slots=2"]))
    app = build_app(eng, phase_log=log)
    with TestClient(app) as client:
        for p in (list(range(20, 60)), list(range(70, 99))):
            assert client.post("/v1/completions", json={"prompt": p, "max_tokens": 12}).status_code == 200
        m = client.get("/metrics").text
    app.state.loop.close()
    recs = [json.loads(l) for l in open(log)]
    assert len(recs) == 2 and all(r["output_tokens"] == 12 for r in recs)
    assert all(sum(b["committed"] for b in r["blocks"]) == 11 for r in recs)   # the first token is the prefill's
    rep = acceptance_report_requests([r["blocks"] for r in recs])
    assert f"q38_committed_tokens_per_block {rep['mean_committed_per_block']}" in m
    out = subprocess.run([sys.executable, "-m", "qwen38_b200.spec.analysis", log], capture_output=True, text=True,
                         timeout=120)
    assert out.returncode == 0 and json.loads(out.stdout)["requests"] == 2


def test_engine_fault_fails_requests_and_serving_continues(tiny):
    """An exception escaping an engine step fails the requests in flight (their waiters get the
    error) and releases them; the loop keeps serving the next request."""
    from qwen38_b200.serving.api import EngineLoop
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16),
                       max_slots=3)
    eng = ServingEngine(tgt, None, verifier_rows=4)
    free0 = tgt.allocator.num_free
    real = eng.step
    state = {"n": 0}

    def flaky():
        state["n"] += 1
        if state["n"] == 3:
            raise RuntimeError("injected engine fault")
        return real()
    eng.step = flaky
    loop = EngineLoop(eng)
    d1, b1 = loop.submit(list(range(10, 40)), 30)
    assert d1.wait(60) and b1["request"].state == ABORTED and "injected" in b1["request"].error
    d2, b2 = loop.submit(list(range(50, 70)), 6)
    assert d2.wait(60) and b2["request"].output == greedy_reference(tgt, list(range(50, 70)), 6)
    assert loop.faults == 1 and tgt.allocator.num_free == free0
    loop.close()


def test_sampled_requests_speculate_exactly(tiny):
    """With counter-based Gumbel noise a sampled token depends only on its prefix, seed and position,
    so block speculation on a sampled request commits several tokens per block and still yields
    exactly the one-token-per-step sample."""
    tgt, dr = _setup(tiny, slots=2)
    p = _prompt(43, 44)
    ref = tgt.sample(torch.tensor(p), 24, temperature=0.8, seed=9)
    for speculate, pinned in ((True, PinnedAcceptance(ref, seed=4, mean_accepted=2)), (True, None), (False, None)):
        eng = ServingEngine(tgt, dr, verifier_rows=4, speculate_sampled=speculate)
        eng.add_request(p, 24, request_id="s", temperature=0.8, seed=9, pinned=pinned)
        req = {r.request_id: r for r in eng.run()}["s"]
        assert req.output == ref
        if pinned is not None:
            assert max(b["committed"] for b in req.blocks) > 1 and len(req.blocks) < 23
        if not speculate:
            assert all(b["rows"] == 1 for b in req.blocks)


def test_completion_echo():
    from fastapi.testclient import TestClient

    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.api import build_app
    from qwen38_b200.serving.factory import build_engine
    eng = build_engine(load_run_config(profile="tiny-cpu"))
    app = build_app(eng)
    with TestClient(app) as client:
        a = client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 4}).json()["choices"][0]
        b = client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 4, "echo": True}).json()["choices"][0]
        assert b["text"] == "abc" + a["text"] and b["token_ids"] == a["token_ids"]
    app.state.loop.close()


def test_text_stream_keeps_split_characters_whole():
    """A multi-byte UTF-8 character whose bytes arrive in two engine steps goes out once, whole,
    with and without stop strings (the streamed text equals the non-streamed text)."""
    from qwen38_b200.serving.api import ByteTokenizer, TextStream
    tok = ByteTokenizer()
    text = "a€b→c"
    ids = tok.encode(text)
    steps = [ids[:2], ids[2:3], ids[3:6], ids[6:8], ids[8:]]       # '€' and '→' split over steps
    for stops in ([], ["x"], ["zz"]):
        ts = TextStream(tok, stops)
        parts = [ts.push(s) for s in steps]
        assert not any(stopped for _, stopped in parts)
        streamed = "".join(p for p, _ in parts) + ts.finish()[0]
        assert streamed == text and "�" not in streamed
    ts = TextStream(tok, ["→"])
    parts = [ts.push(s) for s in steps]
    stopped_at = [i for i, (_, st) in enumerate(parts) if st]
    assert stopped_at and "".join(p for p, _ in parts[:stopped_at[0] + 1]) == "a€b"


def test_streaming_completion_echo():
    """``echo`` on a streamed completion: the prompt text is the first event, then the completion
    text, which together equal the non-streamed echoed text."""
    import json

    from fastapi.testclient import TestClient

    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.api import build_app
    from qwen38_b200.serving.factory import build_engine
    eng = build_engine(load_run_config(profile="tiny-cpu"))
    app = build_app(eng)
    with TestClient(app) as client:
        ref = client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 4, "echo": True}).json()
        r = client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 4, "echo": True, "stream": True})
        events = [json.loads(l[6:]) for l in r.text.split("\n") if l.startswith("data: {")]
        assert events[0]["choices"][0]["text"] == "abc"
        assert "".join(e["choices"][0]["text"] for e in events) == ref["choices"][0]["text"]
        lp = client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 3, "echo": True,
                                                  "logprobs": 2}).json()["choices"][0]["logprobs"]
        assert lp["token_ids"][:3] == [97, 98, 99] and lp["token_logprobs"][0] is None
        assert len(lp["token_logprobs"]) == 3 + 3 and all(v is not None for v in lp["token_logprobs"][1:])
    app.state.loop.close()


def test_packed_verify_rows_capped_by_the_targets_batch_invariant_rows(tiny):
    """A target whose kernels keep at most ``max_pack_rows`` rows batch-invariant gets packed verifies
    of at most that many rows; the other running requests rotate into the next packs and every
    request still equals its single-stream greedy output."""
    tgt, dr = _setup(tiny)
    tgt.max_pack_rows = 8                       # two 4-row blocks per packed verify
    prompts = [_prompt(11, 80), _prompt(12, 60), _prompt(13, 90)]
    golds = [greedy_reference(tgt, p, 12) for p in prompts]
    eng = ServingEngine(tgt, dr, verifier_rows=4)
    assert eng.sched.max_step_rows == 8
    reqs = [eng.add_request(p, 12, pinned=PinnedAcceptance(g, seed=i, mean_accepted=1))
            for i, (p, g) in enumerate(zip(prompts, golds))]
    eng.run()
    for r, g in zip(reqs, golds):
        assert r.state == FINISHED, r.error
        assert r.output == g
