"""TP agreement tool: scores are the engine's own (the greedy token is each row's top-1), identical
collections agree, a near-tie flip agrees while a confident flip does not, and a gloo TP2
collection agrees with TP1."""
import copy
import os
import socket

import torch
import torch.multiprocessing as mp

from qwen38_b200.config import RuntimeConfig
from qwen38_b200.models.target import HybridTarget
from qwen38_b200.utils.tp_agreement import collect, compare, repo_prompts, score

RT = RuntimeConfig(max_context=2048, prefill_chunk=256, gdn_chunk=16)


def _prompts():
    return [(n, ids[:300]) for n, ids in repo_prompts()][:2]


def test_scores_match_the_engines_greedy_choice(tiny):
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RT)
    rec = collect(tgt, _prompts(), max_tokens=24)
    assert len(rec["prompts"]) == 2
    for p in rec["prompts"]:
        assert len(p["tokens"]) == 24 and all(lp <= 0 for lp in p["logprobs"])
        for i, t in enumerate(p["tokens"]):
            assert p["top_ids"][i][0] == t                      # greedy = the scored argmax
            assert abs(p["top_logprobs"][i][0] - p["logprobs"][i]) < 1e-9
    rep = compare(rec, copy.deepcopy(rec))
    assert rep["ok"] and all(r["common_prefix"] == 24 for r in rep["prompts"])


def _flip(rec, k, tok, gap):
    """A copy whose prompt 0 diverges at k to ``tok`` with a top-1/top-2 gap of ``gap`` nats on both sides."""
    ref, cand = copy.deepcopy(rec), copy.deepcopy(rec)
    a, c = ref["prompts"][0], cand["prompts"][0]
    c["tokens"][k] = tok
    for side, other in ((a, tok), (c, a["tokens"][k])):
        ids = side["top_ids"][k]
        lps = side["top_logprobs"][k]
        side["top_ids"][k] = [ids[0], other] + [i for i in ids[1:] if i != other][:len(ids) - 2]
        side["top_logprobs"][k] = [lps[0], lps[0] - gap] + lps[2:len(ids)]
    return ref, cand


def test_divergence_judged_by_margin(tiny):
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RT)
    rec = collect(tgt, _prompts()[:1], max_tokens=40)
    t = rec["prompts"][0]["tokens"]
    alt = (t[30] + 1) % tiny["cfg"].vocab_size
    ref, cand = _flip(rec, 30, alt, 0.1)
    r = compare(ref, cand)
    assert r["ok"] and r["prompts"][0]["common_prefix"] == 30
    ref, cand = _flip(rec, 30, alt, 3.0)
    assert not compare(ref, cand)["ok"]
    ref, cand = _flip(rec, 3, alt, 0.1)                          # too short a common prefix
    assert not compare(ref, cand)["ok"]
    cand = copy.deepcopy(rec)
    cand["prompts"][0]["prompt_sha256"] = "0"
    assert compare(rec, cand)["prompts"][0]["verdict"] == "NOT_COMPARABLE"


def _worker(rank, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        from qwen38_b200.checkpoint import random_target_source
        from qwen38_b200.config import tiny_model_config
        from qwen38_b200.parallel.comm import TorchComm
        cfg = tiny_model_config()
        tgt = HybridTarget(cfg, random_target_source(cfg, 0), RT, comm=TorchComm())
        q.put((rank, collect(tgt, _prompts(), max_tokens=24)))
    except BaseException as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_tp2_gloo_agrees_with_tp1(tiny):
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RT)
    ref = collect(tgt, _prompts(), max_tokens=24)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted((q.get(timeout=300) for _ in procs), key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
    for rank, rec in out:
        assert isinstance(rec, dict), rec
        assert rec["tp"] == 2
        rep = compare(ref, rec)
        assert rep["ok"], rep
    assert out[0][1]["prompts"] == out[1][1]["prompts"]


def test_http_collection_equals_in_process(tiny):
    """Collecting through the server's logprobs gives the in-process record of the same engine."""
    import threading
    import time

    import uvicorn

    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.api import build_app
    from qwen38_b200.serving.factory import build_engine
    from qwen38_b200.utils.tp_agreement import collect_http
    eng = build_engine(load_run_config(profile="tiny-cpu", overrides=["spec.drafter=none", "serving.slots=1"]))
    prompts = [(n, ids[:120]) for n, ids in _prompts()]
    local = collect(eng.target, prompts, max_tokens=12, top_k=3)
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
        remote = collect_http(f"http://127.0.0.1:{port}", prompts, max_tokens=12, top_k=3, tp=1)
    finally:
        server.should_exit = True
        th.join(timeout=30)
        app.state.loop.close()
    assert compare(local, remote)["ok"]
    for a, b in zip(local["prompts"], remote["prompts"]):
        assert a["tokens"] == b["tokens"] and a["top_ids"] == b["top_ids"]
        assert max(abs(x - y) for x, y in zip(a["logprobs"], b["logprobs"])) < 1e-9
