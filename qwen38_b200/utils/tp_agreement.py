"""Token agreement between two tensor-parallel configurations of one model.

Different TP degrees sum each layer's partial products in a different order, so their greedy
tokens are not bit-equal: a near-tie can flip and the texts drift apart after it.  That is
expected, not a fault.  What a new TP degree has to show instead (the reference's
``scripts/ci/tp_agreement.py``) is: (1) coherent output (long enough, not a loop), (2) a long
common prefix before the first flip, (3) at the first flip each side's token inside the other's
top-k and within ``margin`` nats of the other's choice (a rounding flip is a near-tie; a broken
model's is not), and (4) a similar perplexity of each side's own text.

``collect`` answers a fixed prompt set greedily through the engine and scores every emitted token
with the engine's own final norm and LM head (log-probability of the chosen token and the top-k);
``compare`` judges two collections.  Prompts are this repository's own sources as byte-level token
ids, so a run needs no corpus and no tokenizer download.

    python -m qwen38_b200.utils.tp_agreement collect --profile single-stream-4k --out tp1.json
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m qwen38_b200.utils.tp_agreement collect \\
        --profile single-stream-4k --set parallel.tp=2 --out tp2.json
    python -m qwen38_b200.utils.tp_agreement compare tp1.json tp2.json --report agreement.json
    python -m qwen38_b200.utils.tp_agreement collect --url http://127.0.0.1:8000 --tp 2 --out srv.json
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os

import torch

TOP_K = 5
MIN_PREFIX = 24
DIVERGENCE_MARGIN = 0.5        # nats: a bf16 rounding flip sits within this of the other choice
MAX_PPL_RATIO = 1.10
MIN_UNIQUE_RATIO = 0.25

PROMPT_FILES = (
    ("doc", "README.md", 3000, "Summarise the key argument of this document in five bullet points."),
    ("code-attention", "qwen38_b200/csrc/attention.cu", 6000, "Explain what this kernel file does, part by part."),
    ("code-engine", "qwen38_b200/spec/engine.py", 6000, "Describe the control flow of this module."),
)


def repo_prompts(root: str | None = None, limit_chars: int | None = None):
    """[(name, token ids)] from this repository's files (UTF-8 bytes as ids)."""
    root = root or os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    out = []
    for name, path, chars, instruction in PROMPT_FILES:
        full = os.path.join(root, path)
        if not os.path.isfile(full):
            continue
        with open(full, encoding="utf-8", errors="replace") as f:
            text = f.read()[:limit_chars or chars]
        out.append((name, list(f"{instruction}\n\n---\n{text}\n---\n".encode("utf-8"))))
    return out


@torch.no_grad()
def score(target, prompt, output, top_k: int = TOP_K):
    """Log-probabilities the target assigns to ``output`` after ``prompt``: (chosen [n],
    top-k ids [n, k], top-k log-probs [n, k]), from the last layer's rows through the final norm and
    the (vocab-sharded, gathered) LM head."""
    last = target.cfg.num_hidden_layers - 1
    seq = target.new_sequence()
    try:
        toks = torch.as_tensor(list(prompt) + list(output[:-1]), dtype=torch.long, device=target.device)
        _, feats = target.prefill(seq, toks, taps=(last,))
    finally:
        target.release(seq)
    rows = feats[len(prompt) - 1:]
    hn = target.ops.rms_norm(rows, target.final_norm, target.eps, target.dtype)
    logits = target.ops.linear(hn, target.lm_head, out_dtype=torch.float32)
    if target.tp > 1:
        logits = target.comm.all_gather_cat(logits.contiguous(), 1)
    lp = torch.log_softmax(logits.double(), -1)
    out = torch.as_tensor(list(output), dtype=torch.long, device=lp.device)
    chosen = lp.gather(1, out[:, None])[:, 0]
    tv, ti = lp.topk(top_k, -1)
    return chosen.cpu(), ti.cpu(), tv.cpu()


def collect(target, prompts, max_tokens: int = 64, top_k: int = TOP_K, runtime=None):
    """Greedy answers (through ``runtime.generate`` when a ``SpecRuntime`` is given, else plain
    greedy decode) with per-token scores.  Returns the JSON-able record."""
    recs = []
    for name, ids in prompts:
        if runtime is not None:
            toks = runtime.generate(ids, max_tokens)["tokens"]
        else:
            toks = target.greedy(torch.as_tensor(ids, dtype=torch.long, device=target.device), max_tokens)
        chosen, ti, tv = score(target, ids, toks, top_k)
        recs.append(dict(name=name, prompt_sha256=hashlib.sha256(bytes(str(list(ids)), "utf-8")).hexdigest(),
                         tokens=[int(t) for t in toks], logprobs=[float(v) for v in chosen],
                         top_ids=ti.tolist(), top_logprobs=tv.tolist()))
    return dict(schema=1, tp=int(getattr(target, "tp", 1)), top_k=top_k, prompts=recs)


def collect_http(base_url: str, prompts, max_tokens: int = 64, top_k: int = TOP_K, model: str | None = None,
                 tp: int | None = None, timeout: float = 1800.0):
    """``collect`` through a running server's ``/v1/completions`` (greedy, ``logprobs=top_k``), as
    the reference collects over the OpenAI API."""
    import urllib.request
    recs = []
    for name, ids in prompts:
        payload = dict(prompt=list(ids), max_tokens=max_tokens, temperature=0.0, logprobs=top_k)
        if model:
            payload["model"] = model
        req = urllib.request.Request(base_url.rstrip("/") + "/v1/completions", json.dumps(payload).encode(),
                                     {"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=timeout) as resp:
            ch = json.loads(resp.read())["choices"][0]
        lp = ch["logprobs"]
        recs.append(dict(name=name, prompt_sha256=hashlib.sha256(bytes(str(list(ids)), "utf-8")).hexdigest(),
                         tokens=list(ch["token_ids"]), logprobs=list(lp["token_logprobs"]),
                         top_ids=lp["top_token_ids"], top_logprobs=lp["top_token_logprobs"]))
    return dict(schema=1, tp=tp, top_k=top_k, prompts=recs)


def _coherent(tokens):
    return len(tokens) >= 2 and len(set(tokens)) / len(tokens) >= MIN_UNIQUE_RATIO


def _perplexity(logprobs):
    return math.exp(-sum(logprobs) / max(1, len(logprobs)))


def compare(ref: dict, cand: dict, *, margin: float = DIVERGENCE_MARGIN, max_ratio: float = MAX_PPL_RATIO,
            min_prefix: int = MIN_PREFIX) -> dict:
    """Per-prompt and overall verdict of ``cand`` against ``ref`` (see the module docstring)."""
    by_name = {p["name"]: p for p in ref["prompts"]}
    rows, ok = [], True
    for c in cand["prompts"]:
        r = by_name.get(c["name"])
        if r is None or r["prompt_sha256"] != c["prompt_sha256"]:
            rows.append(dict(name=c["name"], verdict="NOT_COMPARABLE"))
            ok = False
            continue
        a, b = r["tokens"], c["tokens"]
        n = min(len(a), len(b))
        k = next((i for i in range(n) if a[i] != b[i]), n)
        row = dict(name=c["name"], common_prefix=k, tokens=(len(a), len(b)),
                   ppl_ref=_perplexity(r["logprobs"]), ppl_cand=_perplexity(c["logprobs"]))
        row["ppl_ratio"] = row["ppl_cand"] / row["ppl_ref"]
        checks = {"coherent": _coherent(a) and _coherent(b),
                  "ppl_ratio": 1 / max_ratio <= row["ppl_ratio"] <= max_ratio}
        if k < n:
            # each side's token at the split must be a near-tie in the other side's distribution
            def near_tie(rec, other_tok):
                ids, lps = rec["top_ids"][k], rec["top_logprobs"][k]
                return other_tok in ids and lps[0] - lps[ids.index(other_tok)] <= margin
            checks["near_tie_flip"] = near_tie(r, b[k]) and near_tie(c, a[k])
            checks["prefix"] = k >= min(min_prefix, n)
        row["checks"] = checks
        row["verdict"] = "AGREE" if all(checks.values()) else "DISAGREE"
        ok = ok and row["verdict"] == "AGREE"
        rows.append(row)
    return dict(ok=ok, tp=(ref.get("tp"), cand.get("tp")), prompts=rows,
                thresholds=dict(margin=margin, max_ppl_ratio=max_ratio, min_prefix=min_prefix,
                                min_unique_ratio=MIN_UNIQUE_RATIO))


def main(argv=None):
    ap = argparse.ArgumentParser(description="TP-vs-TP greedy token agreement")
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("collect")
    c.add_argument("--profile", default=None)
    c.add_argument("--config", default=None)
    c.add_argument("--set", action="append", default=[])
    c.add_argument("--max-tokens", type=int, default=64)
    c.add_argument("--url", default=None, help="collect through a running server's /v1/completions instead")
    c.add_argument("--tp", type=int, default=None, help="TP degree of that server (recorded only)")
    c.add_argument("--out", required=True)
    m = sub.add_parser("compare")
    m.add_argument("ref")
    m.add_argument("cand")
    m.add_argument("--report", default=None)
    a = ap.parse_args(argv)
    if a.cmd == "compare":
        with open(a.ref) as f:
            ref = json.load(f)
        with open(a.cand) as f:
            cand = json.load(f)
        rep = compare(ref, cand)
        if a.report:
            with open(a.report, "w") as f:
                json.dump(rep, f, indent=1)
        print(json.dumps({k: v for k, v in rep.items() if k != "prompts"}))
        return 0 if rep["ok"] else 1
    if a.url:
        rec = collect_http(a.url, repo_prompts(), a.max_tokens, tp=a.tp)
        with open(a.out, "w") as f:
            json.dump(rec, f)
        return 0
    from ..parallel.comm import init_distributed
    from ..runconfig import load_run_config
    from ..serving.factory import build_engine
    rank, world, local = init_distributed()
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    eng = build_engine(load_run_config(a.config, profile=a.profile, overrides=a.set))
    rec = collect(eng.target, repo_prompts(), a.max_tokens)
    if rank == 0:
        with open(a.out, "w") as f:
            json.dump(rec, f)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
