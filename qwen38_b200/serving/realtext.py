"""Real-text exactness: the same prompts answered one at a time and all at once must give the same
bytes.

The reference compares concurrent against sequential serving output on real text
(``scripts/ci/real_text_compare.py``, prompts from ``real_text_prompts.py``).  Here the prompts are
text files (this repository's own documents and sources by default, so no corpus download), encoded
with the byte-level tokenizer; each is answered greedily by the serving engine alone, then every
prompt is admitted at once (continuous batching, packed verify) and the token ids and decoded bytes
are compared per prompt.

    python -m qwen38_b200.serving.realtext --profile multi-stream-8x4k --max-tokens 256
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os

from .api import ByteTokenizer

DEFAULT_FILES = ("README.md", "qwen38_b200/spec/greedy.py", "qwen38_b200/serving/engine.py",
                 "qwen38_b200/csrc/attention.cu")


def text_prompts(paths=None, chars: int = 4000, root: str | None = None):
    """[(name, token ids)] from text files (UTF-8 bytes as ids)."""
    root = root or os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    tok = ByteTokenizer()
    out = []
    for p in paths or DEFAULT_FILES:
        full = p if os.path.isabs(p) else os.path.join(root, p)
        if not os.path.isfile(full):
            continue
        with open(full, encoding="utf-8", errors="replace") as f:
            text = f.read()[:chars]
        out.append((os.path.basename(p), tok.encode("Continue this text:\n\n" + text)))
    return out


def compare(engine, prompts, max_tokens: int) -> dict:
    tok = ByteTokenizer()
    alone = {}
    for name, ids in prompts:
        engine.add_request(ids, max_tokens, request_id=f"seq-{name}")
        done = engine.run()
        alone[name] = [r for r in done if r.request_id == f"seq-{name}"][0].output
    for name, ids in prompts:
        engine.add_request(ids, max_tokens, request_id=f"con-{name}")
    together = {r.request_id[4:]: r.output for r in engine.run()}
    rows = []
    for name, _ in prompts:
        a, b = alone[name], together.get(name)
        ba, bb = tok.decode(a).encode(), tok.decode(b or []).encode()
        rows.append(dict(name=name, tokens=len(a), equal_ids=a == b, equal_bytes=ba == bb,
                         sha256=hashlib.sha256(ba).hexdigest(),
                         first_difference=None if a == b else next(
                             (i for i, (x, y) in enumerate(zip(a, b or [])) if x != y), min(len(a), len(b or [])))))
    return dict(passed=all(r["equal_ids"] and r["equal_bytes"] for r in rows), prompts=rows,
                concurrent=len(prompts), max_tokens=max_tokens)


def main(argv=None):
    from ..runconfig import load_run_config
    from .factory import build_engine
    ap = argparse.ArgumentParser(description="concurrent vs sequential serving output on real text")
    ap.add_argument("--profile", default=None)
    ap.add_argument("--config", default=None)
    ap.add_argument("--set", action="append", default=[])
    ap.add_argument("--files", nargs="*", default=None)
    ap.add_argument("--chars", type=int, default=4000)
    ap.add_argument("--max-tokens", type=int, default=128)
    a = ap.parse_args(argv)
    eng = build_engine(load_run_config(a.config, profile=a.profile, overrides=a.set))
    prompts = text_prompts(a.files, a.chars)
    if len(prompts) > eng.max_running:
        prompts = prompts[:eng.max_running]
    rep = compare(eng, prompts, a.max_tokens)
    print(json.dumps(rep, indent=1))
    return 0 if rep["passed"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
