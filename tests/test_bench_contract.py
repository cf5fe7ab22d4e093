"""The bench's command-line contract on a machine without a GPU: defaults (one GPU, at least three
warm-up steps), the options the driver passes, and the reference arm's one-line answer."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          timeout=300, cwd=ROOT)


def test_help_lists_the_contract_options():
    r = _run("--help")
    assert r.returncode == 0
    for opt in ("--gpus", "--steps", "--warmup", "--impl", "--drafter", "--weights"):
        assert opt in r.stdout


def test_defaults():
    src = open(os.path.join(ROOT, "bench.py")).read()
    assert 'add_argument("--gpus", type=int, default=1)' in src
    warm = [l for l in src.splitlines() if 'add_argument("--warmup"' in l][0]
    assert int(warm.split("default=")[1].split(")")[0]) >= 3


def test_reference_arm_prints_one_json_line():
    for extra in ((), ("--gpus", "1", "--steps", "2", "--warmup", "3")):
        r = _run("--impl", "reference", *extra)
        assert r.returncode == 0, r.stderr
        lines = [l for l in r.stdout.splitlines() if l.strip()]
        assert len(lines) == 1
        d = json.loads(lines[0])
        assert d["impl"] == "reference" and d["unavailable"]
