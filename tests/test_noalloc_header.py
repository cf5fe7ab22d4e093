"""The allocation-free GEMM's C header (csrc/q38_noalloc.h) against its definitions, its ctypes
binding and the built extension's exported symbols (CPU only: nothing is launched)."""
import os
import re
import shutil
import subprocess

import pytest

from qwen38_b200.ops import noalloc
from qwen38_b200.ops.build import CSRC, so_path

HEADER = os.path.join(CSRC, "q38_noalloc.h")


def _prototypes(text):
    """{name: (return type, [parameter types])} of the function declarations in C source text."""
    out = {}
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    for m in re.finditer(r"\b(int)\s+(q38_\w+)\s*\(([^)]*)\)\s*[;{]", text):
        params = [p.strip() for p in m.group(3).split(",")]
        types = []
        for p in params:
            if p in ("", "void"):
                continue
            p = re.sub(r"\s+", " ", p)
            name = re.match(r"(.*?)(\w+)$", p)
            t = name.group(1).strip().replace(" *", "*")
            types.append(t)
        out[m.group(2)] = (m.group(1), types)
    return out


def test_header_declares_the_binding_prototypes():
    with open(HEADER) as f:
        decl = _prototypes(f.read())
    assert decl == noalloc.PROTOTYPES


def test_definitions_match_the_header():
    with open(os.path.join(CSRC, "gemm_noalloc.cu")) as f:
        src = f.read()
    assert '#include "q38_noalloc.h"' in src
    defs = _prototypes(src.replace('extern "C" __attribute__((visibility("default")))', ""))
    with open(HEADER) as f:
        decl = _prototypes(f.read())
    assert defs == decl


def test_header_compiles_as_c():
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    if not os.path.exists(os.path.join(inc, "cuda_runtime_api.h")):
        pytest.skip("CUDA headers not found")
    src = '#include "q38_noalloc.h"\nint f(void) { return Q38_NOALLOC_ESIZE + Q38_NOALLOC_EPI_ADD_F32; }\n'
    r = subprocess.run([cc, "-x", "c", "-std=c99", "-fsyntax-only", "-Wall", "-Werror", "-I", CSRC, "-I", inc, "-"],
                       input=src, text=True, capture_output=True)
    assert r.returncode == 0, r.stderr


def test_extension_exports_the_symbols():
    so = so_path()
    nm = shutil.which("nm")
    if so is None or nm is None:
        pytest.skip("extension not built or nm missing")
    r = subprocess.run([nm, "-D", "--defined-only", so], text=True, capture_output=True, check=True)
    exported = {ln.split()[-1] for ln in r.stdout.splitlines() if ln.strip()}
    for name in noalloc.PROTOTYPES:
        assert name in exported, name
