"""Builds and loads the in-tree CUDA extension (sm_100a only).

``build()`` compiles ``qwen38_b200/csrc/*`` with ``-gencode arch=compute_100a,code=sm_100a`` into
``qwen38_b200/_build/qwen38_b200_C*.so`` (nvcc cross-compiles without a GPU).  ``load()`` imports
that file directly; on a CUDA machine without it, ops fail loudly rather than falling back.
"""
from __future__ import annotations

import glob
import hashlib
import importlib.machinery
import importlib.util
import os
import sys

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
NAME = "qwen38_b200_C"

CUDA_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "--use_fast_math",
    "--expt-relaxed-constexpr", "-Xptxas=-warn-spills",
]

_mod = None


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


STAMP = os.path.join(BUILD, "sources.sha256")


def sources_digest() -> str:
    """One sha256 over every compiled source and header (name and content) plus the nvcc flags."""
    h = hashlib.sha256(" ".join(CUDA_FLAGS).encode())
    for path in sorted(sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))):
        h.update(os.path.basename(path).encode())
        with open(path, "rb") as f:
            h.update(hashlib.sha256(f.read()).digest())
    return h.hexdigest()


def stale() -> bool | None:
    """True when the built extension was compiled from other sources than the tree now holds (its
    stamp differs), None when there is no build or no stamp."""
    if so_path() is None or not os.path.exists(STAMP):
        return None
    with open(STAMP) as f:
        return f.read().strip() != sources_digest()


def build(verbose: bool = False):
    from torch.utils.cpp_extension import load
    os.makedirs(BUILD, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(min(8, os.cpu_count() or 4)))
    digest = sources_digest()
    mod = load(name=NAME, sources=sources(), extra_cuda_cflags=CUDA_FLAGS, extra_cflags=["-O3", "-std=c++17"],
               build_directory=BUILD, verbose=verbose, with_cuda=True)
    with open(STAMP, "w") as f:
        f.write(digest + "\n")
    global _mod
    _mod = mod
    return mod


def so_path():
    cands = sorted(glob.glob(os.path.join(BUILD, NAME + "*.so")))
    return cands[0] if cands else None


def load():
    """Import the built extension (no compilation)."""
    global _mod
    if _mod is not None:
        return _mod
    path = so_path()
    if path is None:
        raise RuntimeError(f"qwen38_b200 CUDA extension not built ({BUILD}); run __graft_entry__.build() "
                           "or python -m qwen38_b200.ops.build")
    if stale():
        import warnings
        warnings.warn(f"{path} was built from other sources than {CSRC} now holds; rebuild it")
    import torch  # noqa: F401  (loads libtorch symbols first)
    loader = importlib.machinery.ExtensionFileLoader(NAME, path)
    spec = importlib.util.spec_from_file_location(NAME, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[NAME] = mod
    _mod = mod
    return mod


if __name__ == "__main__":
    build(verbose=True)
    print(so_path())
