"""Provenance of a run: what code, build and environment produced a number.

``manifest()`` returns the sha256 of the loaded CUDA extension, one combined digest of every
source file (per-file digests with ``full=True``), the nvcc flags, and torch / CUDA / driver
versions.  ``bench.py`` prints the short form in its JSON line; the serving image pins the same
fields (the reference's overlay provenance, ``scripts/ci/c2_image_provenance.py``).

    python -m qwen38_b200.utils.provenance            # full manifest as JSON
"""
from __future__ import annotations

import hashlib
import json
import platform

import torch

from ..ops import build
from .trace import source_digests


def _sha(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def manifest(full: bool = False) -> dict:
    src = source_digests()
    combined = hashlib.sha256("".join(f"{k}:{v}\n" for k, v in src.items()).encode()).hexdigest()
    so = build.so_path()
    out = {
        "sources_sha256": combined,
        "extension_sha256": _sha(so) if so else None,
        "extension_matches_sources": None if build.stale() is None else not build.stale(),
        "nvcc_flags": " ".join(build.CUDA_FLAGS),
        "torch": torch.__version__,
        "cuda_runtime": torch.version.cuda,
        "python": platform.python_version(),
    }
    if torch.cuda.is_available():
        out["device"] = torch.cuda.get_device_name(0)
        out["capability"] = ".".join(map(str, torch.cuda.get_device_capability(0)))
        try:
            import pynvml
            pynvml.nvmlInit()
            out["driver"] = pynvml.nvmlSystemGetDriverVersion()
        except Exception:
            pass
    if full:
        out["source_files"] = src
    return out


if __name__ == "__main__":
    print(json.dumps(manifest(full=True), indent=1))
