"""Builds a serving engine (target, drafter, prefix registry, communicator) from a ``RunConfig``.

Weights come from an HF-layout checkpoint directory (``RunConfig.model``; a ``drafter/``
subdirectory holds the DSpark drafter, ``mtp.*`` tensors the MTP head) or, for the ``full`` /
``tiny`` presets, from seeded random initialisation of that architecture.
"""
from __future__ import annotations

import os

import torch

from ..checkpoint import (SafetensorsSource, load_drafter_config, random_drafter_source,
                          random_target_source)
from ..config import ModelConfig, full_drafter_config, full_model_config, tiny_drafter_config, tiny_model_config
from ..runconfig import RunConfig


def _model(rc: RunConfig):
    if rc.model == "full":
        return full_model_config(), full_drafter_config(), None
    if rc.model == "tiny":
        return tiny_model_config(), tiny_drafter_config(), None
    if not os.path.isdir(rc.model):
        raise ValueError(f"model must be 'full', 'tiny' or a checkpoint directory: {rc.model}")
    cfg = ModelConfig.from_pretrained(rc.model)
    dpath = os.path.join(rc.model, "drafter")
    dcfg = load_drafter_config(dpath) if os.path.isdir(dpath) else None
    return cfg, dcfg, rc.model


def _is_mxfp8_checkpoint(path) -> bool:
    if not path:
        return False
    import json
    cfg = os.path.join(path, "config.json")
    if not os.path.exists(cfg):
        return False
    with open(cfg) as f:
        return (json.load(f).get("quantization_config") or {}).get("quant_method") == "mxfp8"


def _checkpoint_id(path: str) -> str:
    """Identity of a checkpoint directory for the weight cache: its path, and the names, sizes and
    modification times of its files."""
    import hashlib
    h = hashlib.sha256(os.path.abspath(path).encode())
    for f in sorted(os.listdir(path)):
        st = os.stat(os.path.join(path, f))
        h.update(f"{f}:{st.st_size}:{int(st.st_mtime)}".encode())
    return h.hexdigest()


def build_engine(rc: RunConfig, *, device=None, seed: int = 0, comm=None):
    """Returns ``ServingEngine``.  ``comm``: an existing communicator (TP > 1), else one is made."""
    from ..models.drafter import BlockDrafter
    from ..models.target import HybridTarget
    from .engine import ServingEngine
    rc.validate()
    cfg, dcfg, ckpt = _model(rc)
    from ..parallel.plan import check_tp_plan
    bad = check_tp_plan(cfg, dcfg if rc.spec.drafter == "dspark" else None, rc.parallel.tp)
    if bad:
        raise ValueError(f"TP={rc.parallel.tp} cannot run this shape: " + "; ".join(bad))
    native = rc.kernels.ops == "native"
    if native and not torch.cuda.is_available():
        raise RuntimeError("kernels.ops=native needs a CUDA device")
    os.environ["Q38_PDL"] = "1" if rc.kernels.pdl else "0"
    device = device or ("cuda" if torch.cuda.is_available() and native else "cpu")
    dtype = torch.bfloat16 if torch.device(device).type == "cuda" else torch.float32
    ops = None
    if native:
        from ..ops.native import NativeOps
        ops = NativeOps(device=device, max_keys=rc.runtime.max_context + 64, weight_format=rc.runtime.weight_format)
    if comm is None and rc.parallel.tp > 1:
        from ..parallel.comm import make_comm
        from ..parallel.topology import check_topology
        if torch.cuda.is_available():          # GPU ranks: peer access / NVLink preflight
            check_topology(rc.parallel.tp, comm=rc.parallel.comm if native else "nccl")
        comm = make_comm(rc.parallel.tp, device=device, hidden=cfg.hidden_size,
                         peer=native and rc.parallel.comm != "nccl", fused=rc.parallel.comm == "fused",
                         prefill_rows=rc.runtime.prefill_chunk if rc.parallel.comm == "fused" else 0)
    slots = rc.serving.slots
    src = SafetensorsSource(ckpt) if ckpt else random_target_source(cfg, seed)
    if rc.runtime.weight_format == "mxfp8" and not _is_mxfp8_checkpoint(ckpt):
        from ..checkpoint import MXFP8Source
        src = MXFP8Source(src)              # compute with the MXFP8 round trip of the weights
    if ckpt and rc.weight_cache:
        from ..checkpoint import CachedSource
        src = CachedSource(src, rc.weight_cache, base_id=_checkpoint_id(ckpt) + ":" + rc.runtime.weight_format)
    rt = rc.runtime
    tgt = HybridTarget(cfg, src, rt, device=device, dtype=dtype, ops=ops, comm=comm, max_slots=slots + 1,
                       max_verify_rows=slots * rc.spec.block_rows)
    drafter = None
    if rc.spec.drafter == "dspark":
        if dcfg is None:
            raise ValueError("the checkpoint has no drafter/ directory for spec.drafter=dspark")
        import dataclasses
        dcfg = dataclasses.replace(dcfg, block_rows=rc.spec.block_rows)
        dsrc = SafetensorsSource(os.path.join(ckpt, "drafter")) if ckpt else \
            random_drafter_source(dcfg, cfg.vocab_size, seed + 1)
        drafter = BlockDrafter(dcfg, dsrc, tgt, slots=slots)
    elif rc.spec.drafter == "dflash2":
        import dataclasses
        from ..checkpoint import load_window_drafter_config, random_window_drafter_source
        from ..config import tiny_window_drafter_config, WindowDrafterConfig
        from ..models.window_drafter import WindowDrafter
        wpath = os.path.join(ckpt, "window_drafter") if ckpt else None
        if wpath is not None and not os.path.isdir(wpath):
            raise ValueError("the checkpoint has no window_drafter/ directory for spec.drafter=dflash2")
        wcfg = load_window_drafter_config(wpath) if wpath else \
            (tiny_window_drafter_config() if rc.model == "tiny" else WindowDrafterConfig())
        wcfg = dataclasses.replace(wcfg, block_rows=rc.spec.block_rows)
        wsrc = SafetensorsSource(wpath) if wpath else random_window_drafter_source(wcfg, cfg.vocab_size, seed + 3)
        drafter = WindowDrafter(wcfg, wsrc, tgt, slots=slots)
    elif rc.spec.drafter == "mtp":
        from ..models.mtp import MTPDrafter, random_mtp_source
        msrc = SafetensorsSource(ckpt) if ckpt else random_mtp_source(cfg, seed + 2)
        drafter = MTPDrafter(msrc, tgt, steps=rc.spec.mtp_steps, slots=slots)
    prefix = None
    if rc.serving.prefix_budget_gb > 0:
        from ..prefix.registry import PrefixRegistry
        prefix = PrefixRegistry(tgt, int(rc.serving.prefix_budget_gb * (1 << 30)), boundary=rt.prefill_chunk)
    return ServingEngine(tgt, drafter, verifier_rows=rc.spec.block_rows, lookup=rc.spec.lookup, prefix=prefix)
