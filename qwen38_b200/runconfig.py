"""One typed run configuration: model, runtime, parallelism, speculation, kernels, serving.

Loaded from defaults, then a named profile (``serving/profiles.yaml``), then a YAML file, then
``section.field=value`` overrides (CLI ``--set``), and validated once: incompatible combinations
raise instead of being silently adjusted.  This replaces the reference's hundreds of environment
flags and per-profile argv/env pins (``scripts/ci/serving_c2_contract.py``,
``scripts/ci/serving_fast_policy.py:1-60``, ``scripts/ci/qwen_c2_profiles.json``) with a small,
checked set of fields.
"""
from __future__ import annotations

import dataclasses
import os
from dataclasses import dataclass, field

from .config import RuntimeConfig

PROFILES = os.path.join(os.path.dirname(os.path.abspath(__file__)), "serving", "profiles.yaml")


@dataclass
class ParallelConfig:
    tp: int = 1
    comm: str = "fused"          # fused | peer | nccl


@dataclass
class SpecConfig:
    drafter: str = "dspark"      # dspark | dflash2 | mtp | lookup | none
    block_rows: int = 16
    lookup: bool = False         # lookup drafter first, neural drafter second
    mtp_steps: int = 3


@dataclass
class KernelConfig:
    ops: str = "native"          # native | torch
    cuda_graphs: bool = True
    pdl: bool = True             # programmatic dependent launch (native kernels)


@dataclass
class ServingConfig:
    slots: int = 4
    host: str = "127.0.0.1"
    port: int = 8000
    output_budget_multiple: int = 0      # > 0: max_tokens must be a multiple of it
    prefix_budget_gb: float = 0.0        # 0: prefix reuse off
    request_timeout_s: float = 600.0
    phase_log: str = ""                  # file for one JSON line per finished request ("": off)


@dataclass
class RunConfig:
    model: str = "full"                  # "full", "tiny" or an HF checkpoint directory
    weight_cache: str = ""               # directory of converted target weights ("" : off)
    runtime: RuntimeConfig = field(default_factory=RuntimeConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    spec: SpecConfig = field(default_factory=SpecConfig)
    kernels: KernelConfig = field(default_factory=KernelConfig)
    serving: ServingConfig = field(default_factory=ServingConfig)

    def validate(self) -> "RunConfig":
        p, s, k, v = self.parallel, self.spec, self.kernels, self.serving
        if p.tp not in (1, 2, 4, 8):
            raise ValueError("parallel.tp must be 1, 2, 4 or 8")
        if p.comm not in ("fused", "peer", "nccl"):
            raise ValueError("parallel.comm must be fused, peer or nccl")
        if k.ops not in ("native", "torch"):
            raise ValueError("kernels.ops must be native or torch")
        if p.tp > 1 and k.ops == "torch" and p.comm != "nccl":
            raise ValueError("peer-memory collectives run inside the native kernels: use parallel.comm=nccl "
                             "with kernels.ops=torch")
        if s.drafter not in ("dspark", "dflash2", "mtp", "lookup", "none"):
            raise ValueError("spec.drafter must be dspark, dflash2, mtp, lookup or none")
        if s.block_rows not in (2, 4, 8, 16, 32):
            raise ValueError("spec.block_rows must be a verifier bucket of at least 2")
        if s.drafter == "mtp" and s.block_rows != s.mtp_steps + 1:
            raise ValueError("an MTP drafter proposes mtp_steps tokens: spec.block_rows must be mtp_steps + 1")
        if s.drafter == "lookup" and not s.lookup:
            raise ValueError("spec.drafter=lookup needs spec.lookup=true")
        if v.slots < 1 or v.output_budget_multiple < 0 or v.prefix_budget_gb < 0:
            raise ValueError("serving.slots >= 1, non-negative budgets required")
        return self


def _coerce(value, like):
    if isinstance(like, bool):
        if isinstance(value, str):
            if value.lower() in ("1", "true", "yes", "on"):
                return True
            if value.lower() in ("0", "false", "no", "off"):
                return False
            raise ValueError(f"not a boolean: {value}")
        return bool(value)
    if isinstance(like, int):
        return int(value)
    if isinstance(like, float):
        return float(value)
    if isinstance(like, tuple):
        return tuple(int(x) for x in (value.split(",") if isinstance(value, str) else value))
    return value if not isinstance(like, str) else str(value)


def _apply(obj, tree: dict, where: str = ""):
    names = {f.name for f in dataclasses.fields(obj)}
    for key, val in tree.items():
        if key not in names:
            raise ValueError(f"unknown configuration field {where}{key}")
        cur = getattr(obj, key)
        if dataclasses.is_dataclass(cur):
            if not isinstance(val, dict):
                raise ValueError(f"{where}{key} is a section")
            sub = dataclasses.replace(cur)
            _apply(sub, val, f"{where}{key}.")
            if isinstance(sub, RuntimeConfig):
                sub.__post_init__()
            setattr(obj, key, sub)
        else:
            setattr(obj, key, _coerce(val, cur))


def parse_override(text: str) -> dict:
    """``"spec.block_rows=8"`` -> ``{"spec": {"block_rows": "8"}}``."""
    if "=" not in text:
        raise ValueError(f"override must look like section.field=value: {text}")
    path, value = text.split("=", 1)
    tree: dict = {}
    node = tree
    parts = path.strip().split(".")
    for p in parts[:-1]:
        node = node.setdefault(p, {})
    node[parts[-1]] = value
    return tree


def load_profiles(path: str = PROFILES) -> dict:
    import yaml
    with open(path) as f:
        return yaml.safe_load(f) or {}


def load_run_config(path: str | None = None, *, profile: str | None = None, overrides=()) -> RunConfig:
    cfg = RunConfig()
    if profile is not None:
        profiles = load_profiles()
        if profile not in profiles:
            raise ValueError(f"unknown profile {profile}; known: {sorted(profiles)}")
        _apply(cfg, profiles[profile])
    if path is not None:
        import yaml
        with open(path) as f:
            _apply(cfg, yaml.safe_load(f) or {})
    for o in overrides:
        _apply(cfg, parse_override(o))
    return cfg.validate()
