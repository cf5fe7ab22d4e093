"""Per-rank shape plan for tensor parallelism and the kernels' shape constraints.

Every constraint the sm_100a kernels put on a shape (TMA row strides a multiple of 16 bytes, the
SwiGLU prefill tile of 256 output columns, 64-row gate/up blocks, GQA groups of at most 8 heads,
head dims the attention and GDN kernels are built for, the fused all-reduce's tile count, the
chunked GDN prefill's 16-byte row loads) is checked here for a model / drafter / TP degree before
any weight is loaded, so a TP degree that cannot run fails on the host with the reason instead of
inside a kernel.
"""
from __future__ import annotations

from ..config import DrafterConfig, ModelConfig, tp_widths

GU_BLOCK = 64
PREFILL_BN = 256
FUSED_AR_TILES_MAX = 64


def gdn_in_width(cfg: ModelConfig, tp: int) -> int:
    """Per-rank GDN in-projection rows (q|k|v|z|b|a), padded to a multiple of 8."""
    nkl, nvl = cfg.linear_num_key_heads // tp, cfg.linear_num_value_heads // tp
    w = 2 * nkl * cfg.linear_key_head_dim + 2 * nvl * cfg.linear_value_head_dim + 2 * nvl
    return -(-w // 8) * 8


def tp_plan(cfg: ModelConfig, dcfg: DrafterConfig | None, tp: int) -> dict:
    w = tp_widths(cfg, tp)
    plan = dict(tp=tp, **w)
    plan["gdn_in"] = gdn_in_width(cfg, tp)
    plan["attn_in"] = 2 * w["n_heads"] * cfg.head_dim + 2 * w["n_kv"] * cfg.head_dim
    plan["gemm_k"] = {"hidden": cfg.hidden_size, "attn_out": w["n_heads"] * cfg.head_dim,
                      "gdn_out": w["gdn_nv"] * cfg.linear_value_head_dim, "mlp_down": w["inter"]}
    plan["swiglu_n"] = {"target": 2 * w["inter"]}
    if dcfg is not None:
        if dcfg.num_attention_heads % tp or dcfg.intermediate_size % tp:
            raise ValueError(f"drafter heads / intermediate do not divide by TP={tp}")
        dkv = max(1, dcfg.num_key_value_heads // tp)
        plan["drafter"] = dict(n_heads=dcfg.num_attention_heads // tp, n_kv=dkv, inter=dcfg.intermediate_size // tp)
        plan["gemm_k"].update(drafter_fc=len(dcfg.taps) * dcfg.hidden_size // tp,
                              drafter_attn_out=dcfg.num_attention_heads // tp * dcfg.head_dim,
                              drafter_down=dcfg.intermediate_size // tp)
        plan["swiglu_n"]["drafter"] = 2 * dcfg.intermediate_size // tp
    return plan


def check_tp_plan(cfg: ModelConfig, dcfg: DrafterConfig | None, tp: int) -> list:
    """Violations of the kernels' shape constraints (empty: this TP degree can run)."""
    try:
        p = tp_plan(cfg, dcfg, tp)
    except ValueError as e:
        return [str(e)]
    bad = []
    for name, k in p["gemm_k"].items():
        if k % 8:
            bad.append(f"GEMM K={k} ({name}) is not a multiple of 8 (TMA rows must be 16-byte multiples)")
    for name, n in p["swiglu_n"].items():
        if n % PREFILL_BN:
            bad.append(f"SwiGLU width {n} ({name}) is not a multiple of the 256-column prefill tile")
        if (n // 2) % GU_BLOCK:
            bad.append(f"MLP width {n // 2} ({name}) is not a multiple of the 64-row gate/up block")
    rep = p["n_heads"] // p["n_kv"]
    if p["n_heads"] % p["n_kv"] or not 1 <= rep <= 8:
        bad.append(f"GQA group of {rep} heads: the attention kernels serve 1..8")
    if cfg.head_dim not in (64, 128, 256):
        bad.append(f"attention head dim {cfg.head_dim} not built (64/128/256)")
    if "drafter" in p:
        d = p["drafter"]
        drep = d["n_heads"] // d["n_kv"]
        if d["n_heads"] % d["n_kv"] or not 1 <= drep <= 8:
            bad.append(f"drafter GQA group of {drep} heads: the attention kernels serve 1..8")
    if cfg.linear_key_head_dim != cfg.linear_value_head_dim or cfg.linear_key_head_dim not in (32, 128):
        bad.append("GDN head dims must be equal and 32 or 128")
    if p["gdn_nv"] % p["gdn_nk"]:
        bad.append("GDN value heads must be a multiple of key heads per rank")
    if -(-cfg.hidden_size // 128) > FUSED_AR_TILES_MAX:
        bad.append(f"hidden {cfg.hidden_size} exceeds the fused all-reduce's {FUSED_AR_TILES_MAX} tiles")
    if p["gdn_in"] % 8:
        bad.append("GDN in-projection rows must be 16-byte aligned")
    return bad
