"""Typed configuration for the hybrid target, the block drafter and the runtime.

The target follows the HF ``text_config`` layout of the Qwen3.5/3.6/3.8 hybrid family
(``layer_types`` of ``linear_attention`` / ``full_attention``, ``linear_*`` GDN widths,
``rope_parameters`` with ``partial_rotary_factor``); the reference reads the same keys in
``docker/qwen-c2-graft/graft/model_config.py:85-116``.  Per-rank widths for tensor
parallelism mirror ``model_config.py:138-194`` (heads split evenly, KV heads replicated
when TP exceeds their count, ``model_config.py:159-163``).

One dataclass per concern, each validated on construction; no environment-flag sprawl.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any


LINEAR = "linear_attention"
FULL = "full_attention"


@dataclass
class ModelConfig:
    vocab_size: int = 151936
    hidden_size: int = 5120
    intermediate_size: int = 17408
    num_hidden_layers: int = 64
    num_attention_heads: int = 24
    num_key_value_heads: int = 4
    head_dim: int = 256
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1.0e7
    partial_rotary_factor: float = 0.25
    max_position_embeddings: int = 262144
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 48
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    layer_types: list = field(default_factory=list)
    tie_word_embeddings: bool = False
    eos_token_id: int | None = None

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = [FULL if (i + 1) % 4 == 0 else LINEAR for i in range(self.num_hidden_layers)]
        if len(self.layer_types) != self.num_hidden_layers:
            raise ValueError("layer_types must name every decoder layer")
        if any(t not in (LINEAR, FULL) for t in self.layer_types):
            raise ValueError("layer_types entries must be linear_attention or full_attention")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("query heads must be a multiple of KV heads")
        if self.linear_num_value_heads % self.linear_num_key_heads:
            raise ValueError("GDN value heads must be a multiple of key heads")
        if self.rope_dim % 2 or self.rope_dim > self.head_dim:
            raise ValueError("rotary width must be even and at most head_dim")

    # ---- derived widths -------------------------------------------------------------
    @property
    def rope_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def gdn_key_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def gdn_value_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def gdn_conv_dim(self) -> int:
        return 2 * self.gdn_key_dim + self.gdn_value_dim

    @property
    def linear_layers(self) -> list:
        return [i for i, t in enumerate(self.layer_types) if t == LINEAR]

    @property
    def full_layers(self) -> list:
        return [i for i, t in enumerate(self.layer_types) if t == FULL]

    def num_params(self) -> int:
        h, i, v = self.hidden_size, self.intermediate_size, self.vocab_size
        n = v * h * (1 if self.tie_word_embeddings else 2) + h
        for t in self.layer_types:
            n += 2 * h + 3 * h * i
            if t == LINEAR:
                n += h * (self.gdn_conv_dim + self.gdn_value_dim + 2 * self.linear_num_value_heads)
                n += self.gdn_conv_dim * self.linear_conv_kernel_dim + 2 * self.linear_num_value_heads
                n += self.linear_value_head_dim + self.gdn_value_dim * h
            else:
                qd = self.num_attention_heads * self.head_dim
                kd = self.num_key_value_heads * self.head_dim
                n += h * (2 * qd + 2 * kd) + qd * h + 2 * self.head_dim
        return n

    # ---- HF interop -----------------------------------------------------------------
    def to_hf_text_config(self) -> dict:
        return {
            "model_type": "qwen3_5_text",
            "architectures": ["Qwen3_5ForCausalLM"],
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads,
            "head_dim": self.head_dim,
            "hidden_act": "silu",
            "rms_norm_eps": self.rms_norm_eps,
            "max_position_embeddings": self.max_position_embeddings,
            "rope_parameters": {
                "rope_type": "default",
                "rope_theta": self.rope_theta,
                "partial_rotary_factor": self.partial_rotary_factor,
            },
            "linear_num_key_heads": self.linear_num_key_heads,
            "linear_num_value_heads": self.linear_num_value_heads,
            "linear_key_head_dim": self.linear_key_head_dim,
            "linear_value_head_dim": self.linear_value_head_dim,
            "linear_conv_kernel_dim": self.linear_conv_kernel_dim,
            "layer_types": list(self.layer_types),
            "tie_word_embeddings": self.tie_word_embeddings,
            "eos_token_id": self.eos_token_id,
            "attention_bias": False,
        }

    @classmethod
    def from_hf_dict(cls, cfg: dict) -> "ModelConfig":
        """Accepts a composite (``text_config`` nested) or a text-only HF config dict."""
        if "text_config" in cfg and isinstance(cfg["text_config"], dict):
            cfg = cfg["text_config"]
        rope = cfg.get("rope_parameters") or {}
        kw = {}
        for f in dataclasses.fields(cls):
            if f.name in cfg:
                kw[f.name] = cfg[f.name]
        kw["rope_theta"] = float(rope.get("rope_theta", cfg.get("rope_theta", 1.0e7)))
        kw["partial_rotary_factor"] = float(
            rope.get("partial_rotary_factor", cfg.get("partial_rotary_factor", 1.0)))
        eos = cfg.get("eos_token_id")
        if isinstance(eos, list):
            eos = eos[0] if eos else None
        kw["eos_token_id"] = eos
        return cls(**kw)

    @classmethod
    def from_pretrained(cls, path: str) -> "ModelConfig":
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_hf_dict(json.load(f))


@dataclass
class DrafterConfig:
    """Block drafter conditioned on target hidden states (DSpark family).

    Shape pinned by the reference's intake contract ``scripts/ci/dspark_intake.py:27-86``:
    ``fc`` projects the concatenated tap features (``len(taps) * hidden``) to ``hidden``;
    ``num_hidden_layers`` full-attention layers attend over the projected context rows plus the
    block rows; the target LM head is shared; a rank-``markov_rank`` Markov bias selects tokens
    sequentially (``scripts/ci/dspark_markov.py:4-29``).  RoPE is YaRN
    (``scripts/ci/dspark_rope_tables.py:8-32``).
    """
    hidden_size: int = 5120
    intermediate_size: int = 17408
    num_hidden_layers: int = 5
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    taps: list = field(default_factory=lambda: [5, 19, 33, 47, 61])
    block_rows: int = 16          # verify rows per block: anchor + (block_rows - 1) proposals
    markov_rank: int = 256
    mask_token_id: int = -1       # -1: last vocabulary id
    rope_theta: float = 1.0e7
    rope_type: str = "yarn"
    yarn_factor: float = 32.0
    yarn_beta_fast: float = 32.0
    yarn_beta_slow: float = 1.0
    yarn_original_max_position: int = 8192
    max_position_embeddings: int = 262144

    def __post_init__(self):
        if self.block_rows not in (2, 4, 8, 16, 32):
            raise ValueError("block_rows must be a verifier bucket (2, 4, 8, 16 or 32)")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("drafter query heads must be a multiple of KV heads")
        if not self.taps:
            raise ValueError("at least one target tap is required")

    @property
    def proposals(self) -> int:
        return self.block_rows - 1

    def mask_id(self, vocab_size: int) -> int:
        return vocab_size - 1 if self.mask_token_id < 0 else self.mask_token_id


@dataclass
class WindowDrafterConfig(DrafterConfig):
    """Windowed block drafter (DFlash2 family), the DSpark drafter's predecessor in the reference.

    Shape and geometry pinned by ``scripts/ci/dflash_device.py:515-560`` (five layers, 8/16/32-row
    blocks, a 2,048-row sliding history window), ``scripts/ci/draft_attention.py:4-18`` (the window
    mask), ``scripts/ci/draft_convolution.py:6-37`` (group-16 dynamic causal convolutions, two
    taps), ``scripts/ci/draft_shared_head.py`` (top-16 candidates per row) and
    ``scripts/ci/draft_selector.py`` (rank-256 predecessor / successor codebooks).  RoPE is the plain
    rotary table over the whole head (``scripts/ci/draft_head_preparation.py:4-12``, theta 1e7).
    """
    block_rows: int = 8
    window: int = 2048            # block row at position p sees history keys k with p - k < window
    conv_group: int = 16          # channels sharing one dynamic convolution weight
    selector_rank: int = 256
    candidates: int = 16          # top candidates per row handed to the selector
    rope_type: str = "default"

    def __post_init__(self):
        super().__post_init__()
        if self.hidden_size % self.conv_group:
            raise ValueError("hidden size must be a multiple of the convolution group")
        if self.window < self.block_rows:
            raise ValueError("the history window must cover a whole block")
        if not 1 <= self.candidates <= 32:
            raise ValueError("1..32 selector candidates per row")

    @property
    def proposals(self) -> int:
        return self.block_rows - 1

    @property
    def conv_groups(self) -> int:
        return self.hidden_size // self.conv_group


@dataclass
class RuntimeConfig:
    """Serving/runtime knobs (paged KV, prefill chunking, verifier buckets, graphs)."""
    max_context: int = 8192
    kv_block_size: int = 16
    prefill_chunk: int = 2048
    gdn_chunk: int = 64
    verify_buckets: tuple = (1, 2, 4, 8, 16, 32)
    use_cuda_graphs: bool = True
    weight_format: str = "bf16"     # "bf16" or "mxfp8"
    state_dtype: str = "fp32"       # GDN recurrent state

    def __post_init__(self):
        if self.kv_block_size not in (16, 32, 64):
            raise ValueError("kv_block_size must be 16, 32 or 64")
        if self.prefill_chunk % self.gdn_chunk:
            raise ValueError("prefill_chunk must be a multiple of gdn_chunk")
        if self.weight_format not in ("bf16", "mxfp8"):
            raise ValueError("weight_format must be bf16 or mxfp8")


def tiny_model_config() -> ModelConfig:
    """CPU plumbing shape: vocab 4096, hidden 256, 4 layers [GDN, GDN, GDN, attention]."""
    return ModelConfig(
        vocab_size=4096, hidden_size=256, intermediate_size=768, num_hidden_layers=4,
        num_attention_heads=4, num_key_value_heads=2, head_dim=64, rms_norm_eps=1e-6,
        rope_theta=1.0e7, partial_rotary_factor=0.5, max_position_embeddings=4096,
        linear_num_key_heads=4, linear_num_value_heads=8, linear_key_head_dim=32,
        linear_value_head_dim=32, linear_conv_kernel_dim=4,
        layer_types=[LINEAR, LINEAR, LINEAR, FULL])


def tiny_drafter_config() -> DrafterConfig:
    """One-layer drafter of the tiny target's width that reads the last layer's output and
    proposes 4-row blocks."""
    return DrafterConfig(hidden_size=256, intermediate_size=768, num_hidden_layers=1,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=64, taps=[3],
                         block_rows=4, markov_rank=16, yarn_original_max_position=512,
                         max_position_embeddings=4096)


def tiny_window_drafter_config() -> WindowDrafterConfig:
    """Windowed drafter of the tiny target's width: one layer, 4-row blocks, a 24-row window (so
    CPU tests reach the sliding part), 8 candidates."""
    return WindowDrafterConfig(hidden_size=256, intermediate_size=768, num_hidden_layers=1,
                               num_attention_heads=4, num_key_value_heads=2, head_dim=64, taps=[3],
                               block_rows=4, window=24, selector_rank=16, candidates=8,
                               max_position_embeddings=4096)


def full_model_config() -> ModelConfig:
    """Full-size 27B-class hybrid: vocab 151,936, hidden 5,120, 64 layers (3 GDN : 1 attention),
    SwiGLU 17,408, GDN 16 QK / 48 V heads of 128, attention 24 Q / 4 KV heads of 256."""
    return ModelConfig()


def full_drafter_config() -> DrafterConfig:
    return DrafterConfig()


def tp_widths(cfg: ModelConfig, tp: int) -> dict:
    """Per-rank widths for tensor parallelism ``tp``.

    Attention heads, GDN key/value heads and the MLP intermediate split evenly.  KV heads are
    replicated when ``tp`` exceeds their count: rank r serves KV head ``r * n_kv // tp`` (as in
    the reference's ``replicate_kv_weight`` path).
    """
    if cfg.num_attention_heads % tp or cfg.linear_num_key_heads % tp or cfg.linear_num_value_heads % tp:
        raise ValueError(f"head counts do not divide by TP={tp}")
    if cfg.intermediate_size % tp or cfg.vocab_size % tp:
        raise ValueError(f"intermediate/vocab do not divide by TP={tp}")
    if tp > cfg.num_key_value_heads and tp % cfg.num_key_value_heads:
        raise ValueError("TP above the KV head count must be a multiple of it")
    if tp <= cfg.num_key_value_heads and cfg.num_key_value_heads % tp:
        raise ValueError("KV heads must divide by TP")
    nkv = max(1, cfg.num_key_value_heads // tp)
    return dict(
        n_heads=cfg.num_attention_heads // tp,
        n_kv=nkv,
        kv_replication=tp > cfg.num_key_value_heads,
        gdn_nk=cfg.linear_num_key_heads // tp,
        gdn_nv=cfg.linear_num_value_heads // tp,
        inter=cfg.intermediate_size // tp,
        vocab=cfg.vocab_size // tp,
    )


def to_json(obj: Any) -> str:
    return json.dumps(dataclasses.asdict(obj), indent=1, sort_keys=True)
