"""HF-layout checkpoints: random-init generation, safetensors save/load, lazy tensor sources.

Target tensor names follow HF ``Qwen3_5ForCausalLM`` (``model.layers.N.linear_attn.in_proj_qkv``,
``...self_attn.q_proj`` with per-head ``[query | gate]`` rows, ``model.norm``, ``lm_head``), the
layout the reference loads in ``docker/qwen-c2-graft/graft/model_config.py:366-403``.  Drafter
names follow the DSpark inventory in ``scripts/ci/dspark_intake.py:27-57`` (``fc``,
``hidden_norm``, ``layers.N.*``, ``norm``, ``markov_head.markov_w{1,2}``).

Block-FP8 checkpoints (``quantization_config.quant_method == "fp8"``, the format the reference
dequantises in ``model_config.py:375-377``): a quantised weight is stored as ``float8_e4m3fn``
with a companion ``<name>_scale_inv`` of one fp32 scale per ``weight_block_size`` block (128 x 128
by default); ``SafetensorsSource`` dequantises on read (weight = fp8 value x block scale).
``save_pretrained(..., fp8_block=(128, 128))`` writes that format.

A ``TensorSource`` hands out one tensor at a time so the runtime can pack and shard layer by
layer without materialising a second full copy of a 27B model; ``RandomSource`` derives every
tensor from ``(seed, name)`` so all TP ranks see identical full tensors.
"""
from __future__ import annotations

import json
import math
import os
import zlib
from typing import Iterable

import torch

from .config import LINEAR, DrafterConfig, ModelConfig


def target_shapes(cfg: ModelConfig) -> dict:
    h, it = cfg.hidden_size, cfg.intermediate_size
    out = {"model.embed_tokens.weight": (cfg.vocab_size, h), "model.norm.weight": (h,)}
    if not cfg.tie_word_embeddings:
        out["lm_head.weight"] = (cfg.vocab_size, h)
    for i, t in enumerate(cfg.layer_types):
        p = f"model.layers.{i}."
        out[p + "input_layernorm.weight"] = (h,)
        out[p + "post_attention_layernorm.weight"] = (h,)
        out[p + "mlp.gate_proj.weight"] = (it, h)
        out[p + "mlp.up_proj.weight"] = (it, h)
        out[p + "mlp.down_proj.weight"] = (h, it)
        if t == LINEAR:
            q = p + "linear_attn."
            nv = cfg.linear_num_value_heads
            out[q + "in_proj_qkv.weight"] = (cfg.gdn_conv_dim, h)
            out[q + "in_proj_z.weight"] = (cfg.gdn_value_dim, h)
            out[q + "in_proj_b.weight"] = (nv, h)
            out[q + "in_proj_a.weight"] = (nv, h)
            out[q + "conv1d.weight"] = (cfg.gdn_conv_dim, 1, cfg.linear_conv_kernel_dim)
            out[q + "dt_bias"] = (nv,)
            out[q + "A_log"] = (nv,)
            out[q + "norm.weight"] = (cfg.linear_value_head_dim,)
            out[q + "out_proj.weight"] = (h, cfg.gdn_value_dim)
        else:
            q = p + "self_attn."
            d = cfg.head_dim
            out[q + "q_proj.weight"] = (2 * cfg.num_attention_heads * d, h)
            out[q + "k_proj.weight"] = (cfg.num_key_value_heads * d, h)
            out[q + "v_proj.weight"] = (cfg.num_key_value_heads * d, h)
            out[q + "o_proj.weight"] = (h, cfg.num_attention_heads * d)
            out[q + "q_norm.weight"] = (d,)
            out[q + "k_norm.weight"] = (d,)
    return out


def drafter_shapes(d: DrafterConfig, vocab: int) -> dict:
    h = d.hidden_size
    out = {
        "fc.weight": (h, len(d.taps) * h),
        "hidden_norm.weight": (h,),
        "norm.weight": (h,),
        "markov_head.markov_w1.weight": (vocab, d.markov_rank),
        "markov_head.markov_w2.weight": (vocab, d.markov_rank),
    }
    for l in range(d.num_hidden_layers):
        p = f"layers.{l}."
        out[p + "input_layernorm.weight"] = (h,)
        out[p + "post_attention_layernorm.weight"] = (h,)
        out[p + "mlp.gate_proj.weight"] = (d.intermediate_size, h)
        out[p + "mlp.up_proj.weight"] = (d.intermediate_size, h)
        out[p + "mlp.down_proj.weight"] = (h, d.intermediate_size)
        out[p + "self_attn.q_proj.weight"] = (d.num_attention_heads * d.head_dim, h)
        out[p + "self_attn.k_proj.weight"] = (d.num_key_value_heads * d.head_dim, h)
        out[p + "self_attn.v_proj.weight"] = (d.num_key_value_heads * d.head_dim, h)
        out[p + "self_attn.o_proj.weight"] = (h, d.num_attention_heads * d.head_dim)
        out[p + "self_attn.q_norm.weight"] = (d.head_dim,)
        out[p + "self_attn.k_norm.weight"] = (d.head_dim,)
    return out


def window_drafter_shapes(d, vocab: int) -> dict:
    """Tensor names and shapes of the windowed (DFlash2) drafter; per-layer names follow the
    reference's prepared layer dicts (``scripts/ci/draft_attention_branch.py:55-63``,
    ``scripts/ci/draft_mlp_branch.py:27-45``, ``scripts/ci/draft_selector_fixture.py:11-13``)."""
    h, g = d.hidden_size, d.conv_groups
    out = {
        "fc.weight": (h, len(d.taps) * h),
        "hidden_norm.weight": (h,),
        "norm.weight": (h,),
        "candidate_selector.hidden_projection.weight": (d.selector_rank, h),
        "candidate_selector.predecessor_codebook": (vocab, d.selector_rank),
        "candidate_selector.successor_codebook": (vocab, d.selector_rank),
    }
    for l in range(d.num_hidden_layers):
        p = f"layers.{l}."
        out[p + "input_layernorm.weight"] = (h,)
        out[p + "post_attention_layernorm.weight"] = (h,)
        for branch in ("attention_conv", "mlp_conv"):
            out[p + branch + ".kernel_projection.weight"] = (4 * g, h)
            out[p + branch + ".base_kernel"] = (2, 2, h)
        out[p + "mlp.gate_proj.weight"] = (d.intermediate_size, h)
        out[p + "mlp.up_proj.weight"] = (d.intermediate_size, h)
        out[p + "mlp.down_proj.weight"] = (h, d.intermediate_size)
        out[p + "self_attn.q_proj.weight"] = (d.num_attention_heads * d.head_dim, h)
        out[p + "self_attn.k_proj.weight"] = (d.num_key_value_heads * d.head_dim, h)
        out[p + "self_attn.v_proj.weight"] = (d.num_key_value_heads * d.head_dim, h)
        out[p + "self_attn.o_proj.weight"] = (h, d.num_attention_heads * d.head_dim)
        out[p + "self_attn.q_norm.weight"] = (d.head_dim,)
        out[p + "self_attn.k_norm.weight"] = (d.head_dim,)
    return out


def _init_kind(name: str) -> str:
    if name.endswith("base_kernel"):
        return "conv_base"
    if name.endswith("A_log"):
        return "alog"
    if name.endswith("dt_bias"):
        return "dt"
    if name.endswith("conv1d.weight"):
        return "conv"
    if name.endswith("linear_attn.norm.weight"):
        return "one"
    if name.endswith("norm.weight") or name.endswith("layernorm.weight"):
        return "zc"      # zero-centred (1+w) norm weight
    return "normal"


class TensorSource:
    """Hands out tensors by HF name."""

    def get(self, name: str, device=None, dtype=None) -> torch.Tensor:
        raise NotImplementedError

    def names(self) -> Iterable[str]:
        raise NotImplementedError


class RandomSource(TensorSource):
    """Seeded random init of the named shapes; a tensor depends only on (seed, name)."""

    def __init__(self, shapes: dict, seed: int = 0, std: float = 0.02, direct_norms: bool = False):
        self.shapes, self.seed, self.std = shapes, seed, std
        self.direct_norms = direct_norms     # drafter norms multiply by w directly (w near 1)

    def names(self):
        return list(self.shapes)

    def get(self, name, device=None, dtype=None):
        shape = self.shapes[name]
        device = torch.device(device or "cpu")
        gen = torch.Generator(device=device)
        gen.manual_seed((self.seed * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFF)
        kind = _init_kind(name)
        f32 = dict(device=device, dtype=torch.float32)
        if kind == "normal":
            t = torch.randn(shape, generator=gen, **f32) * self.std
        elif kind == "zc":
            t = (torch.rand(shape, generator=gen, **f32) - 0.5) * 0.2
            if self.direct_norms:
                t = t + 1.0
        elif kind == "one":
            t = 1.0 + (torch.rand(shape, generator=gen, **f32) - 0.5) * 0.2
        elif kind == "conv":
            k = shape[-1]
            t = (torch.rand(shape, generator=gen, **f32) * 2 - 1) / math.sqrt(k)
        elif kind == "conv_base":
            # [phase, tap, channel]: tap 0 near identity, tap 1 (the previous row) small
            t = torch.randn(shape, generator=gen, **f32) * self.std
            t[:, 0] += 1.0
        elif kind == "alog":
            t = torch.log(1 + 15 * torch.rand(shape, generator=gen, **f32))
        elif kind == "dt":
            t = 1.0 + 0.1 * torch.randn(shape, generator=gen, **f32)
        else:
            raise AssertionError(kind)
        if dtype is not None and kind in ("normal", "zc", "one", "conv", "conv_base"):
            t = t.to(dtype)
        return t


class DictSource(TensorSource):
    def __init__(self, sd: dict):
        self.sd = sd

    def names(self):
        return list(self.sd)

    def get(self, name, device=None, dtype=None):
        t = self.sd[name]
        if device is not None:
            t = t.to(device)
        if dtype is not None and t.is_floating_point() and not name.endswith(("A_log", "dt_bias")):
            t = t.to(dtype)
        return t


class SafetensorsSource(TensorSource):
    """Reads tensors lazily from a (possibly sharded) safetensors checkpoint directory."""

    def __init__(self, path: str, prefix: str = ""):
        from safetensors import safe_open
        self.path, self.prefix = path, prefix
        self.block = (128, 128)
        self.mx_block = MX_BLOCK
        cfg_path = os.path.join(path, "config.json")
        if os.path.exists(cfg_path):
            with open(cfg_path) as f:
                qc = json.load(f).get("quantization_config") or {}
            if qc.get("weight_block_size"):
                self.block = tuple(int(b) for b in qc["weight_block_size"])
            self.mx_block = int(qc.get("mx_block_size", MX_BLOCK))
        index = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(index):
            with open(index) as f:
                wm = json.load(f)["weight_map"]
            files = sorted(set(wm.values()))
        else:
            files = [f for f in sorted(os.listdir(path)) if f.endswith(".safetensors")]
            wm = None
        self._handles = {f: safe_open(os.path.join(path, f), framework="pt") for f in files}
        self._where = {}
        for f, h in self._handles.items():
            for k in h.keys():
                self._where[k] = f
        if wm is not None:
            self._where.update(wm)

    def names(self):
        return [k[len(self.prefix):] for k in self._where
                if k.startswith(self.prefix) and not k.endswith(("_scale_inv", "_scale_e8m0"))]

    def get(self, name, device=None, dtype=None):
        key = self.prefix + name
        t = self._handles[self._where[key]].get_tensor(key)
        if t.dtype == torch.float8_e4m3fn and key + "_scale_inv" in self._where:
            sk = key + "_scale_inv"
            t = dequant_fp8_block(t, self._handles[self._where[sk]].get_tensor(sk), self.block)
        elif t.dtype == torch.float8_e4m3fn and key + "_scale_e8m0" in self._where:
            sk = key + "_scale_e8m0"
            t = dequant_mxfp8(t, self._handles[self._where[sk]].get_tensor(sk), self.mx_block)
        if device is not None:
            t = t.to(device)
        if dtype is not None and t.is_floating_point() and not name.endswith(("A_log", "dt_bias")):
            t = t.to(dtype)
        return t


class CachedSource(TensorSource):
    """A converted-tensor cache in front of another source (the reference keeps per-mesh converted
    tensor caches, ``graft/model_config.py:347-364``).  The first ``get`` of a (name, dtype) pair
    reads the base source (dequantising block-FP8 weights, converting dtype) and writes the result
    to ``cache_dir`` as one safetensors file; later loads, in this process or the next, map that
    file instead.  A ``manifest.json`` pins the base source's description so a cache made from other
    weights is never used."""

    def __init__(self, base: TensorSource, cache_dir: str, base_id: str):
        self.base, self.dir, self.base_id = base, cache_dir, base_id
        os.makedirs(cache_dir, exist_ok=True)
        man = os.path.join(cache_dir, "manifest.json")
        if os.path.exists(man):
            with open(man) as f:
                if json.load(f).get("base") != base_id:
                    raise ValueError(f"{cache_dir} caches another checkpoint; use a fresh directory")
        else:
            with open(man, "w") as f:
                json.dump({"base": base_id}, f)
        self.hits = self.misses = 0

    def names(self):
        return self.base.names()

    def _file(self, name, dtype):
        tag = str(dtype).replace("torch.", "") if dtype is not None else "native"
        safe = name.replace("/", "_")
        return os.path.join(self.dir, f"{safe}.{tag}.safetensors")

    def get(self, name, device=None, dtype=None):
        from safetensors.torch import load_file, save_file
        path = self._file(name, dtype)
        if os.path.exists(path):
            self.hits += 1
            t = load_file(path)["t"]
        else:
            self.misses += 1
            t = self.base.get(name, dtype=dtype).contiguous()
            tmp = path + ".tmp"
            save_file({"t": t}, tmp)
            os.replace(tmp, path)               # readers never see a partial file
        return t.to(device) if device is not None else t


def quant_fp8_block(w: torch.Tensor, block=(128, 128)):
    """2-D weight -> (float8_e4m3fn values, fp32 scale_inv [ceil(N/bn), ceil(K/bk)]) with one
    scale per block chosen so the block's largest magnitude maps to the e4m3 maximum (448)."""
    bn, bk = block
    N, K = w.shape
    nb, kb = -(-N // bn), -(-K // bk)
    wp = torch.zeros(nb * bn, kb * bk, dtype=torch.float32)
    wp[:N, :K] = w.float()
    blocks = wp.view(nb, bn, kb, bk)
    amax = blocks.abs().amax(dim=(1, 3)).clamp(min=1e-12)
    scale_inv = amax / 448.0
    q = (blocks / scale_inv[:, None, :, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.view(nb * bn, kb * bk)[:N, :K].contiguous(), scale_inv.contiguous()


def dequant_fp8_block(q: torch.Tensor, scale_inv: torch.Tensor, block=(128, 128)) -> torch.Tensor:
    bn, bk = block
    N, K = q.shape
    s = scale_inv.float().repeat_interleave(bn, 0).repeat_interleave(bk, 1)[:N, :K]
    return q.float() * s


MX_BLOCK = 32
E4M3_EMAX = 8          # largest normal e4m3 value is 1.75 * 2^8 = 448


def quant_mxfp8(w: torch.Tensor, block: int = MX_BLOCK):
    """2-D weight -> (float8_e4m3fn values [N, K], E8M0 scales uint8 [N, ceil(K / block)]).

    OCP Microscaling (MX) v1.0 format: every ``block`` consecutive elements of a row share one
    power-of-two scale X = 2^(floor(log2(amax)) - emax(e4m3)); elements are stored as e4m3 of
    w / X (saturated to +-448) and the scale as its biased exponent (bias 127)."""
    N, K = w.shape
    kb = -(-K // block)
    wp = torch.zeros(N, kb * block, dtype=torch.float32, device=w.device)
    wp[:, :K] = w.float()
    blocks = wp.view(N, kb, block)
    amax = blocks.abs().amax(-1)
    exp = torch.where(amax > 0, torch.floor(torch.log2(amax.clamp(min=torch.finfo(torch.float32).tiny))),
                      torch.full_like(amax, -127.0)) - E4M3_EMAX
    exp = exp.clamp(-127, 127)
    scale = torch.exp2(exp)
    q = (blocks / scale[..., None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.view(N, kb * block)[:, :K].contiguous(), (exp + 127).to(torch.uint8).contiguous()


def dequant_mxfp8(q: torch.Tensor, scale_e8m0: torch.Tensor, block: int = MX_BLOCK) -> torch.Tensor:
    """fp32 weight from MXFP8 storage (exact: an e4m3 value times a power of two)."""
    N, K = q.shape
    s = torch.exp2(scale_e8m0.float() - 127.0).repeat_interleave(block, 1)[:, :K]
    return q.float() * s


class MXFP8Source(TensorSource):
    """Serves the base source's linear-layer weights as their MXFP8 round trip (e4m3 values with
    32-element power-of-two scales, dequantised exactly), everything else unchanged: a model built
    from it computes with exactly the weights an MXFP8 checkpoint holds."""

    def __init__(self, base: TensorSource, block: int = MX_BLOCK):
        self.base, self.block = base, block

    def names(self):
        return self.base.names()

    def get(self, name, device=None, dtype=None):
        t = self.base.get(name, device=device, dtype=torch.float32).float()     # quantised where it lives
        if _fp8_quantised(name, t):
            t = dequant_mxfp8(*quant_mxfp8(t, self.block), self.block)
        if dtype is not None and t.is_floating_point() and not name.endswith(("A_log", "dt_bias")):
            t = t.to(dtype)
        return t


def _fp8_quantised(name: str, t: torch.Tensor) -> bool:
    """Linear-layer weights are quantised; embeddings, LM head, norms and gate parameters stay."""
    return t.dim() == 2 and name.endswith(("proj.weight", "proj_qkv.weight", "proj_z.weight", "fc.weight"))


def random_target_source(cfg: ModelConfig, seed: int = 0) -> RandomSource:
    return RandomSource(target_shapes(cfg), seed=seed)


def random_drafter_source(d: DrafterConfig, vocab: int, seed: int = 1) -> RandomSource:
    return RandomSource(drafter_shapes(d, vocab), seed=seed, direct_norms=True)


def random_window_drafter_source(d, vocab: int, seed: int = 3) -> RandomSource:
    return RandomSource(window_drafter_shapes(d, vocab), seed=seed, direct_norms=True)


def materialize(src: TensorSource, device="cpu", dtype=torch.float32) -> dict:
    return {n: src.get(n, device=device, dtype=dtype) for n in src.names()}


def save_pretrained(path: str, cfg: ModelConfig, src: TensorSource, dtype=torch.bfloat16,
                    shard_bytes: int = 4 << 30, drafter: tuple | None = None, fp8_block: tuple | None = None,
                    mxfp8: bool = False):
    """Write ``config.json`` and (sharded) ``model.safetensors`` in HF layout.  ``drafter`` is an
    optional ``(DrafterConfig, TensorSource)`` written under ``path/drafter``.  ``fp8_block``
    (e.g. ``(128, 128)``) stores linear-layer weights as block-scaled FP8; ``mxfp8`` stores them as
    MXFP8 (e4m3 values, one E8M0 scale per 32 elements of a row in ``<name>_scale_e8m0``)."""
    from safetensors.torch import save_file
    if fp8_block and mxfp8:
        raise ValueError("choose one weight quantisation")
    os.makedirs(path, exist_ok=True)
    meta = {"model_type": "qwen3_5", "architectures": ["Qwen3_5ForConditionalGeneration"],
            "text_config": cfg.to_hf_text_config(), "tie_word_embeddings": cfg.tie_word_embeddings}
    if fp8_block:
        meta["quantization_config"] = {"quant_method": "fp8", "fmt": "e4m3", "activation_scheme": "dynamic",
                                       "weight_block_size": list(fp8_block)}
    if mxfp8:
        meta["quantization_config"] = {"quant_method": "mxfp8", "fmt": "e4m3", "scale_fmt": "e8m0",
                                       "activation_scheme": "none", "mx_block_size": MX_BLOCK}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(meta, f, indent=1)
    shards, cur, size = [], {}, 0

    def entries():
        for n in src.names():
            if fp8_block:
                t = src.get(n, dtype=torch.float32)
                if _fp8_quantised(n, t):
                    q, si = quant_fp8_block(t, fp8_block)
                    yield n, q
                    yield n + "_scale_inv", si
                    continue
            if mxfp8:
                t = src.get(n, dtype=torch.float32)
                if _fp8_quantised(n, t):
                    q, se = quant_mxfp8(t)
                    yield n, q
                    yield n + "_scale_e8m0", se
                    continue
            yield n, src.get(n, dtype=dtype).contiguous()

    for n, t in entries():
        if size + t.numel() * t.element_size() > shard_bytes and cur:
            shards.append(cur)
            cur, size = {}, 0
        cur[n] = t
        size += t.numel() * t.element_size()
    if cur:
        shards.append(cur)
    wm = {}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(path, fn), metadata={"format": "pt"})
        wm.update({k: fn for k in sh})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wm}, f, indent=1)
    if drafter is not None:
        dcfg, dsrc = drafter
        dpath = os.path.join(path, "drafter")
        os.makedirs(dpath, exist_ok=True)
        import dataclasses
        with open(os.path.join(dpath, "config.json"), "w") as f:
            json.dump(dict(dataclasses.asdict(dcfg), architectures=["DSparkDraftModel"]), f, indent=1)
        save_file({n: dsrc.get(n, dtype=dtype).contiguous() for n in dsrc.names()},
                  os.path.join(dpath, "model.safetensors"), metadata={"format": "pt"})


def load_window_drafter_config(path: str):
    """``WindowDrafterConfig`` from a ``window_drafter/config.json``."""
    import dataclasses
    from .config import WindowDrafterConfig
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    names = {f.name for f in dataclasses.fields(WindowDrafterConfig)}
    return WindowDrafterConfig(**{k: v for k, v in raw.items() if k in names})


def save_window_drafter(path: str, dcfg, src: TensorSource, dtype=torch.bfloat16):
    """Write a windowed drafter as ``path/config.json`` + ``path/model.safetensors``."""
    import dataclasses
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(dict(dataclasses.asdict(dcfg), architectures=["DFlash2DraftModel"]), f, indent=1)
    save_file({n: src.get(n, dtype=dtype).contiguous() for n in src.names()},
              os.path.join(path, "model.safetensors"), metadata={"format": "pt"})


def load_drafter_config(path: str) -> DrafterConfig:
    import dataclasses
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    names = {f.name for f in dataclasses.fields(DrafterConfig)}
    return DrafterConfig(**{k: v for k, v in raw.items() if k in names})
