"""HF-layout checkpoints on disk: bf16 round trip, block-FP8 write + dequantising read, and the
runtime loading either one matches the fp32 reference on the same (dequantised) weights."""
import json
import os

import torch

from qwen38_b200.checkpoint import (SafetensorsSource, dequant_fp8_block, materialize, quant_fp8_block,
                                    save_pretrained)
from qwen38_b200.config import ModelConfig, RuntimeConfig
from qwen38_b200.models.reference import ReferenceModel
from qwen38_b200.models.target import HybridTarget

RT = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)


def test_fp8_block_quantisation_error():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(300, 200, generator=g) * torch.rand(300, 1, generator=g)   # rows of different scale
    q, si = quant_fp8_block(w, (128, 128))
    assert q.dtype == torch.float8_e4m3fn and si.shape == (3, 2)
    d = dequant_fp8_block(q, si, (128, 128))
    rel = ((d - w).norm() / w.norm()).item()
    assert rel < 0.04                         # e4m3: 3 mantissa bits, per-block scale
    assert torch.equal(dequant_fp8_block(*quant_fp8_block(d, (128, 128)), (128, 128)), d)  # idempotent


def test_bf16_checkpoint_round_trip(tiny, tmp_path):
    save_pretrained(str(tmp_path), tiny["cfg"], tiny["src"], shard_bytes=1 << 20)
    idx = json.load(open(os.path.join(tmp_path, "model.safetensors.index.json")))
    assert len(set(idx["weight_map"].values())) > 1                      # sharded
    cfg = ModelConfig.from_pretrained(str(tmp_path))
    assert cfg.layer_types == tiny["cfg"].layer_types and cfg.hidden_size == tiny["cfg"].hidden_size
    src = SafetensorsSource(str(tmp_path))
    assert sorted(src.names()) == sorted(tiny["src"].names())
    for n in list(src.names())[:8]:
        assert torch.equal(src.get(n, dtype=torch.float32),
                           tiny["src"].get(n, dtype=torch.bfloat16).float())


def test_fp8_checkpoint_loads_and_runs(tiny, tmp_path):
    save_pretrained(str(tmp_path), tiny["cfg"], tiny["src"], fp8_block=(32, 32))
    meta = json.load(open(os.path.join(tmp_path, "config.json")))
    assert meta["quantization_config"]["weight_block_size"] == [32, 32]
    src = SafetensorsSource(str(tmp_path))
    names = list(src.names())
    assert not any(n.endswith("_scale_inv") for n in names)
    qn = [n for n in names if n.endswith("proj.weight")][0]
    w0 = tiny["src"].get(qn, dtype=torch.float32)
    w1 = src.get(qn, dtype=torch.float32)
    assert ((w1 - w0).norm() / w0.norm()).item() < 0.05
    sd = materialize(src)
    ref = ReferenceModel(tiny["cfg"], sd)
    toks = torch.tensor(tiny["prompt"][:64])
    tgt = HybridTarget(tiny["cfg"], src, RT)
    assert tgt.greedy(toks, 16) == ref.greedy(toks, 16)


def test_cached_source_roundtrip_and_pinning(tmp_path):
    """The converted-tensor cache returns the base source's tensors (an fp8-block checkpoint is
    dequantised once), serves later loads without the base, and refuses another checkpoint's cache."""
    import pytest
    from qwen38_b200.checkpoint import CachedSource, DictSource, quant_fp8_block, dequant_fp8_block
    g = torch.Generator().manual_seed(0)
    w = torch.randn(256, 384, generator=g)
    q, si = quant_fp8_block(w)
    base = DictSource({"a.weight": dequant_fp8_block(q, si), "b.norm.weight": torch.randn(384, generator=g)})
    calls = []
    real_get = base.get
    base.get = lambda n, device=None, dtype=None: calls.append(n) or real_get(n, device=device, dtype=dtype)
    c = CachedSource(base, str(tmp_path / "cache"), base_id="ckpt-1")
    a = c.get("a.weight", dtype=torch.bfloat16)
    assert torch.equal(a, base.sd["a.weight"].bfloat16()) and c.misses == 1
    c2 = CachedSource(base, str(tmp_path / "cache"), base_id="ckpt-1")
    assert torch.equal(c2.get("a.weight", dtype=torch.bfloat16), a) and c2.hits == 1
    assert calls == ["a.weight"]                      # the second load never read the base
    assert torch.equal(c2.get("b.norm.weight"), base.sd["b.norm.weight"])
    with pytest.raises(ValueError):
        CachedSource(base, str(tmp_path / "cache"), base_id="ckpt-2")


def test_factory_weight_cache(tmp_path):
    """An engine built through the weight cache equals one built from the checkpoint directly; the
    second build reads the cache only."""
    from qwen38_b200.checkpoint import random_target_source, save_pretrained
    from qwen38_b200.config import tiny_model_config
    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.factory import build_engine
    from qwen38_b200.spec.engine import greedy_reference
    cfg = tiny_model_config()
    ck = str(tmp_path / "ckpt")
    save_pretrained(ck, cfg, random_target_source(cfg, 0), dtype=torch.float32)
    base = ["spec.drafter=none", f"model={ck}"]
    plain = build_engine(load_run_config(None, profile="tiny-cpu", overrides=base))
    cache = str(tmp_path / "cache")
    for _ in range(2):
        eng = build_engine(load_run_config(None, profile="tiny-cpu", overrides=base + [f"weight_cache={cache}"]))
    assert len([f for f in os.listdir(cache) if f.endswith(".safetensors")]) > 10
    p = list(range(5, 40))
    assert greedy_reference(eng.target, p, 8) == greedy_reference(plain.target, p, 8)


def test_mxfp8_quantisation():
    """OCP MX e4m3 with 32-element power-of-two scales: scale exponent floor(log2 amax) - 8, values
    within e4m3 precision, dequantised weights exact in bf16."""
    from qwen38_b200.checkpoint import dequant_mxfp8, quant_mxfp8
    g = torch.Generator().manual_seed(3)
    w = torch.randn(64, 100, generator=g) * torch.logspace(-3, 2, 100)[None, :]
    q, se = quant_mxfp8(w)
    assert q.dtype == torch.float8_e4m3fn and q.shape == w.shape and se.shape == (64, 4) and se.dtype == torch.uint8
    d = dequant_mxfp8(q, se)
    assert torch.equal(d.bfloat16().float(), d)                          # exact in bf16
    blocks = torch.nn.functional.pad(w, (0, 28)).view(64, 4, 32)
    amax = blocks.abs().amax(-1)
    assert torch.equal(se.long(), (torch.floor(torch.log2(amax)) - 8 + 127).long())
    scale = torch.exp2(se.float() - 127).repeat_interleave(32, 1)[:, :100]
    err = (d - w).abs()
    sat = w.abs() > 448 * scale                                           # saturated by the MX rule
    assert bool((err[~sat] <= torch.maximum(w.abs()[~sat] * 2.0 ** -4, scale[~sat] * 2.0 ** -9)).all())
    z, sz = quant_mxfp8(torch.zeros(2, 32))
    assert torch.equal(dequant_mxfp8(z, sz), torch.zeros(2, 32))


def test_mxfp8_checkpoint_and_weight_format(tmp_path):
    """An MXFP8 checkpoint reads back the MXFP8 round trip of its weights; runtime.weight_format=mxfp8
    builds the same model from bf16 weights; norms and embeddings stay unquantised."""
    from qwen38_b200.checkpoint import MXFP8Source, random_target_source, save_pretrained
    from qwen38_b200.config import tiny_model_config
    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.factory import build_engine
    from qwen38_b200.spec.engine import greedy_reference
    cfg = tiny_model_config()
    src = random_target_source(cfg, 0)
    ck = str(tmp_path / "mx")
    save_pretrained(ck, cfg, src, dtype=torch.float32, mxfp8=True)
    st = SafetensorsSource(ck)
    mx = MXFP8Source(src)
    for n in st.names():
        assert torch.equal(st.get(n, dtype=torch.float32), mx.get(n, dtype=torch.float32)), n
    name = next(n for n in st.names() if n.endswith("mlp.down_proj.weight"))
    assert not torch.equal(mx.get(name, dtype=torch.float32), src.get(name, dtype=torch.float32))
    assert torch.equal(mx.get("model.norm.weight"), src.get("model.norm.weight"))
    p = list(range(7, 50))
    a = build_engine(load_run_config(None, profile="tiny-cpu", overrides=["spec.drafter=none", f"model={ck}"]))
    ck2 = str(tmp_path / "bf")
    save_pretrained(ck2, cfg, src, dtype=torch.float32)
    b = build_engine(load_run_config(None, profile="tiny-cpu", overrides=[
        "spec.drafter=none", f"model={ck2}", "runtime.weight_format=mxfp8"]))
    assert greedy_reference(a.target, p, 10) == greedy_reference(b.target, p, 10)
