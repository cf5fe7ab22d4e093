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
