"""Every TP degree the bench runs (1, 2, 4, 8) satisfies the kernels' shape constraints at the
flagship shape; a shape that breaks one is reported with the reason."""
import pytest

from qwen38_b200.config import DrafterConfig, ModelConfig, full_drafter_config, full_model_config
from qwen38_b200.models.target import pack_gdn
from qwen38_b200.parallel.plan import check_tp_plan, gdn_in_width, tp_plan


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_flagship_shapes_run_at_every_tp(tp):
    cfg, dcfg = full_model_config(), full_drafter_config()
    assert check_tp_plan(cfg, dcfg, tp) == []
    p = tp_plan(cfg, dcfg, tp)
    assert p["gdn_in"] % 8 == 0
    assert p["gdn_in"] == {1: 16480, 2: 8240, 4: 4120, 8: 2064}[tp]   # TP8: 2060 rows + 4 zero rows


def test_packed_gdn_rows_are_padded():
    cfg = ModelConfig(num_hidden_layers=4, hidden_size=256, intermediate_size=512, vocab_size=512,
                      linear_num_key_heads=8, linear_num_value_heads=24, linear_key_head_dim=32,
                      linear_value_head_dim=32, num_attention_heads=8, num_key_value_heads=4, head_dim=64)

    class Src:
        def get(self, name, device=None, dtype=None):
            import torch
            shapes = {"in_proj_qkv.weight": (2 * 8 * 32 + 24 * 32, 256), "in_proj_z.weight": (24 * 32, 256),
                      "in_proj_b.weight": (24, 256), "in_proj_a.weight": (24, 256),
                      "conv1d.weight": (2 * 8 * 32 + 24 * 32, 1, 4), "out_proj.weight": (256, 24 * 32),
                      "A_log": (24,), "dt_bias": (24,), "norm.weight": (32,)}
            key = name.split("linear_attn.")[1]
            return torch.ones(shapes[key])
    L = pack_gdn(Src(), 0, cfg, 8, 0, "cpu", None)
    raw = 2 * 1 * 32 + 2 * 3 * 32 + 2 * 3             # 262 rows per rank at TP8
    assert L["w_in"].shape[0] == gdn_in_width(cfg, 8) == 264
    assert float(L["w_in"][raw:].abs().sum()) == 0.0


def test_violations_are_reported():
    cfg = ModelConfig(intermediate_size=17408 + 8 * 32)      # 17664 / 8 = 2208: not a multiple of 64
    bad = check_tp_plan(cfg, None, 8)
    assert any("64-row gate/up block" in b for b in bad)
    assert check_tp_plan(full_model_config(), DrafterConfig(intermediate_size=17472), 8)   # 2184 per rank
    assert check_tp_plan(ModelConfig(num_attention_heads=24, num_key_value_heads=2), None, 1)  # group of 12
