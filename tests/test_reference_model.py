"""The fp32 reference hybrid against HF transformers' Qwen3.5 text model (independent oracle),
and the chunked delta rule against the sequential one."""
import torch

from qwen38_b200.models.reference import ReferenceModel
from qwen38_b200.ops import torch_ref as R


def test_reference_matches_hf(tiny):
    tr = __import__("pytest").importorskip("transformers")
    from transformers.models.qwen3_5 import Qwen3_5ForCausalLM, Qwen3_5TextConfig
    cfg = tiny["cfg"]
    hc = Qwen3_5TextConfig(**{k: v for k, v in cfg.to_hf_text_config().items()
                              if k not in ("model_type", "architectures")})
    hc._attn_implementation = "eager"
    m = Qwen3_5ForCausalLM(hc).float().eval()
    missing, unexpected = m.load_state_dict(tiny["sd"], strict=False)
    assert not missing and not unexpected
    toks = torch.tensor(tiny["prompt"][:40])[None]
    with torch.no_grad():
        hl = m(toks).logits[0]
    ref = ReferenceModel(cfg, tiny["sd"])
    rl, _, _ = ref.step(toks[0], ref.new_state())
    assert (hl - rl).abs().max().item() < 1e-4


def test_split_steps_equal_one_pass(tiny):
    cfg = tiny["cfg"]
    toks = torch.tensor(tiny["prompt"][:48])
    ref = ReferenceModel(cfg, tiny["sd"])
    full, _, _ = ref.step(toks, ref.new_state())
    st = ref.new_state()
    parts = [ref.step(toks[a:b], st)[0] for a, b in ((0, 17), (17, 18), (18, 48))]
    assert torch.allclose(torch.cat(parts), full, atol=1e-4)


def test_chunked_delta_rule_matches_recurrent():
    g = torch.Generator().manual_seed(3)
    T, H, Dk, Dv = 70, 3, 16, 8
    q = R.l2norm(torch.randn(T, H, Dk, generator=g)) * Dk ** -0.5
    k = R.l2norm(torch.randn(T, H, Dk, generator=g))
    v = torch.randn(T, H, Dv, generator=g)
    gate = -torch.rand(T, H, generator=g)
    beta = torch.rand(T, H, generator=g)
    S0 = torch.randn(H, Dk, Dv, generator=g) * 0.1
    o1, s1 = R.gdn_recurrent(q, k, v, gate, beta, S0)
    o2, s2 = R.gdn_chunked(q, k, v, gate, beta, S0, chunk=16)
    assert torch.allclose(o1, o2, atol=1e-4) and torch.allclose(s1, s2, atol=1e-4)
