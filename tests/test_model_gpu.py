"""End-to-end runtime on the GPU with the native kernels: speculative decoding is token-exact
against plain greedy decode through the same kernels, the native prefill agrees with the fp32
reference model, and full-width layer shapes run through every kernel."""
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from qwen38_b200.checkpoint import DictSource, materialize, random_drafter_source, random_target_source  # noqa: E402
from qwen38_b200.config import (FULL, LINEAR, DrafterConfig, ModelConfig, RuntimeConfig,  # noqa: E402
                                tiny_drafter_config, tiny_model_config)
from qwen38_b200.models.drafter import BlockDrafter  # noqa: E402
from qwen38_b200.models.reference import ReferenceModel  # noqa: E402
from qwen38_b200.models.target import HybridTarget  # noqa: E402
from qwen38_b200.ops.native import NativeOps  # noqa: E402
from qwen38_b200.spec.engine import PinnedAcceptance, SpecRuntime, greedy_reference  # noqa: E402


@pytest.fixture(scope="module")
def nops():
    return NativeOps()


def _tiny_target(nops):
    cfg = tiny_model_config()
    rt = RuntimeConfig(max_context=1024, prefill_chunk=64, gdn_chunk=16)
    return HybridTarget(cfg, random_target_source(cfg, 0), rt, device="cuda", dtype=torch.bfloat16, ops=nops)


def test_tiny_native_speculative_equals_greedy(nops):
    tgt = _tiny_target(nops)
    cfg, dcfg = tgt.cfg, tiny_drafter_config()
    dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, 1), tgt)
    prompt = torch.randint(0, cfg.vocab_size, (128,), generator=torch.Generator().manual_seed(0)).tolist()
    gold = greedy_reference(tgt, prompt, 40)
    for pinned in (None, PinnedAcceptance(gold, seed=3, mean_accepted=1)):
        res = SpecRuntime(tgt, dr, verifier_rows=4).generate(prompt, 40, gold_check=gold, pinned=pinned)
        assert res["tokens"] == gold
    nops.check()


def test_tiny_native_prefill_close_to_reference(nops):
    cfg = tiny_model_config()
    sd = materialize(random_target_source(cfg, 0))          # generated on the CPU, shared by both
    rt = RuntimeConfig(max_context=1024, prefill_chunk=64, gdn_chunk=16)
    tgt = HybridTarget(cfg, DictSource(sd), rt, device="cuda", dtype=torch.bfloat16, ops=nops)
    ref = ReferenceModel(cfg, sd)
    toks = torch.randint(0, cfg.vocab_size, (150,), generator=torch.Generator().manual_seed(1))
    logits, taps, hn = ref.step(toks, ref.new_state(), taps=(3,))
    seq = tgt.new_sequence()
    nxt, feats = tgt.prefill(seq, toks.cuda(), taps=(3,))
    rel = ((feats.float().cpu() - taps[3]).norm() / taps[3].norm()).item()
    assert rel < 3e-2
    top2 = logits[-1].topk(2).values
    if (top2[0] - top2[1]).item() > 0.05:        # skip near-ties in the bf16 comparison
        assert int(nxt) == int(logits[-1].argmax())
    tgt.release(seq)
    nops.check()


def test_full_width_slice_runs(nops):
    """4 layers at the flagship's widths (hidden 5120, GDN 16/48 heads, attention 24/4 x 256,
    SwiGLU 17408, vocab 151936) through prefill, a 16-row verify, commit and a drafter block."""
    cfg = ModelConfig(num_hidden_layers=4, layer_types=[LINEAR, LINEAR, LINEAR, FULL])
    dcfg = DrafterConfig(num_hidden_layers=1, taps=[1, 3])
    rt = RuntimeConfig(max_context=1024, prefill_chunk=256)
    tgt = HybridTarget(cfg, random_target_source(cfg, 0), rt, device="cuda", dtype=torch.bfloat16, ops=nops)
    dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, 1), tgt)
    prompt = torch.randint(0, cfg.vocab_size, (300,), generator=torch.Generator().manual_seed(2)).tolist()
    gold = greedy_reference(tgt, prompt, 20)
    res = SpecRuntime(tgt, dr, verifier_rows=16).generate(prompt, 20, gold_check=gold,
                                                          pinned=PinnedAcceptance(gold, seed=0, mean_accepted=6))
    assert res["tokens"] == gold
    nops.check()


def test_native_sampled_decoding_is_reproducible(nops):
    tgt = _tiny_target(nops)
    toks = torch.randint(0, tgt.cfg.vocab_size, (64,), generator=torch.Generator().manual_seed(8)).cuda()
    a = tgt.sample(toks, 10, temperature=0.8, seed=3)
    b = tgt.sample(toks, 10, temperature=0.8, seed=3)
    assert a == b and len(set(a)) > 1
    assert tgt.sample(toks, 6, temperature=0.0) == tgt.greedy(toks, 6)
    nops.check()



def test_native_serving_packed_verify_matches_single_stream(nops):
    """Continuous batching on the native kernels: five requests with 16-row verify blocks share
    packed verifies of up to 64 rows (four requests; the fifth rotates in), and every request's
    output equals its own single-stream greedy decode through the same kernels."""
    from qwen38_b200.serving.engine import ServingEngine
    from qwen38_b200.serving.scheduler import FINISHED
    cfg, dcfg = tiny_model_config(), tiny_drafter_config()
    rt = RuntimeConfig(max_context=1024, prefill_chunk=64, gdn_chunk=16)
    tgt = HybridTarget(cfg, random_target_source(cfg, 0), rt, device="cuda", dtype=torch.bfloat16, ops=nops,
                       max_slots=6, max_verify_rows=64)
    dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, 1), tgt, slots=5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(20 + i)).tolist()
               for i, n in enumerate((100, 70, 130, 90, 60))]
    golds = [greedy_reference(tgt, p, 24) for p in prompts]
    eng = ServingEngine(tgt, dr, verifier_rows=16)
    assert eng.sched.max_step_rows == 64
    reqs = [eng.add_request(p, 24, pinned=PinnedAcceptance(g, seed=i, mean_accepted=6))
            for i, (p, g) in enumerate(zip(prompts, golds))]
    eng.run()
    for r, g in zip(reqs, golds):
        assert r.state == FINISHED, r.error
        assert r.output == g
    assert eng.steps["decode"] < sum(len(g) for g in golds)
    nops.check()


def test_mxfp8_weights_stream_and_match_the_bf16_expansion(nops):
    """The multi-user benchmark's weight format on the runtime: the target's linear weights are MXFP8
    (``MXFP8Source``); with ``weight_format="mxfp8"`` the verify / decode GEMMs stream them as e4m3
    + E8M0 bytes, and every prediction equals the bf16 kernels' over the same (exactly expanded)
    weights, speculative output included."""
    from qwen38_b200.checkpoint import MXFP8Source
    from qwen38_b200.ops.native import MXWeight
    cfg, dcfg = tiny_model_config(), tiny_drafter_config()
    rt = RuntimeConfig(max_context=1024, prefill_chunk=64, gdn_chunk=16)
    src = MXFP8Source(random_target_source(cfg, 0))
    mx = NativeOps(weight_format="mxfp8")
    t_mx = HybridTarget(cfg, src, rt, device="cuda", dtype=torch.bfloat16, ops=mx)
    t_bf = HybridTarget(cfg, src, rt, device="cuda", dtype=torch.bfloat16, ops=nops)
    n_mx = sum(isinstance(w, MXWeight) for L in t_mx.layers for w in L.values())
    assert n_mx >= 2 * cfg.num_hidden_layers
    prompt = torch.randint(0, cfg.vocab_size, (100,), generator=torch.Generator().manual_seed(9)).tolist()
    gold = greedy_reference(t_bf, prompt, 24)
    assert greedy_reference(t_mx, prompt, 24) == gold
    dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, 1), t_mx)
    res = SpecRuntime(t_mx, dr, verifier_rows=8).generate(prompt, 24, gold_check=gold,
                                                          pinned=PinnedAcceptance(gold, seed=2, mean_accepted=4))
    assert res["tokens"] == gold
    mx.check()
    nops.check()
