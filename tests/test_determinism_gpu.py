"""Race detection without a sanitizer: every native kernel on the verify path is deterministic
(two runs of the same verify give identical bits), and the GEMM / attention / norm kernels write
nothing outside their outputs (canary words around each output stay intact)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from qwen38_b200.checkpoint import random_target_source  # noqa: E402
from qwen38_b200.config import RuntimeConfig, tiny_drafter_config, tiny_model_config  # noqa: E402
from qwen38_b200.models.target import HybridTarget  # noqa: E402
from qwen38_b200.ops.native import NativeOps  # noqa: E402

CANARY = -12288.0          # exact in bf16 and fp32


@pytest.fixture(scope="module")
def nops():
    return NativeOps()


def test_verify_is_bitwise_deterministic(nops):
    cfg = tiny_model_config()
    rt = RuntimeConfig(max_context=1024, prefill_chunk=64, gdn_chunk=16)
    tgt = HybridTarget(cfg, random_target_source(cfg, 0), rt, device="cuda", dtype=torch.bfloat16, ops=nops)
    prompt = torch.randint(0, cfg.vocab_size, (100,), generator=torch.Generator().manual_seed(3)).cuda()
    block = torch.randint(0, cfg.vocab_size, (16,), generator=torch.Generator().manual_seed(4)).cuda()
    outs = []
    for _ in range(2):
        seq = tgt.new_sequence()
        tgt.prefill(seq, prompt)
        pred, feats = tgt.verify([(seq, block)], taps=(1, 3))
        tgt.commit(seq, 7)
        outs.append((pred.clone(), feats.clone(), tgt.rec[seq.slot].clone(), tgt.conv[seq.slot].clone()))
        tgt.release(seq)
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    nops.check()


def _padded(shape, dtype, pad=256):
    n = 1
    for d in shape:
        n *= d
    buf = torch.full((n + 2 * pad,), CANARY, dtype=torch.float32, device="cuda").to(dtype)
    return buf, buf[pad:pad + n].view(*shape)


def _intact(buf, pad=256):
    return bool((buf[:pad].float() == CANARY).all() and (buf[-pad:].float() == CANARY).all())


@pytest.mark.parametrize("T,N,K", [(16, 640, 384), (5, 1000, 256), (300, 512, 256)])
def test_gemm_and_norm_write_only_their_outputs(nops, T, N, K):
    g = torch.Generator(device="cuda").manual_seed(T + N)
    x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
    w = nops.prepare_weight((torch.randn(N, K, generator=g, device="cuda") * 0.05).to(torch.bfloat16))
    buf, out = _padded((T, N), torch.float32)
    out.zero_()
    nops.C.linear(x, w.t, N, out, 1, nops.ws, nops.counters, nops.err)          # fp32 store
    bbuf, bout = _padded((T, N), torch.bfloat16)
    nops.C.linear(x, w.t, N, bout, 0, nops.ws, nops.counters, nops.err)         # bf16 store
    nbuf, nout = _padded((T, N), torch.bfloat16)
    nops.C.rms_norm(out, torch.ones(N, device="cuda"), 1e-6, nout)
    torch.cuda.synchronize()
    nops.check()
    assert _intact(buf) and _intact(bbuf) and _intact(nbuf)


def test_attention_writes_only_its_output(nops):
    T, H, Hkv, D, bs = 16, 6, 1, 256, 16
    g = torch.Generator(device="cuda").manual_seed(9)
    nb = 600 // bs + 2
    kc = torch.randn(nb, bs, Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(nb, bs, Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    bt = torch.arange(nb, dtype=torch.int32, device="cuda")
    q = torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16)
    pos = torch.arange(580, 580 + T, dtype=torch.int32, device="cuda")
    obuf, out = _padded((T, H * D), torch.bfloat16)
    po, pml = nops._bufs(Hkv, H // Hkv * T, D)
    nops.C.attn_decode(q, kc, vc, bt, bs, pos, D ** -0.5, 1, None, 0, out, po, pml, nops.max_keys, nops.err)
    pbuf, pout = _padded((T, H * D), torch.bfloat16)
    nops.C.attn_prefill(q, kc, vc, bt, bs, pos, D ** -0.5, None, pout)
    torch.cuda.synchronize()
    nops.check()
    assert _intact(obuf) and _intact(pbuf)
    assert ((out.float() - pout.float()).norm() / pout.float().norm()).item() < 2e-2   # two kernels, one answer
