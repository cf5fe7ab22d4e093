"""Commit of every accepted prefix 0..T of a verify block leaves exactly the state that k
single-row decodes of the same tokens leave: GDN recurrent state, conv windows, the valid K/V
rows of the sequence - and nothing in any other slot changes.  CPU (fp32, tolerance) and GPU
(native kernels, bit for bit: the verify path is batch-invariant and commit replays it)."""
import pytest
import torch

from qwen38_b200.config import RuntimeConfig


def _kv_rows(tgt, seq, n):
    """K/V rows 0..n-1 of the sequence, gathered through its block table [layers, n, kv, D]."""
    bs = tgt.block_size
    idx = torch.arange(n, device=tgt.device)
    blk = seq.block_table[(idx // bs).long()].long()
    return tgt.kcache[:, blk, idx % bs], tgt.vcache[:, blk, idx % bs]


def _check(tgt, prompt, block, exact):
    eq = (lambda a, b: torch.equal(a, b)) if exact else (lambda a, b: torch.allclose(a.float(), b.float(), atol=2e-5))
    T = int(block.shape[0])
    for k in range(T + 1):
        a, b, other = tgt.new_sequence(), tgt.new_sequence(), tgt.new_sequence()
        try:
            tgt.prefill(a, prompt)
            tgt.prefill(b, prompt)
            tgt.prefill(other, prompt[: len(prompt) // 2])
            other_state = (tgt.rec[other.slot].clone(), tgt.conv[other.slot].clone())
            other_kv = [t.clone() for t in _kv_rows(tgt, other, other.pos)]
            tgt.verify([(a, block)])
            tgt.commit(a, k)
            for t in block[:k]:
                tgt.decode(b, t.reshape(1))
            assert a.pos == b.pos
            assert eq(tgt.rec[a.slot], tgt.rec[b.slot]), f"GDN state differs after committing {k} rows"
            assert eq(tgt.conv[a.slot], tgt.conv[b.slot]), f"conv window differs after committing {k} rows"
            ka, va = _kv_rows(tgt, a, a.pos)
            kb, vb = _kv_rows(tgt, b, b.pos)
            assert eq(ka, kb) and eq(va, vb), f"valid K/V differ after committing {k} rows"
            assert torch.equal(tgt.rec[other.slot], other_state[0]) and torch.equal(tgt.conv[other.slot], other_state[1])
            for x, y in zip(_kv_rows(tgt, other, other.pos), other_kv):
                assert torch.equal(x, y)                          # inactive slot untouched
        finally:
            for s in (a, b, other):
                tgt.release(s)


def test_every_accepted_prefix_cpu(tiny):
    from qwen38_b200.models.target import HybridTarget
    rt = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)
    tgt = HybridTarget(tiny["cfg"], tiny["src"], rt, max_slots=4)
    prompt = torch.tensor(tiny["prompt"][:90])
    block = torch.tensor(tiny["prompt"][90:94])
    _check(tgt, prompt, block, exact=False)


@pytest.mark.gpu
def test_every_accepted_prefix_gpu_bitwise():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from qwen38_b200.checkpoint import random_target_source
    from qwen38_b200.config import tiny_model_config
    from qwen38_b200.models.target import HybridTarget
    from qwen38_b200.ops.native import NativeOps
    cfg = tiny_model_config()
    rt = RuntimeConfig(max_context=1024, prefill_chunk=64, gdn_chunk=16, use_cuda_graphs=False)
    ops = NativeOps()
    tgt = HybridTarget(cfg, random_target_source(cfg, 0), rt, device="cuda", dtype=torch.bfloat16, ops=ops,
                       max_slots=4)
    g = torch.Generator().manual_seed(12)
    prompt = torch.randint(0, cfg.vocab_size, (150,), generator=g).cuda()
    block = torch.randint(0, cfg.vocab_size, (16,), generator=g).cuda()
    _check(tgt, prompt, block, exact=True)
    ops.check()
