"""Windowed (DFlash2) drafter: the convolution, the window mask and the selector against plain
fp64 statements of the reference's oracles (``scripts/ci/draft_convolution.py:17-37``,
``scripts/ci/draft_attention.py:4-18``, ``scripts/ci/draft_selector.py:37-56``), candidates that
do not depend on the vocabulary sharding, and speculative output equal to plain greedy decode."""
import os
from types import SimpleNamespace

import pytest
import torch

from qwen38_b200.checkpoint import (SafetensorsSource, load_window_drafter_config, random_window_drafter_source,
                                    save_window_drafter)
from qwen38_b200.config import RuntimeConfig, tiny_window_drafter_config
from qwen38_b200.models.target import HybridTarget
from qwen38_b200.models.window_drafter import WindowDrafter
from qwen38_b200.ops import TorchOps
from qwen38_b200.ops import torch_ref as R
from qwen38_b200.spec.engine import PinnedAcceptance, SpecRuntime, greedy_reference


def _conv_oracle(x, dyn, tap0, base, group):
    rows, H = x.shape
    G = H // group
    xb = x.to(torch.bfloat16).double()
    y = torch.zeros(rows, H, dtype=torch.float64)
    for r in range(rows):
        for o in range(2):
            if r - o >= 0:
                k = base[o].double() + dyn[r, (tap0 + o) * G:(tap0 + o + 1) * G].double().repeat_interleave(group)
                y[r] += k * xb[r - o]
    return y


def test_draft_conv_matches_oracle():
    g = torch.Generator().manual_seed(0)
    rows, H, group = 8, 64, 16
    x = torch.randn(rows, H, generator=g)
    dyn = (torch.randn(rows, 4 * H // group, generator=g) * 0.1).bfloat16()
    base = torch.randn(2, H, generator=g)
    ops = TorchOps()
    for tap0 in (0, 2):
        y = R.draft_conv(x, dyn, tap0, base, group)
        assert torch.allclose(y.double(), _conv_oracle(x, dyn, tap0, base, group), atol=1e-5)
        res = torch.ones(rows, H)
        ops.draft_conv(x, dyn, tap0, base, group, residual=res)
        assert torch.equal(res, 1 + y)
        assert torch.equal(ops.draft_conv(x, dyn, tap0, base, group), y.bfloat16())
    # causal over the rows: rows before a change keep their values
    x2 = x.clone()
    x2[5:] += 1
    assert torch.equal(R.draft_conv(x2, dyn, 0, base, group)[:5], R.draft_conv(x, dyn, 0, base, group)[:5])


def _window_case(pos, T, H=4, Hkv=2, D=32, cap=128, seed=0):
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(T, (H + 2 * Hkv) * D, generator=g)
    kc = torch.randn(cap, Hkv, D, generator=g)
    vc = torch.randn(cap, Hkv, D, generator=g)
    qn = 1 + 0.1 * torch.randn(D, generator=g)
    kn = 1 + 0.1 * torch.randn(D, generator=g)
    inv = 1.0 / (1.0e7 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    return qkv, kc, vc, qn, kn, inv, (H, Hkv, D), torch.arange(pos, pos + T, dtype=torch.int32)


def test_window_mask_attention_matches_explicit_keys():
    pos, T, W = 70, 4, 24
    qkv, kc, vc, qn, kn, inv, dims, positions = _window_case(pos, T)
    H, Hkv, D = dims
    ops = TorchOps()
    out = ops.draft_block_attention(qkv, qn, kn, inv, 1.0, dims, 1e-6, positions, kc, vc, torch.float32, window=W)
    # oracle: rotate q as the op does, then attend each row's explicit key set
    q = qkv[:, :H * D].reshape(T, H, D)
    cos, sin = R.rope_cos_sin(positions, D, 1.0, inv, 1.0)
    q = R.apply_rope(ops.rms_norm(q, qn, 1e-6, torch.float32), cos, sin).double()
    rep = H // Hkv
    for t in range(T):
        keys = [k for k in range(pos + T) if pos + t - k < W]
        assert keys[0] == pos + t - W + 1 and keys[-1] == pos + T - 1      # window + every block row
        K, V = kc[keys].double(), vc[keys].double()
        for h in range(H):
            s = (K[:, h // rep] @ q[t, h]) * D ** -0.5
            o = torch.softmax(s, 0) @ V[:, h // rep]
            assert torch.allclose(out[t, h * D:(h + 1) * D].double(), o, atol=1e-5)
    # a window covering the whole history is the unwindowed drafter attention
    kc2, vc2 = kc.clone(), vc.clone()
    wide = ops.draft_block_attention(qkv, qn, kn, inv, 1.0, dims, 1e-6, positions, kc2, vc2, torch.float32,
                                     window=pos + T)
    full = ops.draft_block_attention(qkv, qn, kn, inv, 1.0, dims, 1e-6, positions, kc2, vc2, torch.float32)
    assert torch.allclose(wide, full, atol=1e-6)


def _selector_case(V=300, rank=16, rows=8, C=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    pred = torch.randn(V, rank, generator=g).bfloat16()
    succ = torch.randn(V, rank, generator=g).bfloat16()
    feats = torch.randn(rows, rank, generator=g).bfloat16()
    cand = torch.stack([torch.randperm(V, generator=g)[:C] for _ in range(rows)])
    unary = torch.randn(rows, C, generator=g) * 0.5
    return feats, cand, unary, pred, succ


def test_selector_matches_fp64_oracle():
    feats, cand, unary, pred, succ = _selector_case()
    ops = TorchOps()
    ids = ops.draft_select(feats, cand, unary, torch.tensor([7]), pred, succ)
    ref, scores = R.greedy_select(feats, cand, unary, 7, pred, succ)
    assert ids.tolist() == ref.tolist() and scores.shape == (7, 8)
    # without the learned edges the selector is the per-row argmax of the candidate logits
    ids0 = ops.draft_select(feats, cand, unary, torch.tensor([7]), pred * 0, succ * 0)
    assert ids0.tolist() == [int(cand[i, unary[i].argmax()]) for i in range(1, 8)]
    assert ids.tolist() != ids0.tolist()


def test_candidates_do_not_depend_on_vocab_sharding():
    g = torch.Generator().manual_seed(1)
    rows, V, C = 3, 64, 5
    logits = torch.randn(rows, V, generator=g)
    ref_v, ref_i = torch.topk(logits, C, -1)
    one = SimpleNamespace(n_cand=C, tp=1, comm=None, target=SimpleNamespace(vocab_offset=0))
    ids, vals = WindowDrafter.candidates(one, logits)
    assert torch.equal(ids, ref_i) and torch.equal(vals, ref_v)
    for tp in (2, 4):
        w = V // tp
        loc = [torch.topk(logits[:, r * w:(r + 1) * w], C, -1) for r in range(tp)]
        gathered = {torch.float32: torch.cat([l.values for l in loc], 1),
                    torch.int64: torch.cat([l.indices + r * w for r, l in enumerate(loc)], 1)}
        comm = SimpleNamespace(all_gather_cat=lambda t, dim: gathered[t.dtype])
        me = SimpleNamespace(n_cand=C, tp=tp, comm=comm, target=SimpleNamespace(vocab_offset=0))
        ids, vals = WindowDrafter.candidates(me, logits[:, :w])
        assert torch.equal(ids, ref_i) and torch.equal(vals, ref_v)


def _target(tiny):
    return HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16))


def test_window_drafter_speculative_equals_greedy(tiny):
    tgt = _target(tiny)
    wcfg = tiny_window_drafter_config()
    dr = WindowDrafter(wcfg, random_window_drafter_source(wcfg, tiny["cfg"].vocab_size), tgt)
    assert dr.P == wcfg.block_rows - 1 and dr.rows == wcfg.block_rows
    gold = greedy_reference(tgt, tiny["prompt"], 24)
    sr = SpecRuntime(tgt, dr, verifier_rows=wcfg.block_rows)
    res = sr.generate(tiny["prompt"], 24, gold_check=gold)
    assert res["tokens"] == gold
    assert dr.positions[0] >= len(tiny["prompt"]) > wcfg.window
    res = sr.generate(tiny["prompt"], 24, gold_check=gold, pinned=PinnedAcceptance(gold, seed=3, mean_accepted=2))
    assert res["tokens"] == gold


@pytest.mark.parametrize("rows,window,cand", [(2, 2, 1), (8, 8, 4), (16, 40, 16)])
def test_window_drafter_geometries(tiny, rows, window, cand):
    """Block widths 2..16, a window as small as the block, one candidate: still token-exact."""
    import dataclasses
    tgt = _target(tiny)
    wcfg = dataclasses.replace(tiny_window_drafter_config(), block_rows=rows, window=window, candidates=cand)
    dr = WindowDrafter(wcfg, random_window_drafter_source(wcfg, tiny["cfg"].vocab_size), tgt)
    gold = greedy_reference(tgt, tiny["prompt"], 20)
    res = SpecRuntime(tgt, dr, verifier_rows=rows).generate(tiny["prompt"], 20, gold_check=gold)
    assert res["tokens"] == gold


def test_window_drafter_config_checks():
    import dataclasses
    with pytest.raises(ValueError):
        dataclasses.replace(tiny_window_drafter_config(), window=2)          # smaller than a block
    with pytest.raises(ValueError):
        dataclasses.replace(tiny_window_drafter_config(), conv_group=48)     # 256 % 48 != 0
    with pytest.raises(ValueError):
        dataclasses.replace(tiny_window_drafter_config(), candidates=0)


def test_window_limits_what_the_block_sees(tiny):
    """With a history longer than the window, keys older than the window change nothing; a wider
    window sees them."""
    tgt = _target(tiny)
    wcfg = tiny_window_drafter_config()
    src = random_window_drafter_source(wcfg, tiny["cfg"].vocab_size)
    dr = WindowDrafter(wcfg, src, tgt)
    seq = tgt.new_sequence()
    _, feats = tgt.prefill(seq, torch.tensor(tiny["prompt"]), taps=wcfg.taps)
    tgt.release(seq)
    dr.append(feats, 0)
    anchor = torch.tensor([5])
    logits, sel = dr.forward_block(anchor)
    old = slice(0, len(tiny["prompt"]) - wcfg.window)        # below every block row's window
    dr.kctx_all[0, :, old] += 3.0
    dr.vctx_all[0, :, old] -= 3.0
    logits2, sel2 = dr.forward_block(anchor)
    assert torch.equal(logits, logits2) and torch.equal(sel, sel2)
    dr.window = 10 ** 6
    logits3, _ = dr.forward_block(anchor)
    assert not torch.allclose(logits, logits3)


def test_window_drafter_checkpoint_roundtrip(tiny, tmp_path):
    tgt = _target(tiny)
    wcfg = tiny_window_drafter_config()
    src = random_window_drafter_source(wcfg, tiny["cfg"].vocab_size)
    path = os.path.join(str(tmp_path), "window_drafter")
    save_window_drafter(path, wcfg, src, dtype=torch.float32)
    assert load_window_drafter_config(path) == wcfg
    a = WindowDrafter(wcfg, src, tgt)
    b = WindowDrafter(load_window_drafter_config(path), SafetensorsSource(path), tgt)
    seq = tgt.new_sequence()
    _, feats = tgt.prefill(seq, torch.tensor(tiny["prompt"][:40]), taps=wcfg.taps)
    tgt.release(seq)
    a.append(feats, 0)
    b.append(feats, 0)
    anchor = torch.tensor([11])
    assert torch.equal(a.propose(anchor), b.propose(anchor))


def test_serving_engine_with_window_drafter():
    from qwen38_b200.runconfig import load_run_config
    from qwen38_b200.serving.factory import build_engine
    rc = load_run_config(None, profile="tiny-cpu", overrides=["spec.drafter=dflash2"])
    eng = build_engine(rc)
    assert isinstance(eng.drafter, WindowDrafter)
    prompts = {"a": list(range(3, 40)), "b": list(range(100, 160))}
    for rid, p in prompts.items():
        eng.add_request(p, 12, request_id=rid)
    done = {r.request_id: r.output for r in eng.run()}
    for rid, p in prompts.items():
        assert done[rid] == greedy_reference(eng.target, p, len(done[rid]))


def test_window_drafter_prefix_reuse(tiny):
    """A prefix checkpoint carries the windowed drafter's history: the second request restores it,
    prefills only the suffix and proposes exactly what a cold run proposes."""
    from qwen38_b200.prefix.registry import PrefixRegistry
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16),
                       max_slots=2)
    wcfg = tiny_window_drafter_config()
    src = random_window_drafter_source(wcfg, tiny["cfg"].vocab_size)
    dr = WindowDrafter(wcfg, src, tgt)
    g = torch.Generator().manual_seed(7)
    prefix = torch.randint(0, 4096, (128,), generator=g).tolist()
    a = prefix + torch.randint(0, 4096, (100,), generator=g).tolist()
    b = prefix + torch.randint(0, 4096, (90,), generator=g).tolist()
    gold_b = greedy_reference(tgt, b, 20)
    reg = PrefixRegistry(tgt, budget_bytes=1 << 30, boundary=64)
    sr = SpecRuntime(tgt, dr, verifier_rows=wcfg.block_rows, prefix=reg)
    sr.generate(a, 20)
    rb = sr.generate(b, 20, gold_check=gold_b)
    assert rb["reused_prefix"] == 128 and rb["tokens"] == gold_b
    # warm (restored + suffix) drafter history proposes what a cold full publication proposes
    cold = WindowDrafter(wcfg, src, tgt)
    seq = tgt.new_sequence()
    _, feats = tgt.prefill(seq, torch.tensor(b), taps=wcfg.taps)
    tgt.release(seq)
    cold.append(feats, 0)
    ck = reg.lookup(b)                # b's own deepest boundary by now
    assert ck is not None and 128 <= ck.pos < len(b)
    # only the rows the window can still reach are kept
    assert ck.drafter["lo"] == ck.pos - wcfg.window and ck.drafter["k"].shape[1] == wcfg.window
    seq = reg.restore(ck, dr)
    _, feats = tgt.prefill(seq, torch.tensor(b[ck.pos:]), taps=wcfg.taps)
    tgt.release(seq)
    dr.append(feats, ck.pos)
    anchor = torch.tensor([b[-1]])
    assert torch.equal(dr.propose(anchor), cold.propose(anchor))


def _tp_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qwen38_b200.checkpoint import random_target_source
        from qwen38_b200.config import tiny_model_config
        from qwen38_b200.parallel.comm import TorchComm
        cfg, wcfg = tiny_model_config(), tiny_window_drafter_config()
        rt = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)
        prompt = torch.randint(0, cfg.vocab_size, (128,), generator=torch.Generator().manual_seed(0)).tolist()
        tgt = HybridTarget(cfg, random_target_source(cfg, 0), rt, comm=TorchComm())
        dr = WindowDrafter(wcfg, random_window_drafter_source(wcfg, cfg.vocab_size), tgt)
        seq = tgt.new_sequence()
        _, feats = tgt.prefill(seq, torch.tensor(prompt), taps=wcfg.taps)
        tgt.release(seq)
        dr.append(feats, 0)
        props = dr.propose(torch.tensor([prompt[-1]])).tolist()
        dr.reset()
        gold = greedy_reference(tgt, prompt, 20)
        res = SpecRuntime(tgt, dr, verifier_rows=wcfg.block_rows).generate(prompt, 20, gold_check=gold)
        q.put((rank, props, gold, res["tokens"]))
    except BaseException as e:   # report instead of hanging the parent
        q.put((rank, repr(e), None, None))
    finally:
        dist.destroy_process_group()


def test_window_drafter_tp2_gloo(tiny):
    """Two gloo ranks: identical proposals on both ranks (candidates gathered over the vocabulary
    shards), equal to the single-rank drafter's on this seed, and token-exact speculation."""
    import socket
    import torch.multiprocessing as mp
    tgt = _target(tiny)
    wcfg = tiny_window_drafter_config()
    dr = WindowDrafter(wcfg, random_window_drafter_source(wcfg, tiny["cfg"].vocab_size), tgt)
    seq = tgt.new_sequence()
    _, feats = tgt.prefill(seq, torch.tensor(tiny["prompt"]), taps=wcfg.taps)
    tgt.release(seq)
    dr.append(feats, 0)
    props1 = dr.propose(torch.tensor([tiny["prompt"][-1]])).tolist()
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, props, gold, spec in out:
        assert spec is not None, props
        assert spec == gold
    assert out[0][1] == out[1][1] == props1


# ------------------------------------------------------------------------------------------ GPU
@pytest.fixture(scope="module")
def nops():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from qwen38_b200.ops.native import NativeOps
    return NativeOps()


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [1, 8, 32])
def test_native_draft_conv(nops, rows):
    g = torch.Generator().manual_seed(rows)
    H, group = 5120, 16
    dyn = (torch.randn(rows, 4 * H // group, generator=g) * 0.1).bfloat16().cuda()
    base = torch.randn(2, H, generator=g).cuda()
    tops = TorchOps()
    for xdt in (torch.bfloat16, torch.float32):
        x = torch.randn(rows, H, generator=g).to(xdt).cuda()
        for tap0 in (0, 2):
            ref = R.draft_conv(x.float(), dyn, tap0, base, group)
            out = nops.draft_conv(x, dyn, tap0, base, group)
            torch.testing.assert_close(out.float(), ref.bfloat16().float(), atol=1e-6, rtol=8e-3)
            res = torch.randn(rows, H, generator=g).cuda()
            res2 = res.clone()
            nops.draft_conv(x, dyn, tap0, base, group, residual=res)
            tops.draft_conv(x.float(), dyn, tap0, base, group, residual=res2)
            torch.testing.assert_close(res, res2, atol=1e-5, rtol=1e-5)
    nops.check()


@pytest.mark.gpu
@pytest.mark.parametrize("pos,T,W", [(100, 8, 2048), (3000, 16, 2048), (5000, 8, 300), (70, 4, 24)])
def test_native_window_attention(nops, pos, T, W):
    qkv, kc, vc, qn, kn, inv, dims, positions = _window_case(pos, T, H=32, Hkv=8, D=128, cap=pos + 64)
    tops = TorchOps()
    kc2, vc2 = kc.cuda(), vc.cuda()
    ref = tops.draft_block_attention(qkv.cuda(), qn.cuda(), kn.cuda(), inv.cuda(), 1.0, dims, 1e-6, positions.cuda(),
                                     kc2, vc2, torch.float32, window=W)
    kb, vb = kc.bfloat16().cuda(), vc.bfloat16().cuda()
    out = nops.draft_block_attention(qkv.bfloat16().cuda(), qn.cuda(), kn.cuda(), inv.cuda(), 1.0, dims, 1e-6,
                                     positions.cuda(), kb, vb, torch.bfloat16, window=W)
    rel = (out.float() - ref).norm() / ref.norm()
    assert rel < 2e-2
    nops.check()


@pytest.mark.gpu
def test_native_draft_select(nops):
    for seed in range(4):
        feats, cand, unary, pred, succ = _selector_case(V=5000, rank=256, rows=16, C=16, seed=seed)
        ids = nops.draft_select(feats.cuda(), cand.cuda(), unary.cuda(), torch.tensor([7]).cuda(), pred.cuda(),
                                succ.cuda()).cpu()
        ref, _ = R.greedy_select(feats, cand, unary, 7, pred, succ)
        # fp32 device sums against the fp64 oracle: each choice must be the oracle's best along the
        # device's own path, up to fp32 rounding
        prev = 7
        for i in range(1, 16):
            c = cand[i]
            sc = unary[i].double() + (pred[prev].double() * feats[i].double() * succ[c].double()).sum(-1)
            j = int((c == int(ids[i - 1])).nonzero())
            assert sc[j] >= sc.max() - 1e-3 * (1 + sc.abs().max())
            prev = int(ids[i - 1])
        if ids.tolist() != ref.tolist():
            pytest.fail(f"seed {seed}: device path {ids.tolist()} differs from fp64 path {ref.tolist()}")
    nops.check()


@pytest.mark.gpu
def test_native_window_drafter_speculative_equals_greedy(nops):
    from qwen38_b200.checkpoint import random_target_source
    from qwen38_b200.config import tiny_model_config
    cfg = tiny_model_config()
    rt = RuntimeConfig(max_context=1024, prefill_chunk=64, gdn_chunk=64)
    tgt = HybridTarget(cfg, random_target_source(cfg, 0), rt, device="cuda", dtype=torch.bfloat16, ops=nops)
    wcfg = tiny_window_drafter_config()
    dr = WindowDrafter(wcfg, random_window_drafter_source(wcfg, cfg.vocab_size), tgt)
    prompt = torch.randint(0, cfg.vocab_size, (200,), generator=torch.Generator().manual_seed(0)).tolist()
    gold = greedy_reference(tgt, prompt, 40)
    res = SpecRuntime(tgt, dr, verifier_rows=wcfg.block_rows).generate(prompt, 40, gold_check=gold)
    assert res["tokens"] == gold
    nops.check()
