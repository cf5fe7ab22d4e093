"""Numerics of the sm_100a kernels against the plain-PyTorch fp32 definitions of the same ops,
plus the batch-invariance property the speculative runtime relies on (a verify row is
bit-identical to the same row run alone)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from qwen38_b200.ops import TorchOps, torch_ref as R  # noqa: E402
from qwen38_b200.ops.native import NativeOps  # noqa: E402

DEV = "cuda"


@pytest.fixture(scope="module")
def nops():
    return NativeOps()


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("T", [1, 3, 16, 32, 77, 300])
@pytest.mark.parametrize("N,K", [(1000, 640), (5120, 6144), (384, 17408)])
def test_linear_matches_fp32(nops, T, N, K):
    x, w = _bf(T, K, seed=1), _bf(N, K, scale=0.02, seed=2)
    ref = x.float() @ w.float().t()
    y = nops.linear(x, w)
    assert _rel(y, ref) < 8e-3
    y32 = nops.linear(x, w, out_dtype=torch.float32)
    assert _rel(y32, ref) < 1e-4
    nops.check()


@pytest.mark.parametrize("T", [1, 16, 200])
def test_linear_residual_and_swiglu(nops, T):
    K, I = 1024, 768
    x, wd = _bf(T, K, seed=3), _bf(512, K, scale=0.02, seed=4)
    res = torch.randn(T, 512, device=DEV)
    ref = res + x.float() @ wd.float().t()
    nops.linear_residual(x, wd, res)
    assert _rel(res, ref) < 1e-4
    wgu = _bf(2 * I, K, scale=0.02, seed=5)
    y = nops.linear_swiglu(x, wgu, 64)
    r = (x.float() @ wgu.float().t()).view(T, -1, 2, 64)
    ref = (torch.nn.functional.silu(r[:, :, 0]) * r[:, :, 1]).reshape(T, -1)
    assert _rel(y, ref) < 8e-3
    nops.check()


def test_batch_invariance_of_skinny_gemm(nops):
    K, N = 5120, 17408
    x, w = _bf(16, K, seed=6), _bf(N, K, scale=0.02, seed=7)
    full = nops.linear(x, w, out_dtype=torch.float32)
    for t in (0, 5, 15):
        one = nops.linear(x[t:t + 1], w, out_dtype=torch.float32)
        assert torch.equal(one[0], full[t])
    nops.check()


@pytest.mark.parametrize("T", [40, 64])
def test_packed_rows_equal_single_request_rows(nops, T):
    """A packed verify of up to 64 rows stays on the weight-streaming GEMM (two 32-token tiles):
    each request's 16 rows get the bits they get alone, for the plain, residual-add and deferred
    split-K epilogues, and the normalised rows match too."""
    K, N = 5120, 5120
    x, tw = _bf(T, K, seed=16), nops.prepare_weight(_bf(N, K, scale=0.02, seed=17))
    w = torch.rand(N, device=DEV) + 0.5
    full = nops.linear(x, tw, out_dtype=torch.float32)
    base = torch.randn(T, N, device=DEV)
    r_full = base.clone()
    nops.linear_residual(x, tw, r_full)
    r_split = base.clone()
    S = nops.linear_split(x, tw, r_split)
    n_split = nops.rms_norm_split(r_split, w, 1e-6, torch.bfloat16, S) if S > 1 else None
    for o0 in range(0, T - 15, 16):
        sl = slice(o0, o0 + 16)
        assert torch.equal(nops.linear(x[sl], tw, out_dtype=torch.float32), full[sl])
        r_one = base[sl].clone()
        nops.linear_residual(x[sl], tw, r_one)
        assert torch.equal(r_one, r_full[sl]) and torch.equal(r_one, r_split[sl])
        if n_split is not None:
            assert torch.equal(nops.rms_norm(r_one, w, 1e-6, torch.bfloat16), n_split[sl])
    nops.check()


@pytest.mark.parametrize("T", [1, 16])
def test_lm_head_argmax(nops, T):
    V, K = 50000, 1024
    x, w = _bf(T, K, seed=8), _bf(V, K, scale=0.05, seed=9)
    val, idx = nops.lm_head_argmax(x, w, 100)
    logits = x.float() @ w.float().t()
    ref_v, ref_i = logits.max(-1)
    assert torch.allclose(val, ref_v, rtol=1e-3, atol=1e-3)
    # ties/near-ties aside, the chosen logit must be the max up to accumulation error
    chosen = logits.gather(1, (idx - 100)[:, None])[:, 0]
    assert torch.all(chosen >= ref_v - 1e-2)
    nops.check()


def test_rms_norm_and_embedding(nops):
    x = torch.randn(7, 5120, device=DEV)
    w = torch.rand(5120, device=DEV) + 0.5
    y = nops.rms_norm(x, w, 1e-6, torch.bfloat16)
    assert _rel(y, TorchOps().rms_norm(x, w, 1e-6, torch.float32)) < 5e-3
    table = _bf(1000, 256, seed=10)
    ids = torch.tensor([3, 999, 0, 3], device=DEV)
    assert torch.equal(nops.embedding(ids, table), table[ids].float())


def _gdn_case(T, nk=4, nv=12, D=128, seed=11):
    g = torch.Generator(device=DEV).manual_seed(seed)
    C = 2 * nk * D + nv * D
    width = C + nv * D + 2 * nv
    proj = (torch.randn(T, width, generator=g, device=DEV)).to(torch.bfloat16)
    window = (torch.randn(3, C, generator=g, device=DEV)).to(torch.bfloat16)
    state = torch.randn(nv, D, D, generator=g, device=DEV) * 0.1
    conv_w = torch.rand(C, 4, generator=g, device=DEV) - 0.5
    A_log = torch.log(1 + 15 * torch.rand(nv, generator=g, device=DEV))
    dt = 1 + 0.1 * torch.randn(nv, generator=g, device=DEV)
    norm_w = 1 + 0.1 * torch.randn(D, generator=g, device=DEV)
    return proj, window, state, conv_w, A_log, dt, norm_w, (nk, nv, D, D)


@pytest.mark.parametrize("T", [1, 4, 16, 40])
def test_gdn_verify_matches_reference(nops, T):
    proj, window, state, conv_w, A_log, dt, norm_w, dims = _gdn_case(T)
    ref = TorchOps().gdn_verify(proj.float(), window.float(), state, conv_w, A_log, dt, norm_w, 1e-6, dims,
                                torch.float32)
    out = nops.gdn_verify(proj, window, state, conv_w, A_log, dt, norm_w, 1e-6, dims, torch.bfloat16)
    assert _rel(out, ref) < 1e-2
    nops.check()


def test_gdn_verify_rows_equal_sequential_commit_decode(nops):
    """Row t of a verify == decode after committing rows < t (bitwise), and commit == replay."""
    T = 8
    proj, window, state, conv_w, A_log, dt, norm_w, dims = _gdn_case(T, seed=12)
    out = nops.gdn_verify(proj, window, state, conv_w, A_log, dt, norm_w, 1e-6, dims, torch.bfloat16)
    st, win = state.clone(), window.clone()
    for t in range(T):
        one = nops.gdn_verify(proj[t:t + 1], win, st, conv_w, A_log, dt, norm_w, 1e-6, dims, torch.bfloat16)
        assert torch.equal(one[0], out[t])
        nops.gdn_commit(proj[t:t + 1], 1, win, st, conv_w, A_log, dt, dims)
    st2, win2 = state.clone(), window.clone()
    nops.gdn_commit(proj, T, win2, st2, conv_w, A_log, dt, dims)
    assert torch.equal(st, st2) and torch.equal(win, win2)
    ref_st, ref_win = state.clone(), window.float().clone()
    TorchOps().gdn_commit(proj.float(), T, ref_win, ref_st, conv_w, A_log, dt, dims)
    assert _rel(st2, ref_st) < 1e-3
    nops.check()


def test_gdn_prefill_matches_chunked_reference(nops):
    T = 300
    proj, window, state, conv_w, A_log, dt, norm_w, dims = _gdn_case(T, seed=13)
    ref_st, ref_win = state.clone(), window.float().clone()
    ref = TorchOps().gdn_prefill(proj.float(), ref_win, ref_st, conv_w, A_log, dt, norm_w, 1e-6, dims, 64,
                                 torch.float32)
    st, win = state.clone(), window.clone()
    nops.chunked_prefill = False            # the sequential prefill kernel
    out = nops.gdn_prefill(proj, win, st, conv_w, A_log, dt, norm_w, 1e-6, dims, 64, torch.bfloat16)
    nops.chunked_prefill = True
    assert _rel(out, ref) < 1e-2
    assert _rel(st, ref_st) < 1e-3
    assert torch.equal(win, ref_win.to(torch.bfloat16))
    nops.check()


def _attn_case(T, pos0, H=6, Hkv=1, D=256, bs=16, seed=14):
    g = torch.Generator(device=DEV).manual_seed(seed)
    nblocks = (pos0 + T + bs - 1) // bs + 4
    kc = (torch.randn(nblocks, bs, Hkv, D, generator=g, device=DEV) * 0.5).to(torch.bfloat16)
    vc = torch.randn(nblocks, bs, Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    bt = torch.randperm(nblocks, generator=torch.Generator().manual_seed(seed)).to(torch.int32).to(DEV)
    proj = torch.randn(T, 2 * H * D + 2 * Hkv * D, generator=g, device=DEV).to(torch.bfloat16)
    qn = 1 + 0.1 * torch.randn(D, generator=g, device=DEV)
    kn = 1 + 0.1 * torch.randn(D, generator=g, device=DEV)
    rd = 64
    inv = 1.0 / (1e7 ** (torch.arange(0, rd, 2, dtype=torch.float32, device=DEV) / rd))
    pos = torch.arange(pos0, pos0 + T, device=DEV, dtype=torch.int32)
    return proj, qn, kn, inv, rd, (H, Hkv, D), pos, kc, vc, bt, bs


@pytest.mark.parametrize("T,pos0", [(1, 0), (16, 100), (16, 4000), (5, 700)])
def test_attention_prep_and_decode(nops, T, pos0):
    proj, qn, kn, inv, rd, dims, pos, kc, vc, bt, bs = _attn_case(T, pos0)
    kc2, vc2 = kc.clone(), vc.clone()
    tops = TorchOps()
    q_ref, gate = tops.attn_prep(proj.float(), qn, kn, inv, 1.0, rd, dims, 1e-6, pos, kc2, vc2, bt, bs)
    q, gate_n = nops.attn_prep(proj, qn, kn, inv, 1.0, rd, dims, 1e-6, pos, kc, vc, bt, bs)
    assert _rel(q, q_ref) < 1e-2
    assert _rel(kc.float(), kc2.float()) < 1e-2
    ref = tops.attn_decode(q_ref.float(), gate.float(), kc2.float(), vc2.float(), bt, pos, bs, torch.float32)
    out = nops.attn_decode(q, gate_n, kc, vc, bt, pos, bs, torch.bfloat16)
    assert _rel(out, ref) < 2e-2
    # batch invariance: row t alone == row t of the block
    for t in (0, T - 1):
        one = nops.attn_decode(q[t:t + 1], gate_n[t:t + 1], kc, vc, bt, pos[t:t + 1], bs, torch.bfloat16)
        assert torch.equal(one[0], out[t])
    nops.check()


@pytest.mark.parametrize("T,pos0", [(16, 8180), (16, 9000), (5, 65530), (16, 70000)])
def test_attention_decode_long_context_groups(nops, T, pos0):
    """Across the key-group tiers (1, 4 and 8 chunks per CTA): numerics against the fp32 reference
    and the same bits for a row alone as inside the block."""
    proj, qn, kn, inv, rd, dims, pos, kc, vc, bt, bs = _attn_case(T, pos0)
    kc2, vc2 = kc.clone(), vc.clone()
    tops = TorchOps()
    q_ref, gate = tops.attn_prep(proj.float(), qn, kn, inv, 1.0, rd, dims, 1e-6, pos, kc2, vc2, bt, bs)
    q, gate_n = nops.attn_prep(proj, qn, kn, inv, 1.0, rd, dims, 1e-6, pos, kc, vc, bt, bs)
    ref = tops.attn_decode(q_ref.float(), gate.float(), kc2.float(), vc2.float(), bt, pos, bs, torch.float32)
    out = nops.attn_decode(q, gate_n, kc, vc, bt, pos, bs, torch.bfloat16)
    assert _rel(out, ref) < 2e-2
    for t in (0, T - 1):
        one = nops.attn_decode(q[t:t + 1], gate_n[t:t + 1], kc, vc, bt, pos[t:t + 1], bs, torch.bfloat16)
        assert torch.equal(one[0], out[t])
    nops.check()


@pytest.mark.parametrize("T,pos0,H,Hkv", [(40, 0, 6, 1), (300, 1000, 6, 1), (2048, 2048, 6, 1), (77, 5, 3, 1),
                                           (64, 64, 4, 2)])
def test_attention_prefill_kernel(nops, T, pos0, H, Hkv):
    """Hand-written prefill flash attention (paged, causal, GQA, sigmoid gate) vs the fp32 reference."""
    proj, qn, kn, inv, rd, dims, pos, kc, vc, bt, bs = _attn_case(T, pos0, H=H, Hkv=Hkv)
    kc2, vc2 = kc.clone(), vc.clone()
    tops = TorchOps()
    q_ref, gate = tops.attn_prep(proj.float(), qn, kn, inv, 1.0, rd, dims, 1e-6, pos, kc2, vc2, bt, bs)
    q, gate_n = nops.attn_prep(proj, qn, kn, inv, 1.0, rd, dims, 1e-6, pos, kc, vc, bt, bs)
    ref = tops.attn_decode(q_ref.float(), gate.float(), kc2.float(), vc2.float(), bt, pos, bs, torch.float32)
    out = nops.attn_prefill(q, gate_n, kc, vc, bt, pos, bs, torch.bfloat16)
    assert _rel(out, ref) < 2e-2
    nops.check()


def test_lm_head_gumbel_sampling(nops):
    """Gumbel-max sampling in the LM-head argmax epilogue: the same samples as the fp32 reference
    with the same noise (up to bf16 logit rounding), greedy rows unchanged, vocab offsets respected."""
    from qwen38_b200.ops import torch_ref as R
    T, V, K = 16, 5000, 512
    g = torch.Generator(device=DEV).manual_seed(21)
    x = torch.randn(T, K, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(V, K, generator=g, device=DEV) * 0.1).to(torch.bfloat16)
    scale = torch.tensor([0.0 if t % 4 == 0 else 1.0 / (0.5 + 0.1 * t) for t in range(T)], device=DEV)
    key = torch.tensor([R.sample_key(99, 1000 + t) for t in range(T)], device=DEV)
    _, idx = nops.lm_head_argmax(x, w, 7000, (scale, key))
    _, ref = TorchOps().lm_head_argmax(x.float(), w.float(), 7000, (scale, key))
    _, greedy = nops.lm_head_argmax(x, w, 7000)
    nops.check()
    assert int((idx == ref).sum()) >= T - 1
    assert torch.equal(idx[::4], greedy[::4])
    assert bool((idx >= 7000).all() and (idx < 7000 + V).all())


def test_markov_select(nops):
    P, V, Rk = 5, 3000, 64
    g = torch.Generator(device=DEV).manual_seed(15)
    logits = torch.randn(P, V, generator=g, device=DEV)
    pred = (torch.randn(V, Rk, generator=g, device=DEV) * 0.3).to(torch.bfloat16)
    succ = (torch.randn(V, Rk, generator=g, device=DEV) * 0.3).to(torch.bfloat16)
    anchor = torch.tensor([17], device=DEV)
    out = nops.markov_select(logits, anchor, pred, succ).tolist()
    ref = R.markov_select(logits.cpu(), 17, pred.cpu(), succ.cpu())
    assert out == ref


@pytest.mark.parametrize("P,V,Rk", [(15, 151936, 256), (15, 18992, 256), (3, 1000, 64)])
def test_fused_markov_equals_per_step_kernels(nops, P, V, Rk):
    """The one-launch selector (grid barrier per step) picks exactly what the two-launch per-step
    kernels pick (same dot-product order), call after call."""
    g = torch.Generator(device=DEV).manual_seed(P + V)
    logits = torch.randn(P, V, generator=g, device=DEV) * 2
    pred = (torch.randn(V + 77, Rk, generator=g, device=DEV) * 0.3).to(torch.bfloat16)
    succ = (torch.randn(V, Rk, generator=g, device=DEV) * 0.3).to(torch.bfloat16)
    for anchor_id in (5, V + 70, 12345 % V):
        anchor = torch.tensor([anchor_id], device=DEV)
        fused = nops.markov_select(logits, anchor, pred, succ, vocab_offset=3)
        prev = anchor.clone()
        steps = torch.empty(P, dtype=torch.int64, device=DEV)
        val = torch.empty(1, device=DEV)
        for i in range(P):
            nops.C.markov_step(logits[i].contiguous(), pred, succ, prev, steps[i:i + 1], val, nops.amax_val,
                               nops.amax_idx, 3, True)
        torch.cuda.synchronize()
        nops.check()
        assert fused.tolist() == steps.tolist()


@pytest.mark.parametrize("T", [64, 300, 2048])
def test_gdn_chunked_prefill_matches_reference(nops, T):
    proj, window, state, conv_w, A_log, dt, norm_w, dims = _gdn_case(T, seed=21)
    ref_st, ref_win = state.clone(), window.float().clone()
    ref = TorchOps().gdn_prefill(proj.float(), ref_win, ref_st, conv_w, A_log, dt, norm_w, 1e-6, dims, 64,
                                 torch.float32)
    st, win = state.clone(), window.clone()
    nops.chunked_prefill = True
    out = nops.gdn_prefill(proj, win, st, conv_w, A_log, dt, norm_w, 1e-6, dims, 64, torch.bfloat16)
    assert _rel(out, ref) < 3e-2
    assert _rel(st, ref_st) < 3e-2
    assert torch.equal(win, ref_win.to(torch.bfloat16))
    # the sequential kernel agrees too (two independent implementations)
    st2, win2 = state.clone(), window.clone()
    nops.chunked_prefill = False
    out2 = nops.gdn_prefill(proj, win2, st2, conv_w, A_log, dt, norm_w, 1e-6, dims, 64, torch.bfloat16)
    nops.chunked_prefill = True
    assert _rel(out, out2) < 3e-2
    nops.check()


@pytest.mark.parametrize("T,N,K", [(16, 5120, 17408), (16, 5120, 6144), (3, 384, 17408), (32, 1000, 640)])
def test_cluster_splitk_bits_equal_global_fixup(nops, T, N, K):
    """The skinny GEMM reduces split-K partials inside a thread-block cluster (DSMEM); the
    allocation-free entry point still reduces them through global memory and the last-arriving
    CTA.  Both add the same partials in the same split order, so the fp32 results are identical."""
    import ctypes

    from qwen38_b200.ops.build import so_path
    from qwen38_b200.ops.noalloc import EPI_ADD_F32, EPI_F32, bind
    fn, status = bind(so_path())
    x, tw = _bf(T, K, seed=7), nops.prepare_weight(_bf(N, K, scale=0.02, seed=8))
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    y_cluster = nops.linear(x, tw, out_dtype=torch.float32)
    y_global = torch.empty(T, N, device=DEV)
    assert fn(x.data_ptr(), T, K, tw.t.data_ptr(), N, y_global.data_ptr(), N, EPI_F32, st) == 0
    torch.cuda.synchronize()
    assert status() == 0
    assert torch.equal(y_cluster, y_global)
    base = torch.randn(T, N, device=DEV)
    r1, r2 = base.clone(), base.clone()
    nops.linear_residual(x, tw, r1)
    assert fn(x.data_ptr(), T, K, tw.t.data_ptr(), N, r2.data_ptr(), N, EPI_ADD_F32, st) == 0
    torch.cuda.synchronize()
    assert torch.equal(r1, r2)
    nops.check()


@pytest.mark.parametrize("T,N,K", [(16, 5120, 17408), (16, 5120, 6144), (1, 5120, 6144), (3, 384, 17408),
                                   (32, 1000, 640)])
def test_deferred_splitk_equals_in_gemm_fixup(nops, T, N, K):
    """The split GEMM stores its K slices and the next norm adds them in split order, then the
    residual: the residual and the normalised rows are bit-identical to the GEMM's own fix-up
    followed by the plain norm, and the weight-less completion leaves the same residual."""
    x, tw = _bf(T, K, seed=11), nops.prepare_weight(_bf(N, K, scale=0.02, seed=12))
    w = torch.rand(N, device=DEV) + 0.5
    base = torch.randn(T, N, device=DEV)
    r_ref, r_def, r_set = base.clone(), base.clone(), base.clone()
    nops.linear_residual(x, tw, r_ref)
    n_ref = nops.rms_norm(r_ref, w, 1e-6, torch.bfloat16)
    S = nops.linear_split(x, tw, r_def)
    assert S == nops.C.swap_splits(N, K)
    n_def = nops.rms_norm_split(r_def, w, 1e-6, torch.bfloat16, S) if S > 1 else nops.rms_norm(r_def, w, 1e-6,
                                                                                             torch.bfloat16)
    S2 = nops.linear_split(x, tw, r_set)
    if S2 > 1:
        assert nops.rms_norm_split(r_set, None, 1e-6, torch.bfloat16, S2) is None
    torch.cuda.synchronize()
    nops.check()
    assert torch.equal(r_ref, r_def) and torch.equal(r_ref, r_set)
    assert torch.equal(n_ref, n_def)


@pytest.fixture(scope="module")
def mxops():
    return NativeOps(weight_format="mxfp8")


def _mx_bf(N, K, seed):
    """An MXFP8 weight (its exact bf16 expansion) with every finite e4m3 byte pattern planted in row 0
    (31 per 32-element block, the block's last element 448 so its scale stays the OCP choice)."""
    from qwen38_b200.checkpoint import dequant_mxfp8, quant_mxfp8
    w = torch.randn(N, K, generator=torch.Generator(device=DEV).manual_seed(seed), device=DEV) * 0.02
    q, se = quant_mxfp8(w)
    b = torch.arange(256, device=DEV, dtype=torch.int32)
    b = b[(b & 0x7F) != 0x7F].to(torch.uint8)
    row = q.view(torch.uint8)[0]
    for blk in range(min(K // 32, -(-b.numel() // 31))):
        part = b[blk * 31:(blk + 1) * 31]
        row[blk * 32:blk * 32 + part.numel()] = part
        row[blk * 32 + 31] = 0x7E
    return dequant_mxfp8(q, se).to(torch.bfloat16)


@pytest.mark.parametrize("T", [1, 16, 40, 64])
@pytest.mark.parametrize("N,K", [(5120, 17408), (2064, 5120), (1000, 640), (384, 6144)])
def test_mx_gemm_bits_equal_bf16_weight(nops, mxops, T, N, K):
    """The MXFP8 weight-streaming GEMM expands each e4m3 tile to the exact bf16 weight in shared
    memory and shares the bf16 kernel's MMA order, split-K plan and epilogues: every epilogue's
    output has the same bits as the bf16 GEMM over the dequantised weight."""
    from qwen38_b200.ops.native import MXWeight
    wb = _mx_bf(N, K, 21)
    mw, tw = mxops.prepare_weight(wb), nops.prepare_weight(wb)
    assert isinstance(mw, MXWeight)
    x = _bf(T, K, seed=22)
    assert torch.equal(mxops.linear(x, mw, out_dtype=torch.float32), nops.linear(x, tw, out_dtype=torch.float32))
    assert torch.equal(mxops.linear(x, mw), nops.linear(x, tw))
    base = torch.randn(T, N, device=DEV)
    r_mx, r_bf = base.clone(), base.clone()
    mxops.linear_residual(x, mw, r_mx)
    nops.linear_residual(x, tw, r_bf)
    assert torch.equal(r_mx, r_bf)
    r_mx, r_bf = base.clone(), base.clone()
    S = mxops.linear_split(x, mw, r_mx)
    assert S == nops.linear_split(x, tw, r_bf)
    if S > 1:
        mxops.rms_norm_split(r_mx, None, 1e-6, torch.bfloat16, S)
        nops.rms_norm_split(r_bf, None, 1e-6, torch.bfloat16, S)
    assert torch.equal(r_mx, r_bf)
    if N % 128 == 0:
        assert torch.equal(mxops.linear_swiglu(x, mw, 64), nops.linear_swiglu(x, tw, 64))
    torch.cuda.synchronize()
    mxops.check()
    nops.check()


def test_mx_prefill_rows_use_the_bf16_expansion(nops, mxops):
    wb = _mx_bf(1024, 2048, 23)
    mw, tw = mxops.prepare_weight(wb), nops.prepare_weight(wb)
    x = _bf(300, 2048, seed=24)
    assert torch.equal(mxops.linear(x, mw, out_dtype=torch.float32), nops.linear(x, tw, out_dtype=torch.float32))
    mxops.check()


def test_gdn_chunked_prefill_state_error_does_not_compound(nops):
    """The bench's prefill shape (48 value heads, 16 key heads, 4,096 rows = 64 chunks): the carried
    fp32 state after 1,024 and after 4,096 rows, against the fp32 reference.  The chunked kernel's
    bf16 operands give a bounded per-chunk error; this pins that it does not grow with the number
    of chunks the state is carried through (max over heads of the per-head relative error)."""
    errs = {}
    for T in (1024, 4096):
        proj, window, state, conv_w, A_log, dt, norm_w, dims = _gdn_case(T, nk=16, nv=48, seed=31)
        ref_st = state.clone()
        TorchOps().gdn_prefill(proj.float(), window.float().clone(), ref_st, conv_w, A_log, dt, norm_w, 1e-6, dims,
                               64, torch.float32)
        st = state.clone()
        nops.chunked_prefill = True
        nops.gdn_prefill(proj, window.clone(), st, conv_w, A_log, dt, norm_w, 1e-6, dims, 64, torch.bfloat16)
        per_head = ((st - ref_st).flatten(1).norm(dim=1) / ref_st.flatten(1).norm(dim=1)).max().item()
        errs[T] = per_head
    nops.check()
    assert errs[4096] < 2e-2, errs
    assert errs[4096] < 1.5 * errs[1024] + 2e-3, errs
