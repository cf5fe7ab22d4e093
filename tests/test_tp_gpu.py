"""Tensor parallel on GPUs (one process per GPU): at TP2 the native runtime's speculative output
equals its own greedy decode on full-width layer shapes, with the GEMM kernels that carry the
all-reduce (pushed from the GEMM, reduced in the next norm), with the separate peer-memory
collectives and with NCCL; the pushed all-reduce adds the same bits on both ranks as GEMM -> peer
all-reduce -> add.  Skipped with fewer
than two GPUs."""
import os

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs two CUDA devices", allow_module_level=True)

import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _rdv():
    """File rendezvous (no TCP port to race for between consecutive spawned groups)."""
    import tempfile
    fd, path = tempfile.mkstemp(prefix="q38_rdv_")
    os.close(fd)
    os.unlink(path)
    return path


def _init(rank, world, rdv):
    import datetime
    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{rdv}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))


def _worker(rank, world, rdv, q, mode):
    if mode == "fused":
        os.environ["Q38_PREFILL_AR"] = "1"       # also run the (opt-in) fused prefill all-reduce
        os.environ["Q38_NVLS"] = "1"             # and the (opt-in) multicast push
    _init(rank, world, rdv)
    try:
        from qwen38_b200.checkpoint import random_drafter_source, random_target_source
        from qwen38_b200.config import FULL, LINEAR, DrafterConfig, ModelConfig, RuntimeConfig
        from qwen38_b200.models.drafter import BlockDrafter
        from qwen38_b200.models.target import HybridTarget
        from qwen38_b200.ops.native import NativeOps
        from qwen38_b200.parallel.comm import make_comm
        from qwen38_b200.spec.engine import PinnedAcceptance, SpecRuntime, greedy_reference
        cfg = ModelConfig(num_hidden_layers=4, layer_types=[LINEAR, LINEAR, LINEAR, FULL])
        dcfg = DrafterConfig(num_hidden_layers=1, taps=[1, 3])
        ops = NativeOps(device=f"cuda:{rank}", max_keys=2048)
        tgt = HybridTarget(cfg, random_target_source(cfg, 0), RuntimeConfig(max_context=1024, prefill_chunk=256),
                           device=f"cuda:{rank}", dtype=torch.bfloat16, ops=ops,
                           comm=make_comm(2, device=f"cuda:{rank}", hidden=cfg.hidden_size, peer=(mode != "nccl"),
                                          fused=(mode == "fused"), prefill_rows=256 if mode == "fused" else 0))
        os.environ.pop("Q38_PREFILL_AR", None)
        dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, 1), tgt)
        prompt = torch.randint(0, cfg.vocab_size, (300,), generator=torch.Generator().manual_seed(2)).tolist()
        gold = greedy_reference(tgt, prompt, 24)
        res = SpecRuntime(tgt, dr, verifier_rows=16).generate(prompt, 24, gold_check=gold,
                                                              pinned=PinnedAcceptance(gold, seed=0, mean_accepted=6))
        ops.check()
        if hasattr(tgt.comm, "check"):
            tgt.comm.check()
        q.put((rank, gold, res["tokens"], None))
        dr.release_graphs()             # graphs hold NCCL work: release before teardown
        tgt.release_graphs()
    except BaseException as e:
        q.put((rank, None, None, repr(e)))
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["fused", "peer", "nccl"])
def test_tp2_native_speculative_equals_greedy(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rdv = _rdv()
    procs = [ctx.Process(target=_worker, args=(r, 2, rdv, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        out = [q.get(timeout=600) for _ in procs]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    for rank, gold, spec, err in out:
        assert err is None, err
        assert spec == gold
    assert out[0][1] == out[1][1]          # both ranks agree on every token


def _kernel_worker(rank, world, rdv, q):
    _init(rank, world, rdv)
    comms = []
    try:
        from qwen38_b200.ops.native import NativeOps
        from qwen38_b200.parallel.symm import SymmComm
        ops = NativeOps(device=f"cuda:{rank}")
        H = 5120
        fused, plain = SymmComm(f"cuda:{rank}", H, fused=True), SymmComm(f"cuda:{rank}", H, fused=False)
        comms = [fused, plain]
        res = []
        for T, K in ((1, 3072), (16, 8704), (32, 3072)):
            g = torch.Generator(device="cuda").manual_seed(100 * T + rank)      # rank-local operands
            x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
            w = ops.prepare_weight((torch.randn(H, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16))
            g0 = torch.Generator(device="cuda").manual_seed(T)                  # shared residual
            r0 = torch.randn(T, H, generator=g0, device="cuda")
            a = r0.clone()
            for _ in range(3):                                                  # epochs advance
                a.copy_(r0)
                ops.rms_norm_ar(a, None, 1e-6, torch.bfloat16, fused, ops.linear_push(x, w, fused))
            s, part = plain.slot_out(T, H)
            ops.linear(x, w, out=part)
            b = r0.clone()
            plain.reduce_slot_add(s, b)
            ref = ops.linear(x, w, out_dtype=torch.float32)
            dist.all_reduce(ref)
            torch.cuda.synchronize()
            res.append((T, bool(torch.equal(a, b)), ((a - (r0 + ref)).abs().max().item()), a.cpu()))
        ops.check()
        fused.check()
        plain.check()
        q.put((rank, res, None))
    except BaseException as e:
        q.put((rank, None, repr(e)))
    finally:
        torch.cuda.synchronize()
        for c in comms:
            c.close()
        dist.destroy_process_group()


def test_tp2_fused_gemm_allreduce_bits():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rdv = _rdv()
    procs = [ctx.Process(target=_kernel_worker, args=(r, 2, rdv, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        out = sorted([q.get(timeout=600) for _ in procs], key=lambda o: o[0])
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    for rank, res, err in out:
        assert err is None, err
        for T, same, maxdiff, _ in res:
            assert same, f"rank {rank} T={T}: fused and separate all-reduce differ"
            assert maxdiff < 1e-3
    for (T0, _, _, a0), (T1, _, _, a1) in zip(out[0][1], out[1][1]):
        assert torch.equal(a0, a1)             # replicated residual: identical bits on both ranks


def _prefill_worker(rank, world, rdv, q):
    os.environ["Q38_PREFILL_AR"] = "1"           # the fused prefill all-reduce is opt in
    os.environ["Q38_NVLS"] = "1"                 # (it needs the multicast receive areas)
    _init(rank, world, rdv)
    tgt = None
    try:
        from qwen38_b200.checkpoint import random_target_source
        from qwen38_b200.config import FULL, LINEAR, ModelConfig, RuntimeConfig
        from qwen38_b200.models.target import HybridTarget
        from qwen38_b200.ops.native import NativeOps
        from qwen38_b200.parallel.comm import make_comm
        cfg = ModelConfig(num_hidden_layers=4, layer_types=[LINEAR, LINEAR, LINEAR, FULL])
        ops = NativeOps(device=f"cuda:{rank}", max_keys=2048)
        comm = make_comm(2, device=f"cuda:{rank}", hidden=cfg.hidden_size, peer=True, fused=True, prefill_rows=512)
        tgt = HybridTarget(cfg, random_target_source(cfg, 0), RuntimeConfig(max_context=2048, prefill_chunk=512),
                           device=f"cuda:{rank}", dtype=torch.bfloat16, ops=ops, comm=comm, max_slots=1)
        prompt = torch.randint(0, cfg.vocab_size, (900,), generator=torch.Generator().manual_seed(4)).cuda()
        fused_on = comm._pf is not None

        def run():
            seq = tgt.new_sequence()
            nxt, feats = tgt.prefill(seq, prompt, taps=(1, 3))
            out = (int(nxt.item()), feats.float().cpu(), tgt.rec[seq.slot].clone().cpu())
            tgt.release(seq)
            return out
        a, b = run(), run()
        saved, comm._pf = comm._pf, None            # the NCCL all-reduce path
        c = run()
        comm._pf = saved
        ops.check()
        comm.check()
        q.put((rank, fused_on, a, b, c, None))
    except BaseException as e:
        q.put((rank, None, None, None, None, repr(e)))
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


def test_tp2_fused_prefill_allreduce():
    """The fused prefill all-reduce (reduce-scatter GEMM + owner reduce + multicast broadcast) is
    deterministic, leaves identical residuals (taps, GDN state) on both ranks, and agrees with the
    NCCL all-reduce path to fp32 rounding.  Chunks of 512 and 388 rows (a ragged last tile)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rdv = _rdv()
    procs = [ctx.Process(target=_prefill_worker, args=(r, 2, rdv, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        out = sorted([q.get(timeout=600) for _ in procs], key=lambda o: o[0])
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    for rank, fused_on, a, b, c, err in out:
        assert err is None, err
        if not fused_on:
            pytest.skip("no NVSwitch multicast on this system: the fused prefill all-reduce is off")
        assert a[0] == b[0] and torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])      # deterministic
        assert ((a[1] - c[1]).norm() / c[1].norm()).item() < 2e-2                          # vs NCCL
        assert ((a[2] - c[2]).norm() / c[2].norm()).item() < 2e-2
    assert torch.equal(out[0][2][1], out[1][2][1])        # replicated residual: same taps on both ranks
