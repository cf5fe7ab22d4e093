"""Prefix reuse (BASELINE config 4 on the tiny shape): a request whose prefix matches an earlier
one restores KV blocks + GDN state + drafter history at the boundary and prefills only the
suffix; output, GDN state and logits equal a cold full prefill exactly."""
import torch

from qwen38_b200.config import RuntimeConfig
from qwen38_b200.models.drafter import BlockDrafter
from qwen38_b200.models.target import HybridTarget
from qwen38_b200.prefix.registry import KillSwitch, PrefixRegistry
from qwen38_b200.spec.engine import SpecRuntime, greedy_reference

RT = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)


def _prompts(tiny):
    g = torch.Generator().manual_seed(7)
    prefix = torch.randint(0, 4096, (128,), generator=g).tolist()
    a = prefix + torch.randint(0, 4096, (100,), generator=g).tolist()
    b = prefix + torch.randint(0, 4096, (90,), generator=g).tolist()
    return a, b


def test_prefix_reuse_is_exact(tiny):
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RT, max_slots=2)
    dr = BlockDrafter(tiny["dcfg"], tiny["dsrc"], tgt)
    a, b = _prompts(tiny)
    gold_b = greedy_reference(tgt, b, 24)
    # cold reference state after prefill of b
    seq = tgt.new_sequence()
    cold_next, _ = tgt.prefill(seq, torch.tensor(b))
    cold_rec = tgt.rec[seq.slot].clone()
    tgt.release(seq)

    reg = PrefixRegistry(tgt, budget_bytes=1 << 30, boundary=64)
    sr = SpecRuntime(tgt, dr, verifier_rows=4, prefix=reg)
    ra = sr.generate(a, 24)
    assert ra["reused_prefix"] == 0 and reg.stats["captures"] == 3        # boundaries 64, 128, 192
    rb = sr.generate(b, 24, gold_check=gold_b)
    assert rb["reused_prefix"] == 128 and rb["tokens"] == gold_b
    assert reg.stats["hits"] == 1

    # restored + suffix prefill reproduces the cold state bit for bit
    ck = reg.lookup(b)
    seq = reg.restore(ck, dr)
    warm_next, _ = tgt.prefill(seq, torch.tensor(b[128:]))
    assert int(warm_next) == int(cold_next)
    assert torch.equal(tgt.rec[seq.slot], cold_rec)
    tgt.release(seq)


def test_registry_budget_pins_and_kill_switch(tiny, tmp_path):
    tgt = HybridTarget(tiny["cfg"], tiny["src"], RT, max_slots=2)
    a, b = _prompts(tiny)
    reg = PrefixRegistry(tgt, budget_bytes=1 << 30, boundary=64)
    seq = tgt.new_sequence()
    tgt.prefill(seq, torch.tensor(a[:64]))
    ck1 = reg.capture(seq, a)
    tgt.prefill(seq, torch.tensor(a[64:128]))
    ck2 = reg.capture(seq, a)
    assert reg.lookup(b).pos == 128
    free_before = tgt.allocator.num_free
    tgt.release(seq)
    assert tgt.allocator.num_free == free_before          # blocks still held by the checkpoints
    reg.budget = ck2.nbytes                                 # room for one: the LRU entry goes
    reg.pin(ck2)
    reg._enforce_budget()
    assert ck1.key not in reg.entries and ck2.key in reg.entries
    reg.unpin(ck2)
    flag = tmp_path / "off"
    reg.kill = KillSwitch(str(flag), poll_s=0.0)
    assert reg.lookup(b) is not None
    flag.write_text("1")
    assert reg.lookup(b) is None and reg.export_stats()["disabled"]
    reg.clear()
    assert tgt.allocator.num_free == tgt.allocator.num_blocks


def _tp_rank(rank, port, q):
    import os
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        from qwen38_b200.checkpoint import random_drafter_source, random_target_source
        from qwen38_b200.config import tiny_drafter_config, tiny_model_config
        from qwen38_b200.parallel.comm import TorchComm
        cfg, dcfg = tiny_model_config(), tiny_drafter_config()
        tgt = HybridTarget(cfg, random_target_source(cfg, 0), RT, comm=TorchComm(), max_slots=2)
        dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, 1), tgt)
        a, b = _prompts(None)
        gold_b = greedy_reference(tgt, b, 24)
        seq = tgt.new_sequence()
        tgt.prefill(seq, torch.tensor(b))
        cold = tgt.rec[seq.slot].clone()
        tgt.release(seq)
        reg = PrefixRegistry(tgt, budget_bytes=1 << 30, boundary=64)
        sr = SpecRuntime(tgt, dr, verifier_rows=4, prefix=reg)
        sr.generate(a, 24)
        rb = sr.generate(b, 24, gold_check=gold_b)
        ck = reg.lookup(b)
        seq = reg.restore(ck, dr)
        tgt.prefill(seq, torch.tensor(b[ck.pos:]))
        exact = torch.equal(tgt.rec[seq.slot], cold)
        tgt.release(seq)
        q.put((rank, rb["reused_prefix"], rb["tokens"] == gold_b, exact))
    except BaseException as e:
        q.put((rank, repr(e), False, False))
    finally:
        dist.destroy_process_group()


def test_prefix_reuse_tp2_gloo():
    """BASELINE config 4 at TP2 (gloo ranks): the second request reuses the 128-token prefix on both
    ranks, stays token-exact, and each rank's restored + suffix GDN state equals its cold prefill."""
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, reused, exact_tokens, exact_state in out:
        assert reused == 128, reused
        assert exact_tokens and exact_state


def test_prefix_bench_tool_is_token_exact_and_reuses():
    """The prefix-reuse benchmark tool on the tiny shape (CPU): request B restores request A's
    boundary checkpoint, prefills only its new suffix and stays token-exact against greedy."""
    from qwen38_b200.utils.prefixbench import parse, run
    out = run(parse(["--model", "tiny", "--ctx", "256", "--reuse", "128", "--new-tokens", "16"]))
    assert out["token_exact"] and out["reused_prefix"] == 128
    assert out["registry"]["hits"] == 1 and out["registry"]["captures"] >= 1
