"""Tensor parallel on CPU ranks (gloo, world size 2): the TP2 runtime reproduces the TP1
greedy output and speculative decoding stays token-exact (BASELINE config 1 at TP2)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qwen38_b200.checkpoint import random_drafter_source, random_target_source
        from qwen38_b200.config import RuntimeConfig, tiny_drafter_config, tiny_model_config
        from qwen38_b200.models.drafter import BlockDrafter
        from qwen38_b200.models.target import HybridTarget
        from qwen38_b200.parallel.comm import TorchComm
        from qwen38_b200.spec.engine import PinnedAcceptance, SpecRuntime, greedy_reference
        cfg, dcfg = tiny_model_config(), tiny_drafter_config()
        rt = RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16)
        prompt = torch.randint(0, cfg.vocab_size, (128,), generator=torch.Generator().manual_seed(0)).tolist()
        tgt = HybridTarget(cfg, random_target_source(cfg, 0), rt, comm=TorchComm())
        dr = BlockDrafter(dcfg, random_drafter_source(dcfg, cfg.vocab_size, 1), tgt)
        gold = greedy_reference(tgt, prompt, 32)
        res = SpecRuntime(tgt, dr, verifier_rows=4).generate(
            prompt, 32, gold_check=gold, pinned=PinnedAcceptance(gold, seed=0, mean_accepted=1))
        q.put((rank, gold, res["tokens"]))
    except BaseException as e:   # report instead of hanging the parent
        q.put((rank, repr(e), None))
    finally:
        dist.destroy_process_group()


def test_tp2_gloo_matches_tp1(tiny):
    from qwen38_b200.config import RuntimeConfig
    from qwen38_b200.models.target import HybridTarget
    tp1 = HybridTarget(tiny["cfg"], tiny["src"], RuntimeConfig(max_context=512, prefill_chunk=64, gdn_chunk=16))
    gold1 = tp1.greedy(torch.tensor(tiny["prompt"]), 32)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, gold, spec in out:
        assert spec is not None, gold
        assert spec == gold
        # TP2 sums two partials per element; agreement with TP1 is expected on this seed
        assert gold == gold1
