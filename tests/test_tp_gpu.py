"""Tensor parallel on GPUs (one process per GPU): at TP2 the native runtime's speculative output
equals its own greedy decode on full-width layer shapes, with the in-kernel peer-memory
collectives and with NCCL.  Skipped with fewer than two GPUs."""
import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs two CUDA devices", allow_module_level=True)

import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, mode):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from qwen38_b200.checkpoint import random_drafter_source, random_target_source
        from qwen38_b200.config import FULL, LINEAR, DrafterConfig, ModelConfig, RuntimeConfig
        from qwen38_b200.models.drafter import BlockDrafter
        from qwen38_b200.models.target import HybridTarget
        from qwen38_b200.ops.native import NativeOps
        from qwen38_b200.parallel.comm import TorchComm, make_comm
        from qwen38_b200.spec.engine import PinnedAcceptance, SpecRuntime, greedy_reference
        cfg = ModelConfig(num_hidden_layers=4, layer_types=[LINEAR, LINEAR, LINEAR, FULL])
        dcfg = DrafterConfig(num_hidden_layers=1, taps=[1, 3])
        ops = NativeOps(device=f"cuda:{rank}", max_keys=2048)
        tgt = HybridTarget(cfg, random_target_source(cfg, 0), RuntimeConfig(max_context=1024, prefill_chunk=256),
                           device=f"cuda:{rank}", dtype=torch.bfloat16, ops=ops,
                           comm=make_comm(2, device=f"cuda:{rank}", hidden=cfg.hidden_size, peer=(mode == "peer")))
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


@pytest.mark.parametrize("mode", ["peer", "nccl"])
def test_tp2_native_speculative_equals_greedy(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
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
