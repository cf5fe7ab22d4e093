import os
import sys

# Multi-process tests spawn up to 8 CPU ranks; with every process using all cores' OpenMP threads
# the machine is oversubscribed many times over and spin-waiting threads stall the whole suite.
os.environ.setdefault("OMP_NUM_THREADS", "4")

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")


@pytest.fixture(scope="session")
def tiny():
    import torch
    from qwen38_b200.checkpoint import materialize, random_drafter_source, random_target_source
    from qwen38_b200.config import tiny_drafter_config, tiny_model_config
    cfg, dcfg = tiny_model_config(), tiny_drafter_config()
    src = random_target_source(cfg, 0)
    dsrc = random_drafter_source(dcfg, cfg.vocab_size, 1)
    prompt = torch.randint(0, cfg.vocab_size, (128,), generator=torch.Generator().manual_seed(0)).tolist()
    return dict(cfg=cfg, dcfg=dcfg, src=src, dsrc=dsrc, sd=materialize(src), prompt=prompt)
