"""Failure detection on the device without a GPU fault: a peer-memory barrier whose peer never
signals (the second "rank" aliases this GPU's own buffer, so nothing ever sets its flag) gives up
after its time limit, records the error in the device error word, leaves the output untouched and
returns; the context stays usable and a one-rank barrier completes normally."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from qwen38_b200.ops.build import load  # noqa: E402

AR_CTAS, MAX_RANKS, ERR_PEER = 32, 8, 8


def _setup(C, slots=2, slot_floats=4096):
    data_bytes = slots * slot_floats * 4
    buf = C.peer_alloc(data_bytes + slots * AR_CTAS * MAX_RANKS * 4, torch.cuda.current_device())
    base = buf.data_ptr()
    local = buf[:data_bytes].view(torch.float32).view(slots, slot_floats)
    epochs = torch.zeros(slots * AR_CTAS, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    return buf, base, base + data_bytes, local, epochs, err, slot_floats


def test_peer_barrier_times_out_and_reports():
    C = load()
    buf, data, flags, local, epochs, err, sf = _setup(C)
    local[0, :1024].fill_(1.0)
    residual = torch.full((4, 256), 5.0, device="cuda")
    t0 = time.time()
    # world 2, but "rank 1" is this same buffer: its flag for (slot 0, every CTA) is never written
    C.allreduce_residual([data, data], [flags, flags], 0, 0, sf, residual, epochs, err)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(err.item()) & ERR_PEER
    assert torch.all(residual == 5.0)                   # nothing was added
    assert dt < 30
    # the context is still usable
    err.zero_()
    x = torch.randn(1000, device="cuda")
    assert torch.allclose((x * 2).sum(), x.sum() * 2, rtol=1e-4, atol=1e-3)


def test_single_rank_barrier_completes():
    C = load()
    buf, data, flags, local, epochs, err, sf = _setup(C)
    local[1, :1024].fill_(2.0)
    residual = torch.ones(4, 256, device="cuda")
    for _ in range(2):                                  # epochs advance call after call
        C.allreduce_residual([data], [flags], 0, 1, sf, residual, epochs, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.all(residual == 5.0)
