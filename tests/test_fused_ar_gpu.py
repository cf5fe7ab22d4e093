"""The pushed tensor-parallel all-reduce on one GPU: the GEMM that pushes its tiles
(``linear_push``) plus the reducing RMSNorm (``rms_norm_ar``) add exactly what the plain GEMM's
residual epilogue adds, and the fused norm equals the plain norm bit for bit; when a peer never
publishes its tiles the bounded flag wait gives up, records the peer-timeout bit in the error
word, leaves the residual untouched and the context usable.  Two-rank numerics: test_tp_gpu.py."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from qwen38_b200.ops.native import NativeOps, untile_weight  # noqa: E402
from qwen38_b200.parallel.symm import PUSH_ROWS  # noqa: E402

ERR_PEER = 8


class _Areas:
    """Receive area of a fake communicator; every "rank" maps this GPU's own buffer."""

    def __init__(self, world, hidden, slots=4):
        self.world, self.rank, self.hidden = world, 0, hidden
        self.block_words = PUSH_ROWS * hidden
        self.recv = torch.zeros(slots * world * self.block_words, dtype=torch.int64, device="cuda")
        self.recv_ptrs = [self.recv.data_ptr()] * world
        self.fepochs = torch.zeros(slots * PUSH_ROWS, dtype=torch.int32, device="cuda")
        self.slots, self._n = slots, 0

    def fused_slot(self):
        s = self._n % self.slots
        self._n += 1
        return s


@pytest.fixture(scope="module")
def ops():
    return NativeOps()


@pytest.mark.parametrize("T,N,K", [(1, 5120, 3072), (16, 5120, 8704), (32, 5120, 6144), (7, 1024, 640), (64, 5120, 6144)])
def test_one_rank_equals_residual_epilogue_and_plain_norm(ops, T, N, K):
    g = torch.Generator(device="cuda").manual_seed(T * 7 + K)
    x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
    w = ops.prepare_weight((torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16))
    nw = 1 + 0.1 * torch.randn(N, generator=g, device="cuda")
    r0 = torch.randn(T, N, generator=g, device="cuda")
    comm = _Areas(1, N)
    a = r0.clone()
    for _ in range(3):                                   # epochs advance call after call
        a.copy_(r0)
        slot = ops.linear_push(x, w, comm)
        h = ops.rms_norm_ar(a, nw, 1e-6, torch.bfloat16, comm, slot)
    b = r0.clone()
    ops.linear_residual(x, w, b)
    hb = ops.rms_norm(b, nw, 1e-6, torch.bfloat16)
    c = r0.clone()
    ops.rms_norm_ar(c, None, 1e-6, torch.bfloat16, comm, ops.linear_push(x, w, comm))   # reduce only
    ref = r0 + x.float() @ untile_weight(w).float().t()
    torch.cuda.synchronize()
    ops.check()
    assert torch.equal(a, b) and torch.equal(c, b)
    assert torch.equal(h, hb)
    assert ((a - ref).norm() / ref.norm()).item() < 1e-3


def test_missing_peer_times_out_and_reports(ops):
    T, N, K = 4, 1024, 512
    x = torch.randn(T, K, device="cuda").to(torch.bfloat16)
    w = ops.prepare_weight((torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16))
    comm = _Areas(2, N)          # "rank 1"'s block of this GPU's own area is never written
    r = torch.full((T, N), 3.0, device="cuda")
    t0 = time.time()
    slot = ops.linear_push(x, w, comm)
    out = ops.rms_norm_ar(r, torch.ones(N, device="cuda"), 1e-6, torch.bfloat16, comm, slot)
    torch.cuda.synchronize()
    assert time.time() - t0 < 30
    assert int(ops.err.item()) & ERR_PEER
    assert torch.all(r == 3.0)
    ops.err.zero_()
    ops.counters.zero_()
    y = torch.randn(64, device="cuda")
    assert torch.allclose((y * 2).sum(), 2 * y.sum(), rtol=1e-4, atol=1e-3)
    one = _Areas(1, N)                                    # and the kernels still serve a one-rank call
    a = torch.zeros(T, N, device="cuda")
    ops.rms_norm_ar(a, None, 1e-6, torch.bfloat16, one, ops.linear_push(x, w, one))
    b = torch.zeros(T, N, device="cuda")
    ops.linear_residual(x, w, b)
    torch.cuda.synchronize()
    ops.check()
    assert torch.equal(a, b)
    del out
