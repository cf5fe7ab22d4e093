"""The GEMM kernel that carries the tensor-parallel all-reduce (``linear_allreduce``) on one GPU:
at one rank it adds exactly what the plain GEMM's residual epilogue adds, and when a peer never
publishes its tile the bounded flag wait gives up, records the peer-timeout bit in the error word,
leaves the residual untouched and the context usable.  Two-rank numerics: test_tp_gpu.py."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from qwen38_b200.ops.native import NativeOps, untile_weight  # noqa: E402

ERR_PEER, TILES_MAX = 8, 64


class _Areas:
    """Receive / flag areas of a fake communicator; every "rank" maps this GPU's own buffers."""

    def __init__(self, world, hidden, slots=4):
        self.world, self.rank = world, 0
        self.block_floats = 32 * hidden
        self.tiles_max = TILES_MAX
        self.recv = torch.zeros(slots * world * self.block_floats, device="cuda")
        self.flags = torch.zeros(slots * TILES_MAX * 8, dtype=torch.int32, device="cuda")
        self.recv_ptrs = [self.recv.data_ptr()] * world
        self.fflag_ptrs = [self.flags.data_ptr()] * world
        self.fepochs = torch.zeros(slots * TILES_MAX, dtype=torch.int32, device="cuda")
        self.slots, self._n = slots, 0

    def fused_slot(self):
        s = self._n % self.slots
        self._n += 1
        return s


@pytest.fixture(scope="module")
def ops():
    return NativeOps()


@pytest.mark.parametrize("T,N,K", [(1, 5120, 3072), (16, 5120, 8704), (32, 5120, 6144), (7, 1000, 640)])
def test_one_rank_equals_residual_epilogue(ops, T, N, K):
    g = torch.Generator(device="cuda").manual_seed(T * 7 + K)
    x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
    w = ops.prepare_weight((torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16))
    r0 = torch.randn(T, N, generator=g, device="cuda")
    comm = _Areas(1, N)
    a = r0.clone()
    for _ in range(3):
        a.copy_(r0)
        ops.linear_allreduce(x, w, a, comm)
    b = r0.clone()
    ops.linear_residual(x, w, b)
    ref = r0 + x.float() @ untile_weight(w).float().t()
    torch.cuda.synchronize()
    ops.check()
    assert torch.equal(a, b)
    assert ((a - ref).norm() / ref.norm()).item() < 1e-3


def test_missing_peer_times_out_and_reports(ops):
    T, N, K = 4, 1024, 512
    x = torch.randn(T, K, device="cuda").to(torch.bfloat16)
    w = ops.prepare_weight((torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16))
    comm = _Areas(2, N)          # "rank 1" is this GPU's own area: its flags are never written
    r = torch.full((T, N), 3.0, device="cuda")
    t0 = time.time()
    ops.linear_allreduce(x, w, r, comm)
    torch.cuda.synchronize()
    assert time.time() - t0 < 30
    assert int(ops.err.item()) & ERR_PEER
    assert torch.all(r == 3.0)
    ops.err.zero_()
    ops.counters.zero_()
    y = torch.randn(64, device="cuda")
    assert torch.allclose((y * 2).sum(), 2 * y.sum(), rtol=1e-4, atol=1e-3)
    # and the kernel still serves a one-rank call afterwards
    one = _Areas(1, N)
    a = torch.zeros(T, N, device="cuda")
    ops.linear_allreduce(x, w, a, one)
    b = torch.zeros(T, N, device="cuda")
    ops.linear_residual(x, w, b)
    torch.cuda.synchronize()
    ops.check()
    assert torch.equal(a, b)
