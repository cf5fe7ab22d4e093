"""The allocation-free GEMM entry point (``q38_linear_noalloc``, csrc/gemm_noalloc.cu), called
through its exported C symbol, against the regular (allocating) entry point.

It exists for callers that cannot allocate device memory at call time (a foreign memory pool, an
allocator-free serving loop): they pass only inputs and outputs, and the kernel's scratch lives in
a fixed file-scope device array.  This file sorts last so that a run stopping at the first failure
has already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from qwen38_b200.ops.build import so_path  # noqa: E402
from qwen38_b200.ops.native import NativeOps  # noqa: E402
from qwen38_b200.ops.noalloc import bind  # noqa: E402

EPI_BF16, EPI_F32, EPI_ADD_F32 = 0, 1, 2


@pytest.fixture(scope="module")
def lib():
    NativeOps()                       # loads the extension (and libtorch) into this process
    return bind(so_path())            # argument types from csrc/q38_noalloc.h's prototypes


def _call(fn, x, tw, out, epi):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(x.data_ptr(), x.shape[0], x.shape[1], tw.t.data_ptr(), tw.N, out.data_ptr(), out.stride(0), epi,
              ctypes.c_void_p(stream))


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("T,N,K", [(16, 5120, 17408), (1, 16480, 5120), (32, 1000, 640)])
def test_noalloc_matches_allocating_entry_point(lib, T, N, K):
    fn, status = lib
    ops = NativeOps()
    g = torch.Generator(device="cuda").manual_seed(T + N)
    x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
    tw = ops.prepare_weight((torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16))
    ref32 = ops.linear(x, tw, out_dtype=torch.float32)
    ref16 = ops.linear(x, tw)
    ops.check()
    for _ in range(2):                          # two calls in a row share (and reset) the scratch
        out32 = torch.full((T, N), float("nan"), device="cuda")
        assert _call(fn, x, tw, out32, EPI_F32) == 0
        out16 = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
        assert _call(fn, x, tw, out16, EPI_BF16) == 0
        torch.cuda.synchronize()
        assert status() == 0
        assert _rel(out32, ref32) < 1e-4        # same kernel and split plan: equal in practice
        assert _rel(out16, ref16) < 8e-3
    acc = torch.ones(T, N, device="cuda")
    assert _call(fn, x, tw, acc, EPI_ADD_F32) == 0
    torch.cuda.synchronize()
    assert _rel(acc, ref32 + 1.0) < 1e-4


def test_noalloc_rejects_unserved_sizes(lib):
    fn, _ = lib
    ops = NativeOps()
    x = torch.zeros(64, 256, dtype=torch.bfloat16, device="cuda")          # more than 32 rows
    tw = ops.prepare_weight(torch.zeros(128, 256, dtype=torch.bfloat16, device="cuda"))
    out = torch.zeros(64, 128, device="cuda")
    assert _call(fn, x, tw, out, EPI_F32) == 1
    x1 = torch.zeros(1, 256, dtype=torch.bfloat16, device="cuda")
    assert _call(fn, x1, tw, out, 3) == 1                                 # epilogue not served
    big = ops.prepare_weight(torch.zeros(600_000, 64, dtype=torch.bfloat16, device="cuda"))
    xs = torch.zeros(1, 64, dtype=torch.bfloat16, device="cuda")
    outs = torch.zeros(1, 600_000, device="cuda")
    assert _call(fn, xs, big, outs, EPI_F32) == 2                         # beyond the scratch maximum
