"""MXFP8 weights for the weight-streaming GEMM, checked on the CPU: the tiled byte / scale layout
(``mx_tile_weight``) against ``quant_mxfp8``, the refusal of weights that are not exactly MXFP8,
and the kernel's e4m3 -> bf16 expansion (csrc/gemm_kernel.cuh ``e4m3x4_to_bf16x4_scaled``: the
e4m3 sign to bit 15, exponent+mantissa to bits 10..4, then a bf16 multiply by 2^(scale - 7))
restated with integer and bf16 tensor ops over every e4m3 byte and a range of scales."""
import torch

from qwen38_b200.checkpoint import dequant_mxfp8, quant_mxfp8
from qwen38_b200.ops.native import mx_tile_weight


def _mx_weight(N, K, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * 0.02
    return dequant_mxfp8(*quant_mxfp8(w))


def test_tiled_layout_matches_quantisation():
    N, K = 200, 320                                  # padded to 256 rows, 5 K blocks
    w = _mx_weight(N, K, 0)
    mw = mx_tile_weight(w)
    assert mw is not None and mw.q.dtype == torch.uint8 and mw.s.dtype == torch.uint8
    q, se = quant_mxfp8(w)
    NT, KB = 2, 5
    qt = mw.q.view(NT, KB, 128, 64).permute(0, 2, 1, 3).reshape(NT * 128, KB * 64)
    st = mw.s.view(NT, KB, 128, 2).permute(0, 2, 1, 3).reshape(NT * 128, KB * 2)
    assert torch.equal(qt[:N, :K], q.view(torch.uint8))
    assert torch.equal(st[:N, :K // 32], se)
    assert int(qt[N:].sum()) == 0 and int(st[N:].sum()) == 0
    # the bf16 expansion kept for the prefill tiles is the exact weight
    t = mw.t.view(NT, KB, 128, 64).permute(0, 2, 1, 3).reshape(NT * 128, KB * 64)
    assert torch.equal(t[:N, :K].float(), w)


def test_weights_that_are_not_mxfp8_stay_bf16():
    w = (torch.randn(128, 128, generator=torch.Generator().manual_seed(1)) * 0.02).to(torch.bfloat16).float()
    assert mx_tile_weight(w) is None
    assert mx_tile_weight(_mx_weight(128, 128, 2) * 2.0 ** 20) is None     # scale above 2^7


def _bf16_bits_to_float(bits):
    return (bits.to(torch.int32) << 16).view(torch.float32)


def test_kernel_expansion_of_every_e4m3_byte():
    b = torch.arange(256, dtype=torch.int32)
    b = b[(b & 0x7F) != 0x7F]                        # e4m3fn NaN patterns never occur in weights
    ref_val = b.to(torch.uint8).view(torch.float8_e4m3fn).float()
    f = ((b & 0x80) << 8) | ((b & 0x7F) << 4)        # bf16 bits of value * 2^-120
    base = _bf16_bits_to_float(f)
    assert torch.equal(base, ref_val * 2.0 ** -120)  # exact, subnormal e4m3 included
    for e in (100, 115, 120, 127, 130, 134):          # E8M0 scale bytes
        m = _bf16_bits_to_float(torch.tensor([(e + 120) << 7]))
        got = (base.to(torch.bfloat16) * m.to(torch.bfloat16)).float()   # one bf16 rounding, exact here
        want = dequant_mxfp8(b.to(torch.uint8).view(torch.float8_e4m3fn).view(1, -1).contiguous(),
                             torch.full((1, 8), e, dtype=torch.uint8))[0]
        assert torch.equal(got, want), e
