"""Kernel index math checked on the CPU: the decode attention's key-group partition (Python
mirror against the compiled host function, when the extension is built) and the tile-contiguous
weight layout."""
import pytest
import torch

from qwen38_b200.ops import layout


@pytest.mark.parametrize("n", [1, 2, 33, 64, 65, 68, 69, 511, 512, 513, 520, 521, 1025, 4097])
def test_key_groups_partition(n):
    groups = layout.key_groups(n)
    covered = [c for c0, cnt in groups for c in range(c0, c0 + cnt)]
    assert covered == list(range(n))                       # every chunk once, in key order
    assert all(cnt >= 1 for _, cnt in groups)
    for c0, cnt in groups:
        assert cnt <= (1 if c0 < 64 else 4 if c0 < 512 else 8)
    # the partition is fixed: a shorter context only truncates the last group of a longer one
    longer = layout.key_groups(n + 37)
    assert [c0 for c0, _ in groups] == [c0 for c0, _ in longer][:len(groups)]


def test_key_groups_match_compiled_kernel_math():
    try:
        from qwen38_b200.ops.build import load
        C = load()
    except Exception as e:                                  # extension not built in this checkout
        pytest.skip(f"extension not loaded: {e}")
    if not hasattr(C, "attn_key_groups"):
        pytest.skip("extension built before attn_key_groups existed")
    for n in (1, 64, 65, 300, 512, 513, 1025, 4097):
        assert [tuple(g) for g in C.attn_key_groups(n)] == layout.key_groups(n)


def test_tiled_weight_layout():
    from qwen38_b200.ops.native import tile_weight, untile_weight
    g = torch.Generator().manual_seed(0)
    w = torch.randn(300, 200, generator=g)
    tw = tile_weight(w)
    assert torch.equal(untile_weight(tw), w)
    kblocks = -(-200 // 64)
    for n, k in ((0, 0), (129, 65), (299, 199), (255, 127)):
        r, c = layout.tiled_row(n, k, kblocks)
        assert tw.t[r, c] == w[n, k]
