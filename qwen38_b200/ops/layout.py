"""Python mirrors of the index math the kernels use, for planners and CPU tests.

* ``key_groups(nchunks)``: the decode attention's fixed partition of the absolute key axis into
  groups of 128-key chunks (``csrc/attention.cu``: one chunk per group below chunk 64, four below
  chunk 512, eight beyond).  A row's partial results depend only on this partition, never on how
  many rows run with it.
* ``tiled_row(n, k, kblocks)``: the row of the tile-contiguous weight layout (``ops/native.py``,
  ``tile_weight``) that holds weight element (n, k): tile (n // 128, k // 64) is one 16 KB block.
"""
from __future__ import annotations

CH = 128                 # keys per chunk
TIER0, TIER1 = 64, 512   # chunk indices where groups grow to 4 and to 8 chunks


def groups_for(nchunks: int) -> int:
    if nchunks <= TIER0:
        return nchunks
    if nchunks <= TIER1:
        return TIER0 + -(-(nchunks - TIER0) // 4)
    return TIER0 + (TIER1 - TIER0) // 4 + -(-(nchunks - TIER1) // 8)


def group_first_chunk(g: int) -> int:
    if g < TIER0:
        return g
    if g < TIER0 + (TIER1 - TIER0) // 4:
        return TIER0 + 4 * (g - TIER0)
    return TIER1 + 8 * (g - TIER0 - (TIER1 - TIER0) // 4)


def group_chunks(g: int) -> int:
    return 1 if g < TIER0 else (4 if g < TIER0 + (TIER1 - TIER0) // 4 else 8)


def key_groups(nchunks: int):
    """[(first chunk, chunk count)] covering chunks 0..nchunks-1 in order."""
    return [(group_first_chunk(g), min(group_chunks(g), nchunks - group_first_chunk(g)))
            for g in range(groups_for(nchunks))]


def tiled_row(n: int, k: int, kblocks: int) -> tuple:
    """(row, column) of weight element (n, k) in the tile-contiguous layout."""
    return ((n // 128) * kblocks + k // 64) * 128 + n % 128, k % 64
