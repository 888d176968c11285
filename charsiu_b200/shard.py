"""The column (output-row) split of a tensor over ranks, as the device layer
does it (charsiu_gpu_add_blocks in csrc/charsiu_gpu.cu): rows go in whole
8-row groups, rank r of w takes groups [r * ceil(G / w), (r + 1) * ceil(G / w))
of the G = ceil(N / 8). Every row lands on exactly one rank and no reduction
crosses ranks, so sharded outputs are bit-identical to unsharded ones."""
from __future__ import annotations

RG = 8


def shard_rows(n: int, rank: int, world: int):
    """(first row, row count) of rank's slab of an n-row tensor."""
    groups = -(-n // RG)
    per = -(-groups // world)
    g0 = min(per * rank, groups)
    g1 = min(g0 + per, groups)
    row0 = min(g0 * RG, n)
    return row0, max(0, min(g1 * RG, n) - row0)


def slab_rows(n: int, world: int) -> int:
    """Rows of the widest slab: every rank's output buffer is this long, so an
    all-gather moves equal pieces."""
    return -(-(-(-n // RG)) // world) * RG


def assemble(gathered, n: int, world: int):
    """The full output from the world's equal-length slabs (list or array of
    world x slab_rows), in rank order."""
    import numpy as np
    out = np.empty(n, dtype=np.asarray(gathered[0]).dtype)
    for r in range(world):
        row0, rows = shard_rows(n, r, world)
        out[row0:row0 + rows] = np.asarray(gathered[r])[:rows]
    return out
