"""Column (output-row) sharding of a stack of quantised linears over ranks.

Every ggml block format packs values along K, so splitting a weight's N
output rows cuts no block: rank r of W ranks holds rows
[r * N / W, (r + 1) * N / W) of each N x K matrix (a contiguous byte range
of the row-major ggml buffer), computes its slice of Y = X W^T from the
full, replicated X, and the slices are joined by an all-gather whose output
is [W][M][N / W].  N must divide by the rank count (true for every shape of
the 14B stack at 1, 2, 4 and 8 ranks).
"""
from __future__ import annotations

import numpy as np


def row_range(N: int, world: int, rank: int) -> tuple[int, int]:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if N % world:
        raise ValueError(f"N = {N} does not divide over {world} ranks")
    n = N // world
    return rank * n, (rank + 1) * n


def shard_bytes(w: np.ndarray, N: int, world: int, rank: int) -> np.ndarray:
    """Rank's rows of a row-major ggml weight buffer (N rows of equal bytes)."""
    w = np.ascontiguousarray(w).reshape(N, -1)
    r0, r1 = row_range(N, world, rank)
    return w[r0:r1]


def join_gathered(gathered: np.ndarray) -> np.ndarray:
    """[world][M][N / world] all-gather output -> [M][N] (rank-major columns)."""
    g = np.asarray(gathered)
    world, M, n = g.shape
    return np.ascontiguousarray(g.transpose(1, 0, 2).reshape(M, world * n))
