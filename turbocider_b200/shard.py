"""N-column sharding of quantised linears across ranks (one process per GPU).

Each rank holds a contiguous block of weight rows (output columns of Y); the
K axis is never split, so GGUF super-blocks stay whole.  Rank r computes
Y_r = X * W_r^T ([M, rows_r]) and the ranks all-gather their bf16 slices.
All-gather needs equal slice sizes, so every rank's slice is padded to
ceil(N / world) columns; `assemble` drops the padding and interleaves the
rank-major gather buffer [world, M, rows_per_rank] back into Y[M, N].

This is host logic only (the GEMM itself is tc_cuda_qlinear on each rank).
"""
from __future__ import annotations


def rows_per_rank(n: int, world: int) -> int:
    """Padded slice width: ceil(n / world)."""
    return -(-n // world)


def shard_rows(n: int, world: int, rank: int) -> tuple[int, int]:
    """(n_begin, n_count) of rank's weight rows; n_count may be 0 for the
    last ranks when world does not divide n."""
    per = rows_per_rank(n, world)
    begin = min(n, rank * per)
    return begin, min(n, begin + per) - begin


def assemble(gathered, n: int):
    """Y[M, n] from the rank-major all-gather buffer [world, M, per] (torch or
    numpy); columns past each rank's n_count are padding."""
    world, m, per = gathered.shape
    parts = []
    for r in range(world):
        b, c = shard_rows(n, world, r)
        if c:
            parts.append(gathered[r, :, :c])
    if hasattr(gathered, "permute"):
        import torch
        return torch.cat(parts, dim=1)
    import numpy as np
    return np.concatenate(parts, axis=1)
