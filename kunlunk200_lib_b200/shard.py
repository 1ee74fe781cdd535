"""Row sharding of a matmul over the GPUs of one node.

Each rank owns a contiguous slice of the output rows N of every weight
(W[n_begin:n_begin+n_count, :]) and computes Y[:, slice]; an all-gather of
the slices (NCCL over NVLink) rebuilds the full Y on every rank.  The
reference library has no multi-device matmul of its own: its consumers
split rows across devices and exchange them with kunlun::peer copies
(src/k200.cpp:89-95); here the exchange is one collective.

Slices are as even as possible (the first N % world ranks own one extra
row).  all_gather_into_tensor needs equal sizes, so every rank contributes
a slice padded to the largest one and the padding is dropped afterwards.
"""
from __future__ import annotations


def row_shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of `rank`'s slice of n rows over `world` ranks."""
    if n < 0 or world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad shard request n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def padded_rows(n: int, world: int) -> int:
    """Rows of the largest slice: the per-rank size of the all-gather."""
    return -(-n // world)


def gather_rows(gathered, n: int, world: int, batch: int = 1):
    """Full [batch, n] output from an all-gather of padded slices.

    `gathered` holds world blocks of [batch, padded_rows] (rank-major, as
    all_gather_into_tensor writes them); works for numpy arrays and torch
    tensors alike.
    """
    pad = padded_rows(n, world)
    blocks = gathered.reshape(world, batch, pad)
    parts = []
    for r in range(world):
        _, count = row_shard(n, world, r)
        parts.append(blocks[r, :, :count])
    if hasattr(gathered, "new_empty"):  # torch
        import torch

        return torch.cat(parts, dim=1)
    import numpy as np

    return np.concatenate(parts, axis=1)
