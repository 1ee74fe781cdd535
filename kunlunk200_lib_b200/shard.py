"""Row sharding of a matmul over the GPUs of one node.

Each rank owns a contiguous slice of the output rows N of every weight
(W[n_begin:n_begin+n_count, :]) and computes Y[:, slice]; the slices are
then gathered so every rank holds the full Y.  The reference library has no
multi-device matmul of its own: its consumers split rows across devices and
exchange them with kunlun::peer copies (src/k200.cpp:89-95).  Here the
exchange runs over NVLink peer memory inside the library (PeerExchange with
k200_matmul_q4_gather or k200_gather_rows: every slice is stored at its own
offset, so uneven splits need no padding); row_shard also serves callers
that gather with an NCCL all-gather, which needs equal sizes: padded_rows
and gather_rows pad every slice to the largest one and drop the padding.

Slices are as even as possible (the first N % world ranks own one extra
row).
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


class PeerExchange:
    """One all-gather exchange of a row-sharded matmul over peer memory
    (k200_matmul_q4_gather for the batch-1 Q4_0 GEMV, k200_gather_rows for any
    matmul).

    Every rank owns one device region, zeroed at creation, holding
    ``buffers`` exchanges: their output buffers of [batch][n] floats (each
    padded to a multiple of 64 values), then their tag arrays of as many
    64-bit words {f32, epoch}, then their counters (two words each, 64 bytes
    apart).  ``bases[r]`` is rank r's region as an address valid on this
    rank's device (its own allocation, or an IPC mapping of the other
    rank's); other ranks only ever store into the tag arrays.  ``view(b)`` is
    the k200_gather of exchange b; alternate exchanges between consecutive
    uses, so that a rank that runs ahead never overwrites words another rank
    is still reading.
    """

    def __init__(self, K, device: int, n: int, world: int, rank: int, bases: list[int], buffers: int = 2,
                 owned=None, mapped=(), batch: int = 1):
        if not 1 <= world <= K.GATHER_MAX_RANKS or not 0 <= rank < world or len(bases) != world or batch < 1:
            raise ValueError(f"bad exchange: world={world} rank={rank} bases={len(bases)} batch={batch}")
        self.K, self.device, self.n, self.world, self.rank, self.buffers = K, device, n, world, rank, buffers
        self.batch = batch
        self.n_pad = self.padded(n * batch)
        self._owned, self._mapped = owned, list(mapped)
        tags_off = buffers * self.n_pad * 4
        counters_off = tags_off + buffers * self.n_pad * 8
        self.views = []
        for b in range(buffers):
            v = K.GatherView()
            v.ranks, v.rank = world, rank
            for r in range(world):
                v.tags[r] = bases[r] + tags_off + b * self.n_pad * 8
            v.y = bases[rank] + b * self.n_pad * 4
            v.counter = bases[rank] + counters_off + b * 64
            v.rows, v.batch = n, batch
            self.views.append(v)

    @staticmethod
    def padded(n: int) -> int:
        return -(-n // 64) * 64

    @classmethod
    def region_bytes(cls, n: int, buffers: int = 2, batch: int = 1) -> int:
        return buffers * (cls.padded(n * batch) * 12 + 64)

    @classmethod
    def _region(cls, K, device: int, n: int, buffers: int, batch: int = 1):
        import numpy as np

        nbytes = cls.region_bytes(n, buffers, batch)
        buf = K.Buffer(device, nbytes)
        buf.upload(np.zeros(nbytes, np.uint8))
        return buf

    @classmethod
    def over_group(cls, K, device: int, n: int, world: int, rank: int, all_gather, buffers: int = 2,
                   batch: int = 1):
        """Collective: one region per rank, IPC handles swapped with ``all_gather(obj) -> list``."""
        buf = cls._region(K, device, n, buffers, batch)
        handles = all_gather(K.ipc_handle(buf.data()))
        bases, mapped = [], []
        for r, h in enumerate(handles):
            if r == rank:
                bases.append(buf.data())
            else:
                p = K.ipc_open(device, h)
                bases.append(p)
                mapped.append(p)
        return cls(K, device, n, world, rank, bases, buffers, owned=buf, mapped=mapped, batch=batch)

    @classmethod
    def on_one_device(cls, K, device: int, n: int, world: int, buffers: int = 2, batch: int = 1):
        """All ranks' regions on one device, for running the ranks one after another in one stream."""
        bufs = [cls._region(K, device, n, buffers, batch) for _ in range(world)]
        bases = [b.data() for b in bufs]
        xs = [cls(K, device, n, world, r, bases, buffers, batch=batch) for r in range(world)]
        xs[0]._owned = bufs  # the first rank's object keeps every region alive
        return xs

    def view(self, b: int):
        return self.views[b % self.buffers]

    def output(self, b: int) -> int:
        """Address of this rank's own output buffer b (the full [batch][n] rows once
        k200_gather_wait has run on it; this rank's own rows as soon as they are computed)."""
        return self.views[b % self.buffers].y

    def close(self) -> None:
        for p in self._mapped:
            self.K.ipc_close(self.device, p)
        self._mapped = []
        owned = self._owned if isinstance(self._owned, list) else [self._owned] if self._owned else []
        for b in owned:
            b.close()
        self._owned = None
