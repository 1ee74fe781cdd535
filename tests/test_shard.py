"""Row sharding + all-gather of the multi-GPU matmul path, on CPU.

The arithmetic of every output row is independent of the sharding, so the
gathered result must equal the unsharded oracle result bit for bit.  Two
`gloo` ranks stand in for two GPUs (the data path on GPUs is the same
host logic with NCCL)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kunlunk200_lib_b200.shard import gather_rows, padded_rows, row_shard


@pytest.mark.parametrize("n,world", [(11008, 8), (4096, 2), (8193, 4), (5, 8), (1, 2), (14336, 3)])
def test_row_shard_covers_rows_once(n, world):
    seen = []
    for r in range(world):
        start, count = row_shard(n, world, r)
        assert count <= padded_rows(n, world)
        seen.extend(range(start, start + count))
    assert seen == list(range(n))


def test_gather_rows_numpy_roundtrip():
    n, world, batch = 10, 4, 3
    full = np.arange(batch * n, dtype=np.float32).reshape(batch, n)
    pad = padded_rows(n, world)
    blocks = np.zeros((world, batch, pad), np.float32)
    for r in range(world):
        s, c = row_shard(n, world, r)
        blocks[r, :, :c] = full[:, s:s + c]
    assert np.array_equal(gather_rows(blocks.ravel(), n, world, batch), full)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, k, n, batch, q4, x, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle as O

        start, count = row_shard(n, world, rank)
        row_bytes = k // 32 * 18
        shard = q4[start * row_bytes:(start + count) * row_bytes]
        y = O.matmul_gold(shard, O.WT_Q4_0, x, k, count, batch).astype(np.float32).reshape(batch, count)
        pad = padded_rows(n, world)
        mine = torch.zeros(batch, pad)
        mine[:, :count] = torch.from_numpy(y)
        gathered = torch.empty(world * batch * pad)
        dist.all_gather_into_tensor(gathered, mine.reshape(-1))
        if rank == 0:
            out.put(gather_rows(gathered, n, world, batch).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n,batch", [(4096, 1), (1001, 2)])
def test_sharded_q4_gemv_matches_unsharded(O, n, batch):
    k, world = 256, 2
    w = O.normal(0x7340D123, n * k, 0.0, 0.02)
    q4 = O.q4_0_quantize(w, n, k)
    x = O.uniform(0x09200ABC, k * batch, -1.0, 1.0)
    full = O.matmul_gold(q4, O.WT_Q4_0, x, k, n, batch).astype(np.float32).reshape(batch, n)
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, k, n, batch, q4, x, out)) for r in range(world)]
    for p in procs:
        p.start()
    got = out.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert np.array_equal(got, full)


class _FakeK:
    """Stand-in for the library's IPC and allocation calls (no GPU)."""
    GATHER_MAX_RANKS = 8

    def __init__(self):
        from kunlunk200_lib_b200 import GatherView

        self.GatherView = GatherView
        self.opened, self.closed = [], []

    def ipc_handle(self, ptr):
        return ptr.to_bytes(8, "little") * 8

    def ipc_open(self, device, handle):
        p = int.from_bytes(handle[:8], "little") + 0x1000000  # "mapped" elsewhere
        self.opened.append(p)
        return p

    def ipc_close(self, device, ptr):
        self.closed.append(ptr)


def _ranks_over_gloo(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from kunlunk200_lib_b200.shard import PeerExchange

    class Buf:
        def __init__(self, base):
            self.base = base

        def data(self):
            return self.base

        def close(self):
            pass

    K = _FakeK()
    PeerExchange._region = classmethod(lambda cls, K_, dev, n, buffers, batch=1: Buf(0x10000 * (rank + 1)))

    def all_gather(obj):
        got = [None] * world
        dist.all_gather_object(got, obj)
        return got

    ex = PeerExchange.over_group(K, 0, 1000, world, rank, all_gather)
    v0, v1 = ex.view(0), ex.view(1)
    out.put((rank, [v0.tags[r] for r in range(world)], [v1.tags[r] for r in range(world)], v0.y, v1.y,
             v0.counter, v1.counter, ex.output(1), (v0.rows, v0.batch), list(K.opened)))
    ex.close()
    assert sorted(K.closed) == sorted(K.opened)
    dist.destroy_process_group()


def test_peer_exchange_views_over_gloo():
    """Each rank sees its own region directly and the others through their IPC handles."""
    from kunlunk200_lib_b200.shard import PeerExchange

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_ranks_over_gloo, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    pad = PeerExchange.padded(1000)
    assert pad == 1024
    assert PeerExchange.region_bytes(1000) == 2 * (pad * 12 + 64)
    for rank, t0, t1, y0, y1, c0, c1, out1, shape, opened in res:
        for r in range(world):
            base = 0x10000 * (r + 1) + (0 if r == rank else 0x1000000)
            assert t0[r] == base + 2 * pad * 4 and t1[r] == base + 2 * pad * 4 + pad * 8
        own = 0x10000 * (rank + 1)
        assert y0 == own and y1 == own + pad * 4 and out1 == y1
        assert c0 == own + 2 * pad * 12 and c1 == c0 + 64
        assert shape == (1000, 1)
        assert len(opened) == world - 1
