"""Row-sharded batch-1 Q4_0 GEMV with the fused all-gather (k200_matmul_q4_gather).

The reference's consumers split output rows over devices and gather the
slices with kunlun::peer copies (src/k200.cpp:89-95, docs/common-q4.md:31);
here each rank's GEMV stores its rows as tagged words {f32, epoch} into
every rank's tag array of the exchange.  Checks:
  * ranks run one after another on one GPU (every wait is already satisfied
    when it starts, so no kernel waits on one that has not run): after
    k200_gather_wait every rank's buffer holds every shard, bit-identical to
    k200_matmul on that shard, and a chained second GEMV that reads the first
    exchange's tagged words sees the full vector; every word carries the
    exchange's epoch, one per use;
  * a wait that nothing satisfies runs out and posts the peer-timeout status
    (0x4b03) instead of hanging, and the device stays usable;
  * on two GPUs (when present), the same chain across two processes.
Bar: bit-exact against k200_matmul on the same shard (same kernel, same
shape, so the same arithmetic).
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

from kunlunk200_lib_b200.shard import PeerExchange, row_shard

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PEER_TIMEOUT = 0x4B03


def _q4(O, k, n, seed):
    return O.q4_0_quantize(O.normal(seed, n * k, 0.0, 0.02), n, k)


def _plain(K, dw, dx, k, n, row_begin, x_offset=0):
    """Rows [row_begin, row_begin + n) through k200_matmul."""
    row_bytes = k // 32 * 18
    dy = K.Buffer(0, 4 * n)
    kern = K.Kernel()
    K.matmul(kern, 0, dy, dw.data() + row_begin * row_bytes, dx + x_offset, k, n, 1, K.Q4_0)
    K.select(0)
    K.check(K.wait())
    y = dy.download(np.float32, n)
    kern.close()
    dy.close()
    return y


def _download(K, ptr, n):
    out = np.empty(n, np.float32)
    K.select(0)
    K.check(K.copy(out, ptr, out.nbytes, K.DEVICE_TO_HOST))
    return out


def _epoch(K, view):
    """This rank's current epoch of an exchange (its counter's second word)."""
    out = np.empty(2, np.uint32)
    K.select(0)
    K.check(K.copy(out, view.counter, out.nbytes, K.DEVICE_TO_HOST))
    return int(out[1])


def _tag_epochs(K, view, count):
    """The epochs carried by the first `count` words of this rank's tag array."""
    out = np.empty(count, np.uint64)
    K.select(0)
    K.check(K.copy(out, view.tags[view.rank], out.nbytes, K.DEVICE_TO_HOST))
    return (out >> np.uint64(32)).astype(np.uint32)


@pytest.mark.parametrize("world,n1,k2", [(2, 2000, 2048), (3, 2000, 2048), (2, 2001, 2048), (2, 5100, 5120)])
def test_gather_ranks_on_one_gpu(K, O, gpu, world, n1, k2):
    # the second GEMV reads k2 values of the gathered n1-row output: its
    # tagged rows, then the zeroed padding of the exchange buffer read plainly
    # (2001: a block whose first 17 values are tagged; 5100 of 5120: K cut
    # into two parts of 12 and 8 pairs, the second ending in padding)
    k1 = 4096
    n2 = 1024
    q_up = _q4(O, k1, n1, 0x7340D123)
    q_dn = _q4(O, k2, n2, 0x1234567)
    x = O.uniform(0x09200ABC, k1, -1.0, 1.0)
    dw1, dw2, dx = K.Buffer(0, q_up.nbytes), K.Buffer(0, q_dn.nbytes), K.Buffer(0, x.nbytes)
    dw1.upload(q_up)
    dw2.upload(q_dn)
    dx.upload(x)
    up = PeerExchange.on_one_device(K, 0, n1, world)
    dn = PeerExchange.on_one_device(K, 0, n2, world)
    rb1 = k1 // 32 * 18
    rb2 = k2 // 32 * 18
    scratch = max(K.matmul_q4_gather_scratch(0, k1, row_shard(n1, world, r)[1]) for r in range(world))
    scratch = max([scratch] + [K.matmul_q4_gather_scratch(0, k2, row_shard(n2, world, r)[1]) for r in range(world)])
    assert scratch > 0
    sbuf = K.Buffer(0, scratch)
    sbuf.upload(np.zeros(scratch, np.uint8))
    for step in range(2):  # buffer 0, then buffer 1: epochs 1 and 2
        for r in range(world):
            b, c = row_shard(n1, world, r)
            assert K.matmul_q4_gather(0, up[r].view(step), b, dw1.data() + b * rb1, dx.data(), k1, c,
                                      sbuf.data(), scratch) == 0
        for r in range(world):
            b, c = row_shard(n2, world, r)
            # x of the second GEMV: the first 2048 rows of this rank's gathered up output
            assert K.matmul_q4_gather(0, dn[r].view(step), b, dw2.data() + b * rb2, up[r].output(step), k2, c,
                                      sbuf.data(), scratch, wait_for=up[r].view(step)) == 0
        for r in range(world):
            assert K.gather_wait(0, up[r].view(step)) == 0
            assert K.gather_wait(0, dn[r].view(step)) == 0
        K.select(0)
        assert K.wait() == 0
        full_up = np.concatenate([_plain(K, dw1, dx.data(), k1, row_shard(n1, world, r)[1], row_shard(n1, world, r)[0])
                                  for r in range(world)])
        for r in range(world):
            got = _download(K, up[r].output(step), n1)
            assert np.array_equal(got.view(np.uint32), full_up.view(np.uint32)), f"rank {r} up rows"
            # exchange `step` is used once here (buffer 0, then buffer 1): epoch 1 each
            assert _epoch(K, up[r].view(step)) == 1 and _epoch(K, dn[r].view(step)) == 1
            assert (_tag_epochs(K, up[r].view(step), n1) == 1).all()
            assert (_tag_epochs(K, dn[r].view(step), n2) == 1).all()
        xin = up[0].output(step)
        full_dn = np.concatenate([_plain(K, dw2, xin, k2, row_shard(n2, world, r)[1], row_shard(n2, world, r)[0])
                                  for r in range(world)])
        for r in range(world):
            got = _download(K, dn[r].output(step), n2)
            assert np.array_equal(got.view(np.uint32), full_dn.view(np.uint32)), f"rank {r} down rows"
    for xs in (up, dn):
        for e in reversed(xs):
            e.close()


def test_gather_wait_runs_out(K, gpu):
    """Words that no rank stores: the device-side wait gives up with the peer-timeout status."""
    ex = PeerExchange.on_one_device(K, 0, 64, 2)
    own = np.array([0, 1], np.uint32)  # rank 0 claims epoch 1; nobody stores words of epoch 1
    K.select(0)
    K.check(K.copy(ex[0].view(0).counter, own, 8, K.HOST_TO_DEVICE))
    assert K.gather_wait(0, ex[0].view(0)) == 0
    K.select(0)
    assert K.wait() == PEER_TIMEOUT
    # the context is still usable: a satisfied wait completes cleanly
    assert K.gather_wait(0, ex[1].view(0)) == 0
    assert K.wait() == 0
    for e in reversed(ex):
        e.close()


def test_gather_declines_unsupported_shapes(K, gpu):
    """Only the tensor-core batch-1 GEMV stores rows to peers; other shapes are declined, not rerouted."""
    assert K.matmul_q4_gather_scratch(0, 4096 + 32, 100) == 0  # K % 256 != 0
    ex = PeerExchange.on_one_device(K, 0, 128, 1)
    dw, dx, s = K.Buffer(0, 128 * 130 * 18), K.Buffer(0, 4 * 4160), K.Buffer(0, 4096)
    assert K.matmul_q4_gather(0, ex[0].view(0), 0, dw, dx, 4160, 128, s, 4096) == K.GATHER_UNSUPPORTED
    ex[0].close()


def test_gather_two_gpus(K, gpu):
    """The chain over two processes, one per GPU, with IPC-mapped peer buffers."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29561", os.path.join(ROOT, "tests", "gather_worker.py")]
    p = subprocess.run(["timeout", "-k", "30", "240"] + cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    assert p.stdout.count("gather worker ok") == 2, p.stdout[-2000:]


@pytest.mark.parametrize("wtype,k,n,batch,world", [("f16", 1024, 1025, 8, 2), ("f16", 1024, 1025, 8, 3),
                                                   ("q4_0", 1056, 999, 1, 2), ("f32", 512, 8193, 3, 2)])
def test_gather_rows_uneven_on_one_gpu(K, O, gpu, wtype, k, n, batch, world):
    """k200_gather_rows after a plain k200_matmul of each rank's rows: uneven
    splits (1025 over 2 and 3 ranks, 8193 over 2), batched outputs and a Q4_0
    shape (K % 256 != 0) the fused GEMV gather declines.  Every rank's buffer
    must hold every slice bit for bit as that slice's matmul produced it, and
    the assembled result must match the FP64 gold within the bars of the
    unsharded tests."""
    if wtype == "q4_0":
        wb = _q4(O, k, n, 0x7340D123)
        t, wt, row_bytes = K.Q4_0, O.WT_Q4_0, k // 32 * 18
    elif wtype == "f16":
        wb = O.f16(O.uniform(0x7340D123, n * k, -1.0, 1.0))
        t, wt, row_bytes = K.F16, O.WT_F16, 2 * k
    else:
        wb = O.uniform(0x7340D123, n * k, -1.0, 1.0)
        t, wt, row_bytes = K.F32, O.WT_F32, 4 * k
    x = O.uniform(0x09200ABC, k * batch, -1.0, 1.0)
    raw = np.ascontiguousarray(wb).view(np.uint8).ravel()
    dw, dx = K.Buffer(0, raw.nbytes), K.Buffer(0, x.nbytes)
    dw.upload(raw)
    dx.upload(x)
    ex = PeerExchange.on_one_device(K, 0, n, world, batch=batch)
    kern = K.Kernel()
    shards = []
    for r in range(world):
        b, c = row_shard(n, world, r)
        ys = K.Buffer(0, 4 * c * batch)
        K.matmul(kern, 0, ys, dw.data() + b * row_bytes, dx, k, c, batch, t)
        assert K.gather_rows(0, ex[r].view(0), b, ys, c, batch) == 0
        shards.append(ys)
    for r in range(world):
        assert K.gather_wait(0, ex[r].view(0)) == 0
    K.select(0)
    assert K.wait() == 0
    whole = np.empty((batch, n), np.float32)
    for r in range(world):
        b, c = row_shard(n, world, r)
        whole[:, b:b + c] = shards[r].download(np.float32, c * batch).reshape(batch, c)
    whole = whole.ravel()
    gold = O.matmul_gold(wb, wt, x, k, n, batch)
    bar = 1e-3 if (wtype == "f16" and batch >= 4) else 1e-5
    for r in range(world):
        got = _download(K, ex[r].output(0), n * batch)
        assert np.array_equal(got.view(np.uint32), whole.view(np.uint32)), f"rank {r}"
        assert _epoch(K, ex[r].view(0)) == 1 and (_tag_epochs(K, ex[r].view(0), n * batch) == 1).all()
    assert (np.abs(whole - gold) <= bar * (1 + np.abs(gold))).all()
    kern.close()
    for e in reversed(ex):
        e.close()
