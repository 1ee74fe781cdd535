"""One rank of the two-GPU check of k200_matmul_q4_gather (run by
tests/test_gpu_gather.py under torch.distributed.run; not collected by pytest).

Each rank owns one GPU, maps the other rank's exchange regions over CUDA IPC
(handles swapped through a gloo process group), and runs three chained steps
of the 7B MLP shapes: up K4096xN11008 and down K11008xN4096, each row-sharded
over the ranks, the down GEMV waiting on the device for every rank's up rows.
Every step's gathered outputs must equal, bit for bit, the concatenation of
k200_matmul on each shard computed on this GPU.
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import kunlunk200_lib_b200 as K  # noqa: E402
from kunlunk200_lib_b200.shard import PeerExchange, row_shard  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    torch.cuda.set_device(dev)
    K.select(dev)
    shapes = [(4096, 11008), (11008, 4096)]
    torch.manual_seed(0)
    qs = []
    for k, n in shapes:
        w = torch.randn(n, k, device="cuda") * 0.02
        q = torch.empty(n * k // 32 * 18, dtype=torch.uint8, device="cuda")
        K.quantize_q4_0(dev, q, w, k, n)
        qs.append(q)
    x = torch.rand(shapes[0][0], device="cuda") * 2 - 1
    K.select(dev)
    K.check(K.wait())
    torch.cuda.synchronize()

    def all_gather(obj):
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    xs = [PeerExchange.over_group(K, dev, n, world, rank, all_gather) for _, n in shapes]
    nbytes = max(K.matmul_q4_gather_scratch(dev, k, row_shard(n, world, r)[1]) for k, n in shapes for r in range(world))
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    kern = K.Kernel()

    def plain(i, xptr):
        k, n = shapes[i]
        parts = []
        for r in range(world):
            b, c = row_shard(n, world, r)
            y = torch.empty(c, device="cuda")
            K.matmul(kern, dev, y, qs[i].data_ptr() + b * (k // 32 * 18), xptr, k, c, 1, K.Q4_0)
            parts.append(y)
        K.select(dev)
        K.check(K.wait())
        return torch.cat(parts).cpu().numpy()

    def download(ptr, n):
        out = np.empty(n, np.float32)
        K.select(dev)
        K.check(K.copy(out, ptr, out.nbytes, K.DEVICE_TO_HOST))
        return out

    ok = True
    for step in range(3):
        inp = x.data_ptr()
        for i, (k, n) in enumerate(shapes):
            b, c = row_shard(n, world, rank)
            rc = K.matmul_q4_gather(dev, xs[i].view(step), b, qs[i].data_ptr() + b * (k // 32 * 18), inp, k, c,
                                    scratch.data_ptr(), nbytes, wait_for=None if i == 0 else xs[0].view(step))
            assert rc == 0, rc
            inp = xs[i].output(step)
        # the values of both exchanges as plain rows (the down GEMV read the up
        # exchange's tagged words directly)
        assert K.gather_wait(dev, xs[0].view(step)) == 0
        assert K.gather_wait(dev, xs[1].view(step)) == 0
        K.select(dev)
        status = K.wait()
        assert status == 0, hex(status)
        inp = x.data_ptr()
        for i, (k, n) in enumerate(shapes):
            want = plain(i, inp)
            got = download(xs[i].output(step), n)
            if not np.array_equal(got.view(np.uint32), want.view(np.uint32)):
                bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
                print(f"rank {rank} step {step} gemv {i}: {len(bad)} rows differ, first {bad[:8]}", flush=True)
                ok = False
            inp = xs[i].output(step)
    # k200_gather_rows across the processes: an f16 batched matmul of 1025
    # rows split 513 + 512, each slice stored into both ranks' [8][1025] outputs
    k2, n2, batch = 1024, 1025, 8
    torch.manual_seed(1)
    w2 = (torch.rand(n2, k2, device="cuda") * 2 - 1).half()
    x2 = torch.rand(batch, k2, device="cuda") * 2 - 1
    ex2 = PeerExchange.over_group(K, dev, n2, world, rank, all_gather, batch=batch)
    b2, c2 = row_shard(n2, world, rank)
    mine = torch.empty(batch, c2, device="cuda")
    K.matmul(kern, dev, mine, w2.data_ptr() + b2 * k2 * 2, x2, k2, c2, batch, K.F16)
    dist.barrier()  # both exchanges mapped and zeroed everywhere before any rank stores
    assert K.gather_rows(dev, ex2.view(0), b2, mine, c2, batch) == 0
    assert K.gather_wait(dev, ex2.view(0)) == 0
    K.select(dev)
    status = K.wait()
    assert status == 0, hex(status)
    got = download(ex2.output(0), n2 * batch).reshape(batch, n2)
    for r in range(world):
        b, c = row_shard(n2, world, r)
        ref = torch.empty(batch, c, device="cuda")
        K.matmul(kern, dev, ref, w2.data_ptr() + b * k2 * 2, x2, k2, c, batch, K.F16)
        K.select(dev)
        K.check(K.wait())
        if not np.array_equal(got[:, b:b + c].view(np.uint32), ref.cpu().numpy().view(np.uint32)):
            print(f"rank {rank}: gathered slice of rank {r} differs", flush=True)
            ok = False
    dist.barrier()  # every rank is done with the others' regions
    ex2.close()
    for e in xs:
        e.close()
    kern.close()
    dist.barrier()
    dist.destroy_process_group()
    if ok:
        print(f"gather worker ok rank {rank}", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
