"""k200_graph_*: a decode step (host input copied in, two chained batch-1
Q4_0 GEMVs, output copied back) recorded once through the C ABI and replayed;
each replay must equal the same calls run directly, and must pick up new
contents of the pinned host input buffer.  The copies are copy-engine
transfers (k200_copy_async) or kernels (k200_copy_kernel)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kernel_copies", [False, True])
def test_graph_replays_decode_step(K, O, gpu, kernel_copies):
    import torch

    k1, n1 = 1024, 2048      # up: K1 -> N1
    k2, n2 = n1, 512         # down: N1 -> N2
    w1 = O.q4_0_quantize(O.normal(1, n1 * k1, 0.0, 0.02), n1, k1)
    w2 = O.q4_0_quantize(O.normal(2, n2 * k2, 0.0, 0.02), n2, k2)
    dw1, dw2 = K.Buffer(0, w1.nbytes), K.Buffer(0, w2.nbytes)
    dw1.upload(w1)
    dw2.upload(w2)
    dx, dh, dy = K.Buffer(0, 4 * k1), K.Buffer(0, 4 * n1), K.Buffer(0, 4 * n2)
    xh = torch.empty(k1, dtype=torch.float32).pin_memory()
    yh = torch.empty(n2, dtype=torch.float32).pin_memory()
    kern = K.Kernel()

    def step():
        if kernel_copies:  # k200_copy_kernel: pinned host memory read / written by a kernel
            K.check(K.copy_kernel(dx.data(), xh.data_ptr(), 4 * k1))
        else:
            K.check(K.copy_async(dx.data(), xh.data_ptr(), 4 * k1, K.HOST_TO_DEVICE))
        K.matmul(kern, 0, dh, dw1, dx, k1, n1, 1, K.Q4_0)
        K.matmul(kern, 0, dy, dw2, dh, k2, n2, 1, K.Q4_0)
        if kernel_copies:
            K.check(K.copy_kernel(yh.data_ptr(), dy.data(), 4 * n2))
        else:
            K.check(K.copy_async(yh.data_ptr(), dy.data(), 4 * n2, K.DEVICE_TO_HOST))

    x0 = O.uniform(3, k1, -1.0, 1.0)
    xh.copy_(torch.from_numpy(x0))
    K.select(0)
    step()  # direct run: also grows the Kernel's scratch before recording
    K.check(K.wait())
    direct = yh.numpy().copy()
    before = K.matmul_count(0)
    g = K.Graph(0)
    with g:
        step()
    assert K.matmul_count(0) == before + 2  # recording counts the calls once
    yh.zero_()
    g.launch()
    K.select(0)
    K.check(K.wait())
    assert np.array_equal(yh.numpy().view(np.uint32), direct.view(np.uint32))
    # new input in the same pinned buffer: the replay reads it
    x1 = O.uniform(4, k1, -2.0, 2.0)
    xh.copy_(torch.from_numpy(x1))
    g.launch()
    K.select(0)
    K.check(K.wait())
    replayed = yh.numpy().copy()
    step()
    K.check(K.wait())
    assert np.array_equal(replayed.view(np.uint32), yh.numpy().view(np.uint32))
    assert not np.array_equal(replayed, direct)
    g.close()
    kern.close()
