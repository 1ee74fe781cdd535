"""k200_matmul_i8_noalloc: the rowwise-int8 matmul on the library's static
scratch, checked against k200_matmul (the Kernel-scratch entry point) and the
CPU oracle.

The file is named to be collected last, so that in a full run the static
scratch is used after every other test has exercised the library; it must
pass equally when run alone in a fresh process.  Bar: bit-exact, the
rowwise-int8 bar of the other parity tests (exact int32 dots and the combine
formula of kernels/kunlun-combine.xpu:19).
"""
from __future__ import annotations

import os

import numpy as np
import pytest


def _packed_weights(K, O, k, n, seed):
    w = O.normal(seed, n * k, 0.0, 0.02)
    dw = K.Buffer(0, K.packed_i8_size(k, n))
    K.upload_i8_rows(0, dw, k, n, 0, n, w)
    return w, dw


def _kernel_matmul(K, dw, x, k, n, batch):
    """Y through k200_matmul (Kernel-owned scratch)."""
    dx = K.Buffer(0, x.nbytes)
    dx.upload(x)
    dy = K.Buffer(0, 4 * n * batch)
    kern = K.Kernel()
    K.matmul(kern, 0, dy, dw, dx, k, n, batch, K.ROWWISE_I8, K.packed_i8_scales(dw, k, n),
             K.packed_i8_maxima(dw, k, n))
    K.select(0)
    K.check(K.wait())
    y = dy.download(np.float32, n * batch)
    kern.close()
    return y


# (k, n, batch): batch*k = 1024 takes the single-CTA activation quantiser;
# 262144 the three-pass one whose reduction words must be cleared per call;
# 2097152 is the static limit exactly.
@pytest.mark.gpu
@pytest.mark.parametrize("k,n,batch", [(256, 65, 4), (8192, 512, 32), (16384, 96, 128)])
def test_noalloc_matches_kernel_entry_point(K, O, gpu, k, n, batch):
    w, dw = _packed_weights(K, O, k, n, 0x7340D123)
    # two calls in a row; the second input has a far smaller range, so
    # maxima left over from the first call would change its result
    xs = [O.normal(0x09200ABC, k * batch, 0.0, 1.0), O.normal(0x1234567, k * batch, 0.0, 1e-3)]
    wq, scales = O.i8_pack_rows(w, k, n)
    dx = K.Buffer(0, xs[0].nbytes)
    dy = K.Buffer(0, 4 * n * batch)
    for x in xs:
        expect = _kernel_matmul(K, dw, x, k, n, batch)
        dx.upload(x)
        K.select(0)
        before = K.allocated_bytes(0)
        rc = K.matmul_i8_noalloc(0, dy, dw, dx, k, n, batch, K.packed_i8_scales(dw, k, n),
                                 K.packed_i8_maxima(dw, k, n))
        assert rc == 0
        K.select(0)
        K.check(K.wait())
        assert K.allocated_bytes(0) == before
        y = dy.download(np.float32, n * batch)
        assert np.array_equal(y.view(np.uint32), expect.view(np.uint32))
        if batch * k <= 262144:
            q0, q1, m0, m1 = O.a8_tensor(x)
            oracle = O.i8_matmul(wq, scales, q0, q1, m0, m1, k, n, batch)
            assert np.array_equal(y.view(np.uint32), oracle.view(np.uint32))


_FRESH_PROCESS = r"""
import sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
import kunlunk200_lib_b200 as K
import oracle as O

k, n, batch = 1024, 256, 8
K.select(0)  # device set-up: stream, error word, and the static scratch's module
w = O.normal(0x7340D123, n * k, 0.0, 0.02)
x = O.normal(0x09200ABC, k * batch, 0.0, 1.0)
dw = K.Buffer(0, K.packed_i8_size(k, n))
K.upload_i8_rows(0, dw, k, n, 0, n, w)
dx, dy = K.Buffer(0, x.nbytes), K.Buffer(0, 4 * n * batch)
dx.upload(x)
# k200_matmul loads the quantiser and GEMM kernels the noalloc call also runs
kern = K.Kernel()
K.matmul(kern, 0, dy, dw, dx, k, n, batch, K.ROWWISE_I8, K.packed_i8_scales(dw, k, n), K.packed_i8_maxima(dw, k, n))
K.select(0)
K.check(K.wait())
expect = dy.download(np.float32, n * batch)
torch.cuda.mem_get_info(0)
free_before = torch.cuda.mem_get_info(0)[0]
rc = K.matmul_i8_noalloc(0, dy, dw, dx, k, n, batch, K.packed_i8_scales(dw, k, n), K.packed_i8_maxima(dw, k, n))
K.select(0)
K.check(K.wait())
free_after = torch.cuda.mem_get_info(0)[0]
y = dy.download(np.float32, n * batch)
assert rc == 0, rc
assert np.array_equal(y.view(np.uint32), expect.view(np.uint32))
print("FREE_DROP", free_before - free_after)
kern.close()
"""


@pytest.mark.gpu
def test_noalloc_first_call_takes_no_device_memory(K, gpu, tmp_path):
    """In a fresh process, the first allocation-free call must not make CUDA
    load the module that holds the static array (4 MiB): device free memory
    stays put across it, because k200_select already loaded it.  A drop of
    1 MiB or more would mean a device allocation inside the call."""
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = tmp_path / "fresh_noalloc.py"
    script.write_text(_FRESH_PROCESS)
    res = subprocess.run([sys.executable, str(script), root], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    drop = int(res.stdout.split("FREE_DROP")[1].split()[0])
    assert drop < (1 << 20), f"device free memory fell by {drop} bytes during the first noalloc call"


@pytest.mark.gpu
def test_noalloc_honours_tensor_core_switch(K, O, gpu):
    """KUNLUN_TC=0 (read at device set-up) selects the streaming kernels for both
    entry points; checked in a fresh process so the switch is seen, against
    the oracle, bit for bit."""
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import kunlunk200_lib_b200 as K
import oracle as O
k, n, batch = 512, 96, 16
K.select(0)
w = O.normal(5, n * k, 0.0, 0.02)
x = O.normal(6, k * batch, 0.0, 1.0)
dw = K.Buffer(0, K.packed_i8_size(k, n))
K.upload_i8_rows(0, dw, k, n, 0, n, w)
dx, dy = K.Buffer(0, x.nbytes), K.Buffer(0, 4 * n * batch)
dx.upload(x)
assert K.matmul_i8_noalloc(0, dy, dw, dx, k, n, batch, K.packed_i8_scales(dw, k, n), K.packed_i8_maxima(dw, k, n)) == 0
K.select(0)
K.check(K.wait())
y = dy.download(np.float32, n * batch)
wq, s = O.i8_pack_rows(w, k, n)
q0, q1, m0, m1 = O.a8_tensor(x)
assert np.array_equal(y.view(np.uint32), O.i8_matmul(wq, s, q0, q1, m0, m1, k, n, batch).view(np.uint32))
print("OK")
"""
    env = dict(os.environ, KUNLUN_TC="0")
    res = subprocess.run([sys.executable, "-c", code, root], capture_output=True, text=True, timeout=300, env=env)
    assert res.returncode == 0 and "OK" in res.stdout, res.stdout + res.stderr


def test_noalloc_rejects_oversize_before_any_device_work(K):
    """batch*k above the static limit is refused with a status, before any CUDA call
    (null pointers are never touched, so this runs without a GPU)."""
    k, batch = 16384, 129
    assert k * batch > K.NOALLOC_MAX_ELEMENTS
    rc = K.matmul_i8_noalloc(0, None, None, None, k, 64, batch, None, None)
    assert rc == K.NOALLOC_TOO_LARGE
