"""Row gathers (reference k200.h:339-343; src/get-rows-f32.inc, src/get-rows.inc).

get_rows_f32 copies rows by index; common_q4_get_rows decodes common-Q4 weight
columns by index to F32 ((q - 8) * d, exact).  Bar: bit-exact against numpy,
and an index outside [0, n) or a contract violation returns False with the
output untouched.
"""
from __future__ import annotations

import numpy as np
import pytest

GUARD = np.uint32(0xA5B6C7D8)


def _q4_decode(raw: np.ndarray, k: int, n: int) -> np.ndarray:
    blocks = raw.reshape(n, k // 32, 18)
    d = blocks[:, :, :2].copy().view(np.float16).astype(np.float32)  # [n, k/32, 1]
    q = blocks[:, :, 2:]
    lo = (q & 15).astype(np.int32) - 8
    hi = (q >> 4).astype(np.int32) - 8
    vals = np.concatenate([lo, hi], axis=2).astype(np.float32)  # elements 0-15 low, 16-31 high
    return (vals * d).reshape(n, k)


def _device(K, nbytes):
    b = K.Buffer(0, nbytes + 256)
    return b


@pytest.mark.gpu
@pytest.mark.parametrize("k,n,rows", [(16, 3, 1), (80, 7, 3), (4096, 128, 128), (2048, 1000, 512)])
def test_get_rows_f32_bitwise(K, O, gpu, k, n, rows):
    x = O.uniform(0x7340D123, n * k, -4.0, 4.0)
    x[::17] = np.float32(np.inf)
    idx = ((np.arange(rows) * 1237 + 13) % n).astype(np.int32)
    idx[::7] = n - 1
    dx, dy, di = K.Buffer(0, x.nbytes), K.Buffer(0, rows * k * 4 + 256), K.Buffer(0, idx.nbytes)
    dx.upload(x)
    di.upload(idx)
    guard = np.full(rows * k + 64, GUARD, np.uint32)
    dy.upload(guard)
    kern = K.Kernel()
    assert K.get_rows_f32(kern, 0, dy, rows * k * 4, dx, x.nbytes, di, idx.nbytes, k, n, rows)
    y = dy.download(np.uint32, rows * k + 64)
    assert np.array_equal(y[: rows * k], x.view(np.uint32).reshape(n, k)[idx].ravel())
    assert (y[rows * k:] == GUARD).all()


@pytest.mark.gpu
@pytest.mark.parametrize("bad", [-1, "n"])
def test_get_rows_f32_invalid_index_writes_nothing(K, O, gpu, bad):
    k, n, rows = 64, 10, 5
    x = O.uniform(1, n * k)
    idx = np.arange(rows, dtype=np.int32)
    idx[3] = -1 if bad == -1 else n
    dx, dy, di = K.Buffer(0, x.nbytes), K.Buffer(0, rows * k * 4), K.Buffer(0, idx.nbytes)
    dx.upload(x)
    di.upload(idx)
    dy.upload(np.full(rows * k, GUARD, np.uint32))
    kern = K.Kernel()
    assert not K.get_rows_f32(kern, 0, dy, rows * k * 4, dx, x.nbytes, di, idx.nbytes, k, n, rows)
    assert (dy.download(np.uint32, rows * k) == GUARD).all()
    # contract violations: short output, K % 16, rows > 512, misaligned output
    idx[3] = 0
    di.upload(idx)
    assert not K.get_rows_f32(kern, 0, dy, rows * k * 4 - 1, dx, x.nbytes, di, idx.nbytes, k, n, rows)
    assert not K.get_rows_f32(kern, 0, dy, rows * k * 4, dx, x.nbytes, di, idx.nbytes, 40, n, rows)
    assert not K.get_rows_f32(kern, 0, dy, 1 << 30, dx, x.nbytes, di, 1 << 20, k, n, 513)
    assert not K.get_rows_f32(kern, 0, dy.data() + 4, rows * k * 4, dx, x.nbytes, di, idx.nbytes, k, n, rows)


@pytest.mark.gpu
@pytest.mark.parametrize("k,n,rows", [(64, 33, 1), (4096, 1000, 128), (11008, 300, 7), (16384, 40, 512)])
def test_common_q4_get_rows_bitwise(K, O, gpu, k, n, rows):
    raw = O.fixture_q4(k, n)
    wgt = K.CommonQ4Weight(0, k, n)
    wgt.upload(raw)
    idx = ((np.arange(rows) * 1237 + 13) % n).astype(np.int32)
    idx[::7] = n - 1
    idx[::5] = 0
    dy, di = K.Buffer(0, rows * k * 4 + 256), K.Buffer(0, idx.nbytes)
    di.upload(idx)
    dy.upload(np.full(rows * k + 64, GUARD, np.uint32))
    kern = K.Kernel()
    assert K.common_q4_get_rows(kern, 0, dy, rows * k * 4, wgt, di, idx.nbytes, rows)
    y = dy.download(np.float32, rows * k + 64)
    gold = _q4_decode(raw, k, n)[idx].ravel()
    assert np.array_equal(y[: rows * k].view(np.uint32), gold.view(np.uint32))
    assert (y[rows * k:].view(np.uint32) == GUARD).all()
    # an invalid index: nothing written
    idx[rows // 2] = n
    di.upload(idx)
    dy.upload(np.full(rows * k + 64, GUARD, np.uint32))
    assert not K.common_q4_get_rows(kern, 0, dy, rows * k * 4, wgt, di, idx.nbytes, rows)
    assert (dy.download(np.uint32, rows * k + 64) == GUARD).all()
