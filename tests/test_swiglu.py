"""Fused SwiGLU (reference k200.h:186-199, src/k200.cpp:324-368, kernels/kunlun-swiglu.xpu).

y = (g / (1 + exp(-g))) * u with F32 intermediates and one final rounding.
The device's expf and the host's exp may differ by an ulp, so the bar is the
reference bench's own (bench/swiglu-bench.cpp:84): NMSE < 1e-12 and max error
< 2e-5 (1 + max|ref|) for F32 (1e-6 / 2e-3 for F16), with NaN/Inf results
exactly as the reference kernel's rules give them.
"""
from __future__ import annotations

import numpy as np
import pytest


def test_swiglu_reason_contract(K):
    f32, f16 = K.INPUT_F32, K.INPUT_F16
    assert K.swiglu_reason(256, 2, 1024, 1024, 1024, f32) == ""
    assert K.swiglu_reason(256, 2, 512, 512, 512, f16) == ""
    assert K.swiglu_reason(0, 2, 1024, 1024, 1024, f32) == "shape"
    assert K.swiglu_reason(65537, 1, 1 << 20, 1 << 20, 1 << 20, f32) == "shape"
    assert K.swiglu_reason(256, 0, 1024, 1024, 1024, f32) == "shape"
    assert K.swiglu_reason(256, 2, 1023, 1024, 1024, f32) == "stride"
    assert K.swiglu_reason(256, 2, 1026, 1024, 1024, f32) == "stride"
    assert K.swiglu_reason(256, 2**20, 1 << 12, 1 << 12, 1 << 12, f32) == "byte extent"
    assert K.swiglu_reason(256, 2, 1024, 1024, 1024, 99) == "type"


def _reference(g, u):
    g = g.astype(np.float32)
    u = u.astype(np.float32)
    with np.errstate(all="ignore"):
        act = (g / (np.float32(1) + np.exp(-g.astype(np.float64)).astype(np.float32))).astype(np.float32)
        return (act * u).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("width,rows,f16,packed", [(11008, 4, False, False), (4096, 3, True, False),
                                                   (1000, 7, False, True), (257, 1, True, True)])
def test_swiglu_matches_reference(K, O, gpu, width, rows, f16, packed):
    dt = np.float16 if f16 else np.float32
    nb = 2 if f16 else 4
    g = (O.uniform(11, width * rows, -8, 8)).astype(dt).reshape(rows, width)
    u = (O.uniform(12, width * rows, -4, 4)).astype(dt).reshape(rows, width)
    g[0, :4] = np.array([0.0, -1.0, 1.0, -200.0], dt)
    kern = K.Kernel()
    if packed:
        # gate and up side by side in one row buffer, y written into the gate half (exact alias)
        buf = np.concatenate([g, u], axis=1)
        dbuf = K.Buffer(0, buf.nbytes)
        dbuf.upload(buf)
        stride = 2 * width * nb
        ok = K.swiglu(kern, 0, dbuf, buf.nbytes, dbuf, buf.nbytes, dbuf.data() + width * nb,
                      buf.nbytes - width * nb, width, rows, stride, stride, stride, int(f16))
        assert ok
        got = dbuf.download(dt, 2 * width * rows).reshape(rows, 2 * width)
        y, rest = got[:, :width], got[:, width:]
        assert np.array_equal(rest.view(np.uint16 if f16 else np.uint32), u.view(np.uint16 if f16 else np.uint32))
    else:
        dg, du, dy = K.Buffer(0, g.nbytes), K.Buffer(0, u.nbytes), K.Buffer(0, g.nbytes)
        dg.upload(g)
        du.upload(u)
        stride = width * nb
        assert K.swiglu(kern, 0, dy, g.nbytes, dg, g.nbytes, du, u.nbytes, width, rows, stride, stride, stride,
                        int(f16))
        y = dy.download(dt, width * rows).reshape(rows, width)
    ref = _reference(g, u)
    if f16:
        ref = ref.astype(np.float16).astype(np.float32)
    y = y.astype(np.float32)
    d = y.astype(np.float64) - ref
    nmse = np.sum(d * d) / np.sum(ref.astype(np.float64) ** 2)
    assert nmse < (1e-6 if f16 else 1e-12)
    assert np.abs(d).max() < (2e-3 if f16 else 2e-5) * (1 + np.abs(ref).max())


@pytest.mark.gpu
def test_swiglu_special_values(K, gpu):
    inf, nan = np.float32(np.inf), np.float32(np.nan)
    g = np.array([0.0, -0.0, 1.0, -1.0, -200.0, inf, -inf, 1.0, inf, nan, 2.0, 0.0], np.float32)
    u = np.array([inf, -inf, inf, inf, inf, 0.0, 0.0, nan, 2.0, 1.0, 0.0, 3.0], np.float32)
    n = g.size
    dg, du, dy = K.Buffer(0, 4 * n), K.Buffer(0, 4 * n), K.Buffer(0, 4 * n)
    dg.upload(g)
    du.upload(u)
    assert K.swiglu(K.Kernel(), 0, dy, 4 * n, dg, 4 * n, du, 4 * n, n, 1, 4 * n, 4 * n, 4 * n)
    y = dy.download(np.float32, n)
    # SiLU(g) = 0 times an infinite u, -inf gate, NaN operands, inf gate times 0: NaN;
    # a nonzero SiLU(g) times +-inf, or +inf gate times nonzero u: the product's infinity
    expect_nan = [True, True, False, False, True, True, True, True, False, True, False, False]
    assert list(np.isnan(y)) == expect_nan
    assert y[2] == inf and y[3] == -inf and y[8] == inf and y[10] == 0.0 and y[11] == 0.0


@pytest.mark.gpu
def test_swiglu_rejects_partial_alias(K, gpu):
    width = 256
    buf = K.Buffer(0, 3 * width * 4)
    kern = K.Kernel()
    # y overlaps gate by half a row: rejected before any work
    assert not K.swiglu(kern, 0, buf.data() + 512, width * 4, buf, width * 4, buf.data() + 2048, width * 4, width, 1,
                        width * 4, width * 4, width * 4)
