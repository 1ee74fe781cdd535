"""Native and common Q4 layouts (reference k200.h:127-131,203-335).

CPU: sizes, capacity rules and reason strings, and the host packs against
the oracle's restatement and the committed golden vectors (both pinned to
the reference's own src/q4-layout.cpp and src/q4-common-pack.h).

GPU: native_q4_matmul and common_q4_matmul through the C ABI against the
oracle's restatement of the same arithmetic.  Bar: bit-exact.  The int8 x
int4 dots are exact, and every float step of the device kernels follows the
reference's association (two-component A8: kernels/native-q4/quant.h:4-10;
block partial (dot0*s0 + dot1*s1)*d summed in block order; the fallback's
8-lane kunlun-matvec model; Row A8 then dot*d summed in block order times
the row scale), so the outputs equal the oracle's bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest


def _q4(O, k, n):
    """Q4_0 rows of ceil(k/32) blocks: the reference benches' weight fixture when k % 32 == 0,
    else seeded normal weights quantised with a ragged last block (common layout only)."""
    if k % 32 == 0:
        return O.fixture_q4(k, n)
    kk = (k + 31) // 32 * 32
    return O.q4_0_quantize(O.normal(0x7340D123, n * kk, 0.0, 0.02), n, kk)


@pytest.mark.parametrize("k,n", [(96, 33), (256, 128), (4096, 100), (16384, 40)])
def test_native_size_and_pack_match_oracle(K, O, k, n):
    assert K.native_q4_layout_supported(k, n) == bool(O.native_q4_size(k, n))
    assert K.native_q4_size(k, n) == O.native_q4_size(k, n)
    q4 = _q4(O, k, n)
    assert np.array_equal(K.pack_native_q4(q4, k, n), O.pack_native_q4(q4, k, n))


def test_native_pack_matches_golden(K, golden):
    assert np.array_equal(K.pack_native_q4(golden["fx_q4_k96_n33"], 96, 33), golden["native_k96_n33"])


def test_native_capacity_and_reasons(K):
    assert not K.native_q4_layout_supported(16416, 1)          # K > 16384
    assert not K.native_q4_layout_supported(100, 1)            # K % 32
    assert not K.native_q4_layout_supported(4096, 90000000 // 4096 + 1)
    assert K.native_q4_size(100, 1) == 0
    assert K.native_q4_reason(100, 1, 1) == "K/N/layout capacity"
    assert K.native_q4_reason(4096, 4096, 2) == "batch != 1"
    assert K.native_q4_reason(4096, 4000, 1) == "rows not divisible by 128 (N64 requires 256)"
    # n*(k/32)*4 > 16 MiB ("partial capacity") needs n*k > 2^27, above the layout's 9e7 cap
    assert K.native_q4_size(16384, 90000000 // 16384) > 0
    assert K.native_q4_reason(16384, 90000000 // 16384 // 128 * 128, 1) == ""
    assert K.native_q4_reason(4096, 4096, 1) == ""
    assert K.native_q4_reason(4096, 4096, 1, K.INPUT_F16) == ""


def test_native_pack_rejects_small_or_overlapping_buffers(K, O):
    import ctypes as C
    k, n = 256, 64
    q4 = _q4(O, k, n)
    out = np.empty(K.native_q4_size(k, n) - 1, np.uint8)
    L = K.lib()
    assert L.k200_pack_native_q4(out.ctypes.data, out.nbytes, q4.ctypes.data, k, n) == 0
    big = np.zeros(K.native_q4_size(k, n) + q4.nbytes, np.uint8)
    big[: q4.nbytes] = q4
    assert L.k200_pack_native_q4(big.ctypes.data, K.native_q4_size(k, n), big.ctypes.data, k, n) == 0
    assert L.k200_pack_native_q4(None, 1 << 20, q4.ctypes.data, k, n) == 0


@pytest.mark.parametrize("k,n", [(96, 33), (300, 70), (512, 256), (4096, 100), (16384, 300)])
def test_common_size_and_pack_match_oracle(K, O, k, n):
    info = O.common_info(k, n)
    assert K.common_q4_supported(k, n)
    assert K.common_q4_size(k, n) == info["payload_bytes"]
    q4 = _q4(O, k, n)
    packed = K.common_q4_pack(q4, k, n)
    assert np.array_equal(packed, O.common_pack(q4, k, n))
    assert np.array_equal(O.common_inverse(packed, k, n), q4)


def test_common_pack_matches_golden(K, golden):
    assert np.array_equal(K.common_q4_pack(golden["fx_q4_k96_n33"], 96, 33), golden["common_k96_n33"])


def test_common_capacity(K):
    assert not K.common_q4_supported(0, 1) and not K.common_q4_supported(16385, 1)
    assert not K.common_q4_supported(64, 32001) and K.common_q4_supported(1, 32000)
    assert K.common_q4_size(64, 32001) == 0


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def _x(O, k, batch, dtype, pattern=0):
    """The reference benches' input fixture; returns (device input, its f32 values)."""
    x = O.fixture_input(k, batch, pattern)
    if dtype == 1:
        h = O.f16(x)
        return h, h.view(np.float16).astype(np.float32)
    return x, x


@pytest.mark.gpu
@pytest.mark.parametrize("k,n,dtype,pattern", [(256, 128, 0, 0), (4096, 4096, 0, 0), (4096, 11008, 0, 1),
                                               (11008, 4096, 1, 0), (1024, 384, 1, 1)])
def test_native_w4a8x2_bit_exact(K, O, gpu, k, n, dtype, pattern):
    q4 = _q4(O, k, n)
    xin, xf = _x(O, k, 1, dtype, pattern)
    dq = K.Buffer(0, K.native_q4_size(k, n))
    K.upload_native_q4(0, dq, q4, k, n)
    dx, dy = K.Buffer(0, xin.nbytes), K.Buffer(0, 4 * n)
    dx.upload(xin)
    ws = K.NativeQ4Workspace()
    assert K.native_q4_matmul(ws, 0, dy, dq, dx, k, n, 1, dtype) is True
    y = dy.download(np.float32, n)
    q0, q1, params = O.native_a8(xin, k, dtype)
    gold = O.native_q4_gemv(O.pack_native_q4(q4, k, n), k, n, q0, q1, params)
    assert np.array_equal(y.view(np.uint32), gold.view(np.uint32))
    st = ws.statistics()
    assert st["accelerated"] == 1 and st["fallback"] == 0


@pytest.mark.gpu
@pytest.mark.parametrize("k,n,batch,dtype,offset", [(4096, 4096, 2, 0, 0), (1024, 1000, 1, 1, 0),
                                                     (256, 33, 5, 0, 0), (4096, 512, 1, 0, 4)])
def test_native_exact_fallback_bit_exact(K, O, gpu, k, n, batch, dtype, offset):
    """batch > 1, N % 128 != 0, or X not 64-byte aligned: the kunlun-matvec model, bit for bit."""
    q4 = _q4(O, k, n)
    xin, xf = _x(O, k, batch, dtype)
    dq = K.Buffer(0, K.native_q4_size(k, n))
    K.upload_native_q4(0, dq, q4, k, n)
    dx, dy = K.Buffer(0, xin.nbytes + 64), K.Buffer(0, 4 * n * batch)
    K.select(0)
    K.check(K.copy(dx.data() + offset, xin, xin.nbytes, K.HOST_TO_DEVICE))
    ws = K.NativeQ4Workspace()
    assert K.native_q4_matmul(ws, 0, dy, dq, dx.data() + offset, k, n, batch, dtype) is False
    y = dy.download(np.float32, n * batch)
    gold = O.matvec_model(q4, O.WT_Q4_0, xf, k, n, batch)
    assert np.array_equal(y.view(np.uint32), gold.view(np.uint32))
    assert ws.statistics()["fallback"] == 1


@pytest.mark.gpu
@pytest.mark.parametrize("k,n,dtype,pattern", [(4096, 4096, 0, 0), (300, 1000, 0, 1), (11008, 4096, 1, 0),
                                               (96, 33, 0, 0)])
def test_common_gemv_bit_exact(K, O, gpu, k, n, dtype, pattern):
    q4 = _q4(O, k, n)
    xin, _ = _x(O, k, 1, dtype, pattern)
    wgt = K.CommonQ4Weight(0, k, n)
    wgt.upload(q4)
    info = wgt.info()
    ref_info = O.common_info(k, n)
    assert (info["abi_version"], info["quant_type"], info["layout"], info["scale_order"]) == (1, 2, 1, 1)
    assert (info["kp"], info["np"], info["payload_bytes"]) == (ref_info["kp"], ref_info["np"],
                                                               ref_info["payload_bytes"])
    dx, dy = K.Buffer(0, xin.nbytes), K.Buffer(0, 4 * n)
    dx.upload(xin)
    ws = K.CommonQ4Workspace()
    K.common_q4_matmul(ws, 0, dy, wgt, dx, 1, dtype)
    y = dy.download(np.float32, n)
    q0, q1, params = O.native_a8(xin, k, dtype)
    gold = O.common_q4_gemv(O.common_pack(q4, k, n), k, n, q0, q1, params)
    assert np.array_equal(y.view(np.uint32), gold.view(np.uint32))
    # the activation view: component c of element j at c*2*kp + (j/32)*64 + j%32
    view = ws.quantization()
    kp = info["kp"]
    assert view["components"] == 2 and view["rows"] == 1 and view["kp"] == kp
    raw = np.empty(4 * kp, np.int8)
    K.select(0)
    K.check(K.copy(raw, view["values"], raw.nbytes, K.DEVICE_TO_HOST))
    idx = (np.arange(k) // 32) * 64 + np.arange(k) % 32
    assert np.array_equal(raw[idx], q0) and np.array_equal(raw[2 * kp + idx], q1)
    st = ws.statistics()
    assert st["calls"] == 1 and st["paths"][0] == 1


@pytest.mark.gpu
@pytest.mark.parametrize("k,n,m,dtype", [(4096, 4096, 16, 0), (300, 1000, 7, 0), (2048, 3000, 128, 1),
                                         (1024, 512, 300, 0)])
def test_common_gemm_row_a8_bit_exact(K, O, gpu, k, n, m, dtype):
    q4 = _q4(O, k, n)
    xin, _ = _x(O, k, m, dtype)
    wgt = K.CommonQ4Weight(0, k, n)
    wgt.upload(q4)
    dx, dy = K.Buffer(0, xin.nbytes), K.Buffer(0, 4 * n * m)
    dx.upload(xin)
    ws = K.CommonQ4Workspace()
    K.common_q4_matmul(ws, 0, dy, wgt, dx, m, dtype)
    y = dy.download(np.float32, n * m)
    q, scales = O.row_a8(xin, m, k, dtype)
    gold = O.common_q4_gemm(O.common_pack(q4, k, n), k, n, q, scales, m)
    assert np.array_equal(y.view(np.uint32), gold.view(np.uint32))
    # the view: the last chunk of up to 128 rows, [rows][kp] int8 and one scale every 16 floats;
    # a reader may copy a whole 128-row chunk from it (bench/common-q4-bench.cpp:36-37)
    view = ws.quantization()
    first = (m - 1) // 128 * 128
    kp = wgt.info()["kp"]
    assert view["components"] == 1 and view["rows"] == m - first and view["kp"] == kp
    vq = np.empty(128 * kp, np.int8)
    vs = np.empty(128 * 16, np.float32)
    K.select(0)
    K.check(K.copy(vq, view["values"], vq.nbytes, K.DEVICE_TO_HOST))
    K.check(K.copy(vs, view["scales"], vs.nbytes, K.DEVICE_TO_HOST))
    rows = m - first
    assert np.array_equal(vq.reshape(128, kp)[:rows, :k], q.reshape(m, k)[first:])
    assert not vq.reshape(128, kp)[:rows, k:].any()
    assert np.array_equal(vs[: rows * 16: 16], scales[first:])
