"""CPU: pin the oracle (oracle/oracle.c) to the reference's own code.

Two pins per item: the committed golden vectors (tests/golden/, produced by the
reference's sources through oracle/_ref; see make_golden.py) and, when the
reference glue library is built in this checkout, a live comparison against it
on more shapes.
"""
from __future__ import annotations

import numpy as np
import pytest


# ---- golden vectors -------------------------------------------------------
def test_fixture_weights_match_golden(O, golden):
    q4 = O.fixture_q4(96, 33)
    assert np.array_equal(q4, golden["fx_q4_k96_n33"])
    dec = O.q4_0_dequantize(q4, 33, 96)
    assert np.array_equal(dec.view(np.uint32), golden["fx_decoded_k96_n33"].view(np.uint32))


def test_native_pack_matches_golden(O, golden):
    packed = O.pack_native_q4(golden["fx_q4_k96_n33"], 96, 33)
    assert np.array_equal(packed, golden["native_k96_n33"])


@pytest.mark.parametrize("pattern", range(5))
def test_input_patterns_match_golden(O, golden, pattern):
    x = O.fixture_input(256, 2, pattern)
    assert np.array_equal(x.view(np.uint32), golden[f"input_k256_b2_p{pattern}"].view(np.uint32))


@pytest.mark.parametrize("pattern", [0, 1])
def test_native_a8_matches_reference_activation_model(O, golden, pattern):
    """kunlun-native-q4-{max,main,residual}.xpu restated == native_q4_bench::Activation."""
    x = O.fixture_input(256, 1, pattern)
    q0, q1, params = O.native_a8(x, 256, 0)
    lin = golden[f"a8_linear_p{pattern}"]
    assert np.array_equal(q0, lin[:256])
    assert np.array_equal(q1, lin[256:])
    sc = golden[f"a8_scales_p{pattern}"]
    assert params[0] == sc[0] and params[1] == sc[1]
    # the per-tensor two-pass quantiser of the rowwise-i8 matmul path
    # (src/k200.cpp:209-229) uses the same arithmetic
    a0, a1, m0, m1 = O.a8_tensor(x)
    assert np.array_equal(a0, q0) and np.array_equal(a1, q1)
    assert np.float32(m0 / np.float32(127)) == params[0]


def test_fp64_reference_matches_golden(O, golden):
    q4 = golden["fp64_q4_k256_n65"]
    x = golden["fp64_x_k256_b4"]
    w = O.q4_0_dequantize(q4, 65, 256)
    y = O.reference_fp64(w, x, 256, 65, 4, threads=1)
    assert np.array_equal(y, golden["fp64_gold_k256_n65_b4"])
    # library-bench's serial double gold agrees to rounding
    g2 = O.matmul_gold(q4, O.WT_Q4_0, x, 256, 65, 4)
    np.testing.assert_allclose(g2, y, rtol=0, atol=1e-12)


def test_common_pack_matches_golden(O, golden):
    q4 = golden["fx_q4_k96_n33"]
    packed = O.common_pack(q4, 96, 33)
    assert np.array_equal(packed, golden["common_k96_n33"])
    info = golden["common_info_k96_n33"]
    mine = O.common_info(96, 33)
    assert [mine["k"], mine["n"], mine["kp"], mine["np"], mine["scale_offset"], mine["payload_bytes"]] == list(info)
    assert np.array_equal(O.common_inverse(packed, 96, 33), q4)


# ---- live comparison against the reference glue ---------------------------
needs_ref = pytest.mark.skipif("not __import__('oracle').ref_available()",
                               reason="reference glue (oracle/_ref) not built in this checkout")


@needs_ref
@pytest.mark.parametrize("k,n", [(32, 1), (256, 65), (512, 33), (4096, 40)])
def test_live_fixture_decode_native(O, k, n):
    R = O.ref()
    q4 = np.empty(n * k // 32 * 18, np.uint8)
    dec = np.empty(n * k, np.float32)
    nat = np.empty(((n + 31) // 32 * 32) * k // 2, np.uint8)
    rs = np.empty(n, np.float32)
    R.ref_fixture(k, n, q4.ctypes.data, dec.ctypes.data, nat.ctypes.data, rs.ctypes.data)
    assert np.array_equal(O.fixture_q4(k, n), q4)
    assert np.array_equal(O.q4_0_dequantize(q4, n, k).view(np.uint32), dec.view(np.uint32))
    size = R.ref_native_q4_size(k, n)
    assert size == O.native_q4_size(k, n)
    packed = np.empty(size, np.uint8)
    assert R.ref_pack_native_q4(packed, size, q4, k, n) == 1
    assert np.array_equal(O.pack_native_q4(q4, k, n), packed)
    # the reference bench derives per-row i8 scales from the decoded weights
    _, scales = O.i8_pack_rows(dec, k, n)
    assert np.array_equal(scales.view(np.uint32), rs.view(np.uint32))


@needs_ref
@pytest.mark.parametrize("pattern", range(5))
def test_live_activation(O, pattern):
    R = O.ref()
    k = 512
    x = O.fixture_input(k, 1, pattern)
    lin = np.empty(2 * k, np.int8)
    sc = np.empty(3, np.float32)
    rep = np.empty(k, np.float32)
    R.ref_activation(x, k, 1, 8, 2, lin, sc, rep.ctypes.data)
    q0, q1, params = O.native_a8(x, k, 0)
    assert np.array_equal(q0, lin[:k]) and np.array_equal(q1, lin[k:])
    assert params[0] == sc[0] and params[1] == sc[1]


@needs_ref
@pytest.mark.parametrize("k,n", [(33, 33), (512, 512), (11008, 129), (1000, 300)])
def test_live_common_pack(O, k, n):
    R = O.ref()
    blocks = (k + 31) // 32
    raw = ((np.arange(n * blocks * 18) * 131 + (np.arange(n * blocks * 18) >> 8)) & 255).astype(np.uint8)
    import ctypes as C

    info = (C.c_longlong * 6)()
    assert R.ref_common_pack(raw, raw.size, k, n, 1, 1, None, 0, info) == 1
    payload = np.empty(info[5], np.uint8)
    assert R.ref_common_pack(raw, raw.size, k, n, 1, 1, payload.ctypes.data, payload.size, info) == 1
    assert np.array_equal(O.common_pack(raw, k, n), payload)
    assert np.array_equal(O.common_inverse(payload, k, n), raw)


# ---- restatement self-consistency -----------------------------------------
def test_half_to_float_all_patterns(O):
    """kunlun-matvec.xpu:4-18 over all 65,536 binary16 patterns vs numpy."""
    h = np.arange(65536, dtype=np.uint16)
    ours = np.array([O.half_to_float(int(v)) for v in h[::97]], np.float32)
    ref = h[::97].view(np.float16).astype(np.float32)
    same = (ours.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(ours) & np.isnan(ref))
    assert same.all()


def test_float_to_half_rne(O):
    x = O.uniform(7, 4096, -70000.0, 70000.0)
    x = np.concatenate([x, O.uniform(8, 4096, -1e-4, 1e-4), np.array([0.0, -0.0, 65504.0, 65520.0], np.float32)])
    ours = O.f16(x)
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ref)


def test_library_bench_closed_form_decodes_to_its_f32_weights(O):
    """bench/library-bench.cpp:89-100: the q4_0 bytes decode to the f32 pattern."""
    w, q = O.library_bench_weights(256, 65)
    dec = O.q4_0_dequantize(q, 65, 256)
    assert np.array_equal(dec, w)


def test_q4_0_quantizer_roundtrip_bound(O):
    """GGML Q4_0: elements decode within d/2 of their input, except those clamped
    at q = 15 (inputs near -v, for v the block's largest-magnitude element),
    which land within d."""
    w = O.normal(0x7340D123, 64 * 256, 0.0, 0.02)
    q = O.q4_0_quantize(w, 64, 256)
    dec = O.q4_0_dequantize(q, 64, 256).reshape(64, 8, 32)
    d = np.abs(np.frombuffer(q.reshape(-1, 18)[:, :2].tobytes(), np.float16).astype(np.float32)).reshape(64, 8, 1)
    err = np.abs(dec - w.reshape(64, 8, 32))
    assert (err <= d * (1 + 8 * 2.0 ** -11) + 1e-7).all()  # d itself is rounded to fp16
    assert np.mean(err <= d * (0.5 + 2.0 ** -10) + 1e-7) > 0.99


def test_i8_pack_rows_rounding(O):
    """upload_i8_rows arithmetic: round half away from zero, clamp 127, zero rows."""
    w = np.array([[0.0] * 32, [1.0] + [0.5 * 127 / 127] * 31, [-2.0, 1.0] + [0.0] * 30], np.float32)
    q, s = O.i8_pack_rows(w, 32, 3)
    q = q.reshape(3, 32)
    assert (q[0] == 0).all() and s[0] == 1.0
    assert q[1, 0] == 127 and q[1, 1] == 64  # 63.5 rounds away from zero
    assert q[2, 0] == -127 and q[2, 1] == 64 and s[2] == np.float32(2.0) / np.float32(127)


def test_i8_matmul_exact_dots(O):
    rng = np.random.default_rng(3)
    k, n, b = 128, 7, 3
    wq = rng.integers(-127, 128, n * k).astype(np.int8)
    q0 = rng.integers(-127, 128, b * k).astype(np.int8)
    q1 = rng.integers(-127, 128, b * k).astype(np.int8)
    scales = rng.random(n).astype(np.float32)
    y, p0, p1 = O.i8_matmul(wq, scales, q0, q1, 3.0, 0.25, k, n, b, want_dots=True)
    ref0 = q0.reshape(b, k).astype(np.int64) @ wq.reshape(n, k).astype(np.int64).T
    ref1 = q1.reshape(b, k).astype(np.int64) @ wq.reshape(n, k).astype(np.int64).T
    assert np.array_equal(p0.reshape(b, n), ref0) and np.array_equal(p1.reshape(b, n), ref1)
    s0, s1 = np.float32(3.0) / np.float32(127), np.float32(0.25) / np.float32(127)
    expect = ((ref0.astype(np.float32) * s0 + ref1.astype(np.float32) * s1) * scales).astype(np.float32)
    assert np.array_equal(y.reshape(b, n), expect)


def test_native_gemv_matches_fp64_within_reference_bar(O):
    """native_q4_bench's accelerated bar: NMSE < 1e-5 vs FP64 on the original x."""
    k, n = 512, 64
    q4 = O.fixture_q4(k, n)
    x = O.fixture_input(k, 1, 0)
    q0, q1, params = O.native_a8(x, k, 0)
    y = O.native_q4_gemv(O.pack_native_q4(q4, k, n), k, n, q0, q1, params)
    gold = O.reference_fp64(O.q4_0_dequantize(q4, n, k), x, k, n, 1)
    nmse = np.sum((y - gold) ** 2) / np.sum(gold ** 2)
    assert nmse < 1e-5
    # and the common-layout GEMV computes the identical values
    yc = O.common_q4_gemv(O.common_pack(q4, k, n), k, n, q0, q1, params)
    assert np.array_equal(yc, y)
