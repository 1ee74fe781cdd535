"""Activation lease and gate/up pair (reference k200.h:310-383; src/q4-activation.inc,
src/q4-pair.inc).

common_q4_prepare quantises X once; common_q4_matmul_shared runs the common
GEMV/GEMM on those activations; common_q4_matmul_pair runs both weights of a
gate/up pair on one prepared row in a single pass.  Bar: bit-identical to
common_q4_matmul on the same input (the same quantisation and arithmetic),
and every decline of the reference (wrong device, stale or mismatched lease,
aliases, disabled by GGML_KUNLUN_Q4_GATE_UP_PAIR) leaves the outputs untouched.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

GUARD = np.uint32(0x7A7A7A7A)


def _weights(O, k, n, seed_shift=0):
    raw = O.fixture_q4(k, n)
    if seed_shift:
        raw = np.roll(raw.reshape(n, -1), seed_shift, axis=0).ravel().copy()
    return raw


def _plain(K, k, n, wgt, x_dev, m):
    ws = K.CommonQ4Workspace()
    y = K.Buffer(0, m * n * 4)
    K.common_q4_matmul(ws, 0, y, wgt, x_dev, m)
    return y.download(np.uint32, m * n)


@pytest.mark.gpu
@pytest.mark.parametrize("k,n,m", [(4096, 4096, 1), (300, 1000, 1), (2048, 3000, 16), (1024, 512, 300)])
def test_shared_matches_plain_matmul(K, O, gpu, k, n, m):
    kk = (k + 31) // 32 * 32
    raw = O.q4_0_quantize(O.normal(5, n * kk, 0.0, 0.02), n, kk) if k % 32 else O.fixture_q4(k, n)
    wgt = K.CommonQ4Weight(0, k, n)
    wgt.upload(raw)
    x = O.fixture_input(k, m, 1)
    dx = K.Buffer(0, x.nbytes)
    dx.upload(x)
    gold = _plain(K, k, n, wgt, dx, m)
    ws, lease = K.CommonQ4Workspace(), K.CommonQ4ActivationLease()
    assert K.common_q4_prepare(ws, 0, dx, k, m, K.INPUT_F32, 7, lease)
    assert lease.matches(0, k, m, K.INPUT_F32, 7) and not lease.matches(0, k, m, K.INPUT_F32, 8)
    assert lease.chunks() == (m + 127) // 128
    c = lease.chunk(lease.chunks() - 1)
    assert c["components"] == (2 if m == 1 else 1) and c["first"] == (m - 1) // 128 * 128
    y = K.Buffer(0, m * n * 4)
    for _ in range(2):  # a lease serves any number of consumers
        assert K.common_q4_matmul_shared(ws, 0, y, wgt, lease, 7)
        assert np.array_equal(y.download(np.uint32, m * n), gold)
    st = ws.activation_statistics()
    assert st["prepare_calls"] == 1 and st["prepared_matmuls"] == 2 and st["quant_kernel_launches"] == 1
    # a plain matmul re-quantises: the lease goes stale
    K.common_q4_matmul(ws, 0, y, wgt, dx, m)
    assert not lease.matches(0, k, m, K.INPUT_F32, 7) and lease.chunks() == 0
    assert not K.common_q4_matmul_shared(ws, 0, y, wgt, lease, 7)
    assert ws.activation_statistics()["rejected_calls"] == 1


@pytest.mark.gpu
def test_lease_reset_and_replacement(K, O, gpu):
    k, n = 512, 256
    wgt = K.CommonQ4Weight(0, k, n)
    wgt.upload(O.fixture_q4(k, n))
    x = O.fixture_input(k, 1, 0)
    dx = K.Buffer(0, x.nbytes)
    dx.upload(x)
    ws, a, b = K.CommonQ4Workspace(), K.CommonQ4ActivationLease(), K.CommonQ4ActivationLease()
    assert K.common_q4_prepare(ws, 0, dx, k, 1, K.INPUT_F32, 1, a)
    assert K.common_q4_prepare(ws, 0, dx, k, 1, K.INPUT_F32, 2, b)  # retires a
    assert not a.matches(0, k, 1, K.INPUT_F32, 1) and b.matches(0, k, 1, K.INPUT_F32, 2)
    b.reset()
    assert not b.matches(0, k, 1, K.INPUT_F32, 2)
    assert ws.activation_statistics()["invalidations"] >= 2
    # rejected descriptors: generation 0, K too large, the workspace's own buffer as input
    assert not K.common_q4_prepare(ws, 0, dx, k, 1, K.INPUT_F32, 0, a)
    assert not K.common_q4_prepare(ws, 0, dx, 16385, 1, K.INPUT_F32, 3, a)
    assert K.common_q4_prepare(ws, 0, dx, k, 1, K.INPUT_F32, 4, a)
    own = a.chunk(0)["values"]
    assert not K.common_q4_prepare(ws, 0, own, k, 1, K.INPUT_F32, 5, b)


@pytest.mark.gpu
@pytest.mark.parametrize("k,n", [(4096, 11008), (2048, 5632)])
def test_pair_matches_two_shared(K, O, gpu, k, n):
    raw0, raw1 = O.fixture_q4(k, n), _weights(O, k, n, 7)
    w0, w1 = K.CommonQ4Weight(0, k, n), K.CommonQ4Weight(0, k, n)
    w0.upload(raw0)
    w1.upload(raw1)
    x = (3.3 * np.sin(np.arange(k) * 0.071)).astype(np.float32)
    dx = K.Buffer(0, x.nbytes)
    dx.upload(x)
    ws, lease = K.CommonQ4Workspace(), K.CommonQ4ActivationLease()
    out0, out1 = K.Buffer(0, n * 4 + 512), K.Buffer(0, n * 4 + 512)
    y0, y1 = out0.data() + 256, out1.data() + 256
    guard = np.full(n + 128, GUARD, np.uint32)
    assert K.common_q4_prepare(ws, 0, dx, k, 1, K.INPUT_F32, 1, lease)
    out0.upload(guard)
    out1.upload(guard)
    assert K.common_q4_matmul_shared(ws, 0, y0, w0, lease, 1)
    assert K.common_q4_matmul_shared(ws, 0, y1, w1, lease, 1)
    gold0, gold1 = out0.download(np.uint32, n + 128), out1.download(np.uint32, n + 128)
    c = lease.chunk(0)
    qbits = np.empty(c["values_bytes"], np.uint8)
    K.select(0)
    K.check(K.copy(qbits, c["values"], qbits.nbytes, K.DEVICE_TO_HOST))
    out0.upload(guard)
    out1.upload(guard)
    assert K.common_q4_matmul_pair(ws, 0, y0, y1, w0, w1, lease, 1)
    assert K.common_q4_pair_last_status(ws) == "Success"
    assert np.array_equal(out0.download(np.uint32, n + 128), gold0)
    assert np.array_equal(out1.download(np.uint32, n + 128), gold1)
    after = np.empty_like(qbits)
    K.check(K.copy(after, c["values"], after.nbytes, K.DEVICE_TO_HOST))
    assert np.array_equal(after, qbits)  # the pair reads the prepared activations, never rewrites them
    assert K.common_q4_matmul_shared(ws, 0, y0, w0, lease, 1)  # the lease survives the pair
    st = K.common_q4_pair_statistics(ws)
    assert st["calls"] == 1 and st["declined"] == 0


@pytest.mark.gpu
def test_pair_declines(K, O, gpu, monkeypatch):
    k, n = 2048, 5632
    w0, w1 = K.CommonQ4Weight(0, k, n), K.CommonQ4Weight(0, k, n)
    w0.upload(O.fixture_q4(k, n))
    w1.upload(_weights(O, k, n, 3))
    x = O.fixture_input(k, 2, 0)
    dx = K.Buffer(0, x.nbytes)
    dx.upload(x)
    ws, lease = K.CommonQ4Workspace(), K.CommonQ4ActivationLease()
    out = K.Buffer(0, 2 * n * 4 + 512)
    y0, y1 = out.data(), out.data() + n * 4 + 256
    guard = np.full((2 * n * 4 + 512) // 4, GUARD, np.uint32)
    out.upload(guard)
    assert K.common_q4_prepare(ws, 0, dx, k, 1, K.INPUT_F32, 9, lease)

    def declined(status, *args):
        assert not K.common_q4_matmul_pair(*args)
        assert K.common_q4_pair_last_status(args[0]) == status

    for flag in ("0", "invalid"):
        monkeypatch.setenv("GGML_KUNLUN_Q4_GATE_UP_PAIR", flag)
        declined("Disabled", ws, 0, y0, y1, w0, w1, lease, 9)
    monkeypatch.setenv("GGML_KUNLUN_Q4_GATE_UP_PAIR", "1")
    declined("InvalidInput", ws, K.device_count(), y0, y1, w0, w1, lease, 9)
    declined("Lease", ws, 0, y0, y1, w0, w1, lease, 8)
    declined("Alias", ws, 0, y0, y0, w0, w1, lease, 9)
    declined("Alias", ws, 0, dx.data(), y1, w0, w1, lease, 9)
    declined("Alias", ws, 0, y0 + 4, y1, w0, w1, lease, 9)
    declined("Alias", ws, 0, y0, y1, w0, w0, lease, 9)
    declined("InvalidInput", K.CommonQ4Workspace(), 0, y0, y1, w0, w1, lease, 9)
    small = K.CommonQ4Weight(0, 1024, 512)
    small.upload(O.fixture_q4(1024, 512))
    declined("InvalidInput", ws, 0, y0, y1, small, small, lease, 9)
    # F16 and two-row leases are not pair leases; a plain matmul makes the lease stale
    hx = K.Buffer(0, k * 2)
    hx.upload(O.f16(x[:k]))
    assert K.common_q4_prepare(ws, 0, hx, k, 1, K.INPUT_F16, 10, lease)
    declined("Lease", ws, 0, y0, y1, w0, w1, lease, 10)
    assert K.common_q4_prepare(ws, 0, dx, k, 2, K.INPUT_F32, 11, lease)
    declined("Lease", ws, 0, y0, y1, w0, w1, lease, 11)
    assert K.common_q4_prepare(ws, 0, dx, k, 1, K.INPUT_F32, 12, lease)
    K.common_q4_matmul(ws, 0, K.Buffer(0, n * 4), w0, dx, 1)
    declined("Lease", ws, 0, y0, y1, w0, w1, lease, 12)
    assert (out.download(np.uint32, guard.size) == GUARD).all()  # no decline wrote anything
    st = K.common_q4_pair_statistics(ws)
    assert st["calls"] == 0 and st["declined"] == 12
