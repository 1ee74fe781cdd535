"""Q6_K typed GEMV (reference k200.h:135-165, src/q6-k.inc, kernels/kunlun-q6-*.xpu).

Activations are quantised per 256-value chunk (symmetric A8), weights are the
GGML Q6_K values (q - 32) with one f32 scale d * sub-scale per 16 values, and
each group's int8 dot is exact.  The restatement below follows the device's
order (dot * activation scale * weight scale, summed over groups in order,
FP32 round-to-nearest), so the bar is bit-exact; the reference's own bars
(bench/q6-k-test.cpp) run in tests/test_gpu_consumers.py.
"""
from __future__ import annotations

import numpy as np
import pytest


def q6_blocks(seed: int, k: int, n: int) -> np.ndarray:
    """Random GGML Q6_K rows: ql, qh and int8 sub-scales uniform, fp16 d finite and small."""
    rng = np.random.default_rng(seed)
    blocks = rng.integers(0, 256, size=(n, k // 256, 210), dtype=np.uint8)
    d = (rng.uniform(0.5, 2.0, size=(n, k // 256)) * 1e-3).astype(np.float16)
    blocks[:, :, 208:210] = d.view(np.uint8).reshape(n, k // 256, 2)
    return blocks.reshape(-1)


def q6_decode(raw: np.ndarray, k: int, n: int):
    """(values [n, k] int (q - 32), scales [n, k/16] f32 = d * sub-scale)."""
    b = raw.reshape(n, k // 256, 210)
    p = np.arange(256)
    half, l, lane = p // 128, p % 32, p % 128 // 32
    lo = half * 64 + l + (lane % 2) * 32
    ql = b[:, :, lo].astype(np.int32)
    nib = np.where(lane < 2, ql & 15, ql >> 4)
    qh = (b[:, :, 128 + half * 32 + l].astype(np.int32) >> (lane * 2)) & 3
    vals = (nib | (qh << 4)) - 32
    d = b[:, :, 208:210].copy().view(np.float16).astype(np.float32)  # [n, k/256, 1]
    sub = b[:, :, 192:208].view(np.int8).astype(np.float32)          # [n, k/256, 16]
    return vals.reshape(n, k), (d * sub).astype(np.float32).reshape(n, k // 16)


def a8_chunks(x: np.ndarray):
    c = x.reshape(-1, 256).astype(np.float32)
    mx = np.abs(c).max(axis=1)
    inv = np.where(mx > 0, np.float32(127) / np.where(mx > 0, mx, 1), 0).astype(np.float32)
    t = (c * inv[:, None]).astype(np.float32)
    z = np.trunc((t + np.where(t >= 0, np.float32(0.5), np.float32(-0.5))).astype(np.float32))
    q = np.clip(z, -127, 127).astype(np.int32)
    scale = np.where(mx > 0, (mx / np.float32(127)).astype(np.float32), 0).astype(np.float32)
    return q.reshape(-1), scale


def q6_gemv_gold(raw, k, n, x):
    vals, wscale = q6_decode(raw, k, n)
    q, ascale = a8_chunks(x)
    dots = (vals.reshape(n, k // 16, 16) * q.reshape(k // 16, 16)[None]).sum(axis=2).astype(np.float32)
    acc = np.zeros(n, np.float32)
    for g in range(k // 16):
        term = (dots[:, g] * ascale[g // 16]).astype(np.float32) * wscale[:, g]
        acc = (acc + term.astype(np.float32)).astype(np.float32)
    return acc


def test_q6_sizes(K):
    assert K.q6_k_supported(256, 32) and K.q6_k_supported(4096, 32000)
    assert not K.q6_k_supported(4352, 32) and not K.q6_k_supported(256, 33) and not K.q6_k_supported(128, 32)
    assert K.q6_k_size(4096, 4096) == 4096 * 4096 + 256 * 4096 * 4
    assert K.q6_k_size(256, 33) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("k,n,m", [(256, 32, 1), (4096, 4096, 1), (1024, 32000, 2), (2048, 96, 5)])
def test_q6_k_bit_exact(K, O, gpu, k, n, m):
    raw = q6_blocks(k + n, k, n)
    wgt = K.Q6KWeight(0, k, n)
    wgt.upload(raw)
    x = (np.sin(np.arange(k * m) * 0.123) * 0.4).astype(np.float32)
    x[:256] = 0.0  # an all-zero chunk
    dx, dy = K.Buffer(0, x.nbytes), K.Buffer(0, m * n * 4)
    dx.upload(x)
    ws = K.Q6KWorkspace()
    K.q6_k_matmul(ws, 0, dy, wgt, dx, m)
    y = dy.download(np.float32, m * n).reshape(m, n)
    for r in range(m):
        gold = q6_gemv_gold(raw, k, n, x[r * k:(r + 1) * k])
        assert np.array_equal(y[r].view(np.uint32), gold.view(np.uint32))
    assert ws.statistics()["calls"] == m
