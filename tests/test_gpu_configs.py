"""GPU parity at the exact BASELINE configurations (configs 2-4; configs 0 and
1 are in test_gpu_matmul.py), through kunlun::matmul via the C ABI, against
the CPU oracle on the same seeded inputs.

Each float case prints its achieved error, max |y - g| / (1 + |g|) against
library-bench's FP64 gold (bench/library-bench.cpp:121-127), so the margin to
the bar is on record (run pytest with -s to see it):
  * config 2 (Q4_0, K4096 N14336, batch 16/128/512) and config 3 f16 at
    batch 64 run on the tensor cores; config 3 f32 on the FP32 pipes;
  * config 4 (rowwise int8, K8192 N28672, batch 1/32/256) is bit-exact:
    exact int32 dots and the combine of kernels/kunlun-combine.xpu:19.
"""
from __future__ import annotations

import numpy as np
import pytest

from test_gpu_matmul import TOL, TOL_F16_TC, TOL_Q4_TC, _check_float, _device_matmul, _i8_case

pytestmark = pytest.mark.gpu


def _achieved(name, y, gold):
    rel = np.abs(y.astype(np.float64) - gold) / (1.0 + np.abs(gold))
    nmse = float(np.sum((y - gold) ** 2) / max(np.sum(gold ** 2), 1e-300))
    print(f"\nACHIEVED {name}: max|y-g|/(1+|g|) = {rel.max():.3e}  nmse = {nmse:.3e}")
    return rel.max(), nmse


@pytest.mark.parametrize("batch", [16, 128, 512])
def test_config2_q4_0_gemm(K, O, gpu, batch):
    """Config 2: Q4_0 K=4096 N=14336, W ~ N(0, 0.02) GGML-quantised, X ~ U[-1, 1]."""
    k, n = 4096, 14336
    w = O.normal(0x7340D123, n * k, 0.0, 0.02)
    q4 = O.q4_0_quantize(w, n, k)
    x = O.uniform(0x09200ABC, k * batch, -1.0, 1.0)
    y = _device_matmul(K, K.Q4_0, q4, x, k, n, batch)
    gold = O.matmul_gold(q4, O.WT_Q4_0, x, k, n, batch)
    _achieved(f"config2 q4_0 B{batch}", y, gold)
    _check_float(y, gold, tol=TOL_Q4_TC)


@pytest.mark.parametrize("wtype", ["f16", "f32"])
@pytest.mark.parametrize("n,batch", [(8192, 1), (8192, 64), (8193, 64)])
def test_config3_dense(K, O, gpu, wtype, n, batch):
    """Config 3: F16/F32 K=8192, N=8192 (and the N=8193 tail), W and X ~ U[-1, 1]."""
    k = 8192
    w = O.uniform(0x7340D123, n * k, -1.0, 1.0)
    x = O.uniform(0x09200ABC, k * batch, -1.0, 1.0)
    if wtype == "f16":
        wb, t, wt = O.f16(w), K.F16, O.WT_F16
    else:
        wb, t, wt = w, K.F32, O.WT_F32
    y = _device_matmul(K, t, wb, x, k, n, batch)
    gold = O.matmul_gold(wb, wt, x, k, n, batch)
    _achieved(f"config3 {wtype} N{n} B{batch}", y, gold)
    _check_float(y, gold, tol=TOL_F16_TC if wtype == "f16" and batch >= 4 else TOL)


@pytest.mark.parametrize("batch", [1, 32, 256])
def test_config4_rowwise_i8(K, O, gpu, batch):
    """Config 4: rowwise int8 K=8192 N=28672, W ~ N(0, 0.02), X ~ N(0, 1); bit-exact."""
    k, n = 8192, 28672
    w, x, y, packed = _i8_case(K, O, k, n, batch)
    wq, scales = O.i8_pack_rows(w, k, n)
    assert np.array_equal(packed[: k * n].view(np.int8), wq)
    off = O.aligned(k * n)
    assert np.array_equal(packed[off: off + 4 * n].view(np.uint32), scales.view(np.uint32))
    q0, q1, m0, m1 = O.a8_tensor(x)
    expect = O.i8_matmul(wq, scales, q0, q1, m0, m1, k, n, batch)
    assert np.array_equal(y.view(np.uint32), expect.view(np.uint32))
    print(f"\nACHIEVED config4 i8 B{batch}: bit-exact over {n * batch} outputs")
