"""GPU: the reference's own consumer programs, compiled against the reference
header and linked against this library (oracle/_ref/bin, built by
`make -C oracle consumers`), run unchanged and pass their own checks.

The case list is the reference's hardware smoke list, tools/verify.sh:12-21,
plus bench/fused-bench.cpp at its defaults.  The 2-device `memory` case needs
two visible GPUs.
"""
from __future__ import annotations

import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref", "bin")


def _run(prog, *args, timeout=300):
    path = os.path.join(BIN, prog)
    if not os.path.exists(path):
        pytest.fail(f"{path} missing: build with `make -C oracle consumers REF=<reference>` before shipping")
    r = subprocess.run([path, *map(str, args)], capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, f"{prog} {args} exited {r.returncode}\n{r.stdout}\n{r.stderr}"
    return r.stdout


VERIFY = (
    [("matmul", t, 0, 256, 65, 4) for t in ("f32", "f16", "q4_0", "i8")]
    + [("pipeline", t, 0, 256, 65, 4) for t in ("f32", "f16", "q4_0", "i8")]
    + [(op, "f32", 0) for op in ("add", "multiply", "silu", "rms", "scale")]
    + [("matmul", "q4_0", 0, 4096, 4096, 1), ("matmul", "i8", 0, 4096, 4096, 1)]
)


@pytest.mark.parametrize("args", VERIFY, ids=lambda a: "-".join(map(str, a)))
def test_library_bench_verify_list(K, gpu, args):
    out = _run("library-bench", *args)
    assert "PASS" in out, out


def test_library_bench_memory(K, gpu):
    if K.device_count() < 2:
        pytest.skip("the reference's memory test copies between two devices")
    out = _run("library-bench", "memory", "f32", 0)
    assert "PASS" in out


def test_fused_bench(K, gpu):
    """bench/fused-bench.cpp: direct q4_0 within 1e-3(1+|ref|), fused vs two-FC i8 NMSE <= 1e-8."""
    out = _run("fused-bench", 0, 4096, 4096, 1)
    assert out.count("PASS") == 3, out


def test_memory_example(K, gpu):
    out = _run("memory-example")
    assert "PASS" in out
