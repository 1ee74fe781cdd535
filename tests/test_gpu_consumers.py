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


def test_peer_same_device(K, gpu):
    """kunlun::peer (src/k200.cpp:89-95) with source and destination on one
    device: the bytes arrive, the call completes before returning, and the
    peer counters of Statistics move (src/k200.cpp:94, k200.h:345-350)."""
    import numpy as np

    nbytes = (1 << 20) + 48
    data = (np.arange(nbytes, dtype=np.uint64) * 2654435761 % 251).astype(np.uint8)
    src, dst = K.Buffer(0, nbytes), K.Buffer(0, nbytes)
    src.upload(data)
    before = K.statistics()
    K.peer(0, dst.data(), 0, src.data(), nbytes)
    assert np.array_equal(dst.download(np.uint8, nbytes), data)
    after = K.statistics()
    assert after["peer_copies"] == before["peer_copies"] + 1
    assert after["peer_bytes"] == before["peer_bytes"] + nbytes


def test_fused_bench(K, gpu):
    """bench/fused-bench.cpp: direct q4_0 within 1e-3(1+|ref|), fused vs two-FC i8 NMSE <= 1e-8."""
    out = _run("fused-bench", 0, 4096, 4096, 1)
    assert out.count("PASS") == 3, out


def test_memory_example(K, gpu):
    out = _run("memory-example")
    assert "PASS" in out


def test_cmake_package_consumer(K, gpu):
    """The reference's examples/library project, configured unchanged with
    find_package(KunlunK200) against this repository's CMake install
    (`make -C oracle cmake-consumer`), runs against that installed library."""
    out = _run("cmake-consumer")
    assert "KunlunK200 0.7.12: PASS" in out, out


# bench/native-q4-bench.cpp: mode PD K N batch dtype pattern trials.  The
# program requires NMSE < 1e-5 (W4A8x2 path), < 1e-10 (exact fallback) or
# < 1e-2 (cdnn) against its FP64 reference, and re-checks the native pack
# byte by byte (its lines 40-47).
NATIVE = [
    ("native", 0, 4096, 4096, 1, "f32", 0, 3),
    ("native", 0, 4096, 11008, 1, "f32", 1, 3),
    ("native", 0, 11008, 4096, 1, "f16", 0, 3),
    ("native", 0, 4096, 4096, 2, "f32", 0, 3),    # batch 2: exact fallback
    ("native", 0, 1024, 1000, 1, "f16", 4, 3),    # N % 128 != 0: exact fallback
    ("direct", 0, 4096, 4096, 1, "f32", 0, 3),
    ("cdnn", 0, 4096, 4096, 1, "f32", 0, 3),
]


@pytest.mark.parametrize("args", NATIVE, ids=lambda a: "-".join(map(str, a)))
def test_native_q4_bench(K, gpu, args):
    out = _run("native-q4-bench", *args)
    assert "RESULT mode=" + args[0] in out, out
    expect_accelerated = args[0] == "native" and args[4] == 1 and args[3] % 128 == 0
    if args[0] == "native":
        assert f"accelerated={int(expect_accelerated)}" in out, out


# bench/common-q4-bench.cpp: PD K N M dtype pattern trials common.  The
# program requires implementation NMSE <= 1e-10 against the activations the
# workspace's quantisation view reports, and checks the call and upload counts.
COMMON = [
    (0, 4096, 4096, 1, "f32", 0, 3, "common"),
    (0, 4096, 11008, 1, "f16", 1, 3, "common"),
    (0, 300, 1000, 1, "f32", 0, 3, "common"),      # K and N off the 256 padding
    (0, 4096, 4096, 16, "f32", 0, 3, "common"),
    (0, 2048, 3000, 128, "f16", 4, 3, "common"),
    (0, 1024, 512, 300, "f32", 1, 3, "common"),    # three 128-row chunks
]


@pytest.mark.parametrize("args", COMMON, ids=lambda a: "-".join(map(str, a)))
def test_common_q4_bench(K, gpu, args):
    out = _run("common-q4-bench", *args)
    assert '"correct":true' in out, out


# bench/get-rows-f32-test.cpp: PD.  Bitwise row copies for K in {16, 80, 2048,
# 4096} and M in {1, 3, 128, 512}, guard words around the output, indices -1 and
# N rejected without a write, and short buffers rejected.
def test_get_rows_f32_test(K, gpu):
    out = _run("get-rows-f32-test", 0)
    assert "F32_ROWS" in out and "bitwise=1" in out, out


# bench/get-rows-test.cpp: FILE OFFSET K N PD TIMING.  Decodes common-Q4 weight
# columns by index and compares them bit for bit with its own Q4_0 decode of
# the raw blocks read from FILE at OFFSET; invalid indices must write nothing.
@pytest.mark.parametrize("k,n", [(4096, 1000), (256, 33)])
def test_get_rows_test(K, O, gpu, tmp_path, k, n):
    raw = O.fixture_q4(k, n)
    path = tmp_path / "weights.q4"
    path.write_bytes(b"\0" * 96 + raw.tobytes())
    out = _run("get-rows-test", str(path), 96, k, n, 0, 0)
    assert "GET_ROWS_UNIT_PASS invalid_ids_rejected=1" in out, out
    assert out.count("bitwise=1") == 4, out


# bench/swiglu-contract.cpp: eleven malformed calls rejected before any device
# work or allocation.
def test_swiglu_contract(K, gpu):
    out = _run("swiglu-contract")
    assert out.count("rejected_before_device=1 PASS") == 11, out


# bench/swiglu-bench.cpp: PD WIDTH ROWS BYTES PATTERN PACKED GAP ALIAS; its own
# bar (NMSE, max error, NaN/Inf rules, untouched padding) prints pass=1.
@pytest.mark.parametrize("args", [(0, 11008, 128, 4, 0, 0, 0, 0), (0, 11008, 16, 2, 0, 0, 0, 0),
                                  (0, 4096, 8, 4, 4, 0, 0, 0), (0, 4096, 8, 4, 5, 0, 0, 0),
                                  (0, 1000, 5, 4, 2, 1, 0, 1), (0, 1000, 5, 2, 3, 1, 64, 2),
                                  (0, 777, 3, 4, 0, 0, 32, 1)],
                         ids=lambda a: "-".join(map(str, a)))
def test_swiglu_bench(K, gpu, args):
    out = _run("swiglu-bench", *args)
    assert "pass=1" in out, out


# bench/common-q4-state-bench.cpp: PD F16.  80 calls on one workspace over
# M in {1, 8, 32, 64, 128, 129, 256}: outputs equal those of fresh workspaces,
# the weight pointer and device allocation stay put after the first round.
@pytest.mark.parametrize("f16", [0, 1])
def test_common_q4_state_bench(K, gpu, f16):
    out = _run("common-q4-state-bench", 0, f16)
    assert '"correct":true' in out and '"stable_hbm":true' in out, out


# bench/q6-k-test.cpp: FILE OFFSET K N PD.  Implementation NMSE < 1e-10 against
# its FP64 restatement over the chunk-256 A8 activations, repeat runs bitwise
# equal, zero input gives zero output, and guards untouched.
@pytest.mark.parametrize("k,n", [(4096, 4096), (256, 32), (2048, 11008)])
def test_q6_k_test(K, gpu, tmp_path, k, n):
    from test_q6_k import q6_blocks
    path = tmp_path / "weights.q6k"
    path.write_bytes(b"\0" * 32 + q6_blocks(7, k, n).tobytes())
    out = _run("q6-k-test", str(path), 32, k, n, 0)
    assert "Q6_STANDALONE_PASS" in out and "Q6_CHUNK_SCALE_PASS" in out, out

