"""CPU: the C-ABI library loads, exports every declared symbol, keeps the
reference's packaging contract, and rejects contract violations the way the
reference does (abort with a diagnostic) -- all without touching a GPU."""
from __future__ import annotations

import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_c_symbols() -> set[str]:
    text = open(os.path.join(ROOT, "include", "k200_c.h")).read()
    return set(re.findall(r"\b(k200_[a-z0-9_]+)\s*\(", text))


def _exported(path: str) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_library_loads_without_gpu(K):
    assert K.version() == "0.7.12"


def test_every_c_abi_symbol_is_exported(K):
    declared = _declared_c_symbols()
    assert declared, "no declarations parsed from include/k200_c.h"
    exported = _exported(K.LIB_PATH)
    missing = declared - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    assert declared <= set(K.exported_symbols()) | declared  # python binds a subset; all must exist
    for name in K.exported_symbols():
        assert name in exported


def test_cpp_api_symbols_match_reference_mangling(K):
    """The kunlun:: hot-path API keeps the reference's Itanium-mangled names."""
    exported = _exported(K.LIB_PATH)
    expected = [
        "_ZN6kunlun13runtime_mutexEv",
        "_ZN6kunlun5checkEi",
        "_ZN6kunlun7requireEb",
        "_ZN6kunlun6selectEi",
        "_ZN6kunlun4waitEv",
        "_ZN6kunlun4copyEPvPKvmNS_8CopyKindE",
        "_ZN6kunlun4peerEiPviPKvm",
        "_ZN6kunlun8allocateEim",
        "_ZN6kunlun7releaseEiPvm",
        "_ZN6kunlun15allocated_bytesEi",
        "_ZN6kunlun12device_countEPi",
        "_ZN6kunlun17diagnostic_tensorEPKcPKl",
        "_ZN6kunlun6BufferC1Eim",
        "_ZN6kunlun6BufferD1Ev",
        "_ZN6kunlun6KernelC1Ev",
        "_ZN6kunlun6KernelD1Ev",
        "_ZN6kunlun7alignedEm",
        "_ZN6kunlun14packed_i8_sizeEii",
        "_ZN6kunlun16packed_i8_scalesEPvii",
        "_ZN6kunlun16packed_i8_maximaEPvii",
        "_ZN6kunlun14upload_i8_rowsEiPviiiiPKf",
        "_ZN6kunlun6matmulERNS_6KernelEiPvPKvS4_iiiNS_10WeightTypeEPKfS7_i",
        "_ZN6kunlun11elementwiseERNS_6KernelEiPvPKvS4_iiiNS_13ElementwiseOpEf",
        "_ZN6kunlun10statisticsEv",
        "_ZN6kunlun7versionEv",
        # native and common Q4 layouts (k200.h:127-131, 203-335)
        "_ZN6kunlun26native_q4_layout_supportedEii",
        "_ZN6kunlun14native_q4_sizeEii",
        "_ZN6kunlun14pack_native_q4EPvmPKvii",
        "_ZN6kunlun16upload_native_q4EiPvPKvii",
        "_ZN6kunlun16native_q4_reasonEiiiNS_9InputTypeE",
        "_ZN6kunlun17NativeQ4WorkspaceC1Ev",
        "_ZNK6kunlun17NativeQ4Workspace10statisticsEv",
        "_ZN6kunlun16native_q4_matmulERNS_17NativeQ4WorkspaceEiPvPKvS4_iiiNS_9InputTypeE",
        "_ZN6kunlun19common_q4_supportedEii",
        "_ZN6kunlun14common_q4_sizeEii",
        "_ZN6kunlun14CommonQ4WeightC1EiiiPvm",
        "_ZN6kunlun14CommonQ4Weight6uploadEPKvm",
        "_ZNK6kunlun14CommonQ4Weight4infoEv",
        "_ZN6kunlun17CommonQ4WorkspaceC1Ev",
        "_ZNK6kunlun17CommonQ4Workspace12quantizationEv",
        "_ZN6kunlun16common_q4_matmulERNS_17CommonQ4WorkspaceEiPvRKNS_14CommonQ4WeightEPKviNS_9InputTypeE",
        # row gathers (k200.h:339-343)
        "_ZN6kunlun12get_rows_f32ERNS_6KernelEiPvmPKvmPKimiii",
        "_ZN6kunlun18common_q4_get_rowsERNS_6KernelEiPvmRKNS_14CommonQ4WeightEPKimi",
        # activation lease and gate/up pair (k200.h:310-383)
        "_ZN6kunlun17common_q4_prepareERNS_17CommonQ4WorkspaceEiPKviiNS_9InputTypeEmRNS_23CommonQ4ActivationLeaseE",
        "_ZN6kunlun23common_q4_matmul_sharedERNS_17CommonQ4WorkspaceEiPvRKNS_14CommonQ4WeightERKNS_23CommonQ4ActivationLeaseEm",
        "_ZN6kunlun21common_q4_matmul_pairERNS_17CommonQ4WorkspaceEiPvS2_RKNS_14CommonQ4WeightES5_RKNS_23CommonQ4ActivationLeaseEm",
        "_ZN6kunlun25common_q4_pair_statisticsERKNS_17CommonQ4WorkspaceE",
        "_ZN6kunlun26common_q4_pair_last_statusERKNS_17CommonQ4WorkspaceE",
        "_ZN6kunlun23CommonQ4ActivationLeaseC1Ev",
        "_ZN6kunlun23CommonQ4ActivationLease5resetEv",
        "_ZNK6kunlun23CommonQ4ActivationLease7matchesEiiiNS_9InputTypeEm",
        "_ZNK6kunlun23CommonQ4ActivationLease6chunksEv",
        "_ZNK6kunlun23CommonQ4ActivationLease5chunkEm",
        # Q6_K typed GEMV (k200.h:135-165)
        "_ZN6kunlun14q6_k_supportedEii",
        "_ZN6kunlun9q6_k_sizeEii",
        "_ZN6kunlun9Q6KWeightC1EiiiPvm",
        "_ZN6kunlun9Q6KWeight6uploadEPKvm",
        "_ZN6kunlun12Q6KWorkspaceC1Ev",
        "_ZNK6kunlun12Q6KWorkspace12legacy_callsEv",
        "_ZN6kunlun11q6_k_matmulERNS_12Q6KWorkspaceEiPvRKNS_9Q6KWeightEPKviNS_9InputTypeE",
        # fused SwiGLU (k200.h:186-199)
        "_ZN6kunlun13swiglu_reasonERKNS_12SwiGLULayoutE",
        "_ZN6kunlun6swigluERNS_6KernelEiPvmPKvmS4_mRKNS_12SwiGLULayoutE",
    ]
    missing = [s for s in expected if s not in exported]
    assert not missing, missing


def test_soname_is_reference_packaging(K):
    out = subprocess.run(["readelf", "-d", K.LIB_PATH], capture_output=True, text=True, check=True).stdout
    assert "Library soname: [libkunlunk200.so.0]" in out


def test_reference_consumers_link_against_this_library():
    """Reference programs compiled against the reference header resolve every
    symbol from this library (built by `make -C oracle consumers`)."""
    bindir = os.path.join(ROOT, "oracle", "_ref", "bin")
    progs = [p for p in ("library-bench", "fused-bench", "native-q4-bench", "common-q4-bench",
                         "common-q4-state-bench", "get-rows-test",
                         "get-rows-f32-test", "swiglu-bench", "swiglu-contract", "q6-k-test", "memory-example")
             if os.path.exists(os.path.join(bindir, p))]
    if not progs:
        pytest.skip("reference consumer programs not built in this checkout")
    exported = _exported(os.path.join(ROOT, "kunlunk200_lib_b200", "lib", "libkunlunk200.so.0"))
    for p in progs:
        path = os.path.join(bindir, p)
        out = subprocess.run(["ldd", path], capture_output=True, text=True).stdout
        assert "libkunlunk200.so.0 =>" in out and "not found" not in out, out
        needed = subprocess.run(["nm", "-u", path], capture_output=True, text=True, check=True).stdout
        wanted = {l.split()[-1] for l in needed.splitlines() if "kunlun" in l}
        assert wanted and wanted <= exported, sorted(wanted - exported)


# a well-formed two-rank exchange view (dummy addresses) that each case then breaks
_GATHER = ("v = K.GatherView()\nv.ranks, v.rank = 2, 0\n"
           "for r in range(2):\n    v.tags[r] = 65536 * (r + 1)\n"
           "v.y = 4096\nv.counter = 1 << 20\nv.rows, v.batch = 64, 1\n")


def _run_contract(snippet: str) -> subprocess.CompletedProcess:
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "import kunlunk200_lib_b200 as K\n"
        "kern = K.Kernel()\n" % ROOT
    ) + snippet
    return subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)


@pytest.mark.parametrize(
    "case,call",
    [
        ("k not multiple of 32", "K.matmul(kern, 0, 16, 16, 16, 33, 8, 1, K.Q4_0)"),
        ("k above 16384", "K.matmul(kern, 0, 16, 16, 16, 16416, 8, 1, K.F32)"),
        ("zero batch", "K.matmul(kern, 0, 16, 16, 16, 32, 8, 0, K.F32)"),
        ("null output", "K.matmul(kern, 0, 0, 16, 16, 32, 8, 1, K.F32)"),
        ("bad tile", "K.matmul(kern, 0, 16, 16, 16, 32, 8, 1, K.F32, tile=4)"),
        ("i8 without scales", "K.matmul(kern, 0, 16, 16, 16, 32, 8, 1, K.ROWWISE_I8)"),
        ("q6_k on legacy matmul", "K.matmul(kern, 0, 16, 16, 16, 32, 8, 1, 4)"),
        ("overflowing n*batch", "K.matmul(kern, 0, 16, 16, 16, 32, 1 << 28, 4, K.F32)"),
        ("elementwise width", "K.elementwise(kern, 0, 16, 16, 16, 100, 33, 100, K.ADD)"),
        ("rms epsilon", "K.elementwise(kern, 0, 16, 16, 16, 64, 32, 64, K.RMS_NORM, 0.0)"),
        ("i8 upload bounds", "K.upload_i8_rows(0, 16, 32, 4, 3, 2, 16)"),
        ("gather without ranks", _GATHER + "v.ranks = 0\nK.matmul_q4_gather(0, v, 0, 16, 16, 4096, 16, 16, 64)"),
        ("gather rank out of range", _GATHER + "v.rank = 2\nK.matmul_q4_gather(0, v, 0, 16, 16, 4096, 16, 16, 64)"),
        ("gather null peer tags", _GATHER + "v.tags[1] = None\nK.matmul_q4_gather(0, v, 0, 16, 16, 4096, 16, 16, 64)"),
        ("gather null output", _GATHER + "v.y = None\nK.matmul_q4_gather(0, v, 0, 16, 16, 4096, 16, 16, 64)"),
        ("gather batch 2 for the GEMV", _GATHER + "v.batch = 2\nK.matmul_q4_gather(0, v, 0, 16, 16, 4096, 16, 16, 64)"),
        ("gather x outside wait_for", _GATHER + "K.matmul_q4_gather(0, v, 0, 16, 1 << 16, 4096, 16, 16, 64, "
                                                "wait_for=v)"),
        ("gather rows batch mismatch", _GATHER + "K.gather_rows(0, v, 0, 16, 16, 2)"),
        ("gather wait on a bad exchange", _GATHER + "w = K.GatherView()\n"
                                          "K.matmul_q4_gather(0, v, 0, 16, 16, 4096, 16, 16, 64, wait_for=w)"),
        ("gather negative first row", _GATHER + "K.matmul_q4_gather(0, v, -16, 16, 16, 4096, 16, 16, 64)"),
        ("gather rows past the buffer", _GATHER + "K.matmul_q4_gather(0, v, 56, 16, 16, 4096, 16, 16, 64)"),
        ("gather without a row count", _GATHER + "v.rows = 0\nK.matmul_q4_gather(0, v, 0, 16, 16, 4096, 16, 16, 64)"),
        ("gather wait without ranks", _GATHER + "v.ranks = 0\nK.gather_wait(0, v)"),
        ("gather wait without a batch", _GATHER + "v.batch = 0\nK.gather_wait(0, v)"),
    ],
)
def test_contract_violations_abort(case, call):
    """src/k200.cpp:271-277 and :283-286: invalid calls abort before any launch."""
    r = _run_contract(call)
    assert r.returncode != 0, f"{case}: call was accepted"
    assert "Kunlun invalid argument" in r.stderr, r.stderr
