"""CPU oracle for the k200 matmul hot path -- TEST INFRASTRUCTURE ONLY.

ctypes/numpy front end of ``oracle/liboracle.so`` (the plain-C restatement in
``oracle/oracle.c``) and, when it was built, of ``oracle/_ref/libk200ref.so``
(the reference's own CPU sources compiled where they lie; see the Makefile).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this package, and only as the checker or the timed CPU baseline.
The product library never loads it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libk200ref.so")

_lib = None
_ref = None

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def build(ref: str | None = None) -> None:
    """Compile liboracle.so (and the reference glue when ``ref`` is given)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref and os.path.isdir(ref):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref}"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        sig = {
            "ko_fill_uniform": (None, [C.c_uint32, f32p, C.c_size_t, C.c_float, C.c_float]),
            "ko_fill_normal": (None, [C.c_uint32, f32p, C.c_size_t, C.c_float, C.c_float]),
            "ko_fixture_q4": (None, [C.c_int, C.c_int, u8p]),
            "ko_fixture_input": (None, [C.c_int, C.c_int, C.c_int, f32p]),
            "ko_library_bench_weights": (None, [C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
            "ko_library_bench_input": (None, [C.c_int, C.c_int, f32p]),
            "ko_half_to_float": (C.c_float, [C.c_uint16]),
            "ko_float_to_half": (C.c_uint16, [C.c_float]),
            "ko_f32_to_f16": (None, [f32p, u16p, C.c_size_t]),
            "ko_q4_0_quantize": (None, [f32p, C.c_int, C.c_int, u8p]),
            "ko_q4_0_dequantize": (None, [u8p, C.c_int, C.c_int, f32p]),
            "ko_matmul_gold": (None, [C.c_void_p, C.c_int, f32p, C.c_int, C.c_int, C.c_int, f64p]),
            "ko_matvec_model": (None, [C.c_void_p, C.c_int, f32p, C.c_int, C.c_int, C.c_int, f32p]),
            "ko_reference_fp64": (None, [f32p, f32p, C.c_int, C.c_int, C.c_int, f64p, C.c_int]),
            "ko_q4_gemv_fp64": (None, [u8p, f32p, C.c_int, C.c_int, C.c_int, f32p, C.c_int]),
            "ko_aligned": (C.c_size_t, [C.c_size_t]),
            "ko_packed_i8_size": (C.c_size_t, [C.c_int, C.c_int]),
            "ko_i8_pack_rows": (C.c_int, [f32p, C.c_int, C.c_int, i8p, f32p]),
            "ko_a8_tensor": (C.c_int, [f32p, C.c_size_t, i8p, i8p, C.POINTER(C.c_float), C.POINTER(C.c_float)]),
            "ko_i8_matmul": (None, [i8p, f32p, i8p, i8p, C.c_float, C.c_float, C.c_int, C.c_int, C.c_int,
                                    f32p, C.c_void_p, C.c_void_p]),
            "ko_native_q4_supported": (C.c_int, [C.c_int, C.c_int]),
            "ko_native_q4_size": (C.c_size_t, [C.c_int, C.c_int]),
            "ko_pack_native_q4": (C.c_int, [u8p, C.c_size_t, u8p, C.c_int, C.c_int]),
            "ko_native_a8": (None, [C.c_void_p, C.c_int, C.c_int, i8p, i8p, f32p]),
            "ko_native_q4_gemv": (None, [u8p, C.c_int, C.c_int, i8p, i8p, f32p, f32p]),
            "ko_common_pack": (C.c_int, [u8p, C.c_size_t, C.c_int, C.c_int, u8p]),
            "ko_common_inverse": (C.c_int, [u8p, C.c_int, C.c_int, u8p]),
            "ko_common_q4_gemv": (None, [u8p, C.c_int, C.c_int, i8p, i8p, f32p, f32p]),
            "ko_row_a8": (None, [C.c_void_p, C.c_int, C.c_int, C.c_int, i8p, f32p]),
            "ko_common_q4_gemm": (None, [u8p, C.c_int, C.c_int, i8p, f32p, C.c_int, f32p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref():
    """The reference's own CPU code (oracle/_ref), or None when not built."""
    global _ref
    if _ref is None and ref_available():
        R = C.CDLL(REF_PATH)
        R.ref_fixture.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        R.ref_input.argtypes = [C.c_int, C.c_int, C.c_int, f32p]
        R.ref_activation.argtypes = [f32p, C.c_int, C.c_int, C.c_int, C.c_int, i8p, f32p, C.c_void_p]
        R.ref_reference.argtypes = [f32p, f32p, C.c_int, C.c_int, C.c_int, f64p]
        R.ref_gemv_create.restype = C.c_void_p
        R.ref_gemv_create.argtypes = [f32p, C.c_int, C.c_int, C.c_int]
        R.ref_gemv_run.argtypes = [C.c_void_p, f32p, C.c_int, f64p]
        R.ref_gemv_destroy.argtypes = [C.c_void_p]
        R.ref_native_q4_size.restype = C.c_size_t
        R.ref_native_q4_size.argtypes = [C.c_int, C.c_int]
        R.ref_pack_native_q4.argtypes = [u8p, C.c_size_t, u8p, C.c_int, C.c_int]
        R.ref_common_pack.argtypes = [u8p, C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                      C.c_size_t, C.c_void_p]
        _ref = R
    return _ref


# ---------------------------------------------------------------------------
# numpy helpers over the C restatement
# ---------------------------------------------------------------------------
WT_F32, WT_F16, WT_Q4_0, WT_I8 = 0, 1, 2, 3


def uniform(seed: int, count: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib().ko_fill_uniform(seed, out, count, lo, hi)
    return out


def normal(seed: int, count: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib().ko_fill_normal(seed, out, count, mean, std)
    return out


def fixture_q4(k: int, n: int) -> np.ndarray:
    out = np.empty(n * (k // 32) * 18, np.uint8)
    lib().ko_fixture_q4(k, n, out)
    return out


def fixture_input(k: int, batch: int, pattern: int = 0) -> np.ndarray:
    out = np.empty(k * batch, np.float32)
    lib().ko_fixture_input(k, batch, pattern, out)
    return out


def library_bench_weights(k: int, n: int):
    w = np.empty(n * k, np.float32)
    q = np.empty(n * k // 32 * 18, np.uint8)
    lib().ko_library_bench_weights(k, n, w.ctypes.data, q.ctypes.data)
    return w, q


def library_bench_input(k: int, batch: int) -> np.ndarray:
    x = np.empty(k * batch, np.float32)
    lib().ko_library_bench_input(k, batch, x)
    return x


def f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.empty(x.size, np.uint16)
    lib().ko_f32_to_f16(x, out, x.size)
    return out


def half_to_float(h: int) -> float:
    return lib().ko_half_to_float(h)


def q4_0_quantize(w: np.ndarray, n: int, k: int) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32).ravel()
    out = np.empty(n * (k // 32) * 18, np.uint8)
    lib().ko_q4_0_quantize(w, n, k, out)
    return out


def q4_0_dequantize(q: np.ndarray, n: int, k: int) -> np.ndarray:
    out = np.empty(n * k, np.float32)
    lib().ko_q4_0_dequantize(np.ascontiguousarray(q, np.uint8), n, k, out)
    return out


def matmul_gold(w: np.ndarray, wtype: int, x: np.ndarray, k: int, n: int, batch: int) -> np.ndarray:
    w = np.ascontiguousarray(w)
    y = np.empty(batch * n, np.float64)
    lib().ko_matmul_gold(w.ctypes.data, wtype, np.ascontiguousarray(x, np.float32), k, n, batch, y)
    return y


def matvec_model(w: np.ndarray, wtype: int, x: np.ndarray, k: int, n: int, batch: int) -> np.ndarray:
    w = np.ascontiguousarray(w)
    y = np.empty(batch * n, np.float32)
    lib().ko_matvec_model(w.ctypes.data, wtype, np.ascontiguousarray(x, np.float32), k, n, batch, y)
    return y


def reference_fp64(w: np.ndarray, x: np.ndarray, k: int, n: int, batch: int, threads: int = 0) -> np.ndarray:
    y = np.empty(batch * n, np.float64)
    lib().ko_reference_fp64(np.ascontiguousarray(w, np.float32), np.ascontiguousarray(x, np.float32),
                            k, n, batch, y, threads)
    return y


def q4_gemv_fp64(q: np.ndarray, x: np.ndarray, k: int, n: int, batch: int, threads: int = 0) -> np.ndarray:
    y = np.empty(batch * n, np.float32)
    lib().ko_q4_gemv_fp64(np.ascontiguousarray(q, np.uint8), np.ascontiguousarray(x, np.float32),
                          k, n, batch, y, threads)
    return y


def packed_i8_size(k: int, n: int) -> int:
    return lib().ko_packed_i8_size(k, n)


def aligned(b: int) -> int:
    return lib().ko_aligned(b)


def i8_pack_rows(w: np.ndarray, k: int, n: int):
    q = np.empty(n * k, np.int8)
    s = np.empty(n, np.float32)
    if not lib().ko_i8_pack_rows(np.ascontiguousarray(w, np.float32).ravel(), k, n, q, s):
        raise ValueError("non-finite weight")
    return q, s


def a8_tensor(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32).ravel()
    q0 = np.empty(x.size, np.int8)
    q1 = np.empty(x.size, np.int8)
    m0, m1 = C.c_float(), C.c_float()
    if not lib().ko_a8_tensor(x, x.size, q0, q1, C.byref(m0), C.byref(m1)):
        raise ValueError("non-finite activation")
    return q0, q1, np.float32(m0.value), np.float32(m1.value)


def i8_matmul(wq, scales, q0, q1, max0, max1, k, n, batch, want_dots=False):
    y = np.empty(batch * n, np.float32)
    p0 = np.empty(batch * n, np.int32) if want_dots else None
    p1 = np.empty(batch * n, np.int32) if want_dots else None
    lib().ko_i8_matmul(np.ascontiguousarray(wq, np.int8), np.ascontiguousarray(scales, np.float32),
                       np.ascontiguousarray(q0, np.int8), np.ascontiguousarray(q1, np.int8),
                       float(max0), float(max1), k, n, batch, y,
                       p0.ctypes.data if want_dots else None, p1.ctypes.data if want_dots else None)
    return (y, p0, p1) if want_dots else y


def native_q4_size(k: int, n: int) -> int:
    return lib().ko_native_q4_size(k, n)


def pack_native_q4(q4: np.ndarray, k: int, n: int) -> np.ndarray:
    size = native_q4_size(k, n)
    out = np.empty(size, np.uint8)
    if not lib().ko_pack_native_q4(out, size, np.ascontiguousarray(q4, np.uint8), k, n):
        raise ValueError("unsupported native layout")
    return out


def native_a8(x: np.ndarray, k: int, dtype: int = 0):
    x = np.ascontiguousarray(x)
    q0 = np.empty(k, np.int8)
    q1 = np.empty(k, np.int8)
    params = np.empty(4, np.float32)
    lib().ko_native_a8(x.ctypes.data, k, dtype, q0, q1, params)
    return q0, q1, params


def native_q4_gemv(native: np.ndarray, k: int, n: int, q0, q1, params) -> np.ndarray:
    y = np.empty(n, np.float32)
    lib().ko_native_q4_gemv(native, k, n, q0, q1, np.ascontiguousarray(params, np.float32), y)
    return y


def common_info(k: int, n: int):
    kp = -(-k // (512 if k < 512 else 256)) * (512 if k < 512 else 256)
    np_ = -(-n // 256) * 256
    scale_offset = kp * np_ // 2
    return dict(k=k, n=n, kp=kp, np=np_, scale_offset=scale_offset, payload_bytes=scale_offset + kp * np_ // 16)


def common_pack(q4: np.ndarray, k: int, n: int) -> np.ndarray:
    info = common_info(k, n)
    out = np.empty(info["payload_bytes"], np.uint8)
    q4 = np.ascontiguousarray(q4, np.uint8)
    if not lib().ko_common_pack(q4, q4.size, k, n, out):
        raise ValueError("unsupported common layout")
    return out


def common_inverse(packed: np.ndarray, k: int, n: int) -> np.ndarray:
    out = np.empty(n * ((k + 31) // 32) * 18, np.uint8)
    lib().ko_common_inverse(np.ascontiguousarray(packed, np.uint8), k, n, out)
    return out


def common_q4_gemv(packed, k, n, q0, q1, params) -> np.ndarray:
    y = np.empty(n, np.float32)
    lib().ko_common_q4_gemv(packed, k, n, q0, q1, np.ascontiguousarray(params, np.float32), y)
    return y


def row_a8(x: np.ndarray, m: int, k: int, dtype: int = 0):
    x = np.ascontiguousarray(x)
    q = np.empty(m * k, np.int8)
    s = np.empty(m, np.float32)
    lib().ko_row_a8(x.ctypes.data, m, k, dtype, q, s)
    return q, s


def common_q4_gemm(packed, k, n, q, row_scale, m) -> np.ndarray:
    y = np.empty(m * n, np.float32)
    lib().ko_common_q4_gemm(packed, k, n, q, np.ascontiguousarray(row_scale, np.float32), m, y)
    return y
