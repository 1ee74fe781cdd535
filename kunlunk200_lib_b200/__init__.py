"""Python host side of the B200 k200 library.

Binds ``lib/libkunlunk200.so.0`` (built in-tree by ``kunlunk200_lib_b200.build``)
through its C ABI (``include/k200_c.h``) and mirrors the reference's
``kunlun::`` API (UnagiDojyou/kunlunK200_lib v0.7.12, include/kunlun/k200.h)
with the same names, argument meaning and error behaviour: contract
violations abort the process with the reference's diagnostics, device
statuses come back as ints.

There is no CPU fallback: importing this module on a machine without the
built library raises, and every compute call needs a CUDA device.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(_PKG, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libkunlunk200.so.0")

# kunlun::WeightType / CopyKind / ElementwiseOp values (k200.h:18,40-41)
F32, F16, Q4_0, ROWWISE_I8 = 0, 1, 2, 3
HOST_TO_DEVICE, DEVICE_TO_HOST, DEVICE_TO_DEVICE = 0, 1, 2
ADD, MULTIPLY, SILU, RMS_NORM, SCALE = 0, 1, 2, 3, 4

_lib = None

_SIGNATURES = {
    "k200_version": (C.c_char_p, []),
    "k200_device_count": (C.c_int, [C.POINTER(C.c_int)]),
    "k200_select": (None, [C.c_int]),
    "k200_wait": (C.c_int, []),
    "k200_check": (None, [C.c_int]),
    "k200_require": (None, [C.c_int]),
    "k200_copy": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]),
    "k200_copy_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]),
    "k200_peer": (None, [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_size_t]),
    "k200_allocate": (C.c_void_p, [C.c_int, C.c_size_t]),
    "k200_release": (None, [C.c_int, C.c_void_p, C.c_size_t]),
    "k200_allocated_bytes": (C.c_size_t, [C.c_int]),
    "k200_lock": (None, []),
    "k200_unlock": (None, []),
    "k200_kernel_create": (C.c_void_p, []),
    "k200_kernel_destroy": (None, [C.c_void_p]),
    "k200_aligned": (C.c_size_t, [C.c_size_t]),
    "k200_packed_i8_size": (C.c_size_t, [C.c_int, C.c_int]),
    "k200_packed_i8_scales": (C.c_void_p, [C.c_void_p, C.c_int, C.c_int]),
    "k200_packed_i8_maxima": (C.c_void_p, [C.c_void_p, C.c_int, C.c_int]),
    "k200_upload_i8_rows": (None, [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "k200_pack_i8_rows_device": (None, [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "k200_matmul": (None, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                           C.c_int, C.c_void_p, C.c_void_p, C.c_int]),
    "k200_elementwise": (None, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                C.c_int, C.c_int, C.c_float]),
    "k200_matmul_count": (C.c_size_t, [C.c_int]),
    "k200_peer_copies": (C.c_size_t, []),
    "k200_peer_bytes": (C.c_size_t, []),
    "k200_stream": (C.c_void_p, [C.c_int]),
    "k200_set_stream": (None, [C.c_int, C.c_void_p]),
    "k200_set_static_weights": (None, [C.c_int, C.c_int]),
    "k200_copy_kernel": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "k200_graph_begin": (C.c_int, [C.c_int]),
    "k200_graph_end": (C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    "k200_graph_launch": (C.c_int, [C.c_int, C.c_void_p]),
    "k200_graph_destroy": (C.c_int, [C.c_void_p]),
    "k200_quantize_q4_0": (None, [C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int]),
    "k200_ipc_handle": (C.c_int, [C.c_void_p, C.c_void_p]),
    "k200_ipc_open": (C.c_int, [C.c_int, C.c_void_p, C.POINTER(C.c_void_p)]),
    "k200_ipc_close": (C.c_int, [C.c_int, C.c_void_p]),
    "k200_matmul_q4_gather_scratch": (C.c_size_t, [C.c_int, C.c_int, C.c_int]),
    "k200_matmul_q4_gather": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                        C.c_void_p, C.c_size_t, C.c_void_p]),
    "k200_gather_wait": (C.c_int, [C.c_int, C.c_void_p]),
    "k200_gather_rows": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int]),
    "k200_matmul_i8_noalloc": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                         C.c_void_p, C.c_void_p]),
    # native Q4 layout
    "k200_native_q4_layout_supported": (C.c_int, [C.c_int, C.c_int]),
    "k200_native_q4_size": (C.c_size_t, [C.c_int, C.c_int]),
    "k200_pack_native_q4": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_int, C.c_int]),
    "k200_upload_native_q4": (None, [C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int]),
    "k200_native_q4_reason": (C.c_char_p, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "k200_native_q4_workspace_create": (C.c_void_p, []),
    "k200_native_q4_workspace_destroy": (None, [C.c_void_p]),
    "k200_native_q4_statistics": (None, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "k200_native_q4_matmul": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                        C.c_int, C.c_int]),
    # common Q4 ABI v1
    "k200_common_q4_supported": (C.c_int, [C.c_int, C.c_int]),
    "k200_common_q4_size": (C.c_size_t, [C.c_int, C.c_int]),
    "k200_common_q4_pack": (C.c_int, [C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p, C.c_size_t]),
    "k200_common_q4_weight_create": (C.c_void_p, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_size_t]),
    "k200_common_q4_weight_destroy": (None, [C.c_void_p]),
    "k200_common_q4_weight_upload": (None, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "k200_common_q4_weight_data": (C.c_void_p, [C.c_void_p]),
    "k200_common_q4_weight_info": (None, [C.c_void_p, C.c_void_p]),
    "k200_common_q4_workspace_create": (C.c_void_p, []),
    "k200_common_q4_workspace_destroy": (None, [C.c_void_p]),
    "k200_common_q4_matmul": (None, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int]),
    "k200_common_q4_quantization": (None, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                           C.POINTER(C.c_int)]),
    "k200_common_q4_statistics": (None, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "k200_get_rows_f32": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p,
                                    C.c_size_t, C.c_int, C.c_int, C.c_int]),
    "k200_common_q4_get_rows": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p,
                                          C.c_size_t, C.c_int]),
    "k200_common_q4_lease_create": (C.c_void_p, []),
    "k200_common_q4_lease_destroy": (None, [C.c_void_p]),
    "k200_common_q4_lease_reset": (None, [C.c_void_p]),
    "k200_common_q4_lease_matches": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64]),
    "k200_common_q4_lease_chunks": (C.c_size_t, [C.c_void_p]),
    "k200_common_q4_lease_chunk": (None, [C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                          C.POINTER(C.c_int), C.POINTER(C.c_size_t)]),
    "k200_common_q4_prepare": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_uint64,
                                         C.c_void_p]),
    "k200_common_q4_matmul_shared": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                               C.c_uint64]),
    "k200_common_q4_matmul_pair": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                             C.c_void_p, C.c_uint64]),
    "k200_common_q4_pair_statistics": (None, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "k200_common_q4_pair_last_status": (C.c_int, [C.c_void_p]),
    "k200_common_q4_activation_statistics": (None, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "k200_q6_k_supported": (C.c_int, [C.c_int, C.c_int]),
    "k200_q6_k_size": (C.c_size_t, [C.c_int, C.c_int]),
    "k200_q6_k_weight_create": (C.c_void_p, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_size_t]),
    "k200_q6_k_weight_destroy": (None, [C.c_void_p]),
    "k200_q6_k_weight_upload": (None, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "k200_q6_k_weight_data": (C.c_void_p, [C.c_void_p]),
    "k200_q6_k_workspace_create": (C.c_void_p, []),
    "k200_q6_k_workspace_destroy": (None, [C.c_void_p]),
    "k200_q6_k_workspace_statistics": (None, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "k200_q6_k_matmul": (None, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int]),
    "k200_swiglu_reason": (C.c_char_p, [C.c_int] * 6),
    "k200_swiglu": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p,
                              C.c_size_t] + [C.c_int] * 6),
}

# kunlun::InputType values (k200.h:132)
INPUT_F32, INPUT_F16 = 0, 1


def exported_symbols() -> list[str]:
    """Every C-ABI symbol this package binds (the contents of include/k200_c.h)."""
    return sorted(_SIGNATURES)


def lib():
    """The loaded libkunlunk200.so.0 (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m kunlunk200_lib_b200.build`")
        L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(p) -> int | None:
    """Device/host address of an int, ctypes pointer, numpy array or torch tensor."""
    if p is None:
        return None
    if isinstance(p, int):
        return p
    if isinstance(p, np.ndarray):
        return p.ctypes.data
    if hasattr(p, "data_ptr"):
        return p.data_ptr()
    if isinstance(p, Buffer):
        return p.data()
    return C.cast(p, C.c_void_p).value


# ---------------------------------------------------------------------------
# runtime (k200.h:10-23)
# ---------------------------------------------------------------------------
def version() -> str:
    return lib().k200_version().decode()


def device_count() -> int:
    n = C.c_int(0)
    check(lib().k200_device_count(C.byref(n)))
    return n.value


def select(device: int) -> None:
    lib().k200_select(device)


def wait() -> int:
    return lib().k200_wait()


def check(status: int) -> None:
    lib().k200_check(int(status))


def require(condition: bool) -> None:
    lib().k200_require(1 if condition else 0)


def copy(dst, src, nbytes: int, kind: int) -> int:
    return lib().k200_copy(_ptr(dst), _ptr(src), nbytes, kind)


def copy_async(dst, src, nbytes: int, kind: int) -> int:
    return lib().k200_copy_async(_ptr(dst), _ptr(src), nbytes, kind)


def copy_kernel(dst, src, nbytes: int) -> int:
    """Copy by a kernel on the current device's library stream (k200_copy_kernel);
    either side may be pinned host memory."""
    return lib().k200_copy_kernel(_ptr(dst), _ptr(src), nbytes)


def peer(dst_device: int, dst, src_device: int, src, nbytes: int) -> None:
    lib().k200_peer(dst_device, _ptr(dst), src_device, _ptr(src), nbytes)


def allocate(device: int, nbytes: int) -> int | None:
    return lib().k200_allocate(device, nbytes)


def release(device: int, ptr, nbytes: int) -> None:
    lib().k200_release(device, _ptr(ptr), nbytes)


def allocated_bytes(device: int) -> int:
    return lib().k200_allocated_bytes(device)


def stream(device: int) -> int:
    """The library stream of `device` as an integer cudaStream_t handle."""
    return lib().k200_stream(device) or 0


def set_stream(device: int, stream_handle: int | None) -> None:
    """Issue library work of `device` on a caller stream (None: the library's own)."""
    lib().k200_set_stream(device, stream_handle or None)


def set_static_weights(device: int, enabled: bool) -> None:
    """Weights of `device`'s matmuls are never written by the kernel just before them."""
    lib().k200_set_static_weights(device, 1 if enabled else 0)


class Graph:
    """A recorded sequence of library work on one device (k200_graph_*).

    with K.Graph(dev) as g:        # records instead of running
        K.copy_async(...); K.matmul(...); ...
    g.launch(); K.select(dev); K.check(K.wait())
    """

    def __init__(self, device: int):
        self.device = device
        self.handle = None

    def __enter__(self):
        check(lib().k200_graph_begin(self.device))
        return self

    def __exit__(self, exc_type, exc, tb):
        out = C.c_void_p()
        rc = lib().k200_graph_end(self.device, C.byref(out))
        if exc_type is None:
            check(rc)
            self.handle = out.value
        return False

    def launch(self) -> None:
        check(lib().k200_graph_launch(self.device, self.handle))

    def close(self) -> None:
        if self.handle:
            check(lib().k200_graph_destroy(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class runtime_lock:
    """Context manager holding kunlun::runtime_mutex()."""

    def __enter__(self):
        lib().k200_lock()
        return self

    def __exit__(self, *exc):
        lib().k200_unlock()
        return False


class Buffer:
    """RAII device allocation (kunlun::Buffer, k200.h:25-37)."""

    def __init__(self, device: int, nbytes: int):
        self.device = device
        self.nbytes = nbytes
        self.ptr = allocate(device, nbytes)
        require(bool(self.ptr))

    def data(self) -> int:
        return self.ptr

    def size(self) -> int:
        return self.nbytes

    def upload(self, array: np.ndarray) -> None:
        a = np.ascontiguousarray(array)
        require(a.nbytes <= self.nbytes)
        select(self.device)
        check(copy(self.ptr, a, a.nbytes, HOST_TO_DEVICE))

    def download(self, dtype, count: int, offset: int = 0) -> np.ndarray:
        out = np.empty(count, dtype)
        require(offset + out.nbytes <= self.nbytes)
        select(self.device)
        check(copy(out, self.ptr + offset, out.nbytes, DEVICE_TO_HOST))
        return out

    def close(self) -> None:
        if self.ptr:
            release(self.device, self.ptr, self.nbytes)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Kernel:
    """Per-call state bound to one device (kunlun::Kernel, k200.h:62-88)."""

    def __init__(self):
        self.handle = lib().k200_kernel_create()

    def close(self) -> None:
        if self.handle:
            lib().k200_kernel_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# rowwise int8 packing (k200.h:90-96)
# ---------------------------------------------------------------------------
def aligned(nbytes: int) -> int:
    return lib().k200_aligned(nbytes)


def packed_i8_size(k: int, rows: int) -> int:
    return lib().k200_packed_i8_size(k, rows)


def packed_i8_scales(weights, k: int, rows: int) -> int:
    return lib().k200_packed_i8_scales(_ptr(weights), k, rows)


def packed_i8_maxima(weights, k: int, rows: int) -> int:
    return lib().k200_packed_i8_maxima(_ptr(weights), k, rows)


def upload_i8_rows(device: int, weights, k: int, rows: int, first_row: int, count: int, host_input) -> None:
    if isinstance(host_input, np.ndarray):
        host_input = np.ascontiguousarray(host_input, np.float32)
    lib().k200_upload_i8_rows(device, _ptr(weights), k, rows, first_row, count, _ptr(host_input))


def pack_i8_rows_device(device: int, weights, k: int, rows: int, first_row: int, count: int, device_input) -> None:
    lib().k200_pack_i8_rows_device(device, _ptr(weights), k, rows, first_row, count, _ptr(device_input))


# ---------------------------------------------------------------------------
# matmul / elementwise (k200.h:98-107)
# ---------------------------------------------------------------------------
def matmul(kernel: Kernel, device: int, y, w, x, k: int, n: int, batch: int, type: int,
           scales=None, maxima=None, tile: int = 16) -> None:
    """Submit Y[batch,n] = X[batch,k] . W^T[n,k]; select(device)+check(wait()) completes it."""
    lib().k200_matmul(kernel.handle, device, _ptr(y), _ptr(w), _ptr(x), k, n, batch, int(type),
                      _ptr(scales), _ptr(maxima), tile)


def elementwise(kernel: Kernel, device: int, y, a, b, count: int, width: int, b_count: int, op: int,
                parameter: float = 0.0) -> None:
    lib().k200_elementwise(kernel.handle, device, _ptr(y), _ptr(a), _ptr(b), count, width, b_count, int(op),
                           float(parameter))


def quantize_q4_0(device: int, q4, w, k: int, n: int) -> None:
    """GGML Q4_0 block quantiser on the device (f32 [n][k] -> [n][k/32] blocks)."""
    lib().k200_quantize_q4_0(device, _ptr(q4), _ptr(w), k, n)


NOALLOC_MAX_ELEMENTS, NOALLOC_TOO_LARGE, NOALLOC_NOT_READY = 2097152, -2, -3


def matmul_i8_noalloc(device: int, y, w, x, k: int, n: int, batch: int, scales, maxima) -> int:
    """Rowwise-int8 matmul on the library's static scratch (no allocation; see k200_c.h).

    Returns 0 once submitted, NOALLOC_TOO_LARGE when batch*k > NOALLOC_MAX_ELEMENTS,
    NOALLOC_NOT_READY before the first select(device), else a CUDA error code.
    """
    return lib().k200_matmul_i8_noalloc(device, _ptr(y), _ptr(w), _ptr(x), k, n, batch, _ptr(scales),
                                        _ptr(maxima))


# ---------------------------------------------------------------------------
# native Q4 layout (k200.h:127-131, 203-224)
# ---------------------------------------------------------------------------
def native_q4_layout_supported(k: int, n: int) -> bool:
    return bool(lib().k200_native_q4_layout_supported(k, n))


def native_q4_size(k: int, n: int) -> int:
    return lib().k200_native_q4_size(k, n)


def pack_native_q4(q4: np.ndarray, k: int, n: int) -> np.ndarray:
    """Host pack of N rows of Q4_0 blocks into the native layout (raises if unsupported)."""
    src = np.ascontiguousarray(q4, np.uint8)
    out = np.empty(native_q4_size(k, n), np.uint8)
    if not lib().k200_pack_native_q4(_ptr(out), out.nbytes, _ptr(src), k, n):
        raise ValueError("native Q4 layout unsupported for this shape or buffer")
    return out


def upload_native_q4(device: int, weights, q4: np.ndarray, k: int, n: int) -> None:
    src = np.ascontiguousarray(q4, np.uint8)
    lib().k200_upload_native_q4(device, _ptr(weights), _ptr(src), k, n)


def native_q4_reason(k: int, n: int, batch: int, type: int = INPUT_F32) -> str:
    return lib().k200_native_q4_reason(k, n, batch, int(type)).decode()


class NativeQ4Workspace:
    """kunlun::NativeQ4Workspace (k200.h:205-216): scratch bound to one device."""

    def __init__(self):
        self.handle = lib().k200_native_q4_workspace_create()

    def statistics(self) -> dict:
        out = (C.c_size_t * 4)()
        lib().k200_native_q4_statistics(self.handle, out)
        return {"accelerated": out[0], "fallback": out[1], "hbm_workspace_bytes": out[2],
                "l3_workspace_bytes": out[3]}

    def close(self) -> None:
        if self.handle:
            lib().k200_native_q4_workspace_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def native_q4_matmul(workspace: NativeQ4Workspace, device: int, y, weights, x, k: int, n: int, batch: int = 1,
                     type: int = INPUT_F32) -> bool:
    """Completes before returning; True: W4A8x2 path, False: exact FP32 fallback."""
    return bool(lib().k200_native_q4_matmul(workspace.handle, device, _ptr(y), _ptr(weights), _ptr(x), k, n,
                                            batch, int(type)))


# ---------------------------------------------------------------------------
# common Q4 ABI v1 (k200.h:226-335)
# ---------------------------------------------------------------------------
class _CommonQ4Info(C.Structure):
    _fields_ = [("abi_version", C.c_uint32), ("quant_type", C.c_uint32), ("layout", C.c_uint32),
                ("scale_order", C.c_uint32), ("k", C.c_int), ("n", C.c_int), ("kp", C.c_int), ("np", C.c_int),
                ("device", C.c_int), ("scale_offset", C.c_size_t), ("payload_bytes", C.c_size_t)]


def common_q4_supported(k: int, n: int) -> bool:
    return bool(lib().k200_common_q4_supported(k, n))


def common_q4_size(k: int, n: int) -> int:
    return lib().k200_common_q4_size(k, n)


def common_q4_pack(q4: np.ndarray, k: int, n: int) -> np.ndarray:
    """Host pack of N rows of Q4_0 blocks into the common ABI v1 payload."""
    src = np.ascontiguousarray(q4, np.uint8)
    out = np.empty(common_q4_size(k, n), np.uint8)
    if not lib().k200_common_q4_pack(_ptr(src), src.nbytes, k, n, _ptr(out), out.nbytes):
        raise ValueError("common Q4 layout unsupported for this shape or buffer")
    return out


class CommonQ4Weight:
    """kunlun::CommonQ4Weight (k200.h:242-258): a device weight in the common layout."""

    def __init__(self, device: int, k: int, n: int, storage=None, nbytes: int = 0):
        self.handle = lib().k200_common_q4_weight_create(device, k, n, _ptr(storage), nbytes)

    def upload(self, q4: np.ndarray) -> None:
        src = np.ascontiguousarray(q4, np.uint8)
        lib().k200_common_q4_weight_upload(self.handle, _ptr(src), src.nbytes)

    def data(self) -> int:
        return lib().k200_common_q4_weight_data(self.handle)

    def info(self) -> dict:
        a = _CommonQ4Info()
        lib().k200_common_q4_weight_info(self.handle, C.byref(a))
        return {name: getattr(a, name) for name, _ in _CommonQ4Info._fields_}

    def close(self) -> None:
        if self.handle:
            lib().k200_common_q4_weight_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CommonQ4Workspace:
    """kunlun::CommonQ4Workspace (k200.h:279-303)."""

    def __init__(self):
        self.handle = lib().k200_common_q4_workspace_create()

    def quantization(self) -> dict:
        values, scales, out = C.c_void_p(), C.c_void_p(), (C.c_int * 3)()
        lib().k200_common_q4_quantization(self.handle, C.byref(values), C.byref(scales), out)
        return {"values": values.value, "scales": scales.value, "rows": out[0], "kp": out[1],
                "components": out[2]}

    def statistics(self) -> dict:
        out = (C.c_size_t * 10)()
        lib().k200_common_q4_statistics(self.handle, out)
        return {"paths": list(out[:8]), "calls": out[8], "chunks": out[9]}

    def activation_statistics(self) -> dict:
        out = (C.c_size_t * 8)()
        lib().k200_common_q4_activation_statistics(self.handle, out)
        names = ("prepare_calls", "quantized_chunks", "quant_kernel_launches", "prepared_matmuls",
                 "prepared_chunks", "invalidations", "rejected_calls", "hbm_activation_bytes")
        return dict(zip(names, out))

    def close(self) -> None:
        if self.handle:
            lib().k200_common_q4_workspace_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def common_q4_matmul(workspace: CommonQ4Workspace, device: int, y, weight: CommonQ4Weight, x, m: int,
                     type: int = INPUT_F32) -> None:
    """Y [m,n] = X [m,k] . W^T; completes before returning (M=1: two-component A8, M>1: Row A8)."""
    lib().k200_common_q4_matmul(workspace.handle, device, _ptr(y), weight.handle, _ptr(x), m, int(type))


def q6_k_supported(k: int, n: int) -> bool:
    return bool(lib().k200_q6_k_supported(k, n))


def q6_k_size(k: int, n: int) -> int:
    return lib().k200_q6_k_size(k, n)


class Q6KWeight:
    """kunlun::Q6KWeight (k200.h:139-147): GGML Q6_K rows packed for the device."""

    def __init__(self, device: int, k: int, n: int, storage=None, nbytes: int = 0):
        self.handle = lib().k200_q6_k_weight_create(device, k, n, _ptr(storage), nbytes)

    def upload(self, q6: np.ndarray) -> None:
        src = np.ascontiguousarray(q6, np.uint8)
        lib().k200_q6_k_weight_upload(self.handle, _ptr(src), src.nbytes)

    def data(self) -> int:
        return lib().k200_q6_k_weight_data(self.handle)

    def close(self) -> None:
        if self.handle:
            lib().k200_q6_k_weight_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Q6KWorkspace:
    """kunlun::Q6KWorkspace (k200.h:150-159)."""

    def __init__(self):
        self.handle = lib().k200_q6_k_workspace_create()

    def statistics(self) -> dict:
        out = (C.c_size_t * 4)()
        lib().k200_q6_k_workspace_statistics(self.handle, out)
        return {"calls": out[0], "workspace_bytes": out[3]}

    def close(self) -> None:
        if self.handle:
            lib().k200_q6_k_workspace_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def q6_k_matmul(workspace: Q6KWorkspace, device: int, y, weight: Q6KWeight, x, m: int = 1,
                type: int = INPUT_F32) -> None:
    """kunlun::q6_k_matmul (src/q6-k.inc:104-142): completes before returning."""
    lib().k200_q6_k_matmul(workspace.handle, device, _ptr(y), weight.handle, _ptr(x), m, int(type))


# kunlun::CommonQ4PairStatus values (k200.h:281)
PAIR_STATUS = ("NotAttempted", "Success", "Disabled", "InvalidInput", "Configuration", "WeightAbi", "Lease", "Alias",
               "Workspace")


class CommonQ4ActivationLease:
    """kunlun::CommonQ4ActivationLease (k200.h:310-328): a snapshot of one workspace's quantised activations."""

    def __init__(self):
        self.handle = lib().k200_common_q4_lease_create()

    def reset(self) -> None:
        lib().k200_common_q4_lease_reset(self.handle)

    def matches(self, device: int, k: int, rows: int, type: int, generation: int) -> bool:
        return bool(lib().k200_common_q4_lease_matches(self.handle, device, k, rows, int(type), generation))

    def chunks(self) -> int:
        return lib().k200_common_q4_lease_chunks(self.handle)

    def chunk(self, index: int) -> dict:
        values, scales = C.c_void_p(), C.c_void_p()
        out, nb = (C.c_int * 5)(), (C.c_size_t * 2)()
        lib().k200_common_q4_lease_chunk(self.handle, index, C.byref(values), C.byref(scales), out, nb)
        return {"values": values.value, "scales": scales.value, "first": out[0], "rows": out[1],
                "padded_rows": out[2], "kp": out[3], "components": out[4], "values_bytes": nb[0],
                "scales_bytes": nb[1]}

    def close(self) -> None:
        if self.handle:
            lib().k200_common_q4_lease_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def common_q4_prepare(workspace: "CommonQ4Workspace", device: int, x, k: int, rows: int, type: int,
                      generation: int, lease: CommonQ4ActivationLease) -> bool:
    """kunlun::common_q4_prepare (src/q4-activation.inc:31-76)."""
    return bool(lib().k200_common_q4_prepare(workspace.handle, device, _ptr(x), k, rows, int(type), generation,
                                             lease.handle))


def common_q4_matmul_shared(workspace: "CommonQ4Workspace", device: int, y, weight: "CommonQ4Weight",
                            lease: CommonQ4ActivationLease, generation: int) -> bool:
    """kunlun::common_q4_matmul_shared (src/q4-activation.inc:79-98)."""
    return bool(lib().k200_common_q4_matmul_shared(workspace.handle, device, _ptr(y), weight.handle, lease.handle,
                                                   generation))


def common_q4_matmul_pair(workspace: "CommonQ4Workspace", device: int, y0, y1, w0: "CommonQ4Weight",
                          w1: "CommonQ4Weight", lease: CommonQ4ActivationLease, generation: int) -> bool:
    """kunlun::common_q4_matmul_pair (src/q4-pair.inc:9-80)."""
    return bool(lib().k200_common_q4_matmul_pair(workspace.handle, device, _ptr(y0), _ptr(y1), w0.handle, w1.handle,
                                                 lease.handle, generation))


def common_q4_pair_statistics(workspace: "CommonQ4Workspace") -> dict:
    out = (C.c_size_t * 3)()
    lib().k200_common_q4_pair_statistics(workspace.handle, out)
    return {"calls": out[0], "declined": out[1], "l3_partial_bytes": out[2]}


def common_q4_pair_last_status(workspace: "CommonQ4Workspace") -> str:
    return PAIR_STATUS[lib().k200_common_q4_pair_last_status(workspace.handle)]


def get_rows_f32(kernel: Kernel, device: int, output, output_bytes: int, input, input_bytes: int, indices,
                 index_bytes: int, k: int, n: int, rows: int) -> bool:
    """kunlun::get_rows_f32 (src/get-rows-f32.inc:1-29): completes before returning; False writes nothing."""
    return bool(lib().k200_get_rows_f32(kernel.handle, device, _ptr(output), output_bytes, _ptr(input), input_bytes,
                                        _ptr(indices), index_bytes, k, n, rows))


def common_q4_get_rows(kernel: Kernel, device: int, output, output_bytes: int, weight: CommonQ4Weight, indices,
                       index_bytes: int, rows: int) -> bool:
    """kunlun::common_q4_get_rows (src/get-rows.inc:1-26): decoded F32 weight columns by index."""
    return bool(lib().k200_common_q4_get_rows(kernel.handle, device, _ptr(output), output_bytes, weight.handle,
                                              _ptr(indices), index_bytes, rows))


def swiglu_reason(width: int, rows: int, gate_stride: int, up_stride: int, output_stride: int,
                  type: int = INPUT_F32) -> str:
    """kunlun::swiglu_reason (src/k200.cpp:324-333): "" when the layout is supported."""
    return lib().k200_swiglu_reason(width, rows, gate_stride, up_stride, output_stride, int(type)).decode()


def swiglu(kernel: Kernel, device: int, y, y_bytes: int, gate, gate_bytes: int, up, up_bytes: int, width: int,
           rows: int, gate_stride: int, up_stride: int, output_stride: int, type: int = INPUT_F32) -> bool:
    """kunlun::swiglu (src/k200.cpp:334-368): y = SiLU(gate) * up; completes before returning."""
    return bool(lib().k200_swiglu(kernel.handle, device, _ptr(y), y_bytes, _ptr(gate), gate_bytes, _ptr(up), up_bytes,
                                  width, rows, gate_stride, up_stride, output_stride, int(type)))


def matmul_count(device: int) -> int:
    return lib().k200_matmul_count(device)


def statistics() -> dict:
    return {"matmuls": [matmul_count(d) for d in range(max(1, device_count()))],
            "peer_copies": lib().k200_peer_copies(), "peer_bytes": lib().k200_peer_bytes()}


def weight_bytes(type: int, k: int, n: int) -> int:
    """Bytes of a legacy weight matrix [n,k] in the given encoding."""
    if type == F32:
        return 4 * k * n
    if type == F16:
        return 2 * k * n
    if type == Q4_0:
        return n * (k // 32) * 18
    if type == ROWWISE_I8:
        return packed_i8_size(k, n)
    raise ValueError(type)


# ---------------------------------------------------------------------------
# row-sharded batch-1 Q4_0 GEMV with a fused all-gather over peer memory
# (k200_c.h; replaces the peer-copy gather of a row split, src/k200.cpp:89-95)
# ---------------------------------------------------------------------------
GATHER_MAX_RANKS, GATHER_UNSUPPORTED = 8, -4
IPC_HANDLE_BYTES = 64


class GatherView(C.Structure):
    """k200_gather: one exchange seen from one rank (addresses valid on its device): every
    rank's tag array of [batch][rows] 64-bit words {f32, epoch}, this rank's [batch][rows]
    output buffer and this rank's two counter words."""
    _fields_ = [("ranks", C.c_int), ("rank", C.c_int), ("tags", C.c_void_p * GATHER_MAX_RANKS),
                ("y", C.c_void_p), ("counter", C.c_void_p), ("rows", C.c_int), ("batch", C.c_int)]


def ipc_handle(ptr) -> bytes:
    """64-byte CUDA IPC handle of a device allocation's base address."""
    buf = C.create_string_buffer(IPC_HANDLE_BYTES)
    check(lib().k200_ipc_handle(_ptr(ptr), buf))
    return buf.raw


def ipc_open(device: int, handle: bytes) -> int:
    """Maps another process's allocation on `device`; returns its address here."""
    out = C.c_void_p()
    check(lib().k200_ipc_open(device, C.create_string_buffer(bytes(handle), IPC_HANDLE_BYTES), C.byref(out)))
    return out.value


def ipc_close(device: int, ptr) -> None:
    check(lib().k200_ipc_close(device, _ptr(ptr)))


def matmul_q4_gather_scratch(device: int, k: int, n: int) -> int:
    """Zeroed scratch bytes k200_matmul_q4_gather needs for a shard of n rows (0: not handled)."""
    return lib().k200_matmul_q4_gather_scratch(device, k, n)


def matmul_q4_gather(device: int, out: GatherView, row_begin: int, w, x, k: int, n: int, scratch,
                     scratch_bytes: int, wait_for: GatherView | None = None) -> int:
    """This rank's rows of Y = W.x stored as tagged words into every rank's tag array and as
    plain floats into this rank's y (k200_matmul_q4_gather); with wait_for, x points into that
    exchange's y and is read from its tagged words as they arrive.

    Returns 0, GATHER_UNSUPPORTED or a CUDA error code; asynchronous on the library stream.
    """
    return lib().k200_matmul_q4_gather(device, C.addressof(out), row_begin, _ptr(w), _ptr(x), k, n, _ptr(scratch),
                                       scratch_bytes, None if wait_for is None else C.addressof(wait_for))


def gather_rows(device: int, out: GatherView, row_begin: int, shard, n: int, batch: int = 1) -> int:
    """This rank's [batch][n] slice into columns row_begin.. of every rank's [batch][rows] tag
    array and of this rank's y (k200_gather_rows); 0 or a CUDA error code, asynchronous on the
    library stream."""
    return lib().k200_gather_rows(device, C.addressof(out), row_begin, _ptr(shard), n, batch)


def gather_wait(device: int, exchange: GatherView) -> int:
    """Device-side wait until every tagged word of `exchange` carries this rank's epoch, then
    the values written into this rank's y (k200_gather_wait)."""
    return lib().k200_gather_wait(device, C.addressof(exchange))

