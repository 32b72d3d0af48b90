"""ctypes binding of the C ABI declared in include/nvfp4_b200.h (libnvfp4_b200.so).

This is the binding a non-torch host (or the reference's own C++ launchers) would use. The
functions take raw device pointers (ints) and a cudaStream_t (int; 0 = legacy default stream)
and return an nvfp4 status code; ``check()`` turns a non-zero code into ``NvFp4Error``.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

NVFP4_OK = 0
STATUS_NAMES = {
    0: "NVFP4_OK",
    1: "NVFP4_ERR_INVALID_VALUE",
    2: "NVFP4_ERR_UNSUPPORTED_SHAPE",
    3: "NVFP4_ERR_MISALIGNED",
    4: "NVFP4_ERR_CUDA",
    5: "NVFP4_ERR_NO_DEVICE",
    6: "NVFP4_ERR_DEVICE_TIMEOUT",
    7: "NVFP4_ERR_TOO_LARGE",
}
NVFP4_ERR_INVALID_VALUE = 1
NVFP4_ERR_UNSUPPORTED_SHAPE = 2
NVFP4_ERR_MISALIGNED = 3
NVFP4_ERR_DEVICE_TIMEOUT = 6

# Every symbol include/nvfp4_b200.h declares, with its ctypes signature.
_P, _I64, _F32, _U64, _INT = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64, ctypes.c_int
SIGNATURES = {
    "nvfp4_status_string": ([_INT], ctypes.c_char_p),
    "nvfp4_version": ([], _INT),
    "nvfp4_quantize": ([_P, _P, _I64, _P, _P, _P], _INT),
    "nvfp4_quantize_host_scale": ([_P, _F32, _I64, _P, _P, _P], _INT),
    "nvfp4_quantize_auto_scale_workspace_bytes": ([_I64], _I64),
    "nvfp4_quantize_auto_scale": ([_P, _I64, _P, _P, _P, _P, _I64, _P], _INT),
    "nvfp4_quantize_auto_scale_noalloc": ([_P, _I64, _P, _P, _P, _P], _INT),
    "nvfp4_dequantize": ([_P, _P, _P, _I64, _P, _P], _INT),
    "nvfp4_dequantize_host_scale": ([_P, _F32, _P, _I64, _P, _P], _INT),
    "nvfp4_gemm": ([_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P], _INT),
    "nvfp4_gemm_host_scale": ([_P, _P, _P, _P, _F32, _P, _I64, _I64, _I64, _P], _INT),
    "nvfp4_gemm_plan": ([_I64, _I64, _I64, _INT, ctypes.POINTER(_INT), ctypes.POINTER(_INT),
                         ctypes.POINTER(_INT)], _INT),
    "nvfp4_gemm_quantized": ([_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P], _INT),
    "nvfp4_gemm_swiglu": ([_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P], _INT),
    "nvfp4_gemm_allgather": ([_P, _P, _P, _P, _P, ctypes.POINTER(_P), _INT, _INT, _I64, _I64, _I64, _P], _INT),
    "nvfp4_ipc_export": ([_P, _P, ctypes.POINTER(_I64)], _INT),
    "nvfp4_ipc_open": ([_P, _I64, ctypes.POINTER(_P)], _INT),
    "nvfp4_ipc_close": ([_P, _I64], _INT),
    "nvfp4_blocked_scale_bytes": ([_I64, _I64], _I64),
    "nvfp4_scale_to_blocked": ([_P, _I64, _I64, _P, _P], _INT),
    "nvfp4_scale_from_blocked": ([_P, _I64, _I64, _P, _P], _INT),
    "nvfp4_device_status": ([ctypes.POINTER(_INT), _P], _INT),
    "nvfp4_clear_device_status": ([_P], _INT),
    "nvfp4_selftest_wait_timeout": ([_U64, _P], _INT),
}


class NvFp4Error(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what} failed: {STATUS_NAMES.get(status, status)}")


_lib = None


def lib() -> ctypes.CDLL:
    """Load libnvfp4_b200.so (built in-tree). Raises if it has not been built."""
    global _lib
    if _lib is None:
        path = _build.lib_path()
        if not os.path.exists(path):
            raise ImportError(f"{path} is missing: run `python -m my_nvfp4_gemm_b200.build`")
        L = ctypes.CDLL(path)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != NVFP4_OK:
        raise NvFp4Error(status, what)


def status_string(status: int) -> str:
    return lib().nvfp4_status_string(status).decode()


def quantize(x_ptr, scale_ptr, numel, out_ptr, sf_ptr, stream=0) -> int:
    return lib().nvfp4_quantize(x_ptr, scale_ptr, numel, out_ptr, sf_ptr, stream)


def quantize_host_scale(x_ptr, scale, numel, out_ptr, sf_ptr, stream=0) -> int:
    return lib().nvfp4_quantize_host_scale(x_ptr, scale, numel, out_ptr, sf_ptr, stream)


def quantize_auto_scale_workspace_bytes(numel) -> int:
    return int(lib().nvfp4_quantize_auto_scale_workspace_bytes(numel))


def quantize_auto_scale(x_ptr, numel, out_ptr, sf_ptr, scale_out_ptr, ws_ptr, ws_bytes,
                        stream=0) -> int:
    return lib().nvfp4_quantize_auto_scale(x_ptr, numel, out_ptr, sf_ptr, scale_out_ptr, ws_ptr,
                                           ws_bytes, stream)


def quantize_auto_scale_noalloc(x_ptr, numel, out_ptr, sf_ptr, scale_out_ptr, stream=0) -> int:
    """Same result as quantize_auto_scale, with the library's own fixed device scratch instead
    of a caller workspace (inputs up to 2^30 elements; see include/nvfp4_b200.h)."""
    return lib().nvfp4_quantize_auto_scale_noalloc(x_ptr, numel, out_ptr, sf_ptr, scale_out_ptr,
                                                   stream)


def dequantize(q_ptr, scale_ptr, sf_ptr, n_bytes, out_ptr, stream=0) -> int:
    return lib().nvfp4_dequantize(q_ptr, scale_ptr, sf_ptr, n_bytes, out_ptr, stream)


def dequantize_host_scale(q_ptr, scale, sf_ptr, n_bytes, out_ptr, stream=0) -> int:
    return lib().nvfp4_dequantize_host_scale(q_ptr, scale, sf_ptr, n_bytes, out_ptr, stream)


def gemm(a_ptr, b_ptr, asf_ptr, bsf_ptr, scale_ptr, d_ptr, m, n, k, stream=0) -> int:
    return lib().nvfp4_gemm(a_ptr, b_ptr, asf_ptr, bsf_ptr, scale_ptr, d_ptr, m, n, k, stream)


def gemm_host_scale(a_ptr, b_ptr, asf_ptr, bsf_ptr, scale, d_ptr, m, n, k, stream=0) -> int:
    return lib().nvfp4_gemm_host_scale(a_ptr, b_ptr, asf_ptr, bsf_ptr, scale, d_ptr, m, n, k, stream)


def gemm_plan(m, n, k, sms=0) -> tuple[int, int, int]:
    """(tile rows, tile columns, K split) of the kernel form nvfp4_gemm runs for M x N x K on a
    device with `sms` SMs (0: the current device). Raises on an invalid shape."""
    tm, tn, ks = _INT(0), _INT(0), _INT(0)
    check(lib().nvfp4_gemm_plan(m, n, k, sms, ctypes.byref(tm), ctypes.byref(tn), ctypes.byref(ks)),
          "nvfp4_gemm_plan")
    return tm.value, tn.value, ks.value


def gemm_quantized(a_ptr, b_ptr, asf_ptr, bsf_ptr, scale_ptr, out_scale_ptr, q_ptr, sf_ptr, m, n,
                   k, stream=0) -> int:
    return lib().nvfp4_gemm_quantized(a_ptr, b_ptr, asf_ptr, bsf_ptr, scale_ptr, out_scale_ptr,
                                      q_ptr, sf_ptr, m, n, k, stream)


def gemm_swiglu(a_ptr, b_ptr, asf_ptr, bsf_ptr, scale_ptr, out_ptr, m, n, k, stream=0) -> int:
    return lib().nvfp4_gemm_swiglu(a_ptr, b_ptr, asf_ptr, bsf_ptr, scale_ptr, out_ptr, m, n, k,
                                   stream)


def gemm_allgather(a_ptr, b_ptr, asf_ptr, bsf_ptr, scale_ptr, output_ptrs, rank, m, n_local, k,
                   stream=0) -> int:
    arr = (_P * len(output_ptrs))(*output_ptrs)
    return lib().nvfp4_gemm_allgather(a_ptr, b_ptr, asf_ptr, bsf_ptr, scale_ptr, arr, len(output_ptrs),
                                      rank, m, n_local, k, stream)


IPC_HANDLE_BYTES = 64


def ipc_export(ptr) -> tuple[bytes, int]:
    """(handle bytes, offset) of the device allocation containing ptr."""
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    off = _I64(0)
    check(lib().nvfp4_ipc_export(ptr, buf, ctypes.byref(off)), "nvfp4_ipc_export")
    return buf.raw, off.value


def ipc_open(handle: bytes, offset: int) -> int:
    """Map another process's exported buffer on the current device; returns its address here."""
    p = _P(0)
    check(lib().nvfp4_ipc_open(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES), offset,
                               ctypes.byref(p)), "nvfp4_ipc_open")
    return p.value


def ipc_close(ptr, offset) -> None:
    check(lib().nvfp4_ipc_close(ptr, offset), "nvfp4_ipc_close")


def blocked_scale_bytes(rows, cols) -> int:
    return lib().nvfp4_blocked_scale_bytes(rows, cols)


def scale_to_blocked(sf_ptr, rows, cols, blocked_ptr, stream=0) -> int:
    return lib().nvfp4_scale_to_blocked(sf_ptr, rows, cols, blocked_ptr, stream)


def scale_from_blocked(blocked_ptr, rows, cols, sf_ptr, stream=0) -> int:
    return lib().nvfp4_scale_from_blocked(blocked_ptr, rows, cols, sf_ptr, stream)


def device_status(stream=0) -> int:
    v = ctypes.c_int(0)
    check(lib().nvfp4_device_status(ctypes.byref(v), stream), "nvfp4_device_status")
    return v.value


def clear_device_status(stream=0) -> None:
    check(lib().nvfp4_clear_device_status(stream), "nvfp4_clear_device_status")


def selftest_wait_timeout(timeout_ns: int, stream=0) -> int:
    return lib().nvfp4_selftest_wait_timeout(timeout_ns, stream)
