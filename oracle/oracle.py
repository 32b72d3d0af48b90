"""CPU oracle for the NVFP4 path — TEST INFRASTRUCTURE ONLY.

This module is the checker. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` import it. The product package (``my_nvfp4_gemm_b200``) never imports it and
has no CPU fallback.

It wraps ``oracle/nvfp4_oracle.c`` (a restatement of the reference plugin's arithmetic,
``csrc/quantize/quantize_nvfp4.cu:6-62`` and ``csrc/common/common.h:65-126``) with numpy, and
adds the GEMM reference of ``csrc/gemm/gemm_nvfp4.cu:147,230-231`` for large shapes (decoded
operands, float64 matmul). ``load_reference_kernels()`` exposes the reference's own
quantize/dequant CUDA kernels rebuilt from source for sm_100a (``oracle/_ref``), the GPU
check the oracle is pinned against.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "_build", "libnvfp4_oracle.so")
_REF_PATH = os.path.join(HERE, "_ref", "libref_quantize.so")

_lib = None


def build(ref: bool = False) -> None:
    """Compile the C oracle (and, with ``ref=True``, the reference kernels) via oracle/Makefile."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        f32 = ctypes.c_float
        L.nvfp4_oracle_quantize.argtypes = [p, f32, i64, p, p]
        L.nvfp4_oracle_dequantize.argtypes = [p, f32, p, i64, p]
        L.nvfp4_oracle_decode_scaled.argtypes = [p, p, i64, i64, p]
        L.nvfp4_oracle_gemm.argtypes = [p, p, p, p, f32, i64, i64, i64, p, p, p, p]
        L.nvfp4_oracle_f32_to_e4m3.argtypes = [f32]
        L.nvfp4_oracle_f32_to_e4m3.restype = ctypes.c_uint8
        L.nvfp4_oracle_f32_to_e2m1.argtypes = [f32]
        L.nvfp4_oracle_f32_to_e2m1.restype = ctypes.c_uint8
        L.nvfp4_oracle_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.nvfp4_oracle_e4m3_to_f32.restype = f32
        L.nvfp4_oracle_e2m1_to_f32.argtypes = [ctypes.c_uint8]
        L.nvfp4_oracle_e2m1_to_f32.restype = f32
        L.nvfp4_oracle_f32_to_bf16.argtypes = [f32]
        L.nvfp4_oracle_f32_to_bf16.restype = ctypes.c_uint16
        L.nvfp4_oracle_epilogue.argtypes = [f32, f32]
        L.nvfp4_oracle_epilogue.restype = ctypes.c_uint16
        L.nvfp4_oracle_num_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def num_threads() -> int:
    return int(lib().nvfp4_oracle_num_threads())


# ---- scalar helpers (known-answer tests) -------------------------------------------------
def f32_to_e4m3(x: float) -> int:
    return int(lib().nvfp4_oracle_f32_to_e4m3(x))


def f32_to_e2m1(x: float) -> int:
    return int(lib().nvfp4_oracle_f32_to_e2m1(x))


def e4m3_to_f32(v: int) -> float:
    return float(lib().nvfp4_oracle_e4m3_to_f32(v))


def e2m1_to_f32(v: int) -> float:
    return float(lib().nvfp4_oracle_e2m1_to_f32(v))


def f32_to_bf16(x: float) -> int:
    return int(lib().nvfp4_oracle_f32_to_bf16(x))


# ---- array operations ----------------------------------------------------------------------
def global_scale(x_bf16_bits: np.ndarray) -> np.float32:
    """s = 6*448 / fp32(amax|x|), the reference recipe (test.py:10-11). torch's abs().max() of
    a bf16 tensor is a bf16 value, converted to fp32; ``int / Tensor`` is evaluated by torch as
    ``Tensor.reciprocal() * int`` (two fp32 roundings), which is restated here."""
    mag = (x_bf16_bits.view(np.uint16) & 0x7FFF).astype(np.uint32)
    amax = np.uint32(mag.max()) << np.uint32(16)
    amax_f = np.array([amax], dtype=np.uint32).view(np.float32)[0]
    return np.float32(np.float32(np.float32(1.0) / amax_f) * np.float32(2688.0))


def quantize(x_bf16_bits: np.ndarray, s: float) -> tuple[np.ndarray, np.ndarray]:
    """bf16 bits [..., K] (uint16) -> (packed uint8 [..., K/2], sf uint8 [..., K/16])."""
    x = np.ascontiguousarray(x_bf16_bits.view(np.uint16))
    assert x.shape[-1] % 16 == 0
    q = np.empty(x.shape[:-1] + (x.shape[-1] // 2,), dtype=np.uint8)
    sf = np.empty(x.shape[:-1] + (x.shape[-1] // 16,), dtype=np.uint8)
    lib().nvfp4_oracle_quantize(_ptr(x), float(s), x.size, _ptr(q), _ptr(sf))
    return q, sf


def dequantize(q: np.ndarray, s: float, sf: np.ndarray) -> np.ndarray:
    """packed uint8 [..., K/2] + sf -> bf16 bits uint16 [..., K]."""
    q = np.ascontiguousarray(q)
    sf = np.ascontiguousarray(sf)
    assert sf.size * 8 == q.size
    y = np.empty(q.shape[:-1] + (q.shape[-1] * 2,), dtype=np.uint16)
    lib().nvfp4_oracle_dequantize(_ptr(q), float(s), _ptr(sf), q.size, _ptr(y))
    return y


def decode_scaled(q: np.ndarray, sf: np.ndarray) -> np.ndarray:
    """packed [rows, K/2] + sf [rows, K/16] -> fp32 [rows, K] of e2m1*sf (no global scale)."""
    q = np.ascontiguousarray(q)
    sf = np.ascontiguousarray(sf)
    rows, k = q.shape[0], q.shape[1] * 2
    out = np.empty((rows, k), dtype=np.float32)
    lib().nvfp4_oracle_decode_scaled(_ptr(q), _ptr(sf), rows, k, _ptr(out))
    return out


def gemm_f32(A: np.ndarray, B: np.ndarray, A_sf: np.ndarray, B_sf: np.ndarray,
             scale: float) -> np.ndarray:
    """fp32(sum_k fa*fb) / scale, before the bf16 rounding (float64 matmul; any size)."""
    fa = decode_scaled(A, A_sf).astype(np.float64)
    fb = decode_scaled(B, B_sf).astype(np.float64)
    acc = (fa @ fb.T).astype(np.float32)
    return (acc / np.float32(scale)).astype(np.float32)


def gemm(A: np.ndarray, B: np.ndarray, A_sf: np.ndarray, B_sf: np.ndarray,
         scale: float) -> np.ndarray:
    """Reference GEMM output as bf16 bits uint16 [M, N]."""
    return f32_to_bf16_array(gemm_f32(A, B, A_sf, B_sf, scale))


def gemm_c(A, B, A_sf, B_sf, scale):
    """Same as gemm() through the C loop (double accumulation); for small shapes."""
    M, N, K = A.shape[0], B.shape[0], A.shape[1] * 2
    fa = np.empty((M, K), np.float32)
    fb = np.empty((N, K), np.float32)
    d32 = np.empty((M, N), np.float32)
    d16 = np.empty((M, N), np.uint16)
    A, B, A_sf, B_sf = (np.ascontiguousarray(t) for t in (A, B, A_sf, B_sf))
    lib().nvfp4_oracle_gemm(_ptr(A), _ptr(B), _ptr(A_sf), _ptr(B_sf), float(scale), M, N, K,
                            _ptr(fa), _ptr(fb), _ptr(d32), _ptr(d16))
    return d32, d16


def f32_to_bf16_array(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even; NaN -> 0x7FFF (cvt.rn.bf16x2.f32)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[np.isnan(x)] = 0x7FFF
    return r


def bf16_to_f32_array(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


# ---- the reference's own kernels, rebuilt for sm_100a (GPU box only) -----------------------
def scale_to_blocked(sf: np.ndarray) -> np.ndarray:
    """Row-major scale factors uint8 [rows, cols] -> the 128x4 blocked layout (1-D uint8).

    Not a reference function: the reference's factors only feed its own kernel. This restates
    the published block-scaling-factor layout of library block-scaled GEMMs (cuBLASLt; the one
    torch._scaled_mm takes for float4_e2m1fn_x2 operands): pad rows to a multiple of 128 and
    cols to a multiple of 4 with zeros, cut into 128x4 blocks stored row-block-major, and inside
    a block put row 32*i + j, column c at byte 16*j + 4*i + c.
    """
    rows, cols = sf.shape
    rp, cp = -(-rows // 128) * 128, -(-cols // 4) * 4
    x = np.zeros((rp, cp), dtype=np.uint8)
    x[:rows, :cols] = sf
    # (row-block, i, j, col-block, c) -> (row-block, col-block, j, i, c)
    return np.ascontiguousarray(x.reshape(rp // 128, 4, 32, cp // 4, 4).transpose(0, 3, 2, 1, 4)).reshape(-1)


def scale_from_blocked(blocked: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Inverse of scale_to_blocked: drops the padding."""
    rp, cp = -(-rows // 128) * 128, -(-cols // 4) * 4
    x = blocked.reshape(rp // 128, cp // 4, 32, 4, 4).transpose(0, 3, 2, 1, 4).reshape(rp, cp)
    return np.ascontiguousarray(x[:rows, :cols])


def load_reference_kernels():
    """ctypes handle on oracle/_ref/libref_quantize.so, or None if it was not built."""
    if not os.path.exists(_REF_PATH):
        return None
    L = ctypes.CDLL(_REF_PATH)
    p = ctypes.c_void_p
    L.ref_quantize_nvfp4.argtypes = [p, ctypes.c_float, ctypes.c_int64, p, p, p]
    L.ref_quantize_nvfp4.restype = ctypes.c_int
    L.ref_de_quantize_nvfp4.argtypes = [p, ctypes.c_float, p, ctypes.c_int64, p, p]
    L.ref_de_quantize_nvfp4.restype = ctypes.c_int
    return L
