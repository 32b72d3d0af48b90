"""Seeded input generators shared by the parity tests and tests/golden/make_golden.py.

Values are bf16 bit patterns (numpy uint16), so they are exact and device-independent.
"""
from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (NaN -> 0x7FC0, as torch does)."""
    x = np.asarray(x, dtype=np.float32)
    flat = x.reshape(-1)
    u = flat.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[np.isnan(flat)] = 0x7FC0
    return r.reshape(x.shape)


def bf16_bits_to_f32(h) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


TIES = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0]


def edge_blocks(rng: np.random.Generator) -> np.ndarray:
    """[n, 16] uint16 blocks covering the corners of the quantizer."""
    B = []
    z = np.zeros(16, np.uint16)
    B.append(z)                                                   # all +0
    B.append(np.full(16, 0x8000, np.uint16))                      # all -0
    B.append(np.where(np.arange(16) % 2 == 0, 0, 0x8000).astype(np.uint16))
    nrm = f32_to_bf16_bits(rng.standard_normal(16))
    b = nrm.copy(); b[3] = 0x7FC0; B.append(b)                    # one NaN
    b = nrm.copy(); b[7] = 0xFFC1; B.append(b)                    # negative NaN, payload
    B.append(np.full(16, 0x7FC0, np.uint16))                      # all NaN
    b = nrm.copy(); b[0] = 0x7F80; B.append(b)                    # +inf
    b = nrm.copy(); b[15] = 0xFF80; B.append(b)                   # -inf
    b = nrm.copy(); b[1] = 0x7F80; b[2] = 0xFF80; B.append(b)     # +inf and -inf
    b = nrm.copy(); b[1] = 0x7F80; b[2] = 0x7FC0; B.append(b)     # inf and NaN
    sub = rng.integers(1, 0x80, 16).astype(np.uint16)             # bf16 subnormals
    sub |= (rng.integers(0, 2, 16).astype(np.uint16) << 15)
    B.append(sub)
    b = np.zeros(16, np.uint16); b[5] = 0x0001; B.append(b)       # single smallest subnormal
    B.append(np.array([0x7F7F, 0xFF7F] * 8, np.uint16))           # +-max finite
    B.append(f32_to_bf16_bits(rng.uniform(-1, 1, 16) * 2.0 ** -126))  # near min normal
    # exact E2M1 ties once sf == 1 and os == 1 (s = 1, amax = 6)
    t = np.array(TIES + [-v for v in TIES], np.float32)
    B.append(f32_to_bf16_bits(t))
    B.append(f32_to_bf16_bits(t * 4.0))                           # same at sf == 4
    B.append(f32_to_bf16_bits(t * 0.5))
    # midpoints between codes scaled by amax = 6 (no ties) and tiny nonzeros
    B.append(f32_to_bf16_bits(np.array([6, 0.3, 0.7, 0.8, 1.2, 1.3, 1.7, 1.8,
                                        2.4, 2.6, 3.4, 3.6, 4.9, 5.1, 1e-3, -1e-3], np.float32)))
    # one large value with many tiny ones (tiny ones flush to zero codes)
    b = f32_to_bf16_bits(rng.standard_normal(16) * 1e-4); b[9] = f32_to_bf16_bits(np.float32(1e4)); B.append(b)
    # huge dynamic range per element
    mag = 2.0 ** rng.uniform(-60, 60, 16)
    B.append(f32_to_bf16_bits(mag * rng.choice([-1.0, 1.0], 16)))
    return np.stack(B).astype(np.uint16)


def random_blocks(rng: np.random.Generator, n: int) -> np.ndarray:
    """[n, 16] uint16: normal data, outliers, tiny blocks, wide-range blocks."""
    x = rng.standard_normal((n, 16)).astype(np.float32)
    k = n // 4
    x[:k] *= np.where(rng.random((k, 16)) < 0.05, 50.0, 1.0)            # outliers x50
    x[k:2 * k] *= 1e-6                                                   # sf underflow region
    x[2 * k:3 * k] = (2.0 ** rng.uniform(-30, 30, (k, 16))) * np.sign(rng.standard_normal((k, 16)))
    return f32_to_bf16_bits(x)


def quantize_case_blocks(seed: int = 1234, n_random: int = 4096) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.concatenate([edge_blocks(rng), random_blocks(rng, n_random)]).reshape(-1)


def quantize_case_scales(x_bits: np.ndarray) -> np.ndarray:
    """Per-tensor scales to run every block under: the recipe's, exact ones and IEEE corners."""
    finite = bf16_bits_to_f32(x_bits)
    finite = np.abs(finite[np.isfinite(finite)])
    amax = np.float32(finite.max())
    recipe = np.float32(np.float32(1.0) / amax) * np.float32(2688.0)
    return np.array([recipe, 1.0, 1e-3, 1e3, 3.0e38, 1e-38, 2.0 ** -149, 0.0, -1.0,
                     np.inf, np.nan], dtype=np.float32)


def dequant_exhaustive_inputs() -> tuple[np.ndarray, np.ndarray]:
    """Every scale code paired with every packed byte value: (packed [256*32*8], sf [256*32])."""
    sf = np.repeat(np.arange(256, dtype=np.uint8), 32)
    q = np.tile(np.arange(256, dtype=np.uint8), 256 * 8 // 8)
    return q, sf


DEQUANT_SCALES = np.array([1.0, 0.2475, 1e-30, 3.0e38, 0.0, -1.0, np.inf, np.nan, 2.0 ** -149],
                          dtype=np.float32)


def activation(rng: np.random.Generator, rows: int, cols: int, outlier_frac: float = 0.0,
               std: float = 1.0) -> np.ndarray:
    """bf16 N(0, std^2) matrix with a fraction of elements x50 (the workloads' recipe)."""
    x = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std))
    if outlier_frac > 0:
        n = int(round(outlier_frac * x.size))
        idx = rng.choice(x.size, size=n, replace=False)
        x.reshape(-1)[idx] *= np.float32(50.0)
    return f32_to_bf16_bits(x)
