"""Weight layout for the gate+up GEMM with SwiGLU in the epilogue (``my_plugins.gemm_nvfp4_swiglu``,
``nvfp4_gemm_swiglu`` in the C ABI).

The kernel's 256-row tiles of B must hold the gate rows and the up rows of the same 128
features, so the packed weight and its scale factors are stored with their rows interleaved in
groups of 128: gate rows 128t..128t+127, then up rows 128t..128t+127, for t = 0, 1, ... This is a
one-time re-layout of a weight (a row gather), not part of the per-call path."""
from __future__ import annotations

import torch

GROUP = 128


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[I, X] gate rows and [I, X] up rows (packed codes or scale factors, any dtype) ->
    [2I, X] in the kernel's order. I must be a multiple of 128."""
    if gate.shape != up.shape or gate.dim() != 2:
        raise ValueError(f"gate and up must be 2D and of equal shape, got {tuple(gate.shape)} "
                         f"and {tuple(up.shape)}")
    rows, cols = gate.shape
    if rows % GROUP:
        raise ValueError(f"the number of features ({rows}) must be a multiple of {GROUP}")
    g = gate.reshape(rows // GROUP, GROUP, cols)
    u = up.reshape(rows // GROUP, GROUP, cols)
    return torch.stack((g, u), dim=1).reshape(2 * rows, cols).contiguous()


def split_gate_up(interleaved: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of interleave_gate_up."""
    rows2, cols = interleaved.shape
    x = interleaved.reshape(rows2 // (2 * GROUP), 2, GROUP, cols)
    return (x[:, 0].reshape(rows2 // 2, cols).contiguous(),
            x[:, 1].reshape(rows2 // 2, cols).contiguous())
