"""my_nvfp4_gemm_b200 — NVFP4 quantize / dequantize / GEMM for NVIDIA B200 (sm_100a).

Drop-in for the reference plugin's ``my_plugins`` module (``from csrc import my_plugins``):

    from my_nvfp4_gemm_b200 import my_plugins
    a, a_sf = my_plugins.quantize_nvfp4(A, A_scale)
    d = my_plugins.gemm_nvfp4(a, b, a_sf, b_sf, A_scale * B_scale)

``capi`` is the ctypes view of the C ABI (include/nvfp4_b200.h); ``sharded`` holds the
multi-GPU column-parallel GEMM and row-sharded quantize over torch.distributed.

There is no CPU implementation: the CUDA library must be built
(``python -m my_nvfp4_gemm_b200.build``) and a B200 present for any compute call.
"""
from __future__ import annotations

import importlib
import os

from . import build as _build

__all__ = ["my_plugins", "capi", "load_my_plugins"]
__version__ = "0.1.0"


def load_my_plugins():
    """Import the compiled ``my_plugins`` torch extension (torch is imported first)."""
    import torch  # noqa: F401  (the extension links against libtorch)

    if not os.path.exists(_build.ext_path()):
        raise ImportError(
            f"{_build.ext_path()} is missing: run `python -m my_nvfp4_gemm_b200.build`")
    return importlib.import_module(".my_plugins", __name__)


def __getattr__(name):
    if name == "my_plugins":
        mod = load_my_plugins()
        globals()["my_plugins"] = mod
        return mod
    if name == "capi":
        mod = importlib.import_module(".capi", __name__)
        globals()["capi"] = mod
        return mod
    if name == "sharded":
        mod = importlib.import_module(".sharded", __name__)
        globals()["sharded"] = mod
        return mod
    raise AttributeError(name)
