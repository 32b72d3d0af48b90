"""CPU tests of the drop-in boundary: the C-ABI library loads and exports every declared symbol,
host-side validation returns the documented status codes before any device work, and the torch
module raises RuntimeError on the inputs the reference rejects (no GPU needed for any of it)."""
import ctypes
import os
import re

import pytest
import torch

from my_nvfp4_gemm_b200 import capi

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "nvfp4_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nvfp4_[a-z_0-9]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    names = declared_functions()
    assert len(names) >= 11
    L = capi.lib()
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(capi.SIGNATURES), "ctypes signatures out of sync with the header"


def test_only_the_c_abi_is_exported():
    """Kernel stubs and C++ helpers are local to the library (linker version script): a second
    build loaded into the same process cannot resolve to this one's kernels."""
    import shutil
    import subprocess
    if shutil.which("nm") is None:
        pytest.skip("nm not available")
    out = subprocess.run(["nm", "-D", "--defined-only", capi._build.lib_path()], check=True,
                         capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    exported = {n.split("@")[0] for n in exported}
    assert exported, "no exported symbols"
    assert exported == set(declared_functions()), sorted(exported ^ set(declared_functions()))


def test_status_strings_and_version():
    assert capi.status_string(0) == "NVFP4_OK"
    for code, name in capi.STATUS_NAMES.items():
        assert capi.status_string(code) == name
    assert capi.status_string(99) == "NVFP4_ERR_UNKNOWN"
    assert capi.lib().nvfp4_version() == 0x000100


# Validation happens on the host before any CUDA call, so these run without a GPU. Fake but
# well-aligned addresses are never dereferenced.
FAKE = 0x10000


def test_quantize_validation():
    assert capi.quantize(FAKE, FAKE, 15, FAKE, FAKE) == capi.NVFP4_ERR_UNSUPPORTED_SHAPE
    assert capi.quantize(FAKE, FAKE, -16, FAKE, FAKE) == capi.NVFP4_ERR_INVALID_VALUE
    assert capi.quantize(FAKE, None, 16, FAKE, FAKE) == capi.NVFP4_ERR_INVALID_VALUE
    assert capi.quantize(FAKE + 8, FAKE, 16, FAKE, FAKE) == capi.NVFP4_ERR_MISALIGNED
    assert capi.quantize(FAKE, FAKE, 16, FAKE + 2, FAKE) == capi.NVFP4_ERR_MISALIGNED
    assert capi.quantize(None, FAKE, 16, FAKE, FAKE) == capi.NVFP4_ERR_INVALID_VALUE
    assert capi.quantize(None, FAKE, 0, None, None) == capi.NVFP4_OK  # empty: no-op
    assert capi.quantize_host_scale(FAKE, 1.0, 24, FAKE, FAKE) == capi.NVFP4_ERR_UNSUPPORTED_SHAPE


def test_quantize_auto_scale_validation():
    ws = capi.quantize_auto_scale_workspace_bytes
    assert ws(0) == 4 and ws(16) == 4 and ws(131072) == 4 and ws(131088) == 8
    assert ws(8192 * 8192) == 4 * 512
    q = capi.quantize_auto_scale
    assert q(FAKE, 24, FAKE, FAKE, FAKE, FAKE, 64) == capi.NVFP4_ERR_UNSUPPORTED_SHAPE
    assert q(FAKE, 16, FAKE, FAKE, FAKE, None, 64) == capi.NVFP4_ERR_INVALID_VALUE
    assert q(FAKE, 16, FAKE, FAKE, None, FAKE, 64) == capi.NVFP4_ERR_INVALID_VALUE
    assert q(FAKE, 262144, FAKE, FAKE, FAKE, FAKE, 4) == 7  # workspace too small: TOO_LARGE
    assert q(FAKE + 8, 16, FAKE, FAKE, FAKE, FAKE, 64) == capi.NVFP4_ERR_MISALIGNED


def test_dequantize_validation():
    assert capi.dequantize(FAKE, FAKE, FAKE, 12, FAKE) == capi.NVFP4_ERR_UNSUPPORTED_SHAPE
    assert capi.dequantize(FAKE, FAKE, FAKE, 8, FAKE + 8) == capi.NVFP4_ERR_MISALIGNED
    assert capi.dequantize(FAKE, None, FAKE, 8, FAKE) == capi.NVFP4_ERR_INVALID_VALUE
    assert capi.dequantize_host_scale(FAKE, 1.0, None, 8, FAKE) == capi.NVFP4_ERR_INVALID_VALUE
    assert capi.dequantize(None, FAKE, None, 0, None) == capi.NVFP4_OK


def test_gemm_validation():
    g = capi.gemm
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 128, 200) == capi.NVFP4_ERR_UNSUPPORTED_SHAPE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 12, 256) == capi.NVFP4_ERR_UNSUPPORTED_SHAPE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, -1, 128, 256) == capi.NVFP4_ERR_INVALID_VALUE
    assert g(FAKE, FAKE, FAKE, FAKE, None, FAKE, 128, 128, 256) == capi.NVFP4_ERR_INVALID_VALUE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE + 2, 128, 128, 256) == capi.NVFP4_ERR_MISALIGNED
    assert g(FAKE + 4, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 128, 256) == capi.NVFP4_ERR_MISALIGNED
    assert g(FAKE, FAKE, FAKE, FAKE + 8, FAKE, FAKE, 128, 128, 256) == capi.NVFP4_ERR_MISALIGNED
    assert g(None, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 128, 256) == capi.NVFP4_ERR_INVALID_VALUE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1 << 31, 128, 256) == capi.lib().nvfp4_gemm(
        FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1 << 31, 128, 256, None)
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1 << 31, 128, 256) == 7  # NVFP4_ERR_TOO_LARGE
    assert g(None, None, None, None, FAKE, None, 0, 128, 256) == capi.NVFP4_OK  # M == 0
    assert capi.gemm_host_scale(FAKE, FAKE, FAKE, FAKE, 1.0, FAKE, 1, 8, 100) == \
        capi.NVFP4_ERR_UNSUPPORTED_SHAPE


def test_gemm_quantized_validation():
    g = capi.gemm_quantized
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 48, 256) == capi.NVFP4_ERR_UNSUPPORTED_SHAPE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 32, 0) == capi.NVFP4_ERR_UNSUPPORTED_SHAPE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, None, FAKE, FAKE, 128, 32, 256) == capi.NVFP4_ERR_INVALID_VALUE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE + 8, FAKE, 128, 32, 256) == capi.NVFP4_ERR_MISALIGNED
    assert g(None, None, None, None, None, None, None, None, 0, 32, 256) == capi.NVFP4_OK  # M == 0


def test_gemm_allgather_validation():
    g = capi.gemm_allgather
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, [FAKE, FAKE], 2, 128, 32, 256) == capi.NVFP4_ERR_INVALID_VALUE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, [FAKE] * 9, 0, 128, 32, 256) == capi.NVFP4_ERR_INVALID_VALUE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, [FAKE, FAKE], 0, 128, 12, 256) == capi.NVFP4_ERR_UNSUPPORTED_SHAPE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, [FAKE, None], 0, 128, 32, 256) == capi.NVFP4_ERR_INVALID_VALUE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, [FAKE, FAKE + 8], 0, 128, 32, 256) == capi.NVFP4_ERR_MISALIGNED


def test_status_out_pointer_checked():
    assert capi.lib().nvfp4_device_status(None, None) == capi.NVFP4_ERR_INVALID_VALUE


# ---- the torch module: the reference's TORCH_CHECK behaviour --------------------------------
def test_plugins_reject_like_the_reference(plugins):
    s = torch.tensor(1.0)
    with pytest.raises(RuntimeError, match="bf16 and contiguous"):
        plugins.quantize_nvfp4(torch.zeros(4, 16), s)
    with pytest.raises(RuntimeError, match="float32 and scalar"):
        plugins.quantize_nvfp4(torch.zeros(4, 16, dtype=torch.bfloat16), torch.tensor([1.0]))
    with pytest.raises(RuntimeError, match="cuda device"):
        plugins.quantize_nvfp4(torch.zeros(4, 16, dtype=torch.bfloat16), s)
    with pytest.raises(RuntimeError, match="uint8 and contiguous"):
        plugins.de_quantize_nvfp4(torch.zeros(4, 8), s, torch.zeros(4, 1).to(torch.float8_e4m3fn))
    with pytest.raises(RuntimeError, match="float8_e4m3"):
        plugins.de_quantize_nvfp4(torch.zeros(4, 8, dtype=torch.uint8), s, torch.zeros(4, 1))
    with pytest.raises(RuntimeError, match="A must be uint8"):
        plugins.gemm_nvfp4(torch.zeros(4, 128), torch.zeros(8, 128, dtype=torch.uint8),
                           torch.zeros(4, 16).to(torch.float8_e4m3fn),
                           torch.zeros(8, 16).to(torch.float8_e4m3fn), s)
    with pytest.raises(RuntimeError, match="2D"):
        plugins.gemm_nvfp4(torch.zeros(4, 128, 1, dtype=torch.uint8),
                           torch.zeros(8, 128, dtype=torch.uint8),
                           torch.zeros(4, 16).to(torch.float8_e4m3fn),
                           torch.zeros(8, 16).to(torch.float8_e4m3fn), s)
    with pytest.raises(RuntimeError, match="cuda device"):
        plugins.gemm_nvfp4(torch.zeros(4, 128, dtype=torch.uint8),
                           torch.zeros(8, 128, dtype=torch.uint8),
                           torch.zeros(4, 16).to(torch.float8_e4m3fn),
                           torch.zeros(8, 16).to(torch.float8_e4m3fn), s)


def test_extension_links_the_capi_library():
    """The torch module is a thin layer over libnvfp4_b200.so (loaded from the package dir)."""
    from my_nvfp4_gemm_b200 import build, load_my_plugins
    load_my_plugins()
    maps = open("/proc/self/maps").read()
    assert build.lib_path() in maps
