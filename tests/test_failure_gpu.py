"""Failure detection on the GPU without a GPU fault: a bounded device-side wait runs out (a
barrier nothing completes, 1 ms limit), the kernel records NVFP4_ERR_DEVICE_TIMEOUT in the
library's device status word and returns normally, and the context stays usable."""
import pytest
import torch

from my_nvfp4_gemm_b200 import capi

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    stream = torch.cuda.current_stream().cuda_stream
    capi.clear_device_status(stream)
    assert capi.device_status(stream) == 0
    capi.check(capi.selftest_wait_timeout(1_000_000, stream), "selftest")  # 1 ms
    torch.cuda.synchronize()
    assert capi.device_status(stream) == capi.NVFP4_ERR_DEVICE_TIMEOUT
    capi.clear_device_status(stream)
    assert capi.device_status(stream) == 0
    # the context is intact: ordinary work still runs
    x = torch.randn(1024, device="cuda")
    assert torch.isfinite((x * 2).sum()).item()


def test_plugins_expose_status(plugins):
    plugins.clear_device_status()
    assert plugins.device_status() == 0
