"""CPU checks of the gate/up weight interleave used by the SwiGLU GEMM, and of the C ABI's
shape validation for that entry point (no GPU calls)."""
import pytest
import torch

from my_nvfp4_gemm_b200 import capi
from my_nvfp4_gemm_b200.swiglu import interleave_gate_up, split_gate_up


def test_interleave_order_and_round_trip():
    I, X = 384, 5
    gate = torch.arange(I * X).reshape(I, X)
    up = 100000 + torch.arange(I * X).reshape(I, X)
    w = interleave_gate_up(gate, up)
    assert w.shape == (2 * I, X)
    for t in range(I // 128):
        assert torch.equal(w[256 * t: 256 * t + 128], gate[128 * t: 128 * t + 128])
        assert torch.equal(w[256 * t + 128: 256 * t + 256], up[128 * t: 128 * t + 128])
    g2, u2 = split_gate_up(w)
    assert torch.equal(g2, gate) and torch.equal(u2, up)


def test_interleave_rejects():
    with pytest.raises(ValueError):
        interleave_gate_up(torch.zeros(100, 4), torch.zeros(100, 4))
    with pytest.raises(ValueError):
        interleave_gate_up(torch.zeros(128, 4), torch.zeros(256, 4))


def test_swiglu_capi_validation():
    FAKE = 0x10000
    g = capi.gemm_swiglu
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 384, 256) == capi.NVFP4_ERR_UNSUPPORTED_SHAPE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 512, 0) == capi.NVFP4_ERR_UNSUPPORTED_SHAPE
    assert g(FAKE, FAKE, FAKE, FAKE, None, FAKE, 128, 512, 256) == capi.NVFP4_ERR_INVALID_VALUE
    assert g(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE + 8, 128, 512, 256) == capi.NVFP4_ERR_MISALIGNED
    assert g(None, None, None, None, FAKE, None, 0, 512, 256) == capi.NVFP4_OK
