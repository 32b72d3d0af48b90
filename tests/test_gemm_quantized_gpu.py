"""The GEMM with its output quantized to NVFP4 in the epilogue gives exactly the bytes of the
oracle's quantization (the reference arithmetic, csrc/quantize/quantize_nvfp4.cu:6-35) of this
library's bf16 GEMM output, and of the library's own quantize_nvfp4 of that output, for both
kernel forms, ragged M and N, and per-tensor output scales that leave blocks in range, saturate
them, or push them toward zero."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _operands(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    return A, B


@pytest.mark.parametrize("M,N,K", [(512, 768, 1024), (96, 512, 512), (300, 416, 768),
                                   (128, 28672, 8192), (2048, 4096, 4096), (1, 256, 512),
                                   (37, 1024, 1024)])
@pytest.mark.parametrize("scale_mult", [1.0, 8.0, 1.0 / 256])
def test_quantized_output_matches_gemm_then_quantize(plugins, oracle, M, N, K, scale_mult):
    A, B = _operands(M, N, K, M + N + K)
    sA = 6 * 448 / A.abs().max().float()
    sB = 6 * 448 / B.abs().max().float()
    a, a_sf = plugins.quantize_nvfp4(A, sA)
    b, b_sf = plugins.quantize_nvfp4(B, sB)
    scale = sA * sB
    D = plugins.gemm_nvfp4(a, b, a_sf, b_sf, scale)
    s_out = (6 * 448 / D.abs().max().float() * scale_mult).reshape(())
    q_ref, sf_ref = plugins.quantize_nvfp4(D, s_out)
    q, sf = plugins.gemm_nvfp4_quantized(a, b, a_sf, b_sf, scale, s_out)
    assert q.shape == (M, N // 2) and sf.shape == (M, N // 16)
    assert_oracle_bytes(oracle, D, s_out, q, sf)
    assert torch.equal(sf.view(torch.uint8), sf_ref.view(torch.uint8)), "scale bytes differ"
    assert torch.equal(q, q_ref), "packed codes differ"


def assert_oracle_bytes(oracle, D, s_out, q, sf):
    """q, sf are the oracle's quantization of the bf16 D with the per-tensor scale s_out."""
    bits = D.view(torch.int16).cpu().numpy().view(np.uint16)
    oq, osf = oracle.quantize(bits, s_out.item())
    assert np.array_equal(sf.view(torch.uint8).cpu().numpy(), osf), "scale bytes differ from oracle"
    assert np.array_equal(q.cpu().numpy(), oq), "packed codes differ from oracle"


def test_quantized_output_8192_cube(plugins, oracle):
    A, B = _operands(8192, 8192, 8192, 2)
    sA = 6 * 448 / A.abs().max().float()
    sB = 6 * 448 / B.abs().max().float()
    a, a_sf = plugins.quantize_nvfp4(A, sA)
    b, b_sf = plugins.quantize_nvfp4(B, sB)
    D = plugins.gemm_nvfp4(a, b, a_sf, b_sf, sA * sB)
    s_out = (6 * 448 / D.abs().max().float()).reshape(())
    q_ref, sf_ref = plugins.quantize_nvfp4(D, s_out)
    q, sf = plugins.gemm_nvfp4_quantized(a, b, a_sf, b_sf, sA * sB, s_out)
    assert_oracle_bytes(oracle, D, s_out, q, sf)
    assert torch.equal(sf.view(torch.uint8), sf_ref.view(torch.uint8))
    assert torch.equal(q, q_ref)


def test_quantized_output_rejects(plugins):
    a = torch.zeros(4, 128, dtype=torch.uint8, device="cuda")
    b = torch.zeros(24, 128, dtype=torch.uint8, device="cuda")
    asf = torch.zeros(4, 16, device="cuda").to(torch.float8_e4m3fn)
    bsf = torch.zeros(24, 16, device="cuda").to(torch.float8_e4m3fn)
    s = torch.tensor(1.0, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 32"):
        plugins.gemm_nvfp4_quantized(a, b, asf, bsf, s, s)
    with pytest.raises(RuntimeError, match="on the GPU"):
        plugins.gemm_nvfp4_quantized(a, b[:16].contiguous(), asf, bsf[:16].contiguous(), s, s.cpu())
