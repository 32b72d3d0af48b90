"""Gate+up GEMM with SwiGLU in the epilogue: bit-identical to torch's fp32 silu(Dg) * Du on this
library's own bf16 GEMM output (D against the plain [gate; up] weight), for both kernel forms
and ragged M; and within the GEMM tolerance of the fp32 oracle product."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from my_nvfp4_gemm_b200.swiglu import interleave_gate_up

pytestmark = pytest.mark.gpu


def _case(plugins, M, I, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    X = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(2 * I, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    sX = 6 * 448 / X.abs().max().float()
    sW = 6 * 448 / W.abs().max().float()
    x, x_sf = plugins.quantize_nvfp4(X, sX)
    w, w_sf = plugins.quantize_nvfp4(W, sW)            # [gate; up]
    return x, x_sf, w, w_sf, sX * sW


@pytest.mark.parametrize("M,I,K", [(96, 384, 512), (512, 1024, 1024), (300, 128, 768),
                                   (1024, 28672, 8192), (3, 256, 512), (70, 640, 1024)])
def test_swiglu_matches_torch_on_gemm_output(plugins, M, I, K):
    x, x_sf, w, w_sf, scale = _case(plugins, M, I, K, M + I + K)
    D = plugins.gemm_nvfp4(x, w, x_sf, w_sf, scale)
    want = (F.silu(D[:, :I].float()) * D[:, I:].float()).to(torch.bfloat16)
    wi = interleave_gate_up(w[:I], w[I:])
    wi_sf = interleave_gate_up(w_sf[:I].view(torch.uint8), w_sf[I:].view(torch.uint8)).view(
        torch.float8_e4m3fn)
    out = plugins.gemm_nvfp4_swiglu(x, wi, x_sf, wi_sf, scale)
    assert out.shape == (M, I) and out.dtype == torch.bfloat16
    diff = (out.view(torch.int16) != want.view(torch.int16))
    assert not diff.any(), f"{int(diff.sum())} of {diff.numel()} outputs differ"


def test_swiglu_within_tolerance_of_oracle(plugins, oracle):
    M, I, K = 256, 256, 512
    x, x_sf, w, w_sf, scale = _case(plugins, M, I, K, 5)
    A = oracle.decode_scaled(x.cpu().numpy(), x_sf.view(torch.uint8).cpu().numpy())
    B = oracle.decode_scaled(w.cpu().numpy(), w_sf.view(torch.uint8).cpu().numpy())
    D = (A.astype(np.float64) @ B.astype(np.float64).T) / float(scale)
    ref = torch.from_numpy(D[:, :I] / (1 + np.exp(-D[:, :I])) * D[:, I:]).float()
    wi = interleave_gate_up(w[:I], w[I:])
    wi_sf = interleave_gate_up(w_sf[:I].view(torch.uint8), w_sf[I:].view(torch.uint8)).view(
        torch.float8_e4m3fn)
    out = plugins.gemm_nvfp4_swiglu(x, wi, x_sf, wi_sf, scale).float().cpu()
    rel = ((out - ref).norm() / ref.norm()).item()
    assert rel <= 8e-3, rel   # three bf16 roundings (Dg, Du, the product) on the way
