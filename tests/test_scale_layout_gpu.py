"""GPU checks of the blocked scale-factor export: bytes identical to the oracle's restatement
(through the C ABI and the torch module, aligned and unaligned inputs), the round trip, and a
cross-check of this library's GEMM against a library block-scaled GEMM (cuBLAS through
torch._scaled_mm) fed with the exported factors."""
import numpy as np
import pytest
import torch

from my_nvfp4_gemm_b200 import capi

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1), (130, 5), (97, 33), (300, 64), (1000, 17), (8192, 512)]


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_to_blocked_bit_exact_vs_oracle(oracle, rows, cols):
    rng = np.random.default_rng(rows + 7 * cols)
    sf = rng.integers(0, 256, size=(rows, cols), dtype=np.uint8)
    want = oracle.scale_to_blocked(sf)
    x = torch.from_numpy(sf).cuda()
    out = torch.full((capi.blocked_scale_bytes(rows, cols),), 0xAB, dtype=torch.uint8, device="cuda")
    capi.check(capi.scale_to_blocked(x.data_ptr(), rows, cols, out.data_ptr(), _stream()),
               "nvfp4_scale_to_blocked")
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), want)
    back = torch.full((rows, cols), 0xCD, dtype=torch.uint8, device="cuda")
    capi.check(capi.scale_from_blocked(out.data_ptr(), rows, cols, back.data_ptr(), _stream()),
               "nvfp4_scale_from_blocked")
    torch.cuda.synchronize()
    assert np.array_equal(back.cpu().numpy(), sf)


def test_unaligned_source_uses_the_byte_path(oracle):
    rows, cols = 257, 12
    rng = np.random.default_rng(3)
    sf = rng.integers(0, 256, size=(rows, cols), dtype=np.uint8)
    buf = torch.zeros(rows * cols + 1, dtype=torch.uint8, device="cuda")
    buf[1:] = torch.from_numpy(sf.reshape(-1)).cuda()
    out = torch.empty(capi.blocked_scale_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    capi.check(capi.scale_to_blocked(buf.data_ptr() + 1, rows, cols, out.data_ptr(), _stream()),
               "nvfp4_scale_to_blocked")
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), oracle.scale_to_blocked(sf))


def test_plugins_swizzle_round_trip(plugins, oracle):
    g = torch.Generator(device="cuda").manual_seed(11)
    A = torch.randn(3, 100, 512, device="cuda", generator=g).to(torch.bfloat16)
    s = 6 * 448 / A.abs().max().float()
    _, a_sf = plugins.quantize_nvfp4(A, s)                       # [3, 100, 32]
    blocked = plugins.swizzle_scale_factors(a_sf)
    assert blocked.dtype == torch.float8_e4m3fn and blocked.dim() == 1
    want = oracle.scale_to_blocked(a_sf.view(torch.uint8).reshape(300, 32).cpu().numpy())
    assert np.array_equal(blocked.view(torch.uint8).cpu().numpy(), want)
    back = plugins.unswizzle_scale_factors(blocked, 300, 32)
    assert torch.equal(back.view(torch.uint8), a_sf.view(torch.uint8).reshape(300, 32))
    with pytest.raises(RuntimeError, match="expected"):
        plugins.unswizzle_scale_factors(blocked[:-1], 300, 32)


def _library_gemm(a, b, a_sf, b_sf, plugins):
    """cuBLAS block-scaled NVFP4 GEMM through torch._scaled_mm, fp32 out (acc with no 1/scale)."""
    sa = plugins.swizzle_scale_factors(a_sf)
    sb = plugins.swizzle_scale_factors(b_sf)
    a4 = a.view(torch.float4_e2m1fn_x2)
    b4 = b.view(torch.float4_e2m1fn_x2)
    try:
        return torch._scaled_mm(a4, b4.t(), sa, sb, out_dtype=torch.float32), True
    except (RuntimeError, NotImplementedError):
        try:
            return torch._scaled_mm(a4, b4.t(), sa, sb, out_dtype=torch.bfloat16), False
        except (RuntimeError, NotImplementedError) as e:  # library path absent in this torch build
            pytest.skip(f"torch._scaled_mm has no NVFP4 path here: {e}")


@pytest.mark.parametrize("M,N,K", [(512, 768, 1024), (128, 28672, 8192), (2048, 2048, 4096)])
def test_gemm_matches_library_gemm_on_exported_factors(plugins, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    sA = 6 * 448 / A.abs().max().float()
    sB = 6 * 448 / B.abs().max().float()
    a, a_sf = plugins.quantize_nvfp4(A, sA)
    b, b_sf = plugins.quantize_nvfp4(B, sB)
    scale = sA * sB
    ours = plugins.gemm_nvfp4(a, b, a_sf, b_sf, scale).float()
    lib, fp32_out = _library_gemm(a, b, a_sf, b_sf, plugins)
    if fp32_out:
        # Same bf16 rounding on both sides: only the fp32 summation order differs.
        theirs = (lib / scale).to(torch.bfloat16).float()
        tol = 1e-4
    else:
        theirs = lib.float() / scale    # library rounded to bf16 before the 1/scale
        tol = 4e-3
    rel = ((ours - theirs).norm() / theirs.norm()).item()
    assert rel <= tol, rel
