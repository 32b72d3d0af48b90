"""GPU parity of quantize / dequantize: bit-exact against the CPU oracle and against the
reference's own kernels (rebuilt from source for sm_100a) on the same inputs, through the C ABI
and through the torch module."""
import numpy as np
import pytest
import torch

import nvfp4_cases as cases
from my_nvfp4_gemm_b200 import capi

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def dev_bits(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda()


def capi_quantize(x_bits: np.ndarray, s: float, device_scale: bool = True):
    n = x_bits.size
    x = dev_bits(x_bits)
    q = torch.empty(n // 2, dtype=torch.uint8, device="cuda")
    sf = torch.empty(n // 16, dtype=torch.uint8, device="cuda")
    if device_scale:
        st_t = torch.tensor(s, dtype=torch.float32, device="cuda")
        st = capi.quantize(x.data_ptr(), st_t.data_ptr(), n, q.data_ptr(), sf.data_ptr(), _stream())
    else:
        st = capi.quantize_host_scale(x.data_ptr(), float(s), n, q.data_ptr(), sf.data_ptr(), _stream())
    capi.check(st, "nvfp4_quantize")
    torch.cuda.synchronize()
    return q.cpu().numpy(), sf.cpu().numpy()


def capi_dequantize(q_np: np.ndarray, sf_np: np.ndarray, s: float, device_scale: bool = True):
    q = torch.from_numpy(q_np).cuda()
    sf = torch.from_numpy(sf_np).cuda()
    y = torch.empty(q_np.size * 2, dtype=torch.int16, device="cuda")
    if device_scale:
        st_t = torch.tensor(s, dtype=torch.float32, device="cuda")
        st = capi.dequantize(q.data_ptr(), st_t.data_ptr(), sf.data_ptr(), q_np.size, y.data_ptr(), _stream())
    else:
        st = capi.dequantize_host_scale(q.data_ptr(), float(s), sf.data_ptr(), q_np.size, y.data_ptr(), _stream())
    capi.check(st, "nvfp4_dequantize")
    torch.cuda.synchronize()
    return y.cpu().numpy().view(np.uint16)


def ref_quantize(ref, x_bits, s):
    x = dev_bits(x_bits)
    q = torch.empty(x_bits.size // 2, dtype=torch.uint8, device="cuda")
    sf = torch.empty(x_bits.size // 16, dtype=torch.uint8, device="cuda")
    assert ref.ref_quantize_nvfp4(x.data_ptr(), float(s), x_bits.size, q.data_ptr(), sf.data_ptr(), _stream()) == 0
    torch.cuda.synchronize()
    return q.cpu().numpy(), sf.cpu().numpy()


def ref_dequantize(ref, q_np, sf_np, s):
    q = torch.from_numpy(q_np).cuda()
    sf = torch.from_numpy(sf_np).cuda()
    y = torch.empty(q_np.size * 2, dtype=torch.int16, device="cuda")
    assert ref.ref_de_quantize_nvfp4(q.data_ptr(), float(s), sf.data_ptr(), q_np.size, y.data_ptr(), _stream()) == 0
    torch.cuda.synchronize()
    return y.cpu().numpy().view(np.uint16)


@pytest.fixture(scope="module")
def ref_kernels(oracle):
    ref = oracle.load_reference_kernels()
    if ref is None:
        pytest.skip("reference kernels (oracle/_ref) not built")
    return ref


def _first_mismatch(a, b):
    bad = np.nonzero(a != b)[0]
    return f"{bad.size} mismatches, first at {bad[:8]}: {a[bad[:4]]} vs {b[bad[:4]]}"


@pytest.mark.parametrize("device_scale", [True, False])
def test_quantize_edge_cases_bit_exact_vs_oracle(oracle, device_scale):
    x = cases.quantize_case_blocks()
    for s in cases.quantize_case_scales(x):
        q, sf = capi_quantize(x, s, device_scale)
        oq, osf = oracle.quantize(x, s)
        assert np.array_equal(sf, osf), f"s={s}: sf " + _first_mismatch(sf, osf)
        assert np.array_equal(q, oq), f"s={s}: packed " + _first_mismatch(q, oq)


def test_quantize_edge_cases_bit_exact_vs_reference_kernel(ref_kernels):
    x = cases.quantize_case_blocks(seed=99)
    for s in cases.quantize_case_scales(x):
        q, sf = capi_quantize(x, s)
        rq, rsf = ref_quantize(ref_kernels, x, s)
        assert np.array_equal(sf, rsf), f"s={s}: sf " + _first_mismatch(sf, rsf)
        assert np.array_equal(q, rq), f"s={s}: packed " + _first_mismatch(q, rq)


@pytest.mark.parametrize("device_scale", [True, False])
def test_dequantize_exhaustive_bit_exact(oracle, ref_kernels, device_scale):
    q, sf = cases.dequant_exhaustive_inputs()
    for s in cases.DEQUANT_SCALES:
        y = capi_dequantize(q, sf, s, device_scale)
        assert np.array_equal(y, oracle.dequantize(q, s, sf)), f"s={s} vs oracle"
        assert np.array_equal(y, ref_dequantize(ref_kernels, q, sf, s)), f"s={s} vs reference kernel"


def test_activation_8192x8192_with_outliers_bit_exact(oracle, ref_kernels):
    """The quantize/dequantize workload at full size: 8192x8192 bf16 N(0,1), seed 1, 0.5% of
    elements x50; scale from the reference recipe; bytes identical to oracle and reference."""
    rng = np.random.default_rng(1)
    x = cases.activation(rng, 8192, 8192, outlier_frac=0.005)
    s = oracle.global_scale(x)
    q, sf = capi_quantize(x.reshape(-1), s)
    rq, rsf = ref_quantize(ref_kernels, x.reshape(-1), s)
    assert np.array_equal(sf, rsf) and np.array_equal(q, rq)
    oq, osf = oracle.quantize(x.reshape(-1), s)
    assert np.array_equal(sf, osf) and np.array_equal(q, oq)
    y = capi_dequantize(q, sf, s)
    assert np.array_equal(y, ref_dequantize(ref_kernels, q, sf, s))
    assert np.array_equal(y, oracle.dequantize(q, s, sf))


@pytest.mark.parametrize("shape", [(16,), (3, 48), (2, 5, 64), (1, 8192), (1000, 272)])
def test_plugins_quantize_roundtrip_shapes(plugins, oracle, shape):
    g = torch.Generator(device="cuda").manual_seed(7)
    A = torch.randn(*shape, device="cuda", generator=g, dtype=torch.float32).to(torch.bfloat16)
    s = 6 * 448 / A.abs().max().to(dtype=torch.float32)
    a, a_sf = plugins.quantize_nvfp4(A, s)
    assert a.dtype == torch.uint8 and a.shape == (*shape[:-1], shape[-1] // 2)
    assert a_sf.dtype == torch.float8_e4m3fn and a_sf.shape == (*shape[:-1], shape[-1] // 16)
    bits = A.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
    oq, osf = oracle.quantize(bits, s.item())
    assert np.array_equal(a.cpu().numpy().reshape(-1), oq)
    assert np.array_equal(a_sf.view(torch.uint8).cpu().numpy().reshape(-1), osf)
    # a CPU scale tensor gives the same bytes (host-scale path)
    a2, a_sf2 = plugins.quantize_nvfp4(A, s.cpu())
    assert torch.equal(a2, a) and torch.equal(a_sf2.view(torch.uint8), a_sf.view(torch.uint8))
    r = plugins.de_quantize_nvfp4(a, s, a_sf)
    assert r.dtype == torch.bfloat16 and r.shape == A.shape
    want = oracle.dequantize(oq, s.item(), osf)
    assert np.array_equal(r.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1), want)


def test_plugins_reject_bad_shapes_on_gpu(plugins):
    s = torch.tensor(1.0, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 16"):
        plugins.quantize_nvfp4(torch.zeros(4, 24, dtype=torch.bfloat16, device="cuda"), s)
    q = torch.zeros(4, 8, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError, match="scale factors"):
        plugins.de_quantize_nvfp4(q, s, torch.zeros(4, 2, device="cuda").to(torch.float8_e4m3fn))


def test_empty_tensors(plugins):
    s = torch.tensor(1.0, device="cuda")
    a, a_sf = plugins.quantize_nvfp4(torch.zeros(0, 32, dtype=torch.bfloat16, device="cuda"), s)
    assert a.shape == (0, 16) and a_sf.shape == (0, 2)
    r = plugins.de_quantize_nvfp4(a, s, a_sf)
    assert r.shape == (0, 32)


def _auto_scale_input(case):
    g = torch.Generator(device="cuda").manual_seed(31)
    X = torch.randn(1000, 272, device="cuda", generator=g)
    if case == "outliers":
        X.view(-1)[:: 197] *= 50.0
    elif case == "zeros":
        X.zero_()
    elif case == "nan":
        X[17, 5] = float("nan")
    elif case == "inf":
        X[999, 271] = float("-inf")
    elif case == "tiny":
        X *= 1e-30
    return X.to(torch.bfloat16)


@pytest.mark.parametrize("case", ["normal", "outliers", "zeros", "nan", "inf", "tiny"])
def test_quantize_auto_scale_matches_torch_recipe(plugins, case):
    """The device-computed per-tensor scale equals torch's evaluation of the reference recipe
    (test.py:10-11) bit for bit, and the bytes equal quantize_nvfp4 with that scale."""
    X = _auto_scale_input(case)
    q, sf, s = plugins.quantize_nvfp4_auto_scale(X)
    s_ref = 6 * 448 / X.abs().max().to(dtype=torch.float32)
    assert s.shape == () and s.dtype == torch.float32 and s.device == X.device
    if torch.isnan(s_ref):
        assert torch.isnan(s)
    else:
        assert s.view(torch.int32).item() == s_ref.view(torch.int32).item(), (s.item(), s_ref.item())
    q2, sf2 = plugins.quantize_nvfp4(X, s_ref)
    assert torch.equal(q, q2) and torch.equal(sf.view(torch.uint8), sf2.view(torch.uint8))


def test_quantize_auto_scale_large_activation(plugins):
    """8192 x 8192 activation with 0.5% x50 outliers: many amax chunks, reverse traversal."""
    g = torch.Generator(device="cuda").manual_seed(1)
    X = torch.randn(8192, 8192, device="cuda", generator=g)
    idx = torch.randperm(X.numel(), device="cuda", generator=g)[: int(0.005 * X.numel())]
    X.view(-1)[idx] *= 50.0
    X = X.to(torch.bfloat16)
    q, sf, s = plugins.quantize_nvfp4_auto_scale(X)
    s_ref = 6 * 448 / X.abs().max().to(dtype=torch.float32)
    assert s.view(torch.int32).item() == s_ref.view(torch.int32).item()
    q2, sf2 = plugins.quantize_nvfp4(X, s_ref)
    assert torch.equal(q, q2) and torch.equal(sf.view(torch.uint8), sf2.view(torch.uint8))
