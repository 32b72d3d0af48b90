"""CPU tests of the oracle itself: known answers, internal consistency, and (when present) the
golden vectors produced by the reference's own kernels on a B200 (tests/golden/)."""
import os

import numpy as np
import pytest
import torch

import nvfp4_cases as cases

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_kernels_sm100a.npz")


def test_e2m1_rounding_known_answers(oracle):
    # ties to even, saturation, signed zero (cvt.rn.satfinite.e2m1x2.f32, common.h:65-83)
    table = [(0.0, 0x0), (0.25, 0x0), (0.2501, 0x1), (0.5, 0x1), (0.75, 0x2), (1.0, 0x2),
             (1.25, 0x2), (1.2501, 0x3), (1.5, 0x3), (1.75, 0x4), (2.0, 0x4), (2.5, 0x4),
             (2.5001, 0x5), (3.0, 0x5), (3.5, 0x6), (4.0, 0x6), (5.0, 0x6), (5.0001, 0x7),
             (6.0, 0x7), (1e30, 0x7), (float("inf"), 0x7), (-0.0, 0x8), (-1e-9, 0x8),
             (-0.75, 0xA), (-6.0, 0xF), (-float("inf"), 0xF)]
    for x, code in table:
        assert oracle.f32_to_e2m1(x) == code, (x, oracle.f32_to_e2m1(x), code)
    for code in range(16):
        assert oracle.f32_to_e2m1(oracle.e2m1_to_f32(code)) == code


def test_e4m3_matches_torch_with_saturation(oracle):
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(20000) * 200, rng.uniform(0, 2 ** -6, 20000),
                         [447.9, 448.0, 455.9, 464.0, 1e9, np.inf, -np.inf, 2 ** -10, 2 ** -10 * 1.0001,
                          3 * 2 ** -11]]).astype(np.float32)
    mine = np.array([oracle.f32_to_e4m3(float(v)) for v in xs], np.uint8)
    want = torch.from_numpy(np.clip(xs, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert (mine == want).all()
    assert oracle.f32_to_e4m3(float("nan")) == 0x7F
    for v in range(256):
        f = oracle.e4m3_to_f32(v)
        if (v & 0x7F) == 0x7F:
            assert np.isnan(f)
        else:
            assert oracle.f32_to_e4m3(f) == v


def test_bf16_rounding_matches_torch(oracle):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(100000) * 10.0 ** rng.uniform(-30, 30, 100000)).astype(np.float32)
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert (oracle.f32_to_bf16_array(x) == want).all()


def test_quantize_block_recipe_by_hand(oracle):
    # One block worked through the reference arithmetic (quantize_nvfp4.cu:14-34) by hand:
    # amax = 6, s = 1 -> sf = e4m3(6 * 1 * (1/6)) = 1.0 (0x38), os = 1 -> codes are the values.
    vals = np.array(cases.TIES + [-v for v in cases.TIES], np.float32)
    q, sf = oracle.quantize(cases.f32_to_bf16_bits(vals), 1.0)
    assert sf.tolist() == [0x38]
    codes = [oracle.f32_to_e2m1(float(v)) for v in vals]
    packed = [codes[2 * i] | (codes[2 * i + 1] << 4) for i in range(8)]
    assert q.tolist() == packed
    # zero block: amax floor 2^-133 -> sf 0 -> os = rcp(0) = inf -> 0 * inf = NaN codes
    q0, sf0 = oracle.quantize(np.zeros(16, np.uint16), 1.0)
    assert sf0.tolist() == [0]
    nan_code = oracle.f32_to_e2m1(float("nan"))
    assert q0.tolist() == [nan_code | (nan_code << 4)] * 8


def test_dequantize_inverts_codes(oracle):
    rng = np.random.default_rng(2)
    x = cases.f32_to_bf16_bits(rng.standard_normal(4096).astype(np.float32))
    s = cases.quantize_case_scales(x)[0]
    q, sf = oracle.quantize(x, s)
    y = oracle.dequantize(q, s, sf)
    # re-quantizing the dequantized tensor with the same scale reproduces the codes
    q2, sf2 = oracle.quantize(y, s)
    assert (sf2 == sf).all() and (q2 == q).all()
    # and the reconstruction error is bounded by half the widest code step (2 at 4..6) of each
    # block's scale sf/s, plus the bf16 rounding of the output
    xf, yf = cases.bf16_bits_to_f32(x), cases.bf16_bits_to_f32(y)
    step = np.repeat(np.array([oracle.e4m3_to_f32(int(v)) for v in sf], np.float32), 16) / np.float32(s)
    assert (np.abs(xf - yf) <= step * (1.0 + 2.0 ** -7)).all()


def test_gemm_oracle_paths_agree(oracle):
    rng = np.random.default_rng(3)
    M, N, K = 33, 40, 512
    A = rng.integers(0, 256, (M, K // 2), dtype=np.uint8)
    B = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    Asf = rng.integers(0x20, 0x48, (M, K // 16), dtype=np.uint8)
    Bsf = rng.integers(0x20, 0x48, (N, K // 16), dtype=np.uint8)
    d32_c, d16_c = oracle.gemm_c(A, B, Asf, Bsf, 3.5)
    d32_np = oracle.gemm_f32(A, B, Asf, Bsf, 3.5)
    assert np.array_equal(d32_c, d32_np)
    assert np.array_equal(d16_c, oracle.f32_to_bf16_array(d32_np))


def test_cpu_plumbing_config(oracle):
    """The CPU plumbing workload: A, B bf16 256x256 N(0,1) seed 0, quantize, dequantize, and
    C = bf16(fp32(A_r @ B_r^T)) with alpha = 1 — emulated on the host as in the reference test."""
    g = torch.Generator().manual_seed(0)
    A = torch.randn(256, 256, generator=g).to(torch.bfloat16)
    B = torch.randn(256, 256, generator=g).to(torch.bfloat16)
    a_bits = A.view(torch.int16).numpy().view(np.uint16)
    b_bits = B.view(torch.int16).numpy().view(np.uint16)
    sa, sb = oracle.global_scale(a_bits), oracle.global_scale(b_bits)
    assert sa == np.float32((6 * 448 / A.abs().max().float()).item())
    qa, fa = oracle.quantize(a_bits, sa)
    qb, fb = oracle.quantize(b_bits, sb)
    ar = torch.from_numpy(oracle.dequantize(qa, sa, fa).view(np.int16)).view(torch.bfloat16)
    br = torch.from_numpy(oracle.dequantize(qb, sb, fb).view(np.int16)).view(torch.bfloat16)
    C = (ar.float() @ br.float().T).to(torch.bfloat16)
    # the GEMM oracle on the packed operands gives the same product (scale = s_A * s_B)
    d = oracle.gemm(qa, qb, fa, fb, np.float32(sa) * np.float32(sb))
    Cd = torch.from_numpy(d.view(np.int16)).view(torch.bfloat16).float()
    rel = (Cd - C.float()).norm() / C.float().norm()
    assert rel < 1e-2  # dequantized-bf16 operands vs exact block products
    # quantization error of the whole pipeline against the unquantized fp32 product
    exact = A.float() @ B.float().T
    assert (Cd - exact).norm() / exact.norm() < 0.2


@pytest.mark.skipif(not os.path.exists(GOLDEN), reason="golden vectors not generated yet")
def test_oracle_matches_reference_kernels_golden(oracle):
    """Bit-exact agreement with the reference's own quantize/dequantize kernels (sm_100a)."""
    g = np.load(GOLDEN)
    x = g["q_x"]
    for i, s in enumerate(g["q_scales"]):
        q, sf = oracle.quantize(x, s)
        bad_q = np.nonzero(q != g["q_packed"][i])[0]
        bad_sf = np.nonzero(sf != g["q_sf"][i])[0]
        assert bad_sf.size == 0, f"scale {s}: sf mismatch at blocks {bad_sf[:8]}"
        assert bad_q.size == 0, f"scale {s}: packed mismatch at bytes {bad_q[:8]}"
    for i, s in enumerate(g["dq_scales"]):
        y = oracle.dequantize(g["dq_packed"], s, g["dq_sf"])
        bad = np.nonzero(y != g["dq_out"][i])[0]
        assert bad.size == 0, f"scale {s}: dequant mismatch at {bad[:8]}: {y[bad[:4]]} vs {g['dq_out'][i][bad[:4]]}"
