"""GPU parity of the tcgen05 NVFP4 GEMM against the oracle (decoded operands, float64 sums,
fp32 rounding, / scale, bf16 round-to-nearest-even).

Tolerance (the tensor core's fp32 summation order is unspecified, so the result cannot be
bit-reproducible against any other summation): against bf16_rn(oracle_fp32),
  * relative Frobenius error <= 1e-3, and
  * >= 99.9% of elements within 1 bf16 ulp.
Order-independent properties are checked bit-exactly: each output element depends only on its
own row of A and row of B, so sharding N (or M) reproduces the unsharded result bit for bit."""
import numpy as np
import pytest
import torch

import nvfp4_cases as cases
from my_nvfp4_gemm_b200 import capi

pytestmark = pytest.mark.gpu

FRO_TOL = 1e-3
ULP_FRAC = 0.999


def bf16_ordered(bits: np.ndarray) -> np.ndarray:
    b = bits.astype(np.int32)
    return np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), 0x8000 + (b & 0x7FFF))


def assert_gemm_close(out_bits: np.ndarray, ref_f32: np.ndarray, what: str = ""):
    from oracle import oracle as O
    ref_bits = O.f32_to_bf16_array(ref_f32)
    out_f = cases.bf16_bits_to_f32(out_bits).astype(np.float64)
    ref_f = cases.bf16_bits_to_f32(ref_bits).astype(np.float64)
    assert np.isfinite(out_f).all(), f"{what}: non-finite outputs"
    denom = np.linalg.norm(ref_f)
    fro = np.linalg.norm(out_f - ref_f) / (denom if denom > 0 else 1.0)
    ulp = np.abs(bf16_ordered(out_bits) - bf16_ordered(ref_bits))
    frac = float((ulp <= 1).mean()) if ulp.size else 1.0
    assert fro <= FRO_TOL, f"{what}: relative Frobenius error {fro:.3e} > {FRO_TOL}"
    assert frac >= ULP_FRAC, f"{what}: only {frac:.5f} of elements within 1 bf16 ulp (max {ulp.max()})"


def random_operands(rng, M, N, K, sf_lo=0x28, sf_hi=0x40):
    """Random packed operands: every E2M1 code (incl. -0) and a band of UE4M3 scale codes."""
    A = rng.integers(0, 256, (M, K // 2), dtype=np.uint8)
    B = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    Asf = rng.integers(sf_lo, sf_hi, (M, K // 16), dtype=np.uint8)
    Bsf = rng.integers(sf_lo, sf_hi, (N, K // 16), dtype=np.uint8)
    return A, B, Asf, Bsf


def to_dev(*arrs):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]


def capi_gemm(A, B, Asf, Bsf, scale, device_scale=True):
    M, N, K = A.shape[0], B.shape[0], A.shape[1] * 2
    a, b, asf, bsf = to_dev(A, B, Asf, Bsf)
    d = torch.empty(M, N, dtype=torch.int16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    if device_scale:
        s = torch.tensor(scale, dtype=torch.float32, device="cuda")
        st = capi.gemm(a.data_ptr(), b.data_ptr(), asf.data_ptr(), bsf.data_ptr(), s.data_ptr(),
                       d.data_ptr(), M, N, K, stream)
    else:
        st = capi.gemm_host_scale(a.data_ptr(), b.data_ptr(), asf.data_ptr(), bsf.data_ptr(),
                                  float(scale), d.data_ptr(), M, N, K, stream)
    capi.check(st, "nvfp4_gemm")
    torch.cuda.synchronize()
    return d.cpu().numpy().view(np.uint16)


def plugins_gemm(plugins, A, B, Asf, Bsf, scale):
    a, b, asf, bsf = to_dev(A, B, Asf, Bsf)
    s = torch.tensor(scale, dtype=torch.float32, device="cuda")
    d = plugins.gemm_nvfp4(a, b, asf.view(torch.float8_e4m3fn), bsf.view(torch.float8_e4m3fn), s)
    assert d.dtype == torch.bfloat16 and d.shape == (A.shape[0], B.shape[0])
    return d.view(torch.int16).cpu().numpy().view(np.uint16)


SHAPES = [
    (128, 256, 256),     # one tile, one k-stage
    (256, 512, 1024),    # several tiles and stages
    (1, 8, 256),         # smallest legal problem
    (17, 136, 512),      # ragged M and N inside one tile
    (130, 264, 768),     # ragged across tile boundaries
    (300, 520, 2560),
    (1024, 1024, 2048),
    (16, 4096, 8192),    # decode-like, long K
    (5, 520, 1024),      # M < 128: only the M existing rows of A are loaded
    (127, 264, 512),
    (63, 1024, 2048),
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_random_operands(oracle, M, N, K):
    rng = np.random.default_rng(M * 7 + N * 13 + K)
    A, B, Asf, Bsf = random_operands(rng, M, N, K)
    scale = 3.0
    out = capi_gemm(A, B, Asf, Bsf, scale)
    assert_gemm_close(out, oracle.gemm_f32(A, B, Asf, Bsf, scale), f"{M}x{N}x{K}")


def test_gemm_host_scale_matches_device_scale(oracle):
    rng = np.random.default_rng(5)
    A, B, Asf, Bsf = random_operands(rng, 200, 256, 512)
    assert np.array_equal(capi_gemm(A, B, Asf, Bsf, 0.75, True), capi_gemm(A, B, Asf, Bsf, 0.75, False))


@pytest.mark.parametrize("M", [128, 256])
def test_gemm_single_nonzero_scale_factor_positions(oracle, M):
    """Isolates the scale-factor TMEM layout: one non-unit scale factor at a time, in every
    32-row quarter of the A tile (both CTAs of a pair at M=256), both 128-row halves of the
    B tile and every K step."""
    N, K = 256, 512
    rng = np.random.default_rng(11)
    A, B, _, _ = random_operands(rng, M, N, K)
    one = 0x38  # 1.0
    rows = [(0, 0, 0), (37, 5, 3), (70, 131, 9), (127, 255, 31), (96, 200, 16)]
    if M == 256:
        rows += [(128, 3, 2), (165, 140, 7), (255, 255, 30), (200, 77, 12)]
    for (r, n, kb) in rows:
        Asf = np.full((M, K // 16), one, np.uint8)
        Bsf = np.full((N, K // 16), one, np.uint8)
        Asf[r, kb] = 0x48  # 4.0
        Bsf[n, (kb + 5) % (K // 16)] = 0x30  # 0.5
        out = capi_gemm(A, B, Asf, Bsf, 1.0)
        assert_gemm_close(out, oracle.gemm_f32(A, B, Asf, Bsf, 1.0), f"sf at A[{r},{kb}] B[{n}]")


def test_gemm_quantized_activations_match_dequant_matmul(plugins, oracle):
    """The reference test recipe (test.py:7-20) at its own shape: A 128x1024, B 256x1024,
    quantize both, GEMM with scale = s_A * s_B, compare with the dequantized product."""
    g = torch.Generator(device="cuda").manual_seed(100)
    A = torch.randn(128, 1024, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(256, 1024, device="cuda", generator=g).to(torch.bfloat16)
    sA = 6 * 448 / A.abs().max().to(dtype=torch.float32)
    sB = 6 * 448 / B.abs().max().to(dtype=torch.float32)
    a, a_sf = plugins.quantize_nvfp4(A, sA)
    b, b_sf = plugins.quantize_nvfp4(B, sB)
    d = plugins.gemm_nvfp4(a, b, a_sf, b_sf, sA * sB)
    ref = oracle.gemm_f32(a.cpu().numpy(), b.cpu().numpy(), a_sf.view(torch.uint8).cpu().numpy(),
                          b_sf.view(torch.uint8).cpu().numpy(), (sA * sB).item())
    assert_gemm_close(d.view(torch.int16).cpu().numpy().view(np.uint16), ref, "test.py recipe")
    # and against F.linear of the dequantized operands (what the reference test prints)
    ar = plugins.de_quantize_nvfp4(a, sA, a_sf)
    br = plugins.de_quantize_nvfp4(b, sB, b_sf)
    D = torch.nn.functional.linear(ar.float(), br.float())
    rel = ((d.float() - D).norm() / D.norm()).item()
    assert rel < 1e-2, rel  # dequantized operands are bf16-rounded, the GEMM's are exact


def test_gemm_plugins_path_equals_capi_path(plugins):
    rng = np.random.default_rng(6)
    A, B, Asf, Bsf = random_operands(rng, 384, 640, 1024)
    assert np.array_equal(plugins_gemm(plugins, A, B, Asf, Bsf, 2.0), capi_gemm(A, B, Asf, Bsf, 2.0))


def test_gemm_n_and_m_sharding_bit_identical(plugins):
    """Column-parallel sharding (B rows split across shards) and row splits of A reproduce the
    unsharded output exactly: the property the multi-GPU path relies on."""
    rng = np.random.default_rng(8)
    M, N, K = 512, 2048, 2048
    A, B, Asf, Bsf = random_operands(rng, M, N, K)
    full = plugins_gemm(plugins, A, B, Asf, Bsf, 1.5)
    for P in (2, 4, 8):
        w = N // P
        parts = [plugins_gemm(plugins, A, B[r * w:(r + 1) * w], Asf, Bsf[r * w:(r + 1) * w], 1.5)
                 for r in range(P)]
        assert np.array_equal(np.concatenate(parts, axis=1), full), f"P={P}"
    top = plugins_gemm(plugins, A[:200], B, Asf[:200], Bsf, 1.5)
    assert np.array_equal(top, full[:200])


@pytest.mark.parametrize("M,N,K", [(300, 528, 2560), (96, 1024, 512), (1024, 2048, 2048)])
def test_gemm_allgather_on_one_gpu_matches_gemm(M, N, K):
    """The GEMM with the all-gather fused into its epilogue, with every rank's output a buffer on
    this one GPU: rank r stores its column shard into every rank's output, so after the calls of
    ranks 0 and 1 both outputs equal the plain GEMM bit for bit (world 1: the one output does).
    Covers the multi-destination epilogue and its configuration without a second GPU."""
    rng = np.random.default_rng(M + N + K)
    A, B, Asf, Bsf = random_operands(rng, M, N, K)
    full = capi_gemm(A, B, Asf, Bsf, 1.25)
    a, asf = to_dev(A, Asf)
    s = torch.tensor(1.25, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for world in (1, 2):
        n_loc = N // world
        outs = [torch.full((M, N), -1, dtype=torch.int16, device="cuda") for _ in range(world)]
        for r in range(world):
            b, bsf = to_dev(B[r * n_loc:(r + 1) * n_loc], Bsf[r * n_loc:(r + 1) * n_loc])
            capi.check(capi.gemm_allgather(a.data_ptr(), b.data_ptr(), asf.data_ptr(), bsf.data_ptr(),
                                           s.data_ptr(), [o.data_ptr() for o in outs], r, M, n_loc, K,
                                           stream), "nvfp4_gemm_allgather")
            torch.cuda.synchronize()
        for i, o in enumerate(outs):
            got = o.cpu().numpy().view(np.uint16)
            assert np.array_equal(got, full), f"world {world}: output of rank {i} differs"


@pytest.mark.parametrize("M,world", [(16, 8), (100, 4), (24, 4), (128, 8)])
def test_gemm_allgather_split_decode_on_one_gpu(M, world):
    """Decode shards of a 28672-column weight (K = 2048) with the all-gather fused: each shard
    takes a split-K form (world 8: 128-column tiles over 4 CTAs; world 4: 128-column tiles over
    2 above 32 rows, 256-column tiles over 4 at <= 32), whose epilogue stores every sum into each
    rank's output, here all buffers on this GPU. Every output equals the plain GEMM."""
    N, K = 28672, 2048
    rng = np.random.default_rng(M + world)
    A, B, Asf, Bsf = random_operands(rng, M, N, K)
    full = capi_gemm(A, B, Asf, Bsf, 0.5)
    a, asf = to_dev(A, Asf)
    s = torch.tensor(0.5, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    n_loc = N // world
    assert capi.gemm_plan(M, n_loc, K)[2] > 1  # the shard does split K
    outs = [torch.full((M, N), -1, dtype=torch.int16, device="cuda") for _ in range(world)]
    for r in range(world):
        b, bsf = to_dev(B[r * n_loc:(r + 1) * n_loc], Bsf[r * n_loc:(r + 1) * n_loc])
        capi.check(capi.gemm_allgather(a.data_ptr(), b.data_ptr(), asf.data_ptr(), bsf.data_ptr(),
                                       s.data_ptr(), [o.data_ptr() for o in outs], r, M, n_loc, K,
                                       stream), "nvfp4_gemm_allgather")
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        assert np.array_equal(o.cpu().numpy().view(np.uint16), full), f"output of rank {i} differs"


@pytest.mark.parametrize("M", [16, 128])
def test_gemm_narrow_tiles_of_sharded_decode_bit_identical(plugins, M):
    """A decode-shape weight split into 2, 4 or 8 column shards leaves too few 256-column tiles
    per shard: the 2-way shards run 128-column tiles, the 4- and 8-way shards split K over a
    cluster (fp32 partials summed in a fixed order). The shards reproduce the unsharded product
    bit for bit."""
    rng = np.random.default_rng(M + 11)
    N, K = 28672, 2048
    A, B, Asf, Bsf = random_operands(rng, M, N, K)
    full = plugins_gemm(plugins, A, B, Asf, Bsf, 0.75)
    for P in (2, 4, 8):
        w = N // P
        parts = [plugins_gemm(plugins, A, B[r * w:(r + 1) * w], Asf, Bsf[r * w:(r + 1) * w], 0.75)
                 for r in range(P)]
        assert np.array_equal(np.concatenate(parts, axis=1), full), f"P={P}"


def test_gemm_deterministic(plugins):
    rng = np.random.default_rng(9)
    A, B, Asf, Bsf = random_operands(rng, 1000, 1024, 4096)
    first = plugins_gemm(plugins, A, B, Asf, Bsf, 1.0)
    for _ in range(3):
        assert np.array_equal(plugins_gemm(plugins, A, B, Asf, Bsf, 1.0), first)


def test_gemm_square_8192_full_output(plugins, oracle):
    """The square workload: M = N = K = 8192 from bf16 N(0,1) (seed 2), quantized on the GPU.
    Every element of the 8192 x 8192 output is checked against the oracle (float64 sums), plus
    the row-shard property on 64 sampled rows."""
    g = torch.Generator(device="cuda").manual_seed(2)
    A = torch.randn(8192, 8192, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(8192, 8192, device="cuda", generator=g).to(torch.bfloat16)
    sA = 6 * 448 / A.abs().max().to(dtype=torch.float32)
    sB = 6 * 448 / B.abs().max().to(dtype=torch.float32)
    a, a_sf = plugins.quantize_nvfp4(A, sA)
    b, b_sf = plugins.quantize_nvfp4(B, sB)
    del A, B
    scale = sA * sB
    d = plugins.gemm_nvfp4(a, b, a_sf, b_sf, scale)
    a_np, asf_np = a.cpu().numpy(), a_sf.view(torch.uint8).cpu().numpy()
    b_np, bsf_np = b.cpu().numpy(), b_sf.view(torch.uint8).cpu().numpy()
    ref = oracle.gemm_f32(a_np, b_np, asf_np, bsf_np, scale.item())
    assert_gemm_close(d.view(torch.int16).cpu().numpy().view(np.uint16), ref, "8192^3 full output")
    # the same rows computed as a separate (small-M) problem are bit-identical
    rows = np.sort(np.random.default_rng(0).choice(8192, 64, replace=False))
    idx = torch.from_numpy(rows).cuda()
    d_rows = plugins.gemm_nvfp4(a[idx].contiguous(), b, a_sf[idx].contiguous(), b_sf, scale)
    assert torch.equal(d_rows.view(torch.int16), d.view(torch.int16)[idx])


@pytest.mark.parametrize("M", [16, 32, 64, 128])
def test_gemm_skinny_decode_shape(plugins, oracle, M):
    """Decode-style shape M x 28672 x 8192 for every token count of the decode workload
    (16, 32, 64, 128): weight from N(0, 0.02^2), activations N(0,1), seed 3. M < 128 runs the
    single-CTA form whose A boxes cover only the M existing rows."""
    rng = np.random.default_rng(3)
    Wb = cases.activation(rng, 28672, 8192, std=0.02)
    Xb = cases.activation(rng, M, 8192)
    sW, sX = oracle.global_scale(Wb), oracle.global_scale(Xb)
    W = torch.from_numpy(Wb.view(np.int16)).cuda().view(torch.bfloat16)
    X = torch.from_numpy(Xb.view(np.int16)).cuda().view(torch.bfloat16)
    w, w_sf = plugins.quantize_nvfp4(W, torch.tensor(sW, device="cuda"))
    x, x_sf = plugins.quantize_nvfp4(X, torch.tensor(sX, device="cuda"))
    scale = np.float32(sX) * np.float32(sW)
    d = plugins.gemm_nvfp4(x, w, x_sf, w_sf, torch.tensor(scale, device="cuda"))
    ref = oracle.gemm_f32(x.cpu().numpy(), w.cpu().numpy(), x_sf.view(torch.uint8).cpu().numpy(),
                          w_sf.view(torch.uint8).cpu().numpy(), scale)
    assert_gemm_close(d.view(torch.int16).cpu().numpy().view(np.uint16), ref, f"M={M} skinny")


# Decode shapes whose 256-column tiles fill less than half the SMs split K over a cluster:
# 128-column tiles over 4 CTAs where they fit, else (M > 32) 128-column tiles over 2, else
# 256-column tiles over 4. Each form, with M = 1, M just above 32, one k-block per CTA and
# ragged N (a last tile of 104 and of 8 columns).
SPLIT_SHAPES = [
    (1, 3584, 2048),      # 128-column tiles over 4 (28 tiles, 2 k-blocks per CTA)
    (33, 3584, 1024),     # same form, M just above 32, one k-block per CTA
    (7, 1000, 4096),      # same form, last tile 104 columns wide
    (100, 7168, 2048),    # 128-column tiles over 2 (56 tiles), M > 32
    (24, 7168, 2048),     # 256-column tiles over 4 (28 tiles), M <= 32
    (128, 7176, 1024),    # 128-column tiles over 2, last tile 8 columns wide
]


@pytest.mark.parametrize("M,N,K", SPLIT_SHAPES)
def test_gemm_split_k_decode_shapes(oracle, M, N, K):
    rng = np.random.default_rng(M * 7 + N + K)
    A, B, Asf, Bsf = random_operands(rng, M, N, K)
    ref = oracle.gemm_f32(A, B, Asf, Bsf, 1.5)
    assert_gemm_close(capi_gemm(A, B, Asf, Bsf, 1.5), ref, f"split {M}x{N}x{K}")
    # repeated calls give the same bits (the cluster sum runs in a fixed order)
    assert np.array_equal(capi_gemm(A, B, Asf, Bsf, 1.5), capi_gemm(A, B, Asf, Bsf, 1.5))


@pytest.mark.parametrize("M,N,K", [(5, 520, 1024), (16, 28672, 2048), (100, 1024, 512),
                                   (130, 512, 512)])
def test_gemm_leaves_memory_past_row_m_untouched(M, N, K):
    """With M < 128 the single-CTA form still runs 128-row MMAs; shared-memory rows past M hold
    stale bytes (which may decode as NaN scale factors) and their accumulator lanes must never
    be stored. D is given as the first M rows of a larger buffer filled with a sentinel: the
    rows past M keep the sentinel and the first M rows equal the plain call's output."""
    rng = np.random.default_rng(M + N)
    A, B, Asf, Bsf = random_operands(rng, M, N, K)
    Asf[1::4, 3] = 0x7F                           # NaN scale bytes in some live rows too
    full = capi_gemm(A, B, Asf, Bsf, 1.0)
    a, b, asf, bsf = to_dev(A, B, Asf, Bsf)
    big = torch.full((M + 130, N), 0x1357, dtype=torch.int16, device="cuda")
    s = torch.tensor(1.0, dtype=torch.float32, device="cuda")
    capi.check(capi.gemm(a.data_ptr(), b.data_ptr(), asf.data_ptr(), bsf.data_ptr(), s.data_ptr(),
                         big.data_ptr(), M, N, K, torch.cuda.current_stream().cuda_stream),
               "nvfp4_gemm")
    torch.cuda.synchronize()
    got = big.cpu().numpy().view(np.uint16)
    assert (got[M:] == 0x1357).all(), "rows past M were written"
    assert np.array_equal(got[:M], full)


def test_gemm_k_zero_and_empty(plugins):
    s = torch.tensor(2.0, device="cuda")
    e4 = torch.float8_e4m3fn
    d = plugins.gemm_nvfp4(torch.zeros(5, 0, dtype=torch.uint8, device="cuda"),
                           torch.zeros(8, 0, dtype=torch.uint8, device="cuda"),
                           torch.zeros(5, 0, device="cuda").to(e4), torch.zeros(8, 0, device="cuda").to(e4), s)
    assert d.shape == (5, 8) and (d.float() == 0).all()
    d = plugins.gemm_nvfp4(torch.zeros(0, 128, dtype=torch.uint8, device="cuda"),
                           torch.zeros(8, 128, dtype=torch.uint8, device="cuda"),
                           torch.zeros(0, 16, device="cuda").to(e4), torch.zeros(8, 16, device="cuda").to(e4), s)
    assert d.shape == (0, 8)


def test_gemm_rejects_bad_shapes(plugins):
    s = torch.tensor(1.0, device="cuda")
    e4 = torch.float8_e4m3fn
    u8 = dict(dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 256"):
        plugins.gemm_nvfp4(torch.zeros(4, 64, **u8), torch.zeros(8, 64, **u8),
                           torch.zeros(4, 8, device="cuda").to(e4), torch.zeros(8, 8, device="cuda").to(e4), s)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        plugins.gemm_nvfp4(torch.zeros(4, 128, **u8), torch.zeros(12, 128, **u8),
                           torch.zeros(4, 16, device="cuda").to(e4), torch.zeros(12, 16, device="cuda").to(e4), s)
    with pytest.raises(RuntimeError, match="same K"):
        plugins.gemm_nvfp4(torch.zeros(4, 128, **u8), torch.zeros(8, 256, **u8),
                           torch.zeros(4, 16, device="cuda").to(e4), torch.zeros(8, 32, device="cuda").to(e4), s)
    with pytest.raises(RuntimeError, match="A_sf"):
        plugins.gemm_nvfp4(torch.zeros(4, 128, **u8), torch.zeros(8, 128, **u8),
                           torch.zeros(4, 8, device="cuda").to(e4), torch.zeros(8, 16, device="cuda").to(e4), s)


@pytest.mark.parametrize("M,N,K", [(96, 2048, 4096), (512, 1024, 2048)])
def test_gemm_orders_after_previous_kernels(M, N, K):
    """The GEMM is launched with programmatic stream serialization (it may set up before the
    previous kernel on the stream has completed) and waits for that kernel before touching
    memory: operands written by the kernel just before it are read in full, and an output buffer
    that the kernel just before it reads is not overwritten early. Consecutive GEMMs (the same
    with the epilogue of one and the loads of the next) are covered by the back-to-back launches
    of test_gemm_back_to_back_launches. Six launches alternate between two problems with no
    synchronisation in between."""
    rng = np.random.default_rng(11 + M)
    problems = [random_operands(rng, M, N, K) for _ in range(2)]
    refs = [capi_gemm(*pr, 1.0) for pr in problems]
    assert not np.array_equal(refs[0], refs[1])
    dev = [to_dev(*pr) for pr in problems]
    bufs = [torch.empty_like(t) for t in dev[0]]
    d = torch.empty(M, N, dtype=torch.int16, device="cuda")
    s = torch.tensor(1.0, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    snaps = []
    for it in range(6):
        for dst, src in zip(bufs, dev[it % 2]):
            torch.bitwise_xor(src, 0, out=dst)   # an elementwise kernel writes each operand
        capi.check(capi.gemm(bufs[0].data_ptr(), bufs[1].data_ptr(), bufs[2].data_ptr(),
                             bufs[3].data_ptr(), s.data_ptr(), d.data_ptr(), M, N, K, stream),
                   "nvfp4_gemm")
        snaps.append(torch.bitwise_xor(d, 0))   # a kernel reads D before the next GEMM writes it
    torch.cuda.synchronize()
    for it, snap in enumerate(snaps):
        assert np.array_equal(snap.cpu().numpy().view(np.uint16), refs[it % 2]), f"launch {it}"


@pytest.mark.parametrize("M", [16, 300])
def test_gemm_back_to_back_launches(M):
    """GEMM after GEMM with no other kernel in between: the first M*K/2 bytes of each output
    are read as the next launch's A (packed codes [M, K/2]), a chain of 8 launches on one
    stream. A launch that read A before the previous one's stores were complete would diverge
    from the same chain run with a synchronisation after every launch."""
    rng = np.random.default_rng(40 + M)
    K, N = 1024, 512                      # D is bf16 [M, 512]: M*K bytes, twice the next A
    a, b, asf, bsf = to_dev(*random_operands(rng, M, N, K))
    s = torch.tensor(1.0, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    bufs = [torch.empty(M, N, dtype=torch.bfloat16, device="cuda") for _ in range(8)]

    def chain(sync):
        src = a.data_ptr()
        for i in range(8):
            capi.check(capi.gemm(src, b.data_ptr(), asf.data_ptr(), bsf.data_ptr(),
                                 s.data_ptr(), bufs[i].data_ptr(), M, N, K, stream),
                       "nvfp4_gemm")
            if sync:
                torch.cuda.synchronize()
            src = bufs[i].data_ptr()
        torch.cuda.synchronize()
        return [t.clone() for t in bufs]

    ref = chain(True)
    for _ in range(2):
        assert all(torch.equal(x.view(torch.int16), y.view(torch.int16))
                   for x, y in zip(chain(False), ref))


def test_no_device_timeouts_recorded():
    assert capi.device_status(torch.cuda.current_stream().cuda_stream) == 0
