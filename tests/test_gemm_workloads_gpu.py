"""Parity of the prefill workload at its full size: A 16384 x 8192 bf16 N(0,1) with 0.5% of the
elements x50 (seed 4), weight 57344 x 8192 bf16 N(0, 0.02^2), both quantized on the GPU with the
reference recipe, D = A.B^T / scale as bf16 [16384, 57344] (1.9 GB).

The operands come from bench.py's own generator, so the parity test and the benchmark run the
same bytes. Checked here:
  * both quantized operands, in full, are bit-identical to the oracle's quantization of the
    same bf16 data;
  * 64 sampled rows of D x all 57344 columns are within the GEMM tolerance of the oracle's
    product (float64 sums, then fp32, / scale, bf16): relative Frobenius <= 1e-3 and >= 99.9 %
    of elements within 1 bf16 ulp;
  * the same rows computed as a separate small-M problem are bit-identical (the rows of D do not
    depend on which other rows are in the launch).
The GEMM under test replaces the reference kernel csrc/gemm/gemm_nvfp4.cu:5-240."""
import numpy as np
import pytest
import torch

import bench
from test_gemm_gpu import assert_gemm_close

pytestmark = pytest.mark.gpu


def gemm_f32_column_chunks(oracle, a, asf, b, bsf, scale, chunk=8192):
    """oracle.gemm_f32 over column chunks of B, so the float64 decode of the 57344-row weight is
    never held whole (host memory stays ~1 GB)."""
    parts = [oracle.gemm_f32(a, b[c:c + chunk], asf, bsf[c:c + chunk], scale)
             for c in range(0, b.shape[0], chunk)]
    return np.concatenate(parts, axis=1)


def test_prefill_16384x57344x8192(plugins, oracle):
    inp = bench.sharded_inputs(torch, plugins, "prefill", 0, 1, 0, keep_bf16=True)
    x, x_sf, w, w_sf, scale = inp["x"], inp["x_sf"], inp["w"], inp["w_sf"], inp["scale"]
    assert (inp["M"], inp["N"], inp["K"]) == (16384, 57344, 8192)

    # the quantized operands, every byte
    for bits_t, s, q, sf in ((inp["X"], inp["sX"], x, x_sf), (inp["W"], inp["sW"], w, w_sf)):
        bits = bits_t.view(torch.int16).cpu().numpy().view(np.uint16)
        oq, osf = oracle.quantize(bits, s.item())
        assert np.array_equal(q.cpu().numpy(), oq)
        assert np.array_equal(sf.view(torch.uint8).cpu().numpy(), osf)
    del inp["X"], inp["W"]

    d = plugins.gemm_nvfp4(x, w, x_sf, w_sf, scale)
    assert d.shape == (16384, 57344)
    rows = np.sort(np.random.default_rng(4).choice(16384, 64, replace=False))
    idx = torch.from_numpy(rows).cuda()
    got = d.view(torch.int16)[idx].cpu().numpy().view(np.uint16)
    del d
    b_np, bsf_np = w.cpu().numpy(), w_sf.view(torch.uint8).cpu().numpy()
    ref = gemm_f32_column_chunks(oracle, x.cpu().numpy()[rows], x_sf.view(torch.uint8).cpu().numpy()[rows],
                                 b_np, bsf_np, scale.item())
    assert_gemm_close(got, ref, "prefill 64 sampled rows x 57344")
    d_rows = plugins.gemm_nvfp4(x[idx].contiguous(), w, x_sf[idx].contiguous(), w_sf, scale)
    assert np.array_equal(d_rows.view(torch.int16).cpu().numpy().view(np.uint16), got)
