"""The drop-in at the reference consumer's own import line.

The reference's only consumer (test.py:1) does `from csrc import my_plugins`, where `csrc/` is
the reference's source tree with an empty `__init__.py` (csrc/__init__.py) and the extension
built in place beside it. A project switching to this library keeps that line and replaces
`csrc/__init__.py` with the two-line shim below. This test builds exactly that package in a
temporary directory and runs the consumer's recipe (test.py:4-24: seed 100; A 128 x 1024 and
B 256 x 1024 bf16 N(0,1) moved to the GPU; s = 6*448/amax per tensor; quantize both; GEMM with
s_A * s_B; dequantize both; F.linear of the dequantized operands) in a fresh interpreter, with
assertions where the recipe prints:
  * the module reached through `csrc` is this library's in-tree extension;
  * quantize and dequantize bytes equal the oracle's;
  * the GEMM is within the GEMM tolerance of the oracle product, and within 1e-2 (relative
    Frobenius) of F.linear of the dequantized operands, whose bf16 rounding of the operands is
    the only difference the recipe shows."""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SHIM = "from my_nvfp4_gemm_b200 import my_plugins  # noqa: F401\n"

CONSUMER = textwrap.dedent('''
    from csrc import my_plugins
    import numpy as np
    import torch

    import my_nvfp4_gemm_b200
    from oracle import oracle as O
    from test_gemm_gpu import assert_gemm_close

    assert my_plugins is my_nvfp4_gemm_b200.my_plugins
    assert os.path.dirname(my_plugins.__file__) == os.path.dirname(my_nvfp4_gemm_b200.__file__)

    torch.manual_seed(100)
    A = torch.randn(128, 256 * 4, dtype=torch.bfloat16).to("cuda")
    B = torch.randn(256, 256 * 4, dtype=torch.bfloat16).to("cuda")
    A_scale = 6 * 448 / A.abs().max().to(dtype=torch.float32)
    B_scale = 6 * 448 / B.abs().max().to(dtype=torch.float32)
    a, a_sf = my_plugins.quantize_nvfp4(A, A_scale)
    b, b_sf = my_plugins.quantize_nvfp4(B, B_scale)
    d = my_plugins.gemm_nvfp4(a, b, a_sf, b_sf, A_scale * B_scale)
    a_r = my_plugins.de_quantize_nvfp4(a, A_scale, a_sf)
    b_r = my_plugins.de_quantize_nvfp4(b, B_scale, b_sf)
    D = torch.nn.functional.linear(a_r, b_r)

    def bits(t):
        return t.view(torch.int16).cpu().numpy().view(np.uint16)

    for X, s, q, sf, r in ((A, A_scale, a, a_sf, a_r), (B, B_scale, b, b_sf, b_r)):
        oq, osf = O.quantize(bits(X), s.item())
        assert np.array_equal(q.cpu().numpy(), oq), "quantize bytes"
        assert np.array_equal(sf.view(torch.uint8).cpu().numpy(), osf), "scale bytes"
        assert np.array_equal(bits(r), O.dequantize(oq, s.item(), osf)), "dequantize bytes"

    assert d.dtype == torch.bfloat16 and d.shape == (128, 256)
    ref = O.gemm_f32(a.cpu().numpy(), b.cpu().numpy(), a_sf.view(torch.uint8).cpu().numpy(),
                     b_sf.view(torch.uint8).cpu().numpy(), (A_scale * B_scale).item())
    assert_gemm_close(bits(d), ref, "consumer recipe")
    rel = ((d.float() - D.float()).norm() / D.float().norm()).item()
    assert rel < 1e-2, rel
    print("consumer recipe ok", rel)
''')


def test_consumer_recipe_through_csrc_import(tmp_path):
    pkg = tmp_path / "csrc"
    pkg.mkdir()
    (pkg / "__init__.py").write_text(SHIM)
    script = tmp_path / "consumer.py"
    script.write_text("import os\n" + CONSUMER)
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(tmp_path), ROOT, os.path.join(ROOT, "tests")]
                                        + ([env["PYTHONPATH"]] if env.get("PYTHONPATH") else []))
    r = subprocess.run([sys.executable, str(script)], cwd=str(tmp_path), env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "consumer recipe ok" in r.stdout
