"""Generate the golden vectors that pin the CPU oracle: outputs of the REFERENCE plugin's own
quantize / dequantize kernels (csrc/quantize/quantize_nvfp4.cu, compiled unchanged from the
reference sources for sm_100a by `make -C oracle ref`) on seeded edge-case and random inputs.

Runs on a B200:   python tests/golden/make_golden.py <out.npz>
The committed fixture is tests/golden/ref_kernels_sm100a.npz.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from oracle import oracle as O  # noqa: E402
import nvfp4_cases as cases  # noqa: E402


def run_ref_quantize(ref, x_bits: np.ndarray, s: float):
    x = torch.from_numpy(x_bits.view(np.int16)).cuda()
    q = torch.empty(x_bits.size // 2, dtype=torch.uint8, device="cuda")
    sf = torch.empty(x_bits.size // 16, dtype=torch.uint8, device="cuda")
    st = ref.ref_quantize_nvfp4(x.data_ptr(), float(s), x_bits.size, q.data_ptr(), sf.data_ptr(), None)
    assert st == 0, st
    torch.cuda.synchronize()
    return q.cpu().numpy(), sf.cpu().numpy()


def run_ref_dequantize(ref, q_np: np.ndarray, sf_np: np.ndarray, s: float):
    q = torch.from_numpy(q_np).cuda()
    sf = torch.from_numpy(sf_np).cuda()
    y = torch.empty(q_np.size * 2, dtype=torch.int16, device="cuda")
    st = ref.ref_de_quantize_nvfp4(q.data_ptr(), float(s), sf.data_ptr(), q_np.size, y.data_ptr(), None)
    assert st == 0, st
    torch.cuda.synchronize()
    return y.cpu().numpy().view(np.uint16)


def main(out_path: str) -> None:
    ref = O.load_reference_kernels()
    assert ref is not None, "oracle/_ref/libref_quantize.so is missing (make -C oracle ref)"
    x = cases.quantize_case_blocks()
    scales = cases.quantize_case_scales(x)
    q_out, sf_out = [], []
    for s in scales:
        q, sf = run_ref_quantize(ref, x, s)
        q_out.append(q)
        sf_out.append(sf)
    dq_q, dq_sf = cases.dequant_exhaustive_inputs()
    dq_out = [run_ref_dequantize(ref, dq_q, dq_sf, s) for s in cases.DEQUANT_SCALES]
    np.savez_compressed(
        out_path,
        q_x=x, q_scales=scales, q_packed=np.stack(q_out), q_sf=np.stack(sf_out),
        dq_packed=dq_q, dq_sf=dq_sf, dq_scales=cases.DEQUANT_SCALES, dq_out=np.stack(dq_out),
        device=np.array(torch.cuda.get_device_name()),
    )
    print("wrote", out_path, "quantize cases:", x.size // 16, "blocks x", len(scales), "scales")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <out.npz>")
    main(sys.argv[1])
