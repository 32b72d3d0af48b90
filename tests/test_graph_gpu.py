"""GEMM launches captured into a CUDA graph (torch.cuda.graph) and replayed: every kernel form the
dispatcher picks (both split-K forms, the single-CTA form, narrower single-CTA tiles, the CTA
pair) gives the same bits on replay as in eager calls. Each shape is called once eagerly first:
the per-device setup (shared-memory limits, the SM count) happens on the first call of a form
and is not a stream operation."""
import numpy as np
import pytest
import torch

from my_nvfp4_gemm_b200 import capi

pytestmark = pytest.mark.gpu

SHAPES = [
    (16, 3584, 2048),     # 128-column tiles, K split over 4
    (100, 7168, 2048),    # 128-column tiles, K split over 2
    (16, 28672, 1024),    # single CTA, 256-column tiles
    (16, 14336, 768),     # single CTA, 128-column tiles (3 k-blocks: no split)
    (300, 512, 1024),     # CTA pair
]


def _operands(rng, M, N, K):
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    return (dev(rng.integers(0, 256, (M, K // 2), dtype=np.uint8)),
            dev(rng.integers(0, 256, (N, K // 2), dtype=np.uint8)),
            dev(rng.integers(0x28, 0x40, (M, K // 16), dtype=np.uint8)),
            dev(rng.integers(0x28, 0x40, (N, K // 16), dtype=np.uint8)))


def test_gemm_calls_replay_in_a_cuda_graph():
    rng = np.random.default_rng(17)
    scale = torch.tensor(0.5, dtype=torch.float32, device="cuda")
    cases = []
    for M, N, K in SHAPES:
        a, b, asf, bsf = _operands(rng, M, N, K)
        cases.append((M, N, K, a, b, asf, bsf, torch.empty(M, N, dtype=torch.int16, device="cuda")))

    def run_all(stream_h):
        for M, N, K, a, b, asf, bsf, d in cases:
            capi.check(capi.gemm(a.data_ptr(), b.data_ptr(), asf.data_ptr(), bsf.data_ptr(),
                                 scale.data_ptr(), d.data_ptr(), M, N, K, stream_h), "nvfp4_gemm")

    run_all(torch.cuda.current_stream().cuda_stream)   # eager, also the per-device setup
    torch.cuda.synchronize()
    eager = [d.clone() for *_, d in cases]
    for *_, d in cases:
        d.fill_(0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run_all(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        for *_, d in cases:
            d.fill_(0)
        g.replay()
        torch.cuda.synchronize()
        for (M, N, K, *_), want, (*_, d) in zip(cases, eager, cases):
            assert torch.equal(d, want), f"{M}x{N}x{K}: replay differs from the eager call"
    assert capi.device_status() == 0   # no bounded wait gave up during the replays
