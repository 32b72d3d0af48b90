"""The GEMM with its all-gather fused into the epilogue, all P ranks driven from one process.

Each rank r is GPU r with its own stream; peer access is enabled between every pair of GPUs, so a
rank's output buffer is addressed by the other GPUs directly (no IPC handles: one process). Rank r
holds the replicated activation and its column shard of the weight, and its kernel stores its
tiles into every rank's output, as under torchrun. The GPUs run concurrently; afterwards every
output is compared bit for bit with the single-GPU GEMM of the unsharded weight, and the device
time of one fused launch on GPU 0 is printed (timed alone and with all ranks running).

    python tests/fused_allgather_1proc.py P M N_LOCAL K [REPS]

Used by tests/test_sharded_gpu.py (small shapes) and for ncu captures of the fused kernel
(one process, so ncu can attach to it).
"""
from __future__ import annotations

import os
import statistics
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from my_nvfp4_gemm_b200 import capi  # noqa: E402


def enable_peer_access(world: int) -> None:
    from cuda.bindings import runtime as rt
    for i in range(world):
        rt.cudaSetDevice(i)
        for j in range(world):
            if i != j:
                err = rt.cudaDeviceEnablePeerAccess(j, 0)[0]
                if err not in (rt.cudaError_t.cudaSuccess,
                               rt.cudaError_t.cudaErrorPeerAccessAlreadyEnabled):
                    raise RuntimeError(f"peer access {i} -> {j}: {err}")


def main(world: int, M: int, n_loc: int, K: int, reps: int = 5) -> int:
    assert torch.cuda.device_count() >= world, "not enough GPUs"
    N = world * n_loc
    rng = np.random.default_rng(M + N + K)
    A = rng.integers(0, 256, (M, K // 2), dtype=np.uint8)
    B = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    Asf = rng.integers(0x28, 0x40, (M, K // 16), dtype=np.uint8)
    Bsf = rng.integers(0x28, 0x40, (N, K // 16), dtype=np.uint8)
    enable_peer_access(world)

    ranks = []
    for r in range(world):
        dev = torch.device("cuda", r)
        with torch.cuda.device(dev):
            t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)  # noqa: E731
            ranks.append(dict(
                dev=dev, stream=torch.cuda.Stream(dev), a=t(A), asf=t(Asf),
                b=t(B[r * n_loc:(r + 1) * n_loc]), bsf=t(Bsf[r * n_loc:(r + 1) * n_loc]),
                s=torch.tensor(1.25, dtype=torch.float32, device=dev),
                out=torch.full((M, N), -1, dtype=torch.int16, device=dev)))
    outs = [rk["out"].data_ptr() for rk in ranks]

    def launch(r):
        rk = ranks[r]
        with torch.cuda.device(rk["dev"]):
            capi.check(capi.gemm_allgather(rk["a"].data_ptr(), rk["b"].data_ptr(), rk["asf"].data_ptr(),
                                           rk["bsf"].data_ptr(), rk["s"].data_ptr(), outs, r, M, n_loc,
                                           K, rk["stream"].cuda_stream), "nvfp4_gemm_allgather")

    def sync_all():
        for rk in ranks:
            rk["stream"].synchronize()

    # all ranks at once (each rank's launch on its own GPU and stream)
    for _ in range(2):
        for r in range(world):
            launch(r)
        sync_all()
    dev0 = ranks[0]
    with torch.cuda.device(dev0["dev"]):
        full = torch.empty(M, N, dtype=torch.int16, device=dev0["dev"])
        b_full = torch.from_numpy(B).to(dev0["dev"])
        bsf_full = torch.from_numpy(Bsf).to(dev0["dev"])
        capi.check(capi.gemm(dev0["a"].data_ptr(), b_full.data_ptr(), dev0["asf"].data_ptr(),
                             bsf_full.data_ptr(), dev0["s"].data_ptr(), full.data_ptr(), M, N, K,
                             dev0["stream"].cuda_stream), "nvfp4_gemm")
        dev0["stream"].synchronize()
        want = full.cpu()
    for r, rk in enumerate(ranks):
        if not torch.equal(rk["out"].cpu(), want):
            print(f"rank {r}: output differs from the single-GPU GEMM")
            return 1

    def time_rank0(all_ranks: bool) -> float:
        times = []
        for _ in range(reps):
            sync_all()
            with torch.cuda.device(dev0["dev"]):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(dev0["stream"])
            for r in (range(world) if all_ranks else [0]):
                launch(r)
            with torch.cuda.device(dev0["dev"]):
                e1.record(dev0["stream"])
            sync_all()
            times.append(e0.elapsed_time(e1))
        return statistics.median(times)

    alone, together = time_rank0(False), time_rank0(True)
    out_bytes = 2.0 * M * n_loc * (world - 1)
    print(f"fused gemm+allgather P={world} M={M} N_local={n_loc} K={K}: outputs bit-identical; "
          f"GPU 0 {alone:.3f} ms alone, {together:.3f} ms with all ranks; "
          f"{out_bytes / 1e6:.1f} MB out over NVLink per rank "
          f"({out_bytes / (together * 1e-3) / 1e9:.0f} GB/s)")
    return 0


if __name__ == "__main__":
    a = [int(x) for x in sys.argv[1:]]
    sys.exit(main(*a))
