"""One rank of the multi-GPU check (launched by tests/test_sharded_gpu.py through torchrun).

Each rank: quantize its rows of the activation with the global scale (one all_reduce(MAX)),
all-gather the packed activation, run the column-parallel GEMM on its weight shard with the
chunked NCCL all-gather of D and with the all-gather fused into the GEMM epilogue (stores into
every rank's output over NVLink), and compare with the unsharded single-GPU result on every rank.
"""
import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from my_nvfp4_gemm_b200 import load_my_plugins, sharded  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    P = load_my_plugins()
    M, N, K = 512, 2048, 2048
    g = torch.Generator(device="cuda").manual_seed(42)          # identical on every rank
    X = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)

    # single-GPU reference (every rank computes it locally)
    sX = 6 * 448 / X.abs().max().to(torch.float32)
    sW = 6 * 448 / W.abs().max().to(torch.float32)
    x, x_sf = P.quantize_nvfp4(X, sX)
    w, w_sf = P.quantize_nvfp4(W, sW)
    full = P.gemm_nvfp4(x, w, x_sf, w_sf, sX * sW)

    # row-sharded quantize of X with the global scale, then all-gather of the packed rows
    rows = M // world
    xq, xsf, s_glob = sharded.quantize_row_sharded(X[rank * rows:(rank + 1) * rows].contiguous())
    assert torch.equal(s_glob, sX), "global scale differs from the single-GPU recipe"
    xg = torch.empty(M, K // 2, dtype=torch.uint8, device="cuda")
    xsfg = torch.empty(M, K // 16, dtype=torch.uint8, device="cuda")
    dist.all_gather_into_tensor(xg, xq)
    dist.all_gather_into_tensor(xsfg, xsf.view(torch.uint8))
    assert torch.equal(xg, x) and torch.equal(xsfg, x_sf.view(torch.uint8)), "sharded quantize differs"

    # column-parallel GEMM on this rank's weight shard; local columns and gathered D
    w_sh, w_sf_sh = sharded.shard_weight(w, w_sf, world, rank)
    n0, n1 = sharded.shard_range(N, world, rank)
    local = sharded.gemm_column_parallel(x, w_sh, x_sf, w_sf_sh, sX * sW)
    assert torch.equal(local.view(torch.int16), full[:, n0:n1].view(torch.int16)), "local shard differs"
    gathered = sharded.gemm_column_parallel(x, w_sh, x_sf, w_sf_sh, sX * sW, gather=True, chunks=3)
    assert torch.equal(gathered.view(torch.int16), full.view(torch.int16)), "gathered D differs"

    # the all-gather fused into the GEMM epilogue (stores into every rank's output over
    # NVLink): bit-identical to the single-GPU result, on repeated calls into the same buffers
    for it in range(3):
        fused = sharded.gemm_column_parallel(x, w_sh, x_sf, w_sf_sh, sX * sW, gather=True,
                                             fused=True)
        assert torch.equal(fused.view(torch.int16), full.view(torch.int16)), f"fused D differs ({it})"
    # decode-sized M (on this 1024-column shard: K split over clusters of 4 CTAs, whose epilogue
    # stores every sum into both ranks' outputs) and a ragged M (the CTA-pair form)
    for m in (16, 96, 300):
        fm = sharded.gemm_column_parallel(x[:m].contiguous(), w_sh, x_sf[:m].contiguous(), w_sf_sh,
                                          sX * sW, gather=True, fused=True)
        assert torch.equal(fm.view(torch.int16), full[:m].view(torch.int16)), f"fused D differs (M={m})"
    torch.cuda.synchronize()
    sharded.release_peer_outputs()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}: ok", flush=True)


if __name__ == "__main__":
    main()
