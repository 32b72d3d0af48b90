"""Multi-GPU partitioning of the NVFP4 path over torch.distributed (one process per GPU).

Column-parallel GEMM (N sharding). Rank r owns rows [n0, n1) of the weight B and of B_sf; A and
A_sf are replicated. Each rank computes D[:, n0:n1] with the single-GPU kernel and no
communication: every output element depends only on its own row of A and row of B, so the
shards are bit-identical to the corresponding columns of the unsharded product. An optional
all-gather (NCCL over NVLink/NVSwitch) assembles the full [M, N] on every rank; it is issued per
chunk of M rows as soon as that chunk's GEMM is enqueued, so the transfer of chunk c overlaps
the GEMM of chunk c+1.

Row-sharded quantize. Quantization is independent per 16-element block, so rows shard with no
exchange; the only collective is the per-tensor scale s = 6*448/amax, whose amax is one scalar
all_reduce(MAX) across ranks.

The compute functions default to the CUDA kernels (my_plugins); they are parameters so that the
host-side logic can be exercised on CPU ranks with the gloo backend.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def _plugins():
    from . import load_my_plugins
    return load_my_plugins()


def world_and_rank(group=None) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def shard_range(n: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """[start, stop) of rank's share of n columns. Shares are multiples of `align` (the GEMM's
    N tile) when n allows, else of 8 (the kernel's N % 8 rule); the remainder goes to the
    lowest ranks. Raises if n is not a multiple of 8."""
    if n % 8 != 0:
        raise ValueError(f"N must be a multiple of 8 to shard, got {n}")
    if not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside world of {world}")
    unit = align if n % align == 0 and n // align >= world else 8
    units = n // unit
    base, extra = divmod(units, world)
    start = unit * (rank * base + min(rank, extra))
    stop = start + unit * (base + (1 if rank < extra else 0))
    return start, stop


def shard_weight(B: torch.Tensor, B_sf: torch.Tensor, world: int, rank: int,
                 align: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """This rank's rows of the packed weight and its scale factors (contiguous views)."""
    if B.shape[0] != B_sf.shape[0]:
        raise ValueError(f"B has {B.shape[0]} rows but B_sf has {B_sf.shape[0]}")
    n0, n1 = shard_range(B.shape[0], world, rank, align)
    return B[n0:n1], B_sf[n0:n1]


def amax_all_ranks(x: torch.Tensor, group=None) -> torch.Tensor:
    """max |x| over all ranks' shards, as an fp32 0-dim tensor on x's device."""
    local = x.abs().max().to(torch.float32) if x.numel() else torch.zeros((), dtype=torch.float32,
                                                                          device=x.device)
    world, _ = world_and_rank(group)
    if world > 1:
        t = local.reshape(1).clone()
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        local = t.reshape(())
    return local


def global_scale(x: torch.Tensor, group=None) -> torch.Tensor:
    """The reference recipe s = 6*448 / amax (test.py:10-11) over the whole sharded tensor.
    Evaluated exactly as torch evaluates `int / Tensor`: reciprocal(amax) * 2688."""
    return 6 * 448 / amax_all_ranks(x, group)


def quantize_row_sharded(x_local: torch.Tensor, group=None,
                         quantize_fn: Optional[Callable] = None):
    """Quantize this rank's rows with the global per-tensor scale. Returns (q, sf, s)."""
    s = global_scale(x_local, group)
    fn = quantize_fn or _plugins().quantize_nvfp4
    q, sf = fn(x_local, s)
    return q, sf, s


def gemm_column_parallel(A: torch.Tensor, B_shard: torch.Tensor, A_sf: torch.Tensor,
                         B_sf_shard: torch.Tensor, scale: torch.Tensor, group=None,
                         gather: bool = False, chunks: int = 4,
                         gemm_fn: Optional[Callable] = None) -> torch.Tensor:
    """D[:, shard] = gemm_nvfp4(A, B_shard) on this rank; with gather=True the full D [M, N]
    (all ranks' shards, rank order along N) on every rank.

    The gather needs equal shard widths on all ranks (all_gather_into_tensor); it is issued per
    chunk of M rows right after that chunk's GEMM so NCCL overlaps the next chunk's compute."""
    fn = gemm_fn or _plugins().gemm_nvfp4
    world, _ = world_and_rank(group)
    if not gather or world == 1:
        return fn(A, B_shard, A_sf, B_sf_shard, scale)

    widths = [torch.tensor([B_shard.shape[0]], dtype=torch.int64, device=A.device)
              for _ in range(world)]
    dist.all_gather(widths, widths[0].clone(), group=group)
    w = [int(t.item()) for t in widths]
    if len(set(w)) != 1:
        raise ValueError(f"gather needs equal shard widths on all ranks, got {w}")
    n = w[0]
    M = A.shape[0]
    chunks = max(1, min(chunks, M))
    bounds = [M * i // chunks for i in range(chunks + 1)]
    gathered = torch.empty(world, M, n, dtype=torch.bfloat16, device=A.device)
    works = []
    for c in range(chunks):
        m0, m1 = bounds[c], bounds[c + 1]
        if m1 == m0:
            continue
        d_local = fn(A[m0:m1], B_shard, A_sf[m0:m1], B_sf_shard, scale)
        out = torch.empty(world * (m1 - m0), n, dtype=torch.bfloat16, device=A.device)
        works.append((dist.all_gather_into_tensor(out, d_local.contiguous(), group=group,
                                                  async_op=True), out, m0, m1))
    for work, out, m0, m1 in works:
        work.wait()
        gathered[:, m0:m1] = out.view(world, m1 - m0, n)
    return gathered.permute(1, 0, 2).reshape(M, world * n)
