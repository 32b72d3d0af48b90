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


class PeerOutput:
    """A bf16 [M, N] output buffer on every rank of `group`, each mapped into every rank's
    process (CUDA IPC over NVLink), for the GEMM whose epilogue writes all ranks' outputs.

    ``ptrs[r]`` is rank r's buffer as addressed in this process. The buffer is reused by every
    fused call with the same shape; a call's result stays valid until the next such call."""

    def __init__(self, M: int, N: int, device: torch.device, group=None):
        from . import capi
        self.group = group                  # held so the cache key's group stays alive
        self.world, self.rank = world_and_rank(group)
        self.local = torch.empty(M, N, dtype=torch.bfloat16, device=device)
        # Every rank takes part in the exchange even when its own export failed, so that all
        # ranks see the failure and raise together instead of some waiting in the collective.
        try:
            mine = (True,) + capi.ipc_export(self.local.data_ptr())
        except capi.NvFp4Error as e:
            mine = (False, str(e), 0)
        shared = [None] * self.world
        dist.all_gather_object(shared, mine, group=group)
        failed = [r for r, (ok, _, _) in enumerate(shared) if not ok]
        if failed:
            raise RuntimeError(
                f"fused all-gather: rank(s) {failed} could not export their output buffer for "
                f"CUDA IPC ({shared[failed[0]][1]}). Legacy IPC handles need memory from "
                "cudaMalloc; torch's allocator with PYTORCH_CUDA_ALLOC_CONF=expandable_segments:True "
                "maps its segments with cuMemCreate/cuMemMap, which cannot be exported this way. "
                "Unset expandable_segments, or call gemm_column_parallel(..., fused=False) for "
                "the NCCL all-gather.")
        self.ptrs, self._opened = [], []
        for r, (_, h, off) in enumerate(shared):
            if r == self.rank:
                self.ptrs.append(self.local.data_ptr())
            else:
                p = capi.ipc_open(h, off)
                self._opened.append((p, off))
                self.ptrs.append(p)

    def close(self) -> None:
        from . import capi
        torch.cuda.synchronize(self.local.device)
        for p, off in self._opened:
            capi.ipc_close(p, off)
        self._opened = []


_peer_outputs: dict = {}


def peer_output(M: int, N: int, device: torch.device, group=None) -> PeerOutput:
    """The cached shared output of this shape for `group`. Each cached entry holds a reference
    to its group, so the group's id cannot be reused by a new group while the entry exists; a
    hit is also checked against the group's current world size and rank."""
    key = (M, N, str(device), id(group))
    po = _peer_outputs.get(key)
    if po is not None and (po.group is not group or (po.world, po.rank) != world_and_rank(group)):
        po.close()
        po = None
    if po is None:
        po = _peer_outputs[key] = PeerOutput(M, N, device, group)
    return po


def release_peer_outputs() -> None:
    """Unmap every peer buffer (call on every rank before destroying the process group)."""
    for po in _peer_outputs.values():
        po.close()
    _peer_outputs.clear()


def _rank_barrier(device: torch.device, group=None) -> None:
    # A one-element all-reduce on the current stream: it completes on a rank only after every
    # rank's earlier work on its stream has completed.
    dist.all_reduce(torch.zeros(1, device=device), group=group)


def gemm_column_parallel(A: torch.Tensor, B_shard: torch.Tensor, A_sf: torch.Tensor,
                         B_sf_shard: torch.Tensor, scale: torch.Tensor, group=None,
                         gather: bool = False, chunks: int = 4,
                         gemm_fn: Optional[Callable] = None, fused: bool = False) -> torch.Tensor:
    """D[:, shard] = gemm_nvfp4(A, B_shard) on this rank; with gather=True the full D [M, N]
    (all ranks' shards, rank order along N) on every rank.

    gather=True, fused=False: the GEMM runs per chunk of M rows and each chunk's NCCL
    all_gather_into_tensor overlaps the next chunk's compute. fused=True: one GEMM whose
    epilogue stores this rank's tiles into every rank's output over NVLink (no collective for
    the data; two one-element all-reduces order the ranks before and after). The fused result
    is a shared buffer, valid until the next fused call of the same shape. Both need equal
    shard widths on all ranks."""
    fn = gemm_fn or _plugins().gemm_nvfp4
    world, rank = world_and_rank(group)
    if not gather or world == 1:
        return fn(A, B_shard, A_sf, B_sf_shard, scale)

    widths = [torch.tensor([B_shard.shape[0]], dtype=torch.int64, device=A.device)
              for _ in range(world)]
    dist.all_gather(widths, widths[0].clone(), group=group)
    w = [int(t.item()) for t in widths]
    if len(set(w)) != 1:
        raise ValueError(f"gather needs equal shard widths on all ranks, got {w}")
    n = w[0]
    if fused:
        po = peer_output(A.shape[0], world * n, A.device, group)
        _rank_barrier(A.device, group)      # every rank is done with the previous result
        _plugins().gemm_nvfp4_allgather(A, B_shard, A_sf, B_sf_shard, scale, po.local, po.ptrs,
                                        rank)
        _rank_barrier(A.device, group)      # every rank's stores have landed
        return po.local
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
