"""Host logic of the multi-GPU path on CPU ranks (gloo, world_size 2): shard arithmetic, the
chunked all-gather assembly of a column-parallel GEMM, the row-sharded quantize with a global
amax all-reduce, and failure behaviour (a rank that dies or disagrees ends the others' next
collective with an error instead of a hang). The GEMM/quantize compute is the CPU oracle here;
on GPUs the same functions call the CUDA kernels."""
import datetime
import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

from my_nvfp4_gemm_b200.sharded import shard_range  # noqa: E402


@pytest.mark.parametrize("n", [8, 128, 1024, 8192, 28672, 57344, 1000, 136])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_range_partitions(n, world):
    spans = [shard_range(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    assert all((s1 - s0) % 8 == 0 for s0, s1 in spans)
    if n % (128 * world) == 0:
        assert len({s1 - s0 for s0, s1 in spans}) == 1 and (spans[0][1] % 128 == 0)


def test_shard_range_rejects():
    with pytest.raises(ValueError):
        shard_range(12, 2, 0)
    with pytest.raises(ValueError):
        shard_range(64, 2, 2)


# ---------------------------------------------------------------- multi-process harness
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, scenario, queue):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "tests")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=8))
        out = SCENARIOS[scenario](rank, world)
        queue.put((rank, "ok", out))
    except Exception as e:  # reported to the parent, which asserts on it
        queue.put((rank, "err", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-600:]}"))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def run_ranks(scenario, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, out = q.get(timeout=timeout)
        results[rank] = (status, out)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


# ---------------------------------------------------------------- oracle compute on CPU
def _oracle_gemm(A, B, A_sf, B_sf, scale):
    from oracle import oracle as O
    d = O.gemm(A.numpy(), B.numpy(), A_sf.view(torch.uint8).numpy(), B_sf.view(torch.uint8).numpy(),
               float(scale))
    return torch.from_numpy(d.view(np.int16)).view(torch.bfloat16)


def _oracle_quantize(x, s):
    from oracle import oracle as O
    q, sf = O.quantize(x.view(torch.int16).numpy().view(np.uint16).reshape(-1), float(s))
    return (torch.from_numpy(q).reshape(*x.shape[:-1], x.shape[-1] // 2),
            torch.from_numpy(sf).reshape(*x.shape[:-1], x.shape[-1] // 16).view(torch.float8_e4m3fn))


def _operands(M=96, N=512, K=512, seed=4):
    rng = np.random.default_rng(seed)
    A = torch.from_numpy(rng.integers(0, 256, (M, K // 2), dtype=np.uint8))
    B = torch.from_numpy(rng.integers(0, 256, (N, K // 2), dtype=np.uint8))
    A_sf = torch.from_numpy(rng.integers(0x28, 0x40, (M, K // 16), dtype=np.uint8)).view(torch.float8_e4m3fn)
    B_sf = torch.from_numpy(rng.integers(0x28, 0x40, (N, K // 16), dtype=np.uint8)).view(torch.float8_e4m3fn)
    return A, B, A_sf, B_sf, torch.tensor(2.5)


def scenario_gather(rank, world):
    from my_nvfp4_gemm_b200.sharded import gemm_column_parallel, shard_weight
    A, B, A_sf, B_sf, s = _operands()
    Bs, Bsfs = shard_weight(B, B_sf, world, rank)
    local = gemm_column_parallel(A, Bs, A_sf, Bsfs, s, gather=False, gemm_fn=_oracle_gemm)
    full = gemm_column_parallel(A, Bs, A_sf, Bsfs, s, gather=True, chunks=3, gemm_fn=_oracle_gemm)
    want = _oracle_gemm(A, B, A_sf, B_sf, s)
    n0, n1 = shard_range(B.shape[0], world, rank)
    return (bool(torch.equal(local.view(torch.int16), want[:, n0:n1].view(torch.int16))),
            bool(torch.equal(full.view(torch.int16), want.view(torch.int16))))


def scenario_row_quantize(rank, world):
    from my_nvfp4_gemm_b200.sharded import quantize_row_sharded
    g = torch.Generator().manual_seed(1)
    X = torch.randn(64, 256, generator=g).to(torch.bfloat16)
    X[5, 7] = 300.0 if world == 2 else X[5, 7]            # the global max lives on rank 0
    rows = X.shape[0] // world
    mine = X[rank * rows:(rank + 1) * rows].contiguous()
    q, sf, s = quantize_row_sharded(mine, quantize_fn=_oracle_quantize)
    s_single = 6 * 448 / X.abs().max().to(dtype=torch.float32)
    qw, sfw = _oracle_quantize(mine, s_single)
    return (float(s), float(s_single), bool(torch.equal(q, qw)),
            bool(torch.equal(sf.view(torch.uint8), sfw.view(torch.uint8))))


def scenario_unequal_widths(rank, world):
    from my_nvfp4_gemm_b200.sharded import gemm_column_parallel
    A, B, A_sf, B_sf, s = _operands(N=512)
    n = 256 if rank == 0 else 128
    gemm_column_parallel(A, B[:n], A_sf, B_sf[:n], s, gather=True, gemm_fn=_oracle_gemm)
    return "no error"


def scenario_rank_dies(rank, world):
    """Rank 1 fails between steps (before its next collective); rank 0's next collective must
    end with an error within the process-group timeout rather than wait forever."""
    t = torch.ones(4)
    dist.all_reduce(t)                       # step 1: everyone healthy
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    dist.all_reduce(t)                       # step 2: rank 1 never joins
    return "no error"


def scenario_export_fails(rank, world):
    """The fused all-gather's output buffer cannot be exported on rank 1 (as under torch's
    expandable segments): every rank raises the same explanatory error, none waits."""
    from my_nvfp4_gemm_b200 import capi, sharded
    if rank == 1:
        def export(ptr):
            raise capi.NvFp4Error(4, "nvfp4_ipc_export")
    else:
        def export(ptr):
            return b"\0" * capi.IPC_HANDLE_BYTES, 0
    capi.ipc_export = export
    sharded.PeerOutput(16, 32, torch.device("cpu"))
    return "no error"


SCENARIOS = {
    "export_fails": scenario_export_fails,
    "gather": scenario_gather,
    "row_quantize": scenario_row_quantize,
    "unequal_widths": scenario_unequal_widths,
    "rank_dies": scenario_rank_dies,
}


def test_column_parallel_gather_matches_unsharded():
    res = run_ranks("gather")
    for rank, (status, out) in res.items():
        assert status == "ok", out
        assert out == (True, True), f"rank {rank}: local/gathered mismatch {out}"


def test_row_sharded_quantize_uses_global_amax():
    res = run_ranks("row_quantize")
    for rank, (status, out) in res.items():
        assert status == "ok", out
        s, s_single, q_ok, sf_ok = out
        assert s == s_single and q_ok and sf_ok, (rank, out)


def test_unequal_shard_widths_rejected_on_every_rank():
    res = run_ranks("unequal_widths")
    for rank, (status, out) in res.items():
        assert status == "err" and "equal shard widths" in out, (rank, out)


def test_dead_rank_surfaces_as_error_not_hang():
    res = run_ranks("rank_dies", timeout=90)
    assert res[1][0] == "err" and "injected failure" in res[1][1]
    assert res[0][0] == "err", f"rank 0 should see its collective fail, got {res[0]}"


def test_ipc_export_failure_raises_on_every_rank():
    res = run_ranks("export_fails")
    for rank, (status, out) in res.items():
        assert status == "err" and "expandable_segments" in out and "rank(s) [1]" in out, (rank, out)
