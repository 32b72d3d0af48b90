"""Multi-GPU path on real GPUs (NCCL over NVLink): row-sharded quantize with a global amax,
column-parallel GEMM shards and the chunked all-gather of D, all bit-identical to the single-GPU
result. Runs two ranks under torchrun; skipped when fewer than two GPUs are visible."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_sharded_quantize_gemm_gather():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", os.path.join(HERE, "sharded_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=360)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "rank 0: ok" in r.stdout and "rank 1: ok" in r.stdout


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("M,n_loc,K", [(300, 520, 2560), (96, 1024, 512), (16, 3584, 2048),
                                       (100, 7168, 2048)])
def test_fused_allgather_two_gpus_one_process(M, n_loc, K):
    """The fused GEMM + all-gather with both ranks driven from one process (peer access instead of
    IPC handles): every rank's output equals the single-GPU GEMM bit for bit. The decode shards
    (16 x 3584, 100 x 7168) take split-K forms, whose epilogue stores each sum to both GPUs."""
    cmd = ["timeout", "-k", "30", "300", sys.executable, os.path.join(HERE, "fused_allgather_1proc.py"),
           "2", str(M), str(n_loc), str(K), "2"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=360)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "outputs bit-identical" in r.stdout
