"""bench.py's output contract on the host: rank 0 prints exactly one JSON line on stdout, and
anything else a library writes to file descriptor 1 (NCCL's version banner, for one) is moved to
stderr. The reference arm runs on the CPU, so its whole line is checked here."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_result_line_is_the_only_stdout():
    code = ("import os, bench; bench.keep_stdout_for_result(); "
            "os.write(1, b'NCCL version x.y.z\\n'); print('python-level chatter'); "
            "bench.emit({'metric': 'm', 'value': 1.0})")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.splitlines() == ['{"metric": "m", "value": 1.0}']
    assert "NCCL version x.y.z" in r.stderr and "python-level chatter" in r.stderr


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.splitlines()
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference")
    # the same workload description as the GPU arm's line (so the two lines compare)
    sys.path.insert(0, ROOT)
    import bench
    assert d["config"] == bench.square_config(8192, 1)


def test_sharded_roofline_arithmetic():
    """Per-rank roofline of the sharded keys: algorithmic bytes (weight shard codes + scale
    factors, activation codes + scale factors, bf16 D) and, with a gather, the NVLink bound."""
    sys.path.insert(0, ROOT)
    import bench
    M, K, n_loc, world = 16, 8192, 3584, 8
    inp = {"M": M, "K": K, "n_loc": n_loc}
    ms = 0.008
    r = bench.sharded_roofline(inp, ms, world, 6550.0)
    bytes_rank = n_loc * K * 0.5625 + M * K * 0.5625 + 2.0 * M * n_loc
    assert abs(r["algorithmic_bytes_per_rank"] - bytes_rank) < 1
    assert abs(r["achieved_gbs_per_rank"] - bytes_rank / (ms * 1e-3) / 1e9) < 1e-6
    assert abs(r["frac_hbm_per_rank"] - r["achieved_gbs_per_rank"] / 6550.0) < 1e-9
    assert abs(r["achieved_tflops_per_rank"] - 2.0 * M * n_loc * K / (ms * 1e-3) / 1e12) < 1e-9
    assert "bound_ms" not in r
    g = bench.sharded_roofline(inp, ms, world, 6550.0, gather=True)
    nv = 2.0 * M * n_loc * (world - 1)
    bound = max(2.0 * M * n_loc * K / (bench.NOMINAL_FP4_TFLOPS * 1e12),
                nv / (bench.NVLINK_GBS * 1e9)) * 1e3
    assert g["nvlink_bytes_out_per_rank"] == nv
    assert abs(g["bound_ms"] - bound) < 1e-12 and abs(g["frac_of_bound"] - bound / ms) < 1e-9

