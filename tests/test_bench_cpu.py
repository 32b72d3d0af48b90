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
