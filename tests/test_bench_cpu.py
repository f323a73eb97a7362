"""bench.py's reference arm (the oracle port on the host cores, which the
driver runs beside the GPU arm) prints exactly one JSON line with the
contract's keys; it needs no GPU."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    run = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [line for line in run.stdout.splitlines() if line.strip()]
    assert len(lines) == 1, lines
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] and line["unit"] == "views/s" and line["value"] > 0
    assert line["n_gpus"] == 1 and line["steps"] == 1 and line["higher_is_better"] is True
    assert "config 2" in line["config"]["workload"]
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"],
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_under_torchrun_prints_once_with_every_host_thread():
    """Launched like the driver's N > 1 runs: rank 0 alone runs the oracle,
    with all the host threads it may use (the launcher's OMP_NUM_THREADS=1
    notwithstanding); the other rank exits 0 without output."""
    import os
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    run = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                          "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
                          "--master-port", str(port), "bench.py", "--impl", "reference",
                          "--gpus", "2", "--steps", "1", "--warmup", "0"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [line for line in run.stdout.splitlines() if line.strip()]
    assert len(lines) == 1, lines
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0
    from oracle import oracle as O

    openmp = O.num_threads() > 1 or len(os.sched_getaffinity(0)) == 1
    assert line["cpu_baseline"]["cores"] == (len(os.sched_getaffinity(0)) if openmp else 1)
