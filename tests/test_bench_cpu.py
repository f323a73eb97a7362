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


def _walk_visits(last, offsets, bits, W, H, tw, th):
    """raster_bwd_kernel's walk over the contribution words, one warp at a
    time, in plain loops."""
    rows = 2 if th % 8 == 0 else 1
    blocks_x, block_h = tw // 8, 4 * rows
    warps = blocks_x * (th // block_h)
    tiles_x, tiles_y = -(-W // tw), -(-H // th)
    visits = 0
    for tile in range(tiles_x * tiles_y):
        start = int(offsets[tile])
        for w in range(warps):
            bx0 = (tile % tiles_x) * tw + (w % blocks_x) * 8
            by0 = (tile // tiles_x) * th + (w // blocks_x) * block_h
            top = start
            for y in range(by0, min(by0 + block_h, H)):
                for x in range(bx0, min(bx0 + 8, W)):
                    top = max(top, int(last[y * W + x]))
            if top <= start:
                continue
            top_batch = (top - 1 - start) >> 5
            for batch in range(top_batch + 1):
                word = int(bits[((start >> 5) + tile + batch) * warps + w]) & 0xFFFFFFFF
                if batch == top_batch:
                    k_max = (top - 1 - start) & 31
                    word &= 0xFFFFFFFF if k_max == 31 else (2 << k_max) - 1
                visits += bin(word).count("1")
    return visits


def test_backward_visit_count_follows_the_kernels_walk():
    """bench.py's vectorised count of the contribution bits raster_bwd_kernel
    visits (the roofline's fragment count) equals the kernel's walk."""
    import numpy as np
    import torch

    sys.path.insert(0, str(ROOT))
    from bench import count_visits

    rng = np.random.default_rng(4)
    for W, H, tw, th in ((37, 21, 16, 8), (40, 24, 16, 16), (19, 13, 8, 8), (32, 12, 16, 12)):
        tiles = -(-W // tw) * -(-H // th)
        counts = rng.integers(0, 90, tiles)
        if tiles > 4:
            counts[rng.integers(0, tiles, 2)] = 0  # empty tiles
        offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
        tile_of_pixel = (np.arange(H)[:, None] // th) * -(-W // tw) + np.arange(W)[None, :] // tw
        span = counts[tile_of_pixel]
        last = offsets[tile_of_pixel] + (rng.random((H, W)) * (span + 1)).astype(np.int64)
        rows = 2 if th % 8 == 0 else 1
        warps = (tw // 8) * (th // (4 * rows))
        words = (int(offsets[-1]) // 32 + tiles + 1) * warps
        bits = rng.integers(-2**31, 2**31, words, dtype=np.int64).astype(np.int32)
        got = count_visits(torch.as_tensor(last.reshape(-1).astype(np.int32)),
                           torch.as_tensor(offsets), torch.as_tensor(bits), W, H, tw, th)
        assert got == _walk_visits(last.reshape(-1), offsets, bits, W, H, tw, th) > 0
