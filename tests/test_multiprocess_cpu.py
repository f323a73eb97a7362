"""View-sharded gradient summation on two CPU ranks (gloo), and failure
detection on the host: a rank that never joins makes the collective of the
other rank fail with a timeout instead of hanging."""

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sum_worker(rank, world, port, out):
    from datetime import timedelta

    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.step import scatter_compact

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    config = CapacityConfig(max_gaussians=1000, cluster_size=128, sh_degree=1)
    rng = np.random.default_rng(rank)
    ids = np.sort(rng.choice(8, 5, replace=False)).astype(np.int32)
    clusters = (torch.as_tensor(ids), torch.tensor([5], dtype=torch.int32))
    grads = [torch.as_tensor(rng.normal(0, 1, (1000, k)).astype(np.float32)) for k in (3, 3, 4, 1, 12)]
    pool = scatter_compact(grads, clusters, config)
    flat = torch.cat([t.reshape(-1) for t in pool])
    dist.all_reduce(flat)
    out[rank] = flat.numpy()
    dist.destroy_process_group()


def _expected(world):
    from jaxgs_b200.scene import CapacityConfig

    total = None
    for rank in range(world):
        rng = np.random.default_rng(rank)
        ids = np.sort(rng.choice(8, 5, replace=False))
        grads = [rng.normal(0, 1, (1000, k)).astype(np.float32) for k in (3, 3, 4, 1, 12)]
        parts = []
        for g in grads:
            dst = np.zeros_like(g)
            for j, c in enumerate(ids):
                lo, hi = c * 128, min(c * 128 + 128, 1000)
                if lo < hi:
                    dst[lo:hi] += g[j * 128:j * 128 + (hi - lo)]
            parts.append(dst.reshape(-1))
        flat = np.concatenate(parts)
        total = flat if total is None else total + flat
    return total


def test_view_sharded_gradients_sum_across_ranks():
    world = 2
    port = _free_port()
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_sum_worker, args=(world, port, out), nprocs=world, join=True)
        results = [out[r] for r in range(world)]
    exp = _expected(world)
    for r in results:
        np.testing.assert_allclose(r, exp, rtol=1e-6, atol=1e-6)


def _missing_rank_worker(rank, world, port, out):
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        # This rank leaves between steps without entering the collective.
        out[rank] = "left"
        return
    try:
        dist.all_reduce(torch.ones(4))
        out[rank] = "completed"
    except Exception as exc:  # the collective must fail, not hang
        out[rank] = f"error: {type(exc).__name__}"


def test_a_rank_that_never_joins_is_detected_by_timeout():
    world = 2
    port = _free_port()
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_missing_rank_worker, args=(world, port, out), nprocs=world, join=True)
        assert out[1] == "left"
        assert out[0].startswith("error"), out[0]


def _outputs(losses, overflows, pairs):
    from jaxgs_b200.step import StepOutput

    for loss, overflow, count in zip(losses, overflows, pairs):
        yield StepOutput(torch.tensor(loss), (), (), torch.tensor([count], dtype=torch.int32),
                         torch.tensor([overflow], dtype=torch.int32))


def test_step_monitor_raises_like_the_trainer():
    """training/trainer.py:190-191 (overflow raises at epoch end with the
    peak pair count) and :230-231 (a non-finite loss raises); a healthy
    epoch reports its last loss and peak pairs and clears the record."""
    from jaxgs_b200.step import StepMonitor

    monitor = StepMonitor(100)
    for out in _outputs([0.5, 0.25], [0, 0], [40, 70]):
        monitor.record(out)
    assert monitor.check(3) == {"epoch": 3, "loss": 0.25, "peak_pairs": 70}
    for out in _outputs([0.5, 0.4], [1, 0], [130, 20]):
        monitor.record(out)
    with pytest.raises(RuntimeError, match="epoch 4: 130 pairs exceed 100"):
        monitor.check(4)
    for out in _outputs([0.5], [2], [10]):
        monitor.record(out)
    with pytest.raises(RuntimeError, match="gave up waiting"):
        monitor.check(5)
    for out in _outputs([float("nan")], [0], [10]):
        monitor.record(out)
    with pytest.raises(RuntimeError, match="non-finite training loss"):
        monitor.check(6)
    assert monitor.check(7)["peak_pairs"] == 0


def _raising_rank_worker(rank, world, port, out):
    from datetime import timedelta

    from jaxgs_b200.step import StepMonitor

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    monitor = StepMonitor(100)
    step = 0
    try:
        for step in range(3):
            grads = torch.ones(8)
            dist.all_reduce(grads)
            loss = float("nan") if (rank == 1 and step == 1) else 1.0 / (step + 1)
            for result in _outputs([loss], [0], [10]):
                monitor.record(result)
            # Checked between steps, with no collective in flight.
            monitor.check(step)
        out[rank] = "completed"
    except RuntimeError as exc:
        out[rank] = (step, str(exc).splitlines()[0])
    finally:
        dist.destroy_process_group()


def test_a_rank_that_raises_between_steps_fails_the_job():
    """A rank whose step check raises (a non-finite loss) leaves between
    collectives; the other rank's next all-reduce then fails (peer gone or
    time-out) instead of waiting for good."""
    world = 2
    port = _free_port()
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_raising_rank_worker, args=(world, port, out), nprocs=world, join=True)
        assert out[1] == (1, "non-finite training loss")
        assert out[0] != "completed" and out[0][0] == 2, out[0]
