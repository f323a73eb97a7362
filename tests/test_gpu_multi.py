"""View-sharded step on two GPUs (one rank per GPU): the gradients that the
exchange (ViewShardedExchange over NCCL, or NvlsExchange with this library's
collectives, its all-reduce in the switch or by peer loads and stores) leaves on every rank equal the single-process
sum of the two views' full gradients, over several steps in a row.  Skipped
with fewer than two GPUs (NvlsExchange also without multicast support)."""

import os
import socket
import tempfile

import numpy as np
import pytest

from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _setup(device):
    from jaxgs_b200.scene import CapacityConfig, config0_scene, ring_cameras, world_cluster_bounds
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    pool_np, _, target = config0_scene()
    n = pool_np["xyz"].shape[0]
    config = CapacityConfig(n, 128, 16, 16, 3, n * 64, tile_height=8)
    center, extent, valid = world_cluster_bounds(pool_np, 128)
    bounds = tuple(torch.as_tensor(a, device=device) for a in (center, extent, valid.astype(np.uint8)))
    pool = GaussianArrays.from_numpy(pool_np, device=device)
    cams = [DeviceCamera.from_camera(c, device=device)
            for c in ring_cameras(2, radius=4.0, height=0.5, width=128, height_px=96, focal=110.0)]
    return pool, bounds, cams, torch.as_tensor(target, device=device), config


def _rank(rank, world, port, path, kind):
    import datetime

    import torch.distributed as dist

    from jaxgs_b200.step import GraphedTrainingStep, NvlsExchange, ViewShardedExchange

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=device)
    try:
        pool, bounds, cams, target, config = _setup(device)
        nvls = kind != "nccl"
        if nvls and not NvlsExchange.available():
            if rank == 0:
                np.savez(path, skipped=np.ones(1))
            return
        if nvls:
            exch = NvlsExchange(pool, config, 3, allreduce=kind)
        else:
            exch = ViewShardedExchange(pool, config, 3)
        # NvlsExchange: the exchange is captured into the step's graph.
        step = GraphedTrainingStep(pool, bounds, cams[rank], target, config, 3,
                                   **exch.step_kwargs, exchange=exch if nvls else None)
        for _ in range(3):  # reused buffers: every step must give the same sum
            step()
            grads = step.gradients if nvls else exch.exchange(step.camera.center)
        torch.cuda.synchronize()
        if nvls:
            assert not exch.failed()
        if rank == 0:
            np.savez(path, *[g.cpu().numpy() for g in grads])
        dist.barrier()
        del step
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("kind", ["nccl", "nvls", "p2p"])
def test_two_rank_view_sharded_gradients(kind):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from jaxgs_b200.step import compute_training_step, pool_gradient_buffer

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "grads.npz")
        mp.start_processes(_rank, args=(2, port, path, kind), nprocs=2, join=True,
                           start_method="spawn")
        got = np.load(path)
        if "skipped" in got:
            pytest.skip("no NVLS multicast between the GPUs")
        got = [got[f"arr_{i}"] for i in range(5)]
    pool, bounds, cams, target, config = _setup(torch.device("cuda", 0))
    expected = None
    for cam in cams:
        _, views = pool_gradient_buffer(pool, config, 3)
        compute_training_step(pool, bounds, cam, target, config, 3, pool_grads=views)
        expected = [v.clone() for v in views] if expected is None else [
            e + v for e, v in zip(expected, views)]
    for g, e in zip(got, expected):
        e = e.cpu().numpy()
        assert rel_l2(g.reshape(-1), e.reshape(-1)) < 1e-5
