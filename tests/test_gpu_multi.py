"""View-sharded step on two GPUs (one rank per GPU): the gradients that the
exchange (ViewShardedExchange over NCCL, or NvlsExchange with this library's
collectives, its all-reduce in the switch or by peer loads and stores, with
the SH gradients expanded in the exchange or deferred to the optimizer as
gathered colour rows, pushed as compact entries or sparse chunks) leaves on every rank equal the single-process sum of
the two views' full gradients, over several steps in a row.  Skipped
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
        deferred = "-deferred" in kind
        if nvls:
            exch = NvlsExchange(pool, config, 3, allreduce=kind.split("-")[0],
                                deferred_sh=deferred,
                                colour_push="sparse" if kind.endswith("-sparse") else "compact")
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
        if deferred:
            from jaxgs_b200 import kernels as K
            from jaxgs_b200.optimizer import update_field, update_sh_from_rows

            rows = grads[4]
            sh = K.sh_from_colors(pool.xyz, None, rows, 3, 16)
            # The optimizer's own expansion of the rows equals expanding
            # them first and updating with the result, bit for bit.
            n_clusters = -(-pool.xyz.shape[0] // 128)
            clusters = (torch.arange(n_clusters, dtype=torch.int32, device=device),
                        torch.tensor([n_clusters], dtype=torch.int32, device=device))
            fused = [pool.sh.clone(), torch.full_like(pool.sh, 0.01), torch.full_like(pool.sh, 1e-3)]
            plain = [t.clone() for t in fused]
            update_sh_from_rows(*fused, pool.xyz, rows, pool.alive, clusters, 0.001, 128, 3)
            update_field(*plain, sh, pool.alive, clusters, 0.001, 128, True, False)
            torch.cuda.synchronize()
            assert all(torch.equal(a, b) for a, b in zip(fused, plain))
            grads = (*grads[:4], sh)
        if rank == 0:
            np.savez(path, *[g.cpu().numpy() for g in grads])
        dist.barrier()
        del step
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("kind", ["nccl", "nvls", "p2p", "nvls-deferred", "p2p-deferred",
                                  "p2p-deferred-sparse"])
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


def test_barrier_time_out_sets_the_error_word_and_stops_the_all_reduce():
    """A barrier whose peer never arrives (world 2, one rank running on one
    GPU; the second flag slot is never written) gives up after its bounded
    wait, sets the error word and returns, leaving the GPU usable.  The P2P
    all-reduce that follows reads the word and leaves both copies as they
    are; the same call without the word sums shard 0 into both (control).
    Every address is this GPU's own memory."""
    import ctypes

    from jaxgs_b200 import _lib as L

    dev = torch.device("cuda", 0)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    p = L.ExchangeParams(2, 0)
    flags = torch.zeros(2, dtype=torch.int32, device=dev)  # this rank's slots
    stand_in = torch.zeros(2, dtype=torch.int32, device=dev)  # in place of rank 1's slots
    peer_flags = torch.tensor([flags.data_ptr(), stand_in.data_ptr()], dtype=torch.int64,
                              device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    error = torch.zeros(1, dtype=torch.int32, device=dev)
    L.check(L.lib.gsb_exchange_barrier(stream, L.ref(p), ptr(peer_flags), ptr(flags), ptr(epoch),
                                       ptr(error)), "barrier")
    torch.cuda.synchronize()
    assert int(error.item()) == 1
    assert int(epoch.item()) == 1 and int(stand_in[0].item()) == 1
    a = torch.arange(64, dtype=torch.float32, device=dev)
    b = 100.0 + a
    a0, b0 = a.clone(), b.clone()
    copies = (ctypes.c_void_p * 2)(a.data_ptr(), b.data_ptr())
    L.check(L.lib.gsb_p2p_allreduce(stream, L.ref(p), copies, 64, ptr(error)), "P2P all-reduce")
    torch.cuda.synchronize()
    assert torch.equal(a, a0) and torch.equal(b, b0)
    L.check(L.lib.gsb_p2p_allreduce(stream, L.ref(p), copies, 64, None), "P2P all-reduce")
    torch.cuda.synchronize()
    total = a0[:32] + b0[:32]
    assert torch.equal(a[:32], total) and torch.equal(b[:32], total)
    assert torch.equal(a[32:], a0[32:]) and torch.equal(b[32:], b0[32:])
