"""The whole training step on the GPU vs the oracle's restatement of it.

BASELINE config 0 (4,096 Gaussians, 128x96, 8x16 tiles, SH degree 3, uint8
target): loss within 1e-5 relative; every parameter gradient within 1e-3
relative L2.  The GPU's visible-cluster list is handed to
the oracle so both sides use the same compact gradient order.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _run(pool_np, cam, target, degree=3, tile=(8, 16)):
    from jaxgs_b200.scene import CapacityConfig, world_cluster_bounds
    from jaxgs_b200.step import compute_training_step
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    n = pool_np["xyz"].shape[0]
    config = CapacityConfig(n, 128, 16, tile[1], 3, n * 64, tile_height=tile[0])
    center, extent, valid = world_cluster_bounds(pool_np, 128)
    bounds = (torch.as_tensor(center, device="cuda"), torch.as_tensor(extent, device="cuda"),
              torch.as_tensor(valid.astype(np.uint8), device="cuda"))
    out = compute_training_step(GaussianArrays.from_numpy(pool_np), bounds,
                                DeviceCamera.from_camera(cam), torch.as_tensor(target, device="cuda"),
                                config, degree)
    torch.cuda.synchronize()
    ids = out.visible_clusters[0].cpu().numpy()
    count = int(out.visible_clusters[1].item())
    exp = O.training_step(pool_np, cam, target, degree=degree, sh_dim=16, tile_w=tile[1],
                          tile_h=tile[0], max_pairs=n * 64, clusters=(ids, count))
    return out, exp, count


@pytest.mark.parametrize("tile", [(8, 16), (16, 16)])
def test_training_step_matches_oracle(tile):
    from jaxgs_b200.scene import config0_scene

    pool_np, cam, target = config0_scene()
    out, exp, count = _run(pool_np, cam, target, tile=tile)
    assert count > 0
    loss = float(out.loss)
    assert abs(loss - exp["loss"]) <= 1e-5 * abs(exp["loss"]), (loss, exp["loss"])
    rows = count * 128
    for name, got, ref in zip(("xyz", "log_scale", "rotation", "opacity", "sh"), out.gradients,
                              exp["grads"]):
        g = got.cpu().numpy().reshape(pool_np["xyz"].shape[0], -1)[:rows]
        r = ref.reshape(pool_np["xyz"].shape[0], -1)[:rows]
        err = rel_l2(g, r)
        assert err < 1e-3, (name, err)


def test_training_step_inactive_and_culled_gaussians():
    """Dead slots and a camera that culls part of the pool."""
    from jaxgs_b200.scene import Camera, config0_scene

    pool_np, _, target = config0_scene()
    pool_np["alive"][::3] = False
    cam = Camera.look_at((1.2, 0.4, -3.0), (0.8, 0.0, 0.0), 110.0, 110.0, 128, 96, near=0.01,
                         far=100.0)
    out, exp, count = _run(pool_np, cam, target, degree=1)
    assert abs(float(out.loss) - exp["loss"]) <= 1e-5 * abs(exp["loss"])
    rows = count * 128
    for got, ref in zip(out.gradients, exp["grads"]):
        g = got.cpu().numpy().reshape(4096, -1)[:rows]
        assert rel_l2(g, ref.reshape(4096, -1)[:rows]) < 1e-3


def test_training_step_partial_cluster_and_empty_view():
    """A pool of 1000 slots (its last cluster partial) against the oracle,
    and a camera that sees no cluster at all: the step runs with zero pairs,
    the loss is that of the background image and every gradient is zero."""
    from jaxgs_b200.scene import Camera, config0_scene

    pool_np, cam, target = config0_scene()
    small = {k: np.ascontiguousarray(v[:1000]) for k, v in pool_np.items()}
    out, exp, count = _run(small, cam, target)
    assert count == 8
    assert abs(float(out.loss) - exp["loss"]) <= 1e-5 * abs(exp["loss"])
    for got, ref in zip(out.gradients, exp["grads"]):
        g = got.cpu().numpy().reshape(1000, -1)
        assert rel_l2(g, ref.reshape(1000, -1)) < 1e-3
    away = Camera.look_at((0.0, 0.0, -4.0), (0.0, 0.0, -8.0), 110.0, 110.0, 128, 96,
                          near=0.01, far=100.0)
    out, exp, count = _run(pool_np, away, target)
    assert count == 0 and int(out.pair_count.item()) == 0
    assert abs(float(out.loss) - exp["loss"]) <= 1e-5 * abs(exp["loss"])


def test_pool_order_gradients_for_the_view_sharded_exchange():
    """pool_grads: the step writes pool-order gradients (culled clusters' rows
    zero, stale contents overwritten) into views of one flat buffer, equal to
    the compact gradients scattered to pool order; the graphed step does the
    same on every replay."""
    from jaxgs_b200.scene import Camera, CapacityConfig, config0_scene, world_cluster_bounds
    from jaxgs_b200.step import (GraphedTrainingStep, compute_training_step, pool_gradient_buffer,
                                 scatter_compact)
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    pool_np, _, target = config0_scene()
    # Clusters as x slabs, camera on the +x side: the low-x clusters are culled.
    order = np.argsort(pool_np["xyz"][:, 0], kind="stable")
    pool_np = {k: np.ascontiguousarray(v[order]) for k, v in pool_np.items()}
    cam = Camera.look_at((1.8, 0.0, -2.5), (1.8, 0.0, 0.0), 110.0, 110.0, 128, 96, near=0.01,
                         far=100.0)
    n = pool_np["xyz"].shape[0]
    config = CapacityConfig(n, 128, 16, 16, 3, n * 64, tile_height=8)
    center, extent, valid = world_cluster_bounds(pool_np, 128)
    bounds = (torch.as_tensor(center, device="cuda"), torch.as_tensor(extent, device="cuda"),
              torch.as_tensor(valid.astype(np.uint8), device="cuda"))
    pool = GaussianArrays.from_numpy(pool_np)
    dcam = DeviceCamera.from_camera(cam)
    tgt = torch.as_tensor(target, device="cuda")
    ref = compute_training_step(pool, bounds, dcam, tgt, config, 3)
    count = int(ref.visible_clusters[1].item())
    assert 0 < count < n // 128  # some clusters culled
    expected = scatter_compact(ref.gradients, ref.visible_clusters, config)
    flat, views = pool_gradient_buffer(pool, config, 3)
    flat.fill_(float("nan"))
    out = compute_training_step(pool, bounds, dcam, tgt, config, 3, pool_grads=views)
    torch.cuda.synchronize()
    assert abs(float(out.loss) - float(ref.loss)) <= 1e-6 * abs(float(ref.loss))
    for got, exp in zip(views, expected):
        g, e = got.cpu().numpy().reshape(-1), exp.cpu().numpy().reshape(-1)
        assert np.isfinite(g).all()
        assert rel_l2(g, e) < 1e-5
    graphed = GraphedTrainingStep(pool, bounds, dcam, tgt, config, 3, pool_grads=views)
    flat.fill_(float("nan"))
    graphed()
    torch.cuda.synchronize()
    for got, exp in zip(views, expected):
        assert rel_l2(got.cpu().numpy().reshape(-1), exp.cpu().numpy().reshape(-1)) < 1e-5


def test_training_step_fragment_statistics():
    """collect_stats: the step's [C, 4] fragment statistics equal the oracle's
    for the view; with `stats` they are added into it in place
    (training/step.py:125-126), and a graphed step adds one view's worth on
    every replay."""
    from jaxgs_b200.scene import CapacityConfig, config0_scene, world_cluster_bounds
    from jaxgs_b200.step import GraphedTrainingStep, compute_training_step
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    pool_np, cam, target = config0_scene()
    n = pool_np["xyz"].shape[0]
    config = CapacityConfig(n, 128, 16, 16, 3, n * 64, tile_height=8)
    center, extent, valid = world_cluster_bounds(pool_np, 128)
    bounds = (torch.as_tensor(center, device="cuda"), torch.as_tensor(extent, device="cuda"),
              torch.as_tensor(valid.astype(np.uint8), device="cuda"))
    pool = GaussianArrays.from_numpy(pool_np)
    dcam = DeviceCamera.from_camera(cam)
    tgt = torch.as_tensor(target, device="cuda")
    out = compute_training_step(pool, bounds, dcam, tgt, config, 3, collect_stats=True)
    torch.cuda.synchronize()
    ids = out.visible_clusters[0].cpu().numpy()
    count = int(out.visible_clusters[1].item())
    exp = O.training_step(pool_np, cam, target, degree=3, sh_dim=16, tile_w=16, tile_h=8,
                          max_pairs=n * 64, clusters=(ids, count))
    single = out.stats.cpu().numpy()
    assert single.shape == (n, 4) and exp["stats"][:, 0].sum() > 0
    assert np.mean(single[:, 0] == exp["stats"][:, 0]) >= 0.99
    for col in range(4):
        assert rel_l2(single[:, col], exp["stats"][:, col]) < 1e-3, col
    acc = torch.ones(n, 4, device="cuda")
    again = compute_training_step(pool, bounds, dcam, tgt, config, 3, collect_stats=True,
                                  stats=acc)
    assert again.stats is acc
    torch.cuda.synchronize()
    assert rel_l2(acc.cpu().numpy() - 1.0, single) < 1e-5
    graphed = GraphedTrainingStep(pool, bounds, dcam, tgt, config, 3, collect_stats=True)
    for _ in range(3):
        graphed()
    torch.cuda.synchronize()
    assert rel_l2(graphed.out.stats.cpu().numpy(), 3 * single) < 1e-5


def test_graphed_step_staged_upload_equals_direct_inputs():
    """GraphedTrainingStep.upload stages pinned host inputs on a copy stream;
    the next call consumes them and gives the same loss and gradients as a
    call that passes the same inputs directly."""
    from jaxgs_b200.scene import Camera, CapacityConfig, config0_scene, world_cluster_bounds
    from jaxgs_b200.step import GraphedTrainingStep
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    pool_np, cam, target = config0_scene()
    n = pool_np["xyz"].shape[0]
    config = CapacityConfig(n, 128, 16, 16, 3, n * 64, tile_height=8)
    center, extent, valid = world_cluster_bounds(pool_np, 128)
    bounds = (torch.as_tensor(center, device="cuda"), torch.as_tensor(extent, device="cuda"),
              torch.as_tensor(valid.astype(np.uint8), device="cuda"))
    pool = GaussianArrays.from_numpy(pool_np)
    step = GraphedTrainingStep(pool, bounds, DeviceCamera.from_camera(cam),
                               torch.as_tensor(target, device="cuda"), config, 3)
    other = Camera.look_at((1.0, 0.3, -3.2), (0.2, 0.0, 0.0), cam.fx, cam.fy, cam.width,
                           cam.height, near=cam.near, far=cam.far)
    other_target = np.ascontiguousarray(target[::-1])
    direct = step(DeviceCamera.from_camera(other), torch.as_tensor(other_target, device="cuda"))
    loss_direct = float(direct.loss)
    grads_direct = [g.clone() for g in direct.gradients]
    step(DeviceCamera.from_camera(cam), torch.as_tensor(target, device="cuda"))
    host_cam = DeviceCamera.from_camera(other, device="cpu")
    host_cam = DeviceCamera(*(t.pin_memory() for t in (host_cam.world_to_camera,
                                                        host_cam.intrinsics, host_cam.center,
                                                        host_cam.planes)),
                            other.width, other.height, other.near, other.far)
    step.upload(host_cam, torch.as_tensor(other_target).pin_memory())
    staged = step()
    torch.cuda.synchronize()
    assert float(staged.loss) == loss_direct
    for a, b in zip(staged.gradients, grads_direct):
        assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) < 1e-6
    # The packed camera (one copy) gives the same step again.
    step(DeviceCamera.from_camera(cam), torch.as_tensor(target, device="cuda"))
    step.upload(host_cam.pack().pin_memory(), torch.as_tensor(other_target).pin_memory())
    packed = step()
    torch.cuda.synchronize()
    assert float(packed.loss) == loss_direct
    # Only the captured image size, clip planes and target shape replay.
    for bad in (Camera.look_at((1.0, 0.3, -3.2), (0.2, 0.0, 0.0), cam.fx, cam.fy, cam.width,
                               cam.height, near=cam.near * 2, far=cam.far),
                Camera.look_at((1.0, 0.3, -3.2), (0.2, 0.0, 0.0), cam.fx, cam.fy, cam.width + 16,
                               cam.height, near=cam.near, far=cam.far)):
        with pytest.raises(ValueError, match="captured"):
            step(DeviceCamera.from_camera(bad))
        with pytest.raises(ValueError, match="captured"):
            step.upload(DeviceCamera.from_camera(bad, device="cpu"))
    with pytest.raises(ValueError, match="captured"):
        step(target=torch.as_tensor(target[:, :64].copy(), device="cuda"))
    with pytest.raises(ValueError, match="captured"):
        step.upload(target=torch.as_tensor(target.astype(np.float32) / 255))


def test_graphed_step_double_buffered_inputs_and_loss_readback():
    """Uploads alternate between the two input buffers: every staged step
    gives the loss of a direct call with the same inputs, an upload of only
    the camera keeps the latest target, a call with no inputs repeats the
    latest step, and read_loss delivers each step's loss to pinned host
    memory."""
    from jaxgs_b200.scene import Camera, CapacityConfig, config0_scene, world_cluster_bounds
    from jaxgs_b200.step import GraphedTrainingStep
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    pool_np, cam, target = config0_scene()
    n = pool_np["xyz"].shape[0]
    config = CapacityConfig(n, 128, 16, 16, 3, n * 64, tile_height=8)
    bounds = tuple(torch.as_tensor(a, device="cuda") for a in world_cluster_bounds(pool_np, 128))
    pool = GaussianArrays.from_numpy(pool_np)
    step = GraphedTrainingStep(pool, bounds, DeviceCamera.from_camera(cam),
                               torch.as_tensor(target, device="cuda"), config, 3)
    cams = [cam] + [Camera.look_at((0.8 * k - 1.0, 0.3, -3.5), (0.1 * k, 0.0, 0.0), cam.fx, cam.fy,
                                   cam.width, cam.height, near=cam.near, far=cam.far)
                    for k in range(3)]
    targets = [target, np.ascontiguousarray(target[::-1]), np.ascontiguousarray(target[:, ::-1]),
               np.ascontiguousarray(255 - target)]
    expected = []
    for c, t in zip(cams, targets):
        out = step(DeviceCamera.from_camera(c), torch.as_tensor(t, device="cuda"))
        expected.append(float(out.loss))
    torch.cuda.synchronize()
    assert len(set(expected)) == len(expected)
    host = torch.empty(8, dtype=torch.float32).pin_memory()
    packed = [DeviceCamera.from_camera(c, device="cpu").pack().pin_memory() for c in cams]
    pinned = [torch.as_tensor(t).pin_memory() for t in targets]
    order = [2, 0, 3, 1, 2]
    step.upload(packed[order[0]], pinned[order[0]])
    for i, k in enumerate(order):
        step()
        if i + 1 < len(order):
            step.upload(packed[order[i + 1]], pinned[order[i + 1]])
        read = step.read_loss(host[i])
    read.synchronize()
    for i, k in enumerate(order):
        assert float(host[i]) == expected[k], (i, k)
    # Camera only: the target of the latest step (order[-1]) is kept.
    step.upload(packed[1])
    out = step()
    again = step()
    torch.cuda.synchronize()
    direct = step(DeviceCamera.from_camera(cams[1]), torch.as_tensor(targets[order[-1]], device="cuda"))
    torch.cuda.synchronize()
    assert float(out.loss) == float(again.loss) == float(direct.loss)


def _np_sh_from_colors(xyz, centers, colors, degree, sh_dim):
    """training/sh_pullback.py:18-53 in numpy (float64), summed over views."""
    out = np.zeros((xyz.shape[0], sh_dim, 3))
    for center, gc in zip(centers, colors):
        delta = xyz.astype(np.float64) - center
        norm = np.sqrt(np.maximum((delta * delta).sum(1, keepdims=True), 1e-16))
        dx, dy, dz = (delta / norm).T
        xx, yy, zz = dx * dx, dy * dy, dz * dz
        basis = [np.full_like(dx, 0.28209479177387814), -0.4886025119029199 * dy,
                 0.4886025119029199 * dz, -0.4886025119029199 * dx,
                 1.0925484305920792 * dx * dy, -1.0925484305920792 * dy * dz,
                 0.31539156525252005 * (2 * zz - xx - yy), -1.0925484305920792 * dx * dz,
                 0.5462742152960396 * (xx - yy), -0.5900435899266435 * dy * (3 * xx - yy),
                 2.890611442640554 * dx * dy * dz, -0.4570457994644658 * dy * (4 * zz - xx - yy),
                 0.3731763325901154 * dz * (2 * zz - 3 * xx - 3 * yy),
                 -0.4570457994644658 * dx * (4 * zz - xx - yy), 1.445305721320277 * dz * (xx - yy),
                 -0.5900435899266435 * dx * (xx - 3 * yy)]
        for k in range((degree + 1) ** 2):
            out[:, k, :] += basis[k][:, None] * gc.reshape(-1, 3)
    return out


@pytest.mark.parametrize("degree,sh_dim", [(0, 1), (1, 4), (2, 16), (3, 16)])
def test_sh_from_colors_matches_sh_pullback(degree, sh_dim):
    from jaxgs_b200 import kernels as K

    rng = np.random.default_rng(degree)
    C, V = 1000, 3
    xyz = rng.normal(0, 2, (C, 3)).astype(np.float32)
    centers = rng.normal(0, 5, (V, 3)).astype(np.float32)
    colors = rng.normal(0, 1, (V, C, 3)).astype(np.float32)
    colors[:, ::7] = 0.0  # culled in some views
    xyz[5] = centers[1]   # direction floor (|delta| = 0)
    got = K.sh_from_colors(torch.as_tensor(xyz, device="cuda"), torch.as_tensor(centers, device="cuda"),
                           torch.as_tensor(colors, device="cuda"), degree, sh_dim)
    exp = _np_sh_from_colors(xyz, centers, colors, degree, sh_dim)
    np.testing.assert_allclose(got.cpu().numpy(), exp, rtol=1e-5, atol=1e-6)


def test_view_sharded_exchange_math_equals_summed_per_view_gradients():
    """The exchange's decomposition (summed geometric gradients + per-view
    colour cotangents expanded on each view's SH basis) equals the sum of
    the per-view full gradients, here for three views on one GPU."""
    from jaxgs_b200 import kernels as K
    from jaxgs_b200.scene import CapacityConfig, config0_scene, ring_cameras, world_cluster_bounds
    from jaxgs_b200.step import compute_training_step, pool_gradient_buffer
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    pool_np, _, target = config0_scene()
    n = pool_np["xyz"].shape[0]
    config = CapacityConfig(n, 128, 16, 16, 3, n * 64, tile_height=8)
    center, extent, valid = world_cluster_bounds(pool_np, 128)
    bounds = (torch.as_tensor(center, device="cuda"), torch.as_tensor(extent, device="cuda"),
              torch.as_tensor(valid.astype(np.uint8), device="cuda"))
    pool = GaussianArrays.from_numpy(pool_np)
    tgt = torch.as_tensor(target, device="cuda")
    cams = [DeviceCamera.from_camera(c) for c in ring_cameras(3, radius=4.0, height=0.5, width=128,
                                                                height_px=96, focal=110.0)]
    expected = None
    for cam in cams:
        flat, views = pool_gradient_buffer(pool, config, 3)
        compute_training_step(pool, bounds, cam, tgt, config, 3, pool_grads=views)
        expected = [v.clone() for v in views] if expected is None else [
            e + v for e, v in zip(expected, views)]
    geometric = [torch.zeros_like(e) for e in expected[:4]]
    colors = []
    for cam in cams:
        bufs = tuple(torch.empty_like(e) for e in expected[:4]) + (
            torch.empty(n, 1, 3, device="cuda"),)
        compute_training_step(pool, bounds, cam, tgt, config, 3, pool_grads=bufs,
                              sh_color_only=True)
        geometric = [a + b for a, b in zip(geometric, bufs[:4])]
        colors.append(bufs[4].view(n, 3))
    centers = torch.stack([c.center.reshape(3) for c in cams])
    sh = K.sh_from_colors(pool.xyz, centers, torch.stack(colors), 3, 16)
    torch.cuda.synchronize()
    for got, exp in zip((*geometric, sh), expected):
        g, e = got.cpu().numpy().reshape(-1), exp.cpu().numpy().reshape(-1)
        assert np.abs(e).max() > 0
        assert rel_l2(g, e) < 1e-5
