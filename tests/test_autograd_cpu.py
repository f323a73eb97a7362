"""jaxgs_b200.autograd on the CPU with the kernel bindings it calls replaced
by the oracle (same types in, same types out): the render's backward, which
composes the raster backward over the listed clusters with the pool-order
projection pullback, gives the gradient of its own forward (central
differences, as tests/test_cute.py:328-355 checks the reference's
custom_vjp), every gradient lands on its own parameter tensor with that
tensor's shape, and the loss Function scales its saved image gradient by
the upstream gradient.  The bindings themselves are checked against the
same oracle on the GPU."""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import np_proj

torch = pytest.importorskip("torch")

NAMES = ("xyz", "log_scale", "rotation", "opacity", "sh")


def _table_np(table):
    return {"gaussian_ids": table.gaussian_ids.numpy(), "tile_offsets": table.tile_offsets.numpy()}


@pytest.fixture
def oracle_bindings(monkeypatch):
    from jaxgs_b200 import kernels as K
    from jaxgs_b200.types import ProjectedGaussians, RenderResult, SortedVisibilityTable

    def compact(bounds, camera, config, want_slots=True):
        center, extent, valid = (t.numpy() for t in bounds)
        ids, count, _ = O.cluster_compact(center, extent, valid.astype(np.uint8),
                                          camera.planes.numpy())
        return (torch.as_tensor(ids), torch.tensor([count], dtype=torch.int32)), None

    def project(pool, camera, config, degree, clusters, *, rgb_only=False, active_sh_only=False,
                sh_color_only=False, visible_color_only=False):
        pool_np = {k: getattr(pool, k).detach().numpy() for k in NAMES}
        pool_np["alive"] = pool.alive.numpy().astype(bool)
        ids, count = clusters[0].numpy(), int(clusters[1].item())
        C, sh_dim = config.max_gaussians, int(pool.sh.shape[1])
        p = O.project_fwd(pool_np, camera, degree=degree, sh_dim=sh_dim, clusters=(ids, count),
                          cluster_size=config.cluster_size, visible_color_only=visible_color_only)
        t = torch.as_tensor
        projected = ProjectedGaussians(t(p["mean"]).reshape(C, 2), t(p["depth"]),
                                       t(p["conic"]).reshape(C, 2, 2), t(p["radius"]),
                                       t(p["color"]).reshape(C, 3), t(p["alpha"]), t(p["visible"]))

        def pullback(cot, out=None, compact=True):
            cot_np = {"mean": cot.mean.numpy().reshape(-1), "depth": cot.depth.numpy(),
                      "conic": cot.conic.numpy().reshape(-1), "radius": np.zeros(C, np.float32),
                      "color": cot.color.numpy().reshape(-1), "alpha": cot.alpha.numpy()}
            grads = O.project_bwd(pool_np, camera, p["color"], cot_np, degree=degree,
                                  sh_dim=sh_dim, clusters=(ids, count),
                                  cluster_size=config.cluster_size, compact_gradients=compact,
                                  rgb_only=rgb_only)
            return tuple(torch.as_tensor(g).reshape(getattr(pool, n).shape)
                         for g, n in zip(grads, NAMES))

        return projected, pullback

    def build(projected, camera, config):
        tb = O.bin(np_proj(projected), camera.width, camera.height, config.tile_size,
                   config.raster_tile_height, config.visibility_capacity)
        return SortedVisibilityTable(torch.as_tensor(tb["gaussian_ids"]),
                                     torch.as_tensor(tb["tile_offsets"]),
                                     torch.as_tensor(tb["point_counts"]),
                                     torch.tensor([tb["pair_count"]], dtype=torch.int32),
                                     torch.tensor([int(tb["overflow"])], dtype=torch.int32))

    def raster_fwd(projected, table, camera, config, background=None, want_depth=True,
                   want_alpha=True, splats=None, record=True):
        fwd = O.raster_fwd(np_proj(projected), _table_np(table), camera.width, camera.height,
                           config.tile_size, config.raster_tile_height)
        rgb = torch.as_tensor(fwd["rgb"]).reshape(camera.height, camera.width, 3)
        return RenderResult(rgb, None, None), fwd

    def raster_bwd(projected, table, cache, drgb, camera, config, background=None, ddepth=None,
                   dalpha=None, visible_clusters=None, buffers=None, collect_stats=False):
        C = config.max_gaussians
        cot = O.raster_bwd(np_proj(projected), _table_np(table), cache, drgb.numpy().reshape(-1),
                           camera.width, camera.height, config.tile_size,
                           config.raster_tile_height)
        t = torch.as_tensor
        return projected.replace(mean=t(cot["mean"]).reshape(C, 2),
                                 conic=t(cot["conic"]).reshape(C, 2, 2), depth=t(cot["depth"]),
                                 color=t(cot["color"]).reshape(C, 3), alpha=t(cot["alpha"]),
                                 radius=torch.zeros(C))

    def fused(prediction, target, with_scale, clip_input=False):
        x = prediction.detach().numpy()
        value, grad = O.loss(np.clip(x, 0, 1) if clip_input else x, target.numpy())
        if clip_input:
            grad = grad * O.clip_grad(x)
        return torch.tensor(value, dtype=torch.float32), torch.as_tensor(grad), None

    for name, fake in (("compact_visible_clusters", compact), ("project_with_compact_pullback", project),
                       ("build_sorted_visibility_table_cute", build), ("rasterize_forward", raster_fwd),
                       ("rasterize_backward", raster_bwd), ("_fused_loss", fused)):
        monkeypatch.setattr(K, name, fake)


def _scene(degree):
    from jaxgs_b200.scene import CapacityConfig, world_cluster_bounds
    from jaxgs_b200.types import DeviceCamera, GaussianArrays
    from tests.test_oracle_cpu import _small_pool

    pool_np, cam, target = _small_pool(300, seed=1)
    config = CapacityConfig(300, 128, 1, 16, 3, 300 * 96, tile_height=8)
    pool = GaussianArrays.from_numpy(pool_np, device="cpu")
    for name in NAMES:
        getattr(pool, name).requires_grad_(True)
    center, extent, valid = world_cluster_bounds(pool_np, 128)
    bounds = (torch.as_tensor(center), torch.as_tensor(extent),
              torch.as_tensor(valid.astype(np.uint8)))
    return pool, bounds, DeviceCamera.from_camera(cam, device="cpu"), config, target


@pytest.mark.parametrize("degree", [1, 3])
def test_render_gradients_are_the_derivative_of_its_forward(oracle_bindings, degree):
    from jaxgs_b200.autograd import render

    pool, bounds, camera, config, _ = _scene(degree)
    H, W = camera.height, camera.width
    weights = torch.arange(H * W * 3, dtype=torch.float32).reshape(H, W, 3) / (H * W * 3)
    rgb, overflow = render(pool, bounds, camera, config, degree)
    assert not overflow.requires_grad and int(overflow.item()) == 0
    (rgb * weights).sum().backward()
    for name in NAMES:
        grad = getattr(pool, name).grad
        assert grad is not None and grad.shape == getattr(pool, name).shape, name
    above = pool.sh.grad[:, (degree + 1) ** 2:]
    assert above.numel() == 0 or float(above.abs().max()) == 0
    assert pool.alive.grad is None

    def loss():
        with torch.no_grad():
            return float((render(pool, bounds, camera, config, degree)[0].double()
                          * weights.double()).sum())

    def check(name, index, h):
        param = getattr(pool, name)
        analytic = float(param.grad[index])
        with torch.no_grad():
            saved = param[index].clone()
            param[index] = saved + h
            plus = loss()
            param[index] = saved - h
            minus = loss()
            param[index] = saved
        numeric = (plus - minus) / (2 * h)
        return abs(analytic - numeric) <= 0.003 + 0.04 * abs(numeric)

    top = torch.argsort(-pool.opacity.grad.abs().reshape(-1))[:6].tolist()
    for g in top:
        for name, index in (("log_scale", (g, 1)), ("rotation", (g, 2)), ("opacity", (g, 0)),
                            ("sh", (g, 1, 0))):
            assert check(name, index, 1e-4), (name, index)
    assert np.mean([check("xyz", (g, c), 2e-5) for g in top for c in range(3)]) >= 0.8


def test_fused_loss_scales_its_saved_gradient(oracle_bindings):
    from jaxgs_b200.autograd import fused_loss

    rng = np.random.default_rng(3)
    image = torch.tensor(rng.uniform(-0.1, 1.1, (17, 23, 3)).astype(np.float32), requires_grad=True)
    target = torch.tensor(rng.integers(0, 256, (17, 23, 3), dtype=np.uint8))
    loss = fused_loss(image, target, clip_input=True)
    (3 * loss).backward()
    value, grad = O.loss(np.clip(image.detach().numpy(), 0, 1), target.numpy())
    np.testing.assert_allclose(float(loss.detach()), value, rtol=1e-6)
    np.testing.assert_array_equal(image.grad.numpy(),
                                  (3 * torch.as_tensor(grad * O.clip_grad(image.detach().numpy()))).numpy())
