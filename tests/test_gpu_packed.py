"""The packed rasterizer's entry points (kernels/packed_rasterizer.py:23-216)
on the GPU: packed_forward, packed_backward and packed_loss_and_grad, the
functions the reference's training step calls for 8- and 16-pixel-wide
tiles (training/step.py:74-80).

Checked against the oracle with the packed conventions (image min(rgb, 1)
over no background, the image gradient passed on as given) and against the
float32 entry points they share kernels with: the symmetric conic
convention (conic[0, 1] holds both off-diagonal contributions, conic[1, 0]
stays zero, tests/test_packed.py:79-137) folds the general one exactly,
and the projection pullback gives the same parameter gradients from both.
Bars: images 1e-4 max-abs away from threshold-ambiguous pixels, loss 1e-5
relative, cotangents 1e-3 relative L2.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import np_proj, rel_l2, splats, torch_proj

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _table(table):
    from jaxgs_b200.types import SortedVisibilityTable

    return SortedVisibilityTable(*(torch.as_tensor(table[k], device="cuda") for k in
                                   ("gaussian_ids", "tile_offsets", "point_counts")),
                                 torch.tensor([table["pair_count"]], device="cuda"),
                                 torch.tensor([0], device="cuda"))


def _case(seed, tile_h, tile_w, W=67, H=45, count=300):
    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.types import DeviceCamera

    rng = np.random.default_rng(seed)
    proj = splats(rng, count, W, H, radius=(0.8, 12.0), alpha=(0.05, 0.95))
    proj["visible"][:] = 1
    # Colours above 1 make some pixels exceed 1, where the packed forward clamps.
    proj["color"] = (proj["color"] * 1.6).astype(np.float32)
    table = O.bin(proj, W, H, tile_w, tile_h, count * 64)
    config = CapacityConfig(count, 128, 1, tile_w, 0, len(table["gaussian_ids"]),
                            tile_height=tile_h)
    return proj, table, config, DeviceCamera(None, None, None, None, W, H)


@pytest.mark.parametrize("tile_h,tile_w", [(8, 16), (16, 16), (8, 8), (12, 16)])
def test_packed_forward_is_the_clamped_fp32_forward(tile_h, tile_w):
    from jaxgs_b200 import kernels as K

    proj, table, config, cam = _case(21, tile_h, tile_w)
    projected, t_table = torch_proj(proj), _table(table)
    rgb, cache, stats = K.packed_forward(projected, t_table, cam, config, collect_stats=True)
    plain, _ = K.rasterize_forward(projected, t_table, cam, config, want_depth=False,
                                   want_alpha=False)
    torch.cuda.synchronize()
    assert rgb.shape == (cam.height, cam.width, 3)
    assert (plain.rgb > 1).any(), "the case must exercise the clamp"
    assert torch.equal(rgb, plain.rgb.clamp_max(1.0))
    exp = O.raster_fwd(proj, table, cam.width, cam.height, tile_w, tile_h)
    ok = exp["ambiguous"] == 0
    np.testing.assert_allclose(rgb.cpu().numpy().reshape(-1, 3)[ok],
                               np.minimum(exp["rgb"].reshape(-1, 3)[ok], 1.0), atol=1e-4, rtol=0)
    # Forward fragment statistics (count, weight) equal the backward's.
    bwd = O.raster_bwd(proj, table, exp, np.zeros(cam.width * cam.height * 3, np.float32),
                       cam.width, cam.height, tile_w, tile_h)
    got = stats.cpu().numpy().reshape(-1, 2)
    assert np.mean(got[:, 0] == bwd["stats"][:, 0]) >= 0.99
    assert rel_l2(got[:, 1], bwd["stats"][:, 1]) < 1e-3
    # Without statistics the placeholder has the reference's shape.
    _, _, none = K.packed_forward(projected, t_table, cam, config)
    assert none.shape == (1,)


@pytest.mark.parametrize("tile_h,tile_w", [(8, 16), (16, 16)])
def test_packed_backward_symmetric_conic_folds_the_general_convention(tile_h, tile_w):
    from jaxgs_b200 import kernels as K

    proj, table, config, cam = _case(22, tile_h, tile_w)
    projected, t_table = torch_proj(proj), _table(table)
    rgb, cache, _ = K.packed_forward(projected, t_table, cam, config)
    rng = np.random.default_rng(5)
    grad = torch.as_tensor(rng.normal(0, 1, (cam.height, cam.width, 3)).astype(np.float32),
                           device="cuda")
    general, square = K.packed_backward(projected, t_table, cache, grad, cam, config)
    sym, _ = K.packed_backward(projected, t_table, cache, grad, cam, config,
                               symmetric_conic=True)
    torch.cuda.synchronize()
    assert square.shape == (1,)
    g = general.conic.cpu().numpy().reshape(-1, 4)
    s = sym.conic.cpu().numpy().reshape(-1, 4)
    assert np.all(s[:, 2] == 0)
    assert rel_l2(s[:, 1], g[:, 1] + g[:, 2]) < 1e-6
    for col in (0, 3):
        assert rel_l2(s[:, col], g[:, col]) < 1e-6
    for name in ("mean", "color", "alpha"):
        a = getattr(sym, name).cpu().numpy().reshape(-1)
        b = getattr(general, name).cpu().numpy().reshape(-1)
        assert rel_l2(a, b) < 1e-6, name
    # The general convention against the oracle (image gradient as given).
    fwd = O.raster_fwd(proj, table, cam.width, cam.height, tile_w, tile_h)
    exp = O.raster_bwd(proj, table, fwd, grad.cpu().numpy().reshape(-1), cam.width, cam.height,
                       tile_w, tile_h)
    for name in ("mean", "conic", "color", "alpha"):
        got = getattr(general, name).cpu().numpy().reshape(-1)
        assert rel_l2(got, exp[name]) < 1e-3, (name, rel_l2(got, exp[name]))


def test_packed_loss_and_grad_matches_oracle_and_pullback_is_unchanged():
    """Config 0 through packed_loss_and_grad (symmetric conic, listed
    clusters, as training/step.py:74-79 calls it) against the oracle's packed
    step, and the parameter gradients of both conic conventions."""
    from jaxgs_b200 import kernels as K
    from jaxgs_b200.scene import CapacityConfig, config0_scene, world_cluster_bounds
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    pool_np, cam, target = config0_scene()
    n = pool_np["xyz"].shape[0]
    config = CapacityConfig(n, 128, 16, 16, 3, n * 64, tile_height=8)
    bounds = tuple(torch.as_tensor(a, device="cuda") for a in world_cluster_bounds(pool_np, 128))
    pool = GaussianArrays.from_numpy(pool_np)
    dcam = DeviceCamera.from_camera(cam)
    clusters, _ = K.compact_visible_clusters(bounds, dcam, config, want_slots=False)
    projected, pullback = K.project_with_compact_pullback(
        pool, dcam, config, 3, clusters, rgb_only=True, active_sh_only=True,
        visible_color_only=True)
    table = K.build_sorted_visibility_table_cute(projected, dcam, config)
    tgt = torch.as_tensor(target, device="cuda")
    loss, cot, stats = K.packed_loss_and_grad(projected, table, dcam, config, tgt, True,
                                              symmetric_conic=True, visible_clusters=clusters)
    loss_g, cot_g, _ = K.packed_loss_and_grad(projected, table, dcam, config, tgt, False,
                                              visible_clusters=clusters)
    grads = [g.clone() for g in pullback(cot)]
    grads_g = pullback(cot_g)
    torch.cuda.synchronize()
    assert stats.shape == (n, 4) and float(stats[:, 0].sum()) > 0
    assert float(loss) == float(loss_g)
    ids = clusters[0].cpu().numpy()
    count = int(clusters[1].item())
    exp = O.training_step(pool_np, cam, target, degree=3, sh_dim=16, tile_w=16, tile_h=8,
                          max_pairs=n * 64, clusters=(ids, count), packed=True)
    assert abs(float(loss) - exp["loss"]) <= 1e-5 * abs(exp["loss"]), (float(loss), exp["loss"])
    rows = count * 128
    for name, got, other, ref in zip(("xyz", "log_scale", "rotation", "opacity", "sh"), grads,
                                     grads_g, exp["grads"]):
        g = got.cpu().numpy().reshape(n, -1)[:rows]
        assert rel_l2(g, other.cpu().numpy().reshape(n, -1)[:rows]) < 1e-6, name
        err = rel_l2(g, ref.reshape(n, -1)[:rows])
        assert err < 1e-3, (name, err)
    # The step's fragment statistics come out of the same calls.
    np.testing.assert_allclose(stats[:, 2].cpu().numpy(), cot.alpha.cpu().numpy())
