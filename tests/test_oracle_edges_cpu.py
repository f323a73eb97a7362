"""The oracle against the reference's own edge, bounds, cutoff,
rectangular-tile, infinite-depth and visible-colour cases (CPU):
tests/test_edge_support.py:15-93, tests/test_pipeline.py:136-228 and
tests/test_projection_visibility.py."""

import numpy as np
import pytest

from jaxgs_b200.scene import Camera, CapacityConfig, create_gaussians, seed_gaussians
from oracle import oracle as O


def _edge_scene(edge="left", anisotropic=False):
    """tests/test_edge_support.py:15-40: one Gaussian whose centre lies 24.1
    pixels beyond an image edge, with a screen-space sigma of 8 pixels (so
    its 3-sigma radius stops short of the edge while its 1/255 level does
    not)."""
    vertical = edge in ("top", "bottom")
    width, height = (128, 256) if vertical else (256, 128)
    camera = Camera.from_colmap([1, 0, 0, 0], [0, 0, 0], 128, 128, width / 2, height / 2,
                                width, height)
    config = CapacityConfig(128, 128, 1, 16, 0, 512)
    axis = 1 if vertical else 0
    mean = np.array([width / 2 + 0.5, height / 2 + 0.5])
    mean[axis] = -24.1 if edge in ("left", "top") else 256 + 24.1
    pixel = mean.astype(int)
    pixel[axis] = 0 if edge in ("left", "top") else 255
    scale = np.sqrt(np.array([64.0, 36.0 if anisotropic else 64.0]) - 0.3) / 64
    pool = seed_gaussians(create_gaussians(config),
                          np.array([[(mean[0] - width / 2) / 64, (mean[1] - height / 2) / 64, 2.0]]),
                          np.array([[0.3, 0.5, 0.7]]),
                          scale=np.array([[scale[0], scale[1], 1e-6]]), opacity=0.99)
    angle = (np.pi / 2 if vertical else 0) + (0.2 if anisotropic else 0)
    pool["rotation"][0] = [np.cos(angle / 2), 0, 0, np.sin(angle / 2)]
    return camera, pool, tuple(int(v) for v in pixel)


@pytest.mark.parametrize("edge", ["left", "right", "top", "bottom"])
@pytest.mark.parametrize("anisotropic", [False, True])
def test_oracle_preserves_edge_support(edge, anisotropic):
    """tests/test_edge_support.py:48-65: the splat stays visible, the exact
    1/255 ellipse bins it into the edge tile, and the edge pixel receives
    alpha exp(-d^T C d / 2) times its colour."""
    camera, pool, pixel = _edge_scene(edge, anisotropic)
    W, H = camera.width, camera.height
    proj = O.project_fwd(pool, camera, degree=0, sh_dim=1)
    axis = 1 if edge in ("top", "bottom") else 0
    boundary = 0 if edge in ("left", "top") else 256
    mean = proj["mean"][:2]
    assert abs(float(mean[axis]) - boundary) > float(proj["radius"][0])
    delta = np.array(pixel, np.float64) + 0.5 - mean
    conic = proj["conic"][:4].reshape(2, 2).astype(np.float64)
    expected = proj["alpha"][0] * np.exp(-0.5 * delta @ conic @ delta) * proj["color"][:3]
    assert expected[0] / proj["color"][0] > 1 / 256
    assert proj["visible"][0]
    table = O.bin(proj, W, H, 16, 16, 512)
    assert not table["overflow"]
    image = O.raster_fwd(proj, table, W, H, 16, 16)["rgb"].reshape(H, W, 3)
    np.testing.assert_allclose(image[pixel[1], pixel[0]], expected, rtol=1e-5, atol=1e-7)


def test_oracle_projection_uses_the_coarse_screen_bounds():
    """tests/test_edge_support.py:68-93: a mean within 15% of the screen
    beyond either edge is visible (-38.3, 294.3 on a 256-wide image), just
    past it is not (-38.5, 294.5); so are not an alpha below 1/255, a depth
    before the near plane or beyond the far one."""
    camera, pool, _ = _edge_scene()
    means = np.array([[-38.3, 64], [-38.5, 64], [294.3, 64], [294.5, 64], [128, 64], [128, 64],
                      [128, 64]])
    depths = np.array([2, 2, 2, 2, 2, 0.1, 1001])
    xyz = np.c_[(means - [128, 64]) / 64, depths]
    config = CapacityConfig(128, 128, 1, 16, 0, 512)
    pool = seed_gaussians(create_gaussians(config), xyz, np.full((7, 3), 0.5), scale=2)
    pool["opacity"][4, 0] = np.log(0.001 / 0.999)
    proj = O.project_fwd(pool, camera, degree=0, sh_dim=1)
    np.testing.assert_array_equal(proj["visible"][:7].astype(bool),
                                  [True, False, True, False, False, False, False])


def test_oracle_alpha_cutoff_and_cap():
    """tests/test_pipeline.py:200-228: one splat on a 1x1 image composites
    nothing below alpha 1/256, its own alpha in between, and 255/256 at most,
    in both the colour and the accumulated alpha."""
    for alpha, expected in ((0.001, 0.0), (0.1, 0.1), (1.0, 255.0 / 256)):
        proj = {"mean": np.array([0.5, 0.5], np.float32), "depth": np.array([1.0], np.float32),
                "conic": np.array([1, 0, 0, 1], np.float32),
                "radius": np.array([1.0], np.float32),
                "color": np.array([1.0, 0.0, 0.0], np.float32),
                "alpha": np.array([alpha], np.float32), "visible": np.array([1], np.int8)}
        table = {"gaussian_ids": np.array([0], np.int32), "tile_offsets": np.array([0, 1], np.int32)}
        out = O.raster_fwd(proj, table, 1, 1, 16, 16)
        np.testing.assert_allclose(out["rgb"][0], expected, atol=1e-6)
        np.testing.assert_allclose(out["alpha"][0], expected, atol=1e-6)


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
@pytest.mark.parametrize("empty", [False, True])
def test_oracle_visible_color_only_preserves_render_and_pullback(degree, empty):
    """tests/test_projection_visibility.py: zeroing the colour of culled
    points in listed clusters (visible_color_only) changes no rendered
    pixel and no parameter gradient; the colour clamp (and its zero
    derivative) is kept for visible points."""
    capacity, cluster_size = 131, 65
    config = CapacityConfig(capacity, cluster_size, 16, 16, 3, 4096, tile_height=8)
    camera = Camera.from_colmap([1, 0, 0, 0], [0, 0, 0], 20, 20, 9, 8, 19, 17, far=5.0)
    rng = np.random.default_rng(912)
    xyz = rng.uniform([-0.3, -0.2, 2.0], [0.3, 0.2, 3.0], (capacity, 3)).astype(np.float32)
    # A listed cluster holds points that every projection predicate rejects.
    xyz[1:6] = [[8, 0, 2], [0, -8, 2], [0, 0, -2], [0, 0, 0.1], [0, 0, 6]]
    pool = seed_gaussians(create_gaussians(config), xyz, np.full((capacity, 3), 0.4), scale=0.12)
    slots = np.arange(capacity) // cluster_size != 1
    if empty:
        slots[:] = False
    pool["alive"] = slots.copy()
    pool["alive"][7] = False
    pool["opacity"][6] = -20
    pool["sh"] = rng.normal(0, 0.2, pool["sh"].shape).astype(np.float32)
    pool["sh"][8, 0, 0] = -4
    listed = np.unique(np.nonzero(slots)[0] // cluster_size).astype(np.int32)
    clusters = (np.pad(listed, (0, 3 - len(listed))), len(listed))

    def project(visible_color_only):
        return O.project_fwd(pool, camera, degree=degree, sh_dim=16, clusters=clusters,
                             cluster_size=cluster_size, visible_color_only=visible_color_only)

    expected, actual = project(False), project(True)
    np.testing.assert_array_equal(actual["visible"], expected["visible"])
    visible = expected["visible"].astype(bool)
    for name, width in (("mean", 2), ("depth", 1), ("conic", 4), ("radius", 1), ("alpha", 1)):
        np.testing.assert_array_equal(actual[name].reshape(capacity, width)[slots],
                                      expected[name].reshape(capacity, width)[slots])
    color_a, color_e = actual["color"].reshape(-1, 3), expected["color"].reshape(-1, 3)
    np.testing.assert_array_equal(color_a[visible], color_e[visible])
    np.testing.assert_array_equal(color_a[slots & ~visible], 0)
    if not empty:
        assert visible[0] and visible[-1] and not visible[1:8].any()
        assert np.any(color_e[slots & ~visible] > 0)
        assert color_a[8, 0] == 0

    W, H = camera.width, camera.height
    table = O.bin(expected, W, H, 16, 8, 4096)
    image_grad = rng.normal(0, 0.01, (H, W, 3)).astype(np.float32).reshape(-1)
    fwd_a = O.raster_fwd(actual, table, W, H, 16, 8)
    fwd_e = O.raster_fwd(expected, table, W, H, 16, 8)
    np.testing.assert_array_equal(fwd_a["rgb"], fwd_e["rgb"])
    np.testing.assert_array_equal(fwd_a["last"], fwd_e["last"])
    cot = O.raster_bwd(actual, table, fwd_a, image_grad, W, H, 16, 8)
    cot["radius"] = np.zeros(capacity, np.float32)
    grads = [O.project_bwd(pool, camera, p["color"], cot, degree=degree, sh_dim=16,
                           sh_gradient_dim=(degree + 1) ** 2, clusters=clusters,
                           cluster_size=cluster_size, compact_gradients=True, rgb_only=True)
             for p in (actual, expected)]
    rows = int(slots.sum())
    for got, ref, width in zip(grads[0], grads[1], (3, 3, 4, 1, (degree + 1) ** 2 * 3)):
        np.testing.assert_array_equal(got.reshape(capacity, width)[:rows],
                                      ref.reshape(capacity, width)[:rows])


def _splats(mean, depth, conic, radius, color, alpha, visible):
    return {"mean": np.asarray(mean, np.float32).reshape(-1),
            "depth": np.asarray(depth, np.float32),
            "conic": np.asarray(conic, np.float32).reshape(-1),
            "radius": np.asarray(radius, np.float32),
            "color": np.asarray(color, np.float32).reshape(-1),
            "alpha": np.asarray(alpha, np.float32),
            "visible": np.asarray(visible, np.int8)}


@pytest.mark.parametrize("tile_height", [8, 12])
def test_oracle_rectangular_tiles_keep_rows_apart(tile_height):
    """tests/test_pipeline.py:136-167: two splats in separate tile rows of
    16 x tile_height tiles are binned into their own tiles only, each pixel
    under a splat shows only that splat, and the pixel's gradient reaches
    only its own splat's opacity."""
    W, H = 17, 2 * tile_height + 1
    proj = _splats([[8.0, 4.0], [8.0, tile_height + 4.0]], [1.0, 2.0],
                   np.broadcast_to(np.eye(2) * 2, (2, 2, 2)), [3 / np.sqrt(2)] * 2,
                   [[1.0, 0.0, 0.0], [0.0, 1.0, 0.0]], [0.5, 0.5], [1, 1])
    table = O.bin(proj, W, H, 16, tile_height, 8)
    np.testing.assert_array_equal(np.diff(table["tile_offsets"]), [1, 0, 1, 0, 0, 0])
    assert not table["overflow"]
    fwd = O.raster_fwd(proj, table, W, H, 16, tile_height)
    image = fwd["rgb"].reshape(H, W, 3)
    expected = 0.5 * np.exp(-0.5)
    np.testing.assert_allclose(image[4, 8], [expected, 0, 0], atol=1e-7)
    np.testing.assert_allclose(image[tile_height + 4, 8], [0, expected, 0], atol=1e-7)
    np.testing.assert_array_equal(image[-1, -1], 0)
    drgb = np.zeros((H, W, 3), np.float32)
    drgb[tile_height + 4, 8, 1] = 1
    cot = O.raster_bwd(proj, table, fwd, drgb.reshape(-1), W, H, 16, tile_height)
    np.testing.assert_allclose(cot["alpha"], [0, np.exp(-0.5)], atol=1e-7)


@pytest.mark.parametrize("has_visible", [False, True])
def test_oracle_culled_slots_keep_infinite_depth_out_of_the_gradients(has_visible):
    """tests/test_pipeline.py:170-197: culled slots carry depth = inf; the
    rendered depth (sum of w d) and its gradients stay finite, with
    d depth / d alpha = d and d depth / d d = w for the visible splat."""
    proj = _splats(np.full((2, 2), 0.5), [2.0 if has_visible else np.inf, np.inf],
                   np.broadcast_to(np.eye(2), (2, 2, 2)), [3.0, 3.0], np.full((2, 3), 0.4),
                   [0.5, 0.0], [has_visible, False])
    table = O.bin(proj, 1, 1, 16, 16, 4)
    fwd = O.raster_fwd(proj, table, 1, 1, 16, 16)
    np.testing.assert_allclose(fwd["depth"].sum(), 1.0 if has_visible else 0.0)
    np.testing.assert_allclose(fwd["rgb"], 0.2 if has_visible else 0.0, rtol=1e-6)
    np.testing.assert_allclose(fwd["alpha"], 0.5 if has_visible else 0.0)
    cot = O.raster_bwd(proj, table, fwd, np.zeros(3, np.float32), 1, 1, 16, 16,
                       ddepth=np.ones(1, np.float32))
    for name in ("mean", "depth", "conic", "color", "alpha"):
        assert np.isfinite(cot[name]).all(), name
    np.testing.assert_allclose(cot["alpha"], [2.0 if has_visible else 0.0, 0.0])
    np.testing.assert_allclose(cot["depth"], [0.5 if has_visible else 0.0, 0.0])
