"""CUDA path vs the CPU oracle on the same seeded inputs (through the C ABI).

Bars: bit-exact binning (counts, sorted pairs,
ranges, pair count, overflow); fp32 images within 1e-4 max-abs away from
threshold-ambiguous pixels; loss within 1e-5 relative; gradients within
1e-3 relative L2.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import known_answer_three, np_proj, rel_l2, splats, torch_proj

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _kernels():
    from jaxgs_b200 import kernels as K

    return K


def _dev_camera(cam):
    from jaxgs_b200.types import DeviceCamera

    return DeviceCamera.from_camera(cam)


def _pool(pool):
    from jaxgs_b200.types import GaussianArrays

    return GaussianArrays.from_numpy(pool)


# ---------------------------------------------------------------------------
# Projection
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("degree", [0, 1, 3])
@pytest.mark.parametrize("compacted", [False, True])
def test_projection_matches_oracle(degree, compacted):
    from jaxgs_b200.scene import config0_scene

    K = _kernels()
    pool, cam, _ = config0_scene()
    pool["alive"][::7] = False
    from jaxgs_b200.scene import CapacityConfig

    config = CapacityConfig(4096, 128, 16, 16, 3, tile_height=8)
    clusters = None
    if compacted:
        ids = np.array([0, 3, 5, 6, 31], np.int32)
        clusters = (torch.as_tensor(ids, device="cuda"), torch.tensor([len(ids)], dtype=torch.int32, device="cuda"))
    got = K.project_cute(_pool(pool), _dev_camera(cam), config, degree, clusters)
    torch.cuda.synchronize()
    exp = O.project_fwd(pool, cam, degree=degree, sh_dim=16,
                        clusters=None if clusters is None else (ids, len(ids)))
    g = np_proj(got)
    slots = np.arange(4096) if clusters is None else (ids[:, None] * 128 + np.arange(128)).reshape(-1)
    for name in ("mean", "depth", "conic", "radius", "color", "alpha"):
        width = len(exp[name]) // 4096
        a = g[name].reshape(4096, width)[slots]
        b = exp[name].reshape(4096, width)[slots]
        np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-5, err_msg=name)
    np.testing.assert_array_equal(g["visible"], exp["visible"])


@pytest.mark.parametrize("sh_mode", ["full", "active", "color"])
@pytest.mark.parametrize("rgb_only", [False, True])
def test_projection_pullback_matches_oracle(sh_mode, rgb_only):
    from jaxgs_b200.scene import CapacityConfig, config0_scene
    from jaxgs_b200.types import ProjectedGaussians

    K = _kernels()
    pool, cam, _ = config0_scene()
    degree = 2
    config = CapacityConfig(4096, 128, 16, 16, 3, tile_height=8)
    ids = np.array([1, 2, 7, 30], np.int32)
    clusters = (torch.as_tensor(ids, device="cuda"), torch.tensor([4], dtype=torch.int32, device="cuda"))
    projected, pullback = K.project_with_compact_pullback(
        _pool(pool), _dev_camera(cam), config, degree, clusters, rgb_only=rgb_only,
        active_sh_only=sh_mode == "active", sh_color_only=sh_mode == "color")
    rng = np.random.default_rng(5)
    cot = {k: rng.normal(0, 1, n).astype(np.float32) for k, n in
           (("mean", 4096 * 2), ("depth", 4096), ("conic", 4096 * 4), ("radius", 4096),
            ("color", 4096 * 3), ("alpha", 4096))}
    cot["alpha"][::5] = 0  # rows without any cotangent
    for k in ("mean", "conic", "color", "depth", "radius"):
        cot[k].reshape(4096, -1)[::5] = 0
    t = lambda a, s: torch.as_tensor(a, device="cuda").reshape(s)
    cot_t = ProjectedGaussians(t(cot["mean"], (4096, 2)), t(cot["depth"], (4096,)),
                               t(cot["conic"], (4096, 2, 2)), t(cot["radius"], (4096,)),
                               t(cot["color"], (4096, 3)), t(cot["alpha"], (4096,)), projected.visible)
    grads = [g.cpu().numpy().reshape(4096, -1) for g in pullback(cot_t)]
    color = projected.color.cpu().numpy().reshape(-1)
    shg = {"full": 16, "active": 9, "color": 1}[sh_mode]
    exp = O.project_bwd(pool, cam, color, cot, degree=degree, sh_dim=16, sh_gradient_dim=shg,
                        clusters=(ids, 4), compact_gradients=True, rgb_only=rgb_only,
                        sh_color_only=sh_mode == "color")
    n = 4 * 128
    for name, a, b in zip(("xyz", "log_scale", "rotation", "opacity", "sh"), grads, exp):
        b = b.reshape(4096, -1)
        np.testing.assert_allclose(a[:n], b[:n], rtol=2e-4, atol=2e-5, err_msg=name)


# ---------------------------------------------------------------------------
# Binning (bit-exact)
# ---------------------------------------------------------------------------
def _bin_both(proj, width, height, tw, th, max_pairs):
    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.types import DeviceCamera

    K = _kernels()
    c = len(proj["alpha"])
    config = CapacityConfig(c, 128, 1, tw, 0, max_pairs, tile_height=th)
    cam = DeviceCamera(None, None, None, None, width, height)
    table = K.build_sorted_visibility_table_cute(torch_proj(proj), cam, config)
    torch.cuda.synchronize()
    exp = O.bin(proj, width, height, tw, th, max_pairs)
    return table, exp


def _assert_tables_equal(table, exp):
    pc = int(table.pair_count.item())
    assert pc == exp["pair_count"]
    assert bool(table.overflow.item()) == exp["overflow"]
    np.testing.assert_array_equal(table.point_counts.cpu().numpy(), exp["point_counts"])
    np.testing.assert_array_equal(table.tile_offsets.cpu().numpy(), exp["tile_offsets"])
    used = min(pc, len(exp["gaussian_ids"]))
    np.testing.assert_array_equal(table.gaussian_ids.cpu().numpy()[:used], exp["gaussian_ids"][:used])


def test_binning_known_answer_three_gaussians():
    """tests/test_cute.py:141-159: diff(offsets) == [3,3,3,3], ids [1,2,0]."""
    config, cam, pool = known_answer_three()
    proj = O.project_fwd(pool, cam, degree=0, sh_dim=1)
    table, exp = _bin_both(proj, 8, 8, 4, 4, 16)
    _assert_tables_equal(table, exp)
    np.testing.assert_array_equal(np.diff(table.tile_offsets.cpu().numpy()), [3, 3, 3, 3])
    np.testing.assert_array_equal(table.gaussian_ids.cpu().numpy()[:12].reshape(4, 3),
                                  np.tile([1, 2, 0], (4, 1)))
    table, exp = _bin_both(proj, 8, 8, 4, 4, 4)  # narrow arena overflows
    assert bool(table.overflow.item()) and exp["overflow"]
    _assert_tables_equal(table, exp)


def test_binning_large_ellipse_and_empty_scene():
    """tests/test_cute.py:189-213: pair_count 4 with conic 1e-5 on 17x19."""
    from jaxgs_b200.scene import Camera, CapacityConfig, create_gaussians, seed_gaussians

    cam = Camera.from_colmap([1, 0, 0, 0], [0, 0, 0], 20, 20, 8, 9, 17, 19)
    pool = seed_gaussians(create_gaussians(CapacityConfig(1, 1, 1, 16, 0, 4)),
                          np.array([[0, 0, 2.0]]), np.ones((1, 3)) * 0.5, scale=0.2, opacity=0.5)
    proj = O.project_fwd(pool, cam, degree=0, sh_dim=1)
    proj["conic"] = np.array([1e-5, 0, 0, 1e-5], np.float32)
    table, exp = _bin_both(proj, 17, 19, 16, 16, 4)
    assert int(table.pair_count.item()) == 4
    _assert_tables_equal(table, exp)
    proj["visible"][:] = 0
    table, exp = _bin_both(proj, 17, 19, 16, 16, 4)
    assert int(table.pair_count.item()) == 0
    np.testing.assert_array_equal(table.tile_offsets.cpu().numpy(), 0)
    _assert_tables_equal(table, exp)


@pytest.mark.parametrize("tiles_x", [255, 256])
def test_binning_tile_key_width(tiles_x):
    """tests/test_cute.py:110-138: a point in the last tile of a 255/256-wide grid."""
    from jaxgs_b200.scene import Camera, CapacityConfig, create_gaussians, seed_gaussians

    width, height = tiles_x * 8, 256 * 8
    cam = Camera.from_colmap([1, 0, 0, 0], [0, 0, 0], 20, 20, width - 4, height - 4, width, height)
    pool = seed_gaussians(create_gaussians(CapacityConfig(1, 1, 1, 8, 0, 4)),
                          np.array([[0.0, 0.0, 2.0]]), np.full((1, 3), 0.5), scale=0.02, opacity=0.5)
    proj = O.project_fwd(pool, cam, degree=0, sh_dim=1)
    table, exp = _bin_both(proj, width, height, 8, 8, 4)
    assert int(table.pair_count.item()) == 1
    offsets = table.tile_offsets.cpu().numpy()
    np.testing.assert_array_equal(offsets[:-1], 0)
    assert offsets[-1] == 1
    _assert_tables_equal(table, exp)


@pytest.mark.parametrize("tile_h,tile_w", [(8, 16), (16, 16), (8, 8)])
@pytest.mark.parametrize("seed", [3, 4])
def test_binning_random_ellipses_bit_exact(tile_h, tile_w, seed):
    """Small, huge, thin and degenerate ellipses with depth ties (exercises
    per-lane emission (<= 32 pairs), whole-warp emission (more) and > 32-row
    Gaussians)."""
    rng = np.random.default_rng(seed)
    proj = splats(rng, 2048, 640, 360, radius=(0.4, 60.0), huge=8)
    table, exp = _bin_both(proj, 640, 360, tile_w, tile_h, 1 << 19)
    counts = exp["point_counts"]
    assert np.any((counts > 16) & (counts <= 32)) and np.any(counts > 32)
    _assert_tables_equal(table, exp)


def test_binning_overflow_truncates_like_reference():
    rng = np.random.default_rng(9)
    proj = splats(rng, 1024, 320, 200, radius=(2.0, 30.0))
    full = O.bin(proj, 320, 200, 16, 8, 1 << 18)
    cap = full["pair_count"] // 3
    table, exp = _bin_both(proj, 320, 200, 16, 8, cap)
    assert exp["overflow"] and bool(table.overflow.item())
    _assert_tables_equal(table, exp)


@pytest.mark.parametrize("arena_scale", [1.0, 0.5])
def test_binning_poisoned_outputs_are_written_exactly(arena_scale):
    """Poisoned output buffers (the reference pads its arena with
    fill_padding, sorted_visibility.py:757-766): every counts, offsets and
    arena slot below min(pair_count, arena) is written and equals the
    oracle; no arena slot past it is touched, with and without overflow."""
    from jaxgs_b200 import _lib as L

    K = _kernels()
    rng = np.random.default_rng(21)
    width, height = 320, 200
    proj = splats(rng, 1500, width, height, radius=(0.5, 40.0), huge=4)
    full = O.bin(proj, width, height, 16, 8, 1 << 20)["pair_count"]
    max_pairs = int(full * arena_scale) + 37
    exp = O.bin(proj, width, height, 16, 8, max_pairs)
    assert exp["overflow"] == (arena_scale < 1)
    c = len(proj["alpha"])
    tiles = (-(-width // 16)) * (-(-height // 8))
    poison = -0x5A5A5A5B
    projected = torch_proj(proj)
    counts = torch.full((c,), poison, dtype=torch.int32, device="cuda")
    ids = torch.full((max_pairs,), poison, dtype=torch.int32, device="cuda")
    offsets = torch.full((tiles + 1,), poison, dtype=torch.int32, device="cuda")
    pair_count = torch.full((1,), poison, dtype=torch.int32, device="cuda")
    overflow = torch.full((1,), poison, dtype=torch.int32, device="cuda")
    p = L.BinParams(c, width, height, 16, 8, max_pairs)
    ws = K._workspace(L.lib.gsb_bin_workspace_size(L.ref(p)), "cuda")
    L.check(L.lib.gsb_bin(K._stream(), L.ref(p), K._ptr(ws), ws.numel(),
                          *(K._ptr(t) for t in (projected.mean, projected.conic, projected.alpha,
                                                projected.depth, projected.visible, counts, ids,
                                                offsets, pair_count, overflow))), "binning")
    torch.cuda.synchronize()
    assert int(pair_count.item()) == exp["pair_count"]
    assert bool(overflow.item()) == exp["overflow"]
    np.testing.assert_array_equal(counts.cpu().numpy(), exp["point_counts"])
    np.testing.assert_array_equal(offsets.cpu().numpy(), exp["tile_offsets"])
    used = min(exp["pair_count"], max_pairs)
    got = ids.cpu().numpy()
    np.testing.assert_array_equal(got[:used], exp["gaussian_ids"][:used])
    assert (got[used:] == poison).all()
    assert arena_scale < 1 or used < max_pairs


def test_binning_config1_scene_bit_exact():
    """Full-size BASELINE config 1 (1M Gaussians, 1237x822, 8x16 tiles):
    GPU projection feeds both binnings."""
    from jaxgs_b200.scene import CapacityConfig, config1_camera, config1_scene

    K = _kernels()
    pool = config1_scene()
    cam = config1_camera()
    config = CapacityConfig(1_000_000, 128, 16, 16, 3, 8_000_000, tile_height=8)
    projected = K.project_cute(_pool(pool), _dev_camera(cam), config)
    table = K.build_sorted_visibility_table_cute(projected, _dev_camera(cam), config)
    torch.cuda.synchronize()
    exp = O.bin(np_proj(projected), 1237, 822, 16, 8, 8_000_000)
    _assert_tables_equal(table, exp)


# ---------------------------------------------------------------------------
# fp32 rasterization
# ---------------------------------------------------------------------------
def _raster_case(seed, width=64, height=40, count=300, tw=16, th=8, alpha=(0.05, 0.95)):
    rng = np.random.default_rng(seed)
    proj = splats(rng, count, width, height, radius=(0.8, 12.0), alpha=alpha)
    proj["visible"][:] = 1
    table = O.bin(proj, width, height, tw, th, count * 64)
    return proj, table


@pytest.mark.parametrize("tile_h,tile_w", [(8, 16), (16, 16), (8, 8), (12, 16)])
def test_raster_forward_matches_oracle(tile_h, tile_w):
    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.types import DeviceCamera, SortedVisibilityTable

    K = _kernels()
    W, H = 67, 45
    proj, table = _raster_case(11, W, H, tw=tile_w, th=tile_h)
    c = len(proj["alpha"])
    config = CapacityConfig(c, 128, 1, tile_w, 0, len(table["gaussian_ids"]), tile_height=tile_h)
    bg = np.array([0.1, 0.2, 0.3], np.float32)
    t_table = SortedVisibilityTable(*(torch.as_tensor(table[k], device="cuda") for k in
                                      ("gaussian_ids", "tile_offsets", "point_counts")),
                                    torch.tensor([table["pair_count"]], device="cuda"),
                                    torch.tensor([0], device="cuda"))
    cam = DeviceCamera(None, None, None, None, W, H)
    result, cache = K.rasterize_forward(torch_proj(proj), t_table, cam, config,
                                        torch.as_tensor(bg, device="cuda"))
    torch.cuda.synchronize()
    exp = O.raster_fwd(proj, table, W, H, tile_w, tile_h, bg)
    ok = exp["ambiguous"] == 0
    assert ok.mean() > 0.95
    rgb = result.rgb.cpu().numpy().reshape(-1, 3)
    np.testing.assert_allclose(rgb[ok], exp["rgb"].reshape(-1, 3)[ok], atol=1e-4, rtol=0)
    np.testing.assert_allclose(result.alpha.cpu().numpy().reshape(-1)[ok], exp["alpha"][ok], atol=1e-4)
    np.testing.assert_allclose(result.depth.cpu().numpy().reshape(-1)[ok], exp["depth"][ok], rtol=1e-4, atol=1e-3)
    np.testing.assert_array_equal(cache.last.cpu().numpy()[ok], exp["last"][ok])


def test_raster_forward_saturation_and_empty_tiles():
    """Opaque splats saturate pixels mid-list (T < 1/8192 early stop) and some
    tiles are empty (tests/test_cute.py:216-282 and test_packed.py:241-272)."""
    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.types import DeviceCamera, SortedVisibilityTable

    K = _kernels()
    W, H = 48, 24
    count = 60
    rng = np.random.default_rng(2)
    proj = {
        "mean": rng.uniform(4, 20, (count, 2)).astype(np.float32).reshape(-1),
        "depth": np.linspace(1, 4, count).astype(np.float32),
        "conic": np.tile(np.array([0.014, 0.003, 0.003, 0.025], np.float32), count),
        "radius": np.full(count, 30.0, np.float32),
        "color": rng.uniform(0, 1, count * 3).astype(np.float32),
        "alpha": np.linspace(0.72, 0.97, count).astype(np.float32),
        "visible": np.ones(count, np.int8),
    }
    table = O.bin(proj, W, H, 16, 8, count * 18)
    config = CapacityConfig(count, 128, 1, 16, 0, count * 18, tile_height=8)
    t_table = SortedVisibilityTable(*(torch.as_tensor(table[k], device="cuda") for k in
                                      ("gaussian_ids", "tile_offsets", "point_counts")),
                                    torch.tensor([table["pair_count"]], device="cuda"),
                                    torch.tensor([0], device="cuda"))
    cam = DeviceCamera(None, None, None, None, W, H)
    result, cache = K.rasterize_forward(torch_proj(proj), t_table, cam, config)
    torch.cuda.synchronize()
    exp = O.raster_fwd(proj, table, W, H, 16, 8)
    ok = exp["ambiguous"] == 0
    assert (exp["final_t"] < 1 / 8192).any()
    np.testing.assert_allclose(result.rgb.cpu().numpy().reshape(-1, 3)[ok],
                               exp["rgb"].reshape(-1, 3)[ok], atol=1e-4)
    np.testing.assert_array_equal(cache.last.cpu().numpy()[ok], exp["last"][ok])
    # backward_work[t] = max over the tile's pixels of (last - tile start)
    # (tests/test_work_balance.py:240-246).
    work = cache.backward_work.cpu().numpy()
    last = cache.last.cpu().numpy()
    offs = table["tile_offsets"]
    ys, xs = np.mgrid[0:H, 0:W]
    tile = ((ys // 8) * 3 + xs // 16).reshape(-1)
    expected = np.zeros(len(offs) - 1, np.int64)
    np.maximum.at(expected, tile, last - offs[tile])
    np.testing.assert_array_equal(work, expected)


@pytest.mark.parametrize("tile_h,tile_w", [(8, 16), (16, 16)])
def test_raster_backward_matches_oracle(tile_h, tile_w):
    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.types import DeviceCamera, SortedVisibilityTable

    K = _kernels()
    W, H = 67, 45
    proj, table = _raster_case(12, W, H, tw=tile_w, th=tile_h)
    c = len(proj["alpha"])
    config = CapacityConfig(c, 128, 1, tile_w, 0, len(table["gaussian_ids"]), tile_height=tile_h)
    bg = np.array([0.1, 0.2, 0.3], np.float32)
    t_table = SortedVisibilityTable(*(torch.as_tensor(table[k], device="cuda") for k in
                                      ("gaussian_ids", "tile_offsets", "point_counts")),
                                    torch.tensor([table["pair_count"]], device="cuda"),
                                    torch.tensor([0], device="cuda"))
    cam = DeviceCamera(None, None, None, None, W, H)
    bg_t = torch.as_tensor(bg, device="cuda")
    projected = torch_proj(proj)
    result, cache = K.rasterize_forward(projected, t_table, cam, config, bg_t)
    rng = np.random.default_rng(3)
    drgb = rng.normal(0, 1, (H, W, 3)).astype(np.float32)
    ddepth = rng.normal(0, 0.1, (H, W)).astype(np.float32)
    dalpha = rng.normal(0, 0.5, (H, W)).astype(np.float32)
    cot = K.rasterize_backward(projected, t_table, cache, torch.as_tensor(drgb, device="cuda"), cam,
                               config, bg_t, torch.as_tensor(ddepth, device="cuda"),
                               torch.as_tensor(dalpha, device="cuda"))
    torch.cuda.synchronize()
    fwd = O.raster_fwd(proj, table, W, H, tile_w, tile_h, bg)
    exp = O.raster_bwd(proj, table, fwd, drgb.reshape(-1), W, H, tile_w, tile_h, bg,
                       ddepth.reshape(-1), dalpha.reshape(-1))
    for name in ("mean", "conic", "depth", "color", "alpha"):
        got = getattr(cot, name).cpu().numpy().reshape(-1)
        assert rel_l2(got, exp[name]) < 1e-3, (name, rel_l2(got, exp[name]))


def _assert_stats_close(got, exp):
    """[C, 4] fragment statistics: counts equal for all but threshold-borderline
    Gaussians, every column within 1e-3 relative L2."""
    assert got.shape == exp.shape
    assert np.isfinite(got).all()
    assert exp[:, 0].sum() > 0
    assert np.mean(got[:, 0] == exp[:, 0]) >= 0.99
    for col in range(4):
        assert rel_l2(got[:, col], exp[:, col]) < 1e-3, (col, rel_l2(got[:, col], exp[:, col]))


@pytest.mark.parametrize("tile_h,tile_w,split", [(8, 16, False), (12, 16, True), (16, 16, True)])
def test_fragment_statistics_match_oracle(tile_h, tile_w, split):
    """collect_stats (sorted_rasterize.py:155-203): per Gaussian the composited
    fragment count, the compositing weight sum and the squared opacity
    cotangent sum, stacked with the alpha cotangent as
    sorted_rasterizer.py:227-235 does.  split: the preparation runs on its
    own over NaN-filled buffers with a cluster list, so the statistics and
    the alpha cotangent must be zeroed over the whole pool."""
    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.types import DeviceCamera, SortedVisibilityTable

    K = _kernels()
    W, H = 67, 45
    proj, table = _raster_case(31, W, H, tw=tile_w, th=tile_h)
    c = len(proj["alpha"])
    config = CapacityConfig(c, 128, 1, tile_w, 0, len(table["gaussian_ids"]), tile_height=tile_h)
    t_table = SortedVisibilityTable(*(torch.as_tensor(table[k], device="cuda") for k in
                                      ("gaussian_ids", "tile_offsets", "point_counts")),
                                    torch.tensor([table["pair_count"]], device="cuda"),
                                    torch.tensor([0], device="cuda"))
    cam = DeviceCamera(None, None, None, None, W, H)
    projected = torch_proj(proj)
    rng = np.random.default_rng(8)
    drgb = rng.normal(0, 1, (H, W, 3)).astype(np.float32)
    ddepth = None if split else rng.normal(0, 0.1, (H, W)).astype(np.float32)
    result, cache = K.rasterize_forward(projected, t_table, cam, config)
    drgb_t = torch.as_tensor(drgb, device="cuda")
    if split:
        ids = torch.arange(-(-c // 128), dtype=torch.int32, device="cuda")
        clusters = (ids, torch.tensor([ids.numel()], dtype=torch.int32, device="cuda"))
        buffers = K.BackwardBuffers(t_table, cam, config, visible_clusters=clusters,
                                    collect_stats=True)
        for t in (buffers.gmean, buffers.gconic, buffers.gcolor, buffers.galpha,
                  buffers.fragments):
            t.fill_(float("nan"))
        K.prepare_rasterize_backward(cache, cam, config, buffers)
        cot, stats = K.rasterize_backward(projected, t_table, cache, drgb_t, cam, config,
                                          buffers=buffers)
    else:
        cot, stats = K.rasterize_backward(projected, t_table, cache, drgb_t, cam, config,
                                          ddepth=torch.as_tensor(ddepth, device="cuda"),
                                          collect_stats=True)
    torch.cuda.synchronize()
    fwd = O.raster_fwd(proj, table, W, H, tile_w, tile_h)
    exp = O.raster_bwd(proj, table, fwd, drgb.reshape(-1), W, H, tile_w, tile_h,
                       ddepth=None if ddepth is None else ddepth.reshape(-1))
    _assert_stats_close(stats.cpu().numpy(), exp["stats"])
    for name in ("mean", "conic", "color", "alpha"):
        got = getattr(cot, name).cpu().numpy().reshape(-1)
        assert rel_l2(got, exp[name]) < 1e-3, (name, rel_l2(got, exp[name]))
    # Without statistics the same call returns the cotangents alone.
    plain = K.rasterize_backward(projected, t_table, cache, drgb_t, cam, config,
                                 ddepth=None if ddepth is None else torch.as_tensor(ddepth,
                                                                                   device="cuda"))
    torch.cuda.synchronize()
    assert rel_l2(plain.alpha.cpu().numpy(), exp["alpha"]) < 1e-3


def test_known_answer_early_termination_statistics_on_gpu():
    """tests/test_packed.py:240-273 on the CUDA path: black right half, 0.5
    left half, the fourth splat on collects nothing, and the statistics
    equal the oracle's."""
    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.types import DeviceCamera, SortedVisibilityTable
    from tests.test_oracle_cpu import early_termination_case

    K = _kernels()
    proj, table = early_termination_case()
    config = CapacityConfig(12, 1, 12, 16, 0, 12, tile_height=8)
    t_table = SortedVisibilityTable(torch.as_tensor(table["gaussian_ids"], device="cuda"),
                                    torch.as_tensor(table["tile_offsets"], device="cuda"),
                                    torch.ones(12, dtype=torch.int32, device="cuda"),
                                    torch.tensor([12], device="cuda"),
                                    torch.tensor([0], device="cuda"))
    cam = DeviceCamera(None, None, None, None, 32, 8)
    projected = torch_proj(proj)
    result, cache = K.rasterize_forward(projected, t_table, cam, config)
    drgb = torch.ones(8, 32, 3, device="cuda")
    cot, stats = K.rasterize_backward(projected, t_table, cache, drgb, cam, config,
                                      collect_stats=True)
    torch.cuda.synchronize()
    image = result.rgb.cpu().numpy()
    np.testing.assert_array_equal(image[:, 16:], 0)
    np.testing.assert_allclose(image[:, :16], 0.5, atol=1e-3)
    assert cache.last.cpu().numpy().reshape(8, 32)[:, :16].max() < 12
    np.testing.assert_array_equal(cot.color.cpu().numpy()[3:], 0)
    stats = stats.cpu().numpy()
    np.testing.assert_array_equal(stats[3:, :2], 0)
    fwd = O.raster_fwd(proj, table, 32, 8, 16, 8)
    exp = O.raster_bwd(proj, table, fwd, np.ones(8 * 32 * 3, np.float32), 32, 8, 16, 8)
    np.testing.assert_array_equal(stats[:, 0], exp["stats"][:, 0])
    np.testing.assert_allclose(stats, exp["stats"], rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("tile_h,tile_w", [(16, 8), (12, 16)])
def test_raster_split_stages_match_single_calls(tile_h, tile_w):
    """gsb_raster_pack + gsb_raster_fwd(SPLATS_READY) and gsb_raster_bwd_prepare
    + gsb_raster_bwd(PREPARED), each stage on a second stream, give the
    single calls' forward bit for bit and their cotangents up to the order of
    the atomic additions."""
    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.types import DeviceCamera, SortedVisibilityTable

    K = _kernels()
    W, H = 67, 45
    proj, table = _raster_case(21, W, H, tw=tile_w, th=tile_h)
    c = len(proj["alpha"])
    config = CapacityConfig(c, 128, 1, tile_w, 0, len(table["gaussian_ids"]), tile_height=tile_h)
    t_table = SortedVisibilityTable(*(torch.as_tensor(table[k], device="cuda") for k in
                                      ("gaussian_ids", "tile_offsets", "point_counts")),
                                    torch.tensor([table["pair_count"]], device="cuda"),
                                    torch.tensor([0], device="cuda"))
    cam = DeviceCamera(None, None, None, None, W, H)
    projected = torch_proj(proj)
    drgb = torch.as_tensor(np.random.default_rng(5).normal(0, 1, (H, W, 3)).astype(np.float32),
                           device="cuda")
    ids = torch.arange(-(-c // 128), dtype=torch.int32, device="cuda")
    clusters = (ids, torch.tensor([ids.numel()], dtype=torch.int32, device="cuda"))
    r1, c1 = K.rasterize_forward(projected, t_table, cam, config, want_depth=False, want_alpha=False)
    g1 = K.rasterize_backward(projected, t_table, c1, r1.rgb * 0 + drgb, cam, config,
                              visible_clusters=clusters)
    main, side = torch.cuda.current_stream(), torch.cuda.Stream()
    splats = torch.full((c, 12), float("nan"), device="cuda")
    side.wait_stream(main)
    with torch.cuda.stream(side):
        K.pack_splats(projected, cam, config, out=splats)
    main.wait_stream(side)
    r2, c2 = K.rasterize_forward(projected, t_table, cam, config, want_depth=False,
                                 want_alpha=False, splats=splats)
    buffers = K.BackwardBuffers(t_table, cam, config, visible_clusters=clusters)
    for t in (buffers.gmean, buffers.gconic, buffers.gcolor, buffers.galpha):
        t.fill_(float("nan"))
    side.wait_stream(main)
    with torch.cuda.stream(side):
        K.prepare_rasterize_backward(c2, cam, config, buffers)
    main.wait_stream(side)
    g2 = K.rasterize_backward(projected, t_table, c2, drgb, cam, config, buffers=buffers)
    torch.cuda.synchronize()
    vis = projected.visible != 0
    for a, b in ((r1.rgb, r2.rgb), (c1.final_t, c2.final_t), (c1.last, c2.last),
                 (c1.backward_work, c2.backward_work), (c1.splats[vis], c2.splats[vis])):
        assert torch.equal(a, b)
    # Cotangents accumulate with float atomics, whose order varies per run.
    for name in ("mean", "conic", "color", "alpha"):
        a, b = getattr(g1, name).cpu().numpy(), getattr(g2, name).cpu().numpy()
        assert np.isfinite(b).all(), name
        assert rel_l2(b.reshape(-1), a.reshape(-1)) < 1e-6, name


# ---------------------------------------------------------------------------
# Loss
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("shape", [(3, 5, 3), (17, 31, 3), (64, 49, 3), (96, 128, 3)])
def test_fused_loss_matches_oracle(shape):
    K = _kernels()
    rng = np.random.default_rng(41)
    pred = rng.uniform(0.02, 0.98, shape).astype(np.float32)
    tgt = rng.uniform(0.02, 0.98, shape).astype(np.float32)
    loss, grad = K.fused_loss_and_grad(torch.as_tensor(pred, device="cuda"),
                                       torch.as_tensor(tgt, device="cuda"))
    exp_loss, exp_grad = O.loss(pred, tgt)
    np.testing.assert_allclose(float(loss), exp_loss, rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(grad.cpu().numpy(), exp_grad, rtol=2e-4, atol=2e-7)


def test_fused_loss_uint8_target_and_scale():
    K = _kernels()
    rng = np.random.default_rng(42)
    for shape in ((1, 1, 3), (3, 5, 3), (17, 31, 3), (64, 49, 3)):
        tgt = rng.integers(0, 256, shape, dtype=np.uint8)
        tgt[0, 0] = [0, 128, 255]
        norm = tgt.astype(np.float32) * np.float32(1.0 / 255.0)
        pred = rng.uniform(0, 1, shape).astype(np.float32)
        a = K.fused_loss_and_grad_with_scale(torch.as_tensor(pred, device="cuda"),
                                             torch.as_tensor(tgt, device="cuda"))
        b = K.fused_loss_and_grad_with_scale(torch.as_tensor(pred, device="cuda"),
                                             torch.as_tensor(norm, device="cuda"))
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x.cpu().numpy(), y.cpu().numpy())
        grad, scale = a[1].cpu().numpy(), float(a[2].item())
        assert scale == max(float(np.abs(grad).max()), 1e-12)
    same = torch.full((17, 19, 3), 0.5, device="cuda")
    loss, grad = K.fused_loss_and_grad(same, same)
    assert abs(float(loss)) < 2e-6 and float(grad.abs().max()) < 2e-7


# ---------------------------------------------------------------------------
# Cluster culling
# ---------------------------------------------------------------------------
def test_cluster_compaction_matches_oracle():
    from jaxgs_b200.scene import CapacityConfig, config1_camera, config1_scene, world_cluster_bounds

    K = _kernels()
    pool = config1_scene(n=200_000, seed=7)
    cam = config1_camera()
    center, extent, valid = world_cluster_bounds(pool, 128)
    config = CapacityConfig(200_000, 128, 16, 16, 3, tile_height=8)
    dc = _dev_camera(cam)
    bounds = tuple(torch.as_tensor(a, device="cuda") for a in (center, extent, valid))
    (ids, count), slots = K.compact_visible_clusters(bounds, dc, config)
    torch.cuda.synchronize()
    e_ids, e_count, e_vis = O.cluster_compact(center, extent, valid, cam.frustum_planes())
    assert int(count.item()) == e_count
    np.testing.assert_array_equal(ids.cpu().numpy()[:e_count], e_ids[:e_count])
    np.testing.assert_array_equal(slots.cpu().numpy(), np.repeat(e_vis, 128)[:200_000])
