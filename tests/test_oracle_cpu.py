"""The CPU oracle, pinned (no GPU needed).

1. Known answers transcribed from the reference's own tests
   (tests/golden/known_answers.json, cited per case).
2. The oracle's forward values and analytic gradients against an independent
   PyTorch-autograd restatement of the reference's JAX numerics
   (tests/torch_ref.py): projection, compositing, L1+SSIM.
3. Binning self-consistency properties the reference tests for its GPU
   binning (tests/test_work_balance.py:89-160, test_cute.py:67-107).
4. Golden fixtures of the oracle itself (tests/golden/oracle_small.npz,
   made by tests/golden/make_golden.py) so that an oracle change is noticed.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from jaxgs_b200.scene import (Camera, CapacityConfig, config0_scene, create_gaussians,
                              seed_gaussians)
from oracle import oracle as O
from tests import torch_ref as R
from tests.helpers import known_answer_three, rel_l2, splats

GOLDEN = Path(__file__).resolve().parent / "golden"


# ---------------------------------------------------------------------------
# 1. Known answers of the reference's tests
# ---------------------------------------------------------------------------
def _known():
    return json.loads((GOLDEN / "known_answers.json").read_text())


def test_known_answer_three_gaussians():
    ka = _known()["three_gaussians"]
    config, cam, pool = known_answer_three()
    proj = O.project_fwd(pool, cam, degree=0, sh_dim=1)
    t = O.bin(proj, 8, 8, 4, 4, 16)
    np.testing.assert_array_equal(np.diff(t["tile_offsets"]), ka["diff_offsets"])
    np.testing.assert_array_equal(t["gaussian_ids"][:12].reshape(4, 3), ka["ids_per_tile"])
    assert t["pair_count"] == ka["pair_count"] and t["overflow"] == ka["overflow"]
    narrow = O.bin(proj, 8, 8, 4, 4, 4)
    assert narrow["overflow"] == ka["narrow_overflow"]


def test_known_answer_large_ellipse_and_empty():
    ka = _known()["large_ellipse"]
    cam = Camera.from_colmap([1, 0, 0, 0], [0, 0, 0], 20, 20, 8, 9, 17, 19)
    pool = seed_gaussians(create_gaussians(CapacityConfig(1, 1, 1, 16, 0, 4)),
                          np.array([[0, 0, 2.0]]), np.ones((1, 3)) * 0.5, scale=0.2, opacity=0.5)
    proj = O.project_fwd(pool, cam, degree=0, sh_dim=1)
    proj["conic"] = np.array([1e-5, 0, 0, 1e-5], np.float32)
    t = O.bin(proj, 17, 19, 16, 16, 4)
    assert t["pair_count"] == ka["pair_count"] and t["overflow"] == ka["overflow"]
    proj["visible"][:] = 0
    e = O.bin(proj, 17, 19, 16, 16, 4)
    assert e["pair_count"] == 0 and (e["tile_offsets"] == 0).all()


@pytest.mark.parametrize("tiles_x", [255, 256])
def test_known_answer_tile_key_width(tiles_x):
    ka = _known()["tile_key_width"]
    width, height = tiles_x * 8, 256 * 8
    cam = Camera.from_colmap([1, 0, 0, 0], [0, 0, 0], 20, 20, width - 4, height - 4, width, height)
    pool = seed_gaussians(create_gaussians(CapacityConfig(1, 1, 1, 8, 0, 4)),
                          np.array([[0.0, 0.0, 2.0]]), np.full((1, 3), 0.5), scale=0.02, opacity=0.5)
    t = O.bin(O.project_fwd(pool, cam, degree=0, sh_dim=1), width, height, 8, 8, 4)
    assert t["pair_count"] == ka["pair_count"]
    assert (t["tile_offsets"][:-1] == 0).all() and t["tile_offsets"][-1] == ka["last_offset"]
    assert t["gaussian_ids"][0] == ka["first_id"]


def test_known_answer_digit_plan_of_the_c_library():
    from jaxgs_b200 import _lib

    for num_tiles, expected in _known()["digit_plan"]:
        assert _lib.tile_sort_plan(num_tiles) == tuple(expected)


def test_identical_images_have_zero_loss():
    """tests/test_loss.py:9-12."""
    for value in (0.0, 0.5, 1.0):
        image = np.full((8, 8, 3), value, np.float32)
        loss, grad = O.loss(image, image)
        assert abs(loss) < 1e-7 and np.abs(grad).max() < 1e-7


def test_log_is_within_two_ulp_and_monotone():
    """The binning's project-written log (CUDA's logf is specified to 1 ulp;
    AccuTile only needs a fixed, shared rounding)."""
    rng = np.random.default_rng(0)
    xs = np.concatenate([np.float32(np.exp(rng.uniform(-87, 88, 20000))),
                         np.float32(2.0) ** np.arange(-126, 127, dtype=np.float32),
                         np.float32([1.0, 255.0, 1 / 255.0, 0.70710677, 1.4142135, 1e-40, 3e-45])])
    mine = np.array([O.gs_logf(float(x)) for x in xs], np.float64)
    ref = np.log(xs.astype(np.float64))
    ulp = np.abs(mine - ref) / np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
    ulp[ref == 0] = np.abs(mine[ref == 0]) / np.spacing(np.float32(0))
    assert ulp.max() <= 2.0, ulp.max()
    grid = np.float32(np.linspace(1 / 255, 255, 5000))
    vals = np.array([O.gs_logf(float(x)) for x in grid])
    assert (np.diff(vals) >= 0).all()


# ---------------------------------------------------------------------------
# 2. Oracle vs an independent autograd restatement
# ---------------------------------------------------------------------------
def _small_pool(n=300, seed=1):
    pool_np, cam, target = config0_scene()
    sel = np.random.default_rng(seed).choice(4096, n, replace=False)
    return {k: v[sel].copy() for k, v in pool_np.items()}, cam, target


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
def test_oracle_projection_matches_torch_restatement(degree):
    pool, cam, _ = _small_pool()
    exp = O.project_fwd(pool, cam, degree=degree, sh_dim=16)
    t = {k: torch.as_tensor(v, dtype=torch.float64) for k, v in pool.items() if k != "alive"}
    mean, z, conic, radius, color, alpha, vis = R.project(t["xyz"], t["log_scale"], t["rotation"],
                                                          t["opacity"], t["sh"],
                                                          torch.as_tensor(pool["alive"]), cam, degree)
    np.testing.assert_allclose(exp["mean"], mean.numpy().reshape(-1), rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(exp["conic"], conic.numpy().reshape(-1), rtol=1e-3, atol=1e-5)
    np.testing.assert_allclose(exp["radius"], radius.numpy(), rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(exp["color"], color.numpy().reshape(-1), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(exp["alpha"], alpha.numpy(), rtol=1e-5, atol=1e-7)
    np.testing.assert_array_equal(exp["visible"].astype(bool), vis.numpy())


@pytest.mark.parametrize("degree", [1, 3])
def test_oracle_projection_pullback_matches_autograd(degree):
    """kernels/projection_backward.py vs autograd of render/projection.py
    (the reference's own check is tests/test_cute.py:393-435, 3e-3)."""
    pool, cam, _ = _small_pool(200, seed=4)
    rng = np.random.default_rng(6)
    n = pool["xyz"].shape[0]
    w = {"mean": rng.normal(0, 1, (n, 2)), "depth": rng.normal(0, 1, n),
         "conic": rng.normal(0, 1, (n, 2, 2)), "radius": rng.normal(0, 0.1, n),
         "color": rng.normal(0, 1, (n, 3)), "alpha": rng.normal(0, 1, n)}
    params = [torch.tensor(pool[k], dtype=torch.float64, requires_grad=True)
              for k in ("xyz", "log_scale", "rotation", "opacity", "sh")]
    out = R.project(*params, torch.as_tensor(pool["alive"]), cam, degree)
    names = ("mean", "depth", "conic", "radius", "color", "alpha")
    total = sum((o * torch.as_tensor(w[k])).sum() for k, o in zip(names, out[:6]))
    total.backward()
    proj = O.project_fwd(pool, cam, degree=degree, sh_dim=16)
    cot = {k: np.asarray(w[k], np.float32).reshape(-1) for k in names}
    grads = O.project_bwd(pool, cam, proj["color"], cot, degree=degree, sh_dim=16)
    for name, got, p in zip(("xyz", "log_scale", "rotation", "opacity", "sh"), grads, params):
        ref = p.grad.numpy().reshape(-1)
        if name == "sh":
            ref = ref.reshape(n, 16, 3)
            ref[:, (degree + 1) ** 2:] = 0
            ref = ref.reshape(-1)
        assert rel_l2(got, ref) < 1e-4, (name, rel_l2(got, ref))


def _dense_case(seed=0, count=40, width=23, height=19):
    rng = np.random.default_rng(seed)
    proj = splats(rng, count, width, height, radius=(1.0, 6.0), alpha=(0.2, 0.99))
    proj["visible"][:] = 1
    proj["depth"] = np.arange(count, dtype=np.float32)  # distinct depths -> order by id
    return proj


def _dense_table(count, W, H, tw, th):
    """Every splat listed in every tile in depth (= id) order, so compositing
    is compared without the binning's 1/255-level tile selection (the
    reference's test makes every ellipse cover every tile for the same reason,
    tests/test_cute.py:237-239)."""
    tiles = (-(-W // tw)) * (-(-H // th))
    return {"gaussian_ids": np.tile(np.arange(count, dtype=np.int32), tiles),
            "tile_offsets": (np.arange(tiles + 1) * count).astype(np.int32)}


@pytest.mark.parametrize("tile", [(8, 16), (16, 16), (4, 8)])
def test_oracle_compositing_matches_dense_reference(tile):
    """Sorted compositing == dense compositing with the early stop
    (tests/test_cute.py:216-282 makes the same comparison)."""
    th, tw = tile
    W, H = 23, 19
    proj = _dense_case()
    table = _dense_table(len(proj["alpha"]), W, H, tw, th)
    bg = np.array([0.12, 0.24, 0.36], np.float32)
    fwd = O.raster_fwd(proj, table, W, H, tw, th, bg)
    t = lambda a, s: torch.as_tensor(a, dtype=torch.float64).reshape(s)
    c = len(proj["alpha"])
    rgb, depth, alpha = R.dense_composite(t(proj["mean"], (c, 2)), t(proj["conic"], (c, 2, 2)),
                                          t(proj["color"], (c, 3)), t(proj["alpha"], (c,)),
                                          t(proj["depth"], (c,)), torch.arange(c), W, H, bg)
    ok = fwd["ambiguous"] == 0
    np.testing.assert_allclose(fwd["rgb"].reshape(-1, 3)[ok], rgb.numpy().reshape(-1, 3)[ok], atol=2e-5, rtol=2e-4)
    np.testing.assert_allclose(fwd["alpha"][ok], alpha.numpy().reshape(-1)[ok], atol=2e-5)
    np.testing.assert_allclose(fwd["depth"][ok], depth.numpy().reshape(-1)[ok], atol=2e-4, rtol=2e-4)


def test_oracle_compositing_pullback_matches_autograd():
    W, H = 23, 19
    proj = _dense_case(seed=2)
    table = _dense_table(len(proj["alpha"]), W, H, 16, 8)
    bg = np.array([0.1, 0.2, 0.3], np.float32)
    fwd = O.raster_fwd(proj, table, W, H, 16, 8, bg)
    rng = np.random.default_rng(8)
    drgb = rng.normal(0, 1, (H, W, 3))
    ddepth = rng.normal(0, 0.1, (H, W))
    dalpha = rng.normal(0, 0.5, (H, W))
    c = len(proj["alpha"])
    leaves = {k: torch.tensor(np.asarray(proj[k], np.float64).reshape(s), requires_grad=True)
              for k, s in (("mean", (c, 2)), ("conic", (c, 2, 2)), ("color", (c, 3)),
                           ("alpha", (c,)), ("depth", (c,)))}
    rgb, depth, alpha = R.dense_composite(leaves["mean"], leaves["conic"], leaves["color"],
                                          leaves["alpha"], leaves["depth"], torch.arange(c), W, H, bg)
    total = ((rgb * torch.as_tensor(drgb)).sum() + (depth * torch.as_tensor(ddepth)).sum()
             + (alpha * torch.as_tensor(dalpha)).sum())
    total.backward()
    exp = O.raster_bwd(proj, table, fwd, drgb.reshape(-1), W, H, 16, 8, bg,
                       ddepth.reshape(-1), dalpha.reshape(-1))
    for name in ("mean", "conic", "color", "alpha", "depth"):
        got = exp[name]
        ref = leaves[name].grad.numpy().reshape(-1)
        assert rel_l2(got, ref) < 1e-3, (name, rel_l2(got, ref))


def test_oracle_fragment_statistics_match_dense_autograd():
    """collect_stats (sorted_rasterize.py:155-203) against the dense float64
    restatement: counts exact, the other columns within 1e-4 relative L2."""
    W, H = 23, 19
    proj = _dense_case(seed=4)
    table = _dense_table(len(proj["alpha"]), W, H, 16, 8)
    bg = np.array([0.1, 0.2, 0.3], np.float32)
    fwd = O.raster_fwd(proj, table, W, H, 16, 8, bg)
    drgb = np.random.default_rng(9).normal(0, 1, (H, W, 3))
    exp = O.raster_bwd(proj, table, fwd, drgb.reshape(-1), W, H, 16, 8, bg)
    c = len(proj["alpha"])
    t = lambda a, s: torch.as_tensor(np.asarray(a, np.float64)).reshape(s)
    ref = R.dense_fragment_statistics(t(proj["mean"], (c, 2)), t(proj["conic"], (c, 2, 2)),
                                      t(proj["color"], (c, 3)), t(proj["alpha"], (c,)), W, H,
                                      torch.as_tensor(drgb), bg).numpy()
    stats = exp["stats"]
    assert stats.shape == (c, 4) and ref[:, 0].sum() > 0
    np.testing.assert_array_equal(stats[:, 0], ref[:, 0])
    for col in (1, 2, 3):
        assert rel_l2(stats[:, col], ref[:, col]) < 1e-4, (col, rel_l2(stats[:, col], ref[:, col]))


def early_termination_case():
    """tests/test_packed.py:240-271: twelve coincident near-opaque splats
    (opacity 0.99) over the left 16x8 tile of a 32x8 image; the right tile
    is empty."""
    c = 12
    proj = {"mean": np.full(c * 2, 4.0, np.float32), "depth": np.ones(c, np.float32),
            "conic": np.tile(np.eye(2, dtype=np.float32).reshape(-1) * 1e-4, c),
            "radius": np.ones(c, np.float32), "color": np.full(c * 3, 0.5, np.float32),
            "alpha": np.full(c, 0.99, np.float32), "visible": np.ones(c, np.int8)}
    table = {"gaussian_ids": np.arange(c, dtype=np.int32),
             "tile_offsets": np.array([0, c, c], np.int32)}
    return proj, table


def test_known_answer_early_termination_statistics():
    """tests/test_packed.py:262-273: the right half stays black, the left is
    0.5, no pixel composites all twelve splats, the splats from the fourth
    on collect no statistics and get no colour cotangent, and the squared
    opacity cotangents are finite."""
    proj, table = early_termination_case()
    fwd = O.raster_fwd(proj, table, 32, 8, 16, 8)
    image = fwd["rgb"].reshape(8, 32, 3)
    np.testing.assert_array_equal(image[:, 16:], 0)
    np.testing.assert_allclose(image[:, :16], 0.5, atol=1e-3)
    assert fwd["last"].reshape(8, 32)[:, :16].max() < 12
    bwd = O.raster_bwd(proj, table, fwd, np.ones(8 * 32 * 3, np.float32), 32, 8, 16, 8)
    np.testing.assert_array_equal(bwd["color"].reshape(12, 3)[3:], 0)
    stats = bwd["stats"]
    np.testing.assert_array_equal(stats[3:, :2], 0)
    assert np.isfinite(stats).all()
    # Every pixel of the left tile composites the first two splats.
    np.testing.assert_array_equal(stats[:2, 0], 128)


ADAM_RATES = dict(position_lr_init=0.00016, position_lr_final=0.0000016, feature_lr=0.0025,
                  opacity_lr=0.025, scaling_lr=0.005, rotation_lr=0.001)


def _adam_all_fields(pool, m, v, grads, ids, count, rates, cluster_size, compact):
    out = {}
    for i, name in enumerate(("xyz", "log_scale", "rotation", "opacity", "sh")):
        out[name] = O.sparse_adam(pool[name], m[name], v[name], grads[i], pool["alive"], ids,
                                  count, rates[i], cluster_size=cluster_size,
                                  is_sh=name == "sh", compact_gradients=compact)
    return out


def test_known_answer_sparse_adam_rates_and_mask():
    """tests/test_training_protocol.py:201-224: unit gradients, zero moments,
    step 0, spatial scale 2: each active field moves by rate * 0.1 /
    sqrt(0.001) (rates 0.00032, 0.005, 0.001, 0.025; SH DC 0.0025, the other
    coefficients 0.00025), the inactive slot not at all."""
    config = CapacityConfig(2, 1, 2, 4, 1)
    pool = seed_gaussians(create_gaussians(config), np.ones((2, 3)), np.ones((2, 3)))
    rates = O.parameter_learning_rates(0, 2.0, 30000, **ADAM_RATES)
    zeros = {k: np.zeros_like(pool[k]) for k in ("xyz", "log_scale", "rotation", "opacity", "sh")}
    grads = [np.ones_like(pool[k]) for k in ("xyz", "log_scale", "rotation", "opacity", "sh")]
    # visible = [True, False] with clusters of one slot: cluster 0 listed.
    out = _adam_all_fields(pool, zeros, zeros, grads, np.array([0, 1], np.int32), 1, rates, 1,
                           False)
    for name, rate in zip(("xyz", "log_scale", "rotation", "opacity"), (0.00032, 0.005, 0.001, 0.025)):
        got = out[name][0].reshape(pool[name].shape)
        np.testing.assert_allclose(got[0], pool[name][0] - rate * 0.1 / np.sqrt(0.001), atol=1e-6)
        np.testing.assert_array_equal(got[1], pool[name][1])
    sh = out["sh"][0].reshape(pool["sh"].shape)
    np.testing.assert_allclose(sh[0, 0], pool["sh"][0, 0] - 0.0025 * np.sqrt(10), atol=1e-6)
    np.testing.assert_allclose(sh[0, 1], pool["sh"][0, 1] - 0.00025 * np.sqrt(10), atol=1e-6)
    np.testing.assert_array_equal(sh[1], pool["sh"][1])


def test_oracle_sparse_adam_compact_gradients_and_untouched_slots():
    """tests/test_packed.py:275-330: moments 0.2 / 0.1, gradients 0.3, step
    123, spatial scale 2, clusters of two slots with 1, 3 and 4 listed: the
    compact-gradient update equals the pool-order one, and slots outside the
    listed clusters keep their values and moments."""
    config = CapacityConfig(10, 2, 16, 16, 2, 128, tile_height=8)
    pool = seed_gaussians(create_gaussians(config), np.ones((9, 3)) * 2.0, np.ones((9, 3)) * 0.4)
    names = ("xyz", "log_scale", "rotation", "opacity", "sh")
    visible = np.repeat(np.array([False, True, False, True, True]), 2)
    ids, count = np.array([1, 3, 4, 0, 0], np.int32), 3
    m = {k: np.full_like(pool[k], 0.2) for k in names}
    v = {k: np.full_like(pool[k], 0.1) for k in names}
    grads = [np.full_like(pool[k], 0.3) for k in names]
    rates = O.parameter_learning_rates(123, 2.0, 30000, **ADAM_RATES)
    full = _adam_all_fields(pool, m, v, grads, ids, count, rates, 2, False)
    slots = (ids[:count, None] * 2 + np.arange(2)).reshape(-1)
    compact = [g.reshape(10, -1)[slots].reshape(-1) for g in grads]
    comp = _adam_all_fields(pool, m, v, compact, ids, count, rates, 2, True)
    for name in names:
        for a, b in zip(full[name], comp[name]):
            np.testing.assert_array_equal(a, b)
        x = full[name][0].reshape(10, -1)
        assert np.all(x[visible & pool["alive"]] != pool[name].reshape(10, -1)[visible & pool["alive"]])
        np.testing.assert_array_equal(x[~visible], pool[name].reshape(10, -1)[~visible])
        np.testing.assert_array_equal(full[name][1].reshape(10, -1)[~visible],
                                      m[name].reshape(10, -1)[~visible])


def test_known_answer_densification_scores():
    """tests/test_training_protocol.py:14-29: the first parent's score is
    (4/4 - (2/4)^2) * 3 * sigmoid(0.5 logit)^2, the zero-weight second is
    pruned, dead slots score 0 and are not pruned."""
    config = CapacityConfig(4, 1, 2, 4, 1)
    pool = seed_gaussians(create_gaussians(config), np.array([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]]),
                          np.ones((2, 3)), scale=0.2, opacity=0.5)
    stats = np.array([[3.0, 1.0, 2.0, 4.0], [0.0] * 4, [0.0] * 4, [0.0] * 4])
    score, prune = O.densification_scores(pool["opacity"], pool["alive"], stats)
    np.testing.assert_allclose(score[0], (4 / 4 - (2 / 4) ** 2) * 3 * 0.5 ** 2, rtol=1e-6)
    np.testing.assert_array_equal(prune, [False, True, False, False])
    decayed = O.decay_opacity(pool["opacity"], pool["alive"])
    a = 1 / (1 + np.exp(-decayed))
    np.testing.assert_allclose(a[:2], 0.25, rtol=1e-6)
    np.testing.assert_array_equal(decayed[2:], pool["opacity"].reshape(-1)[2:])


@pytest.mark.parametrize("shape", [(3, 5), (17, 31), (40, 33)])
def test_oracle_loss_matches_autograd(shape):
    """Fused loss value and gradient == autograd of reference/loss.py
    (tests/test_loss.py:15-32 uses rtol 2e-5 / 2e-4)."""
    rng = np.random.default_rng(41)
    pred = rng.uniform(0.02, 0.98, shape + (3,)).astype(np.float32)
    tgt = rng.uniform(0.02, 0.98, shape + (3,)).astype(np.float32)
    x = torch.tensor(pred, dtype=torch.float64, requires_grad=True)
    ref = R.photometric_loss(x, torch.as_tensor(tgt, dtype=torch.float64))
    ref.backward()
    loss, grad = O.loss(pred, tgt)
    np.testing.assert_allclose(loss, float(ref.detach()), rtol=2e-6)
    np.testing.assert_allclose(grad, x.grad.numpy(), rtol=2e-4, atol=1e-7)


def test_oracle_loss_uint8_target_equals_normalised_float():
    rng = np.random.default_rng(42)
    tgt = rng.integers(0, 256, (9, 11, 3), dtype=np.uint8)
    pred = rng.uniform(0, 1, (9, 11, 3)).astype(np.float32)
    a = O.loss(pred, tgt)
    b = O.loss(pred, tgt.astype(np.float32) * np.float32(1.0 / 255.0))
    assert a[0] == b[0]
    np.testing.assert_array_equal(a[1], b[1])


# ---------------------------------------------------------------------------
# 3. Binning properties (reference GPU-binning tests, applied to the oracle)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("tile", [(8, 16), (16, 16)])
def test_oracle_binning_properties(tile):
    th, tw = tile
    rng = np.random.default_rng(3)
    W, H = 640, 360
    proj = splats(rng, 2048, W, H, radius=(0.4, 60.0), huge=8)
    t = O.bin(proj, W, H, tw, th, 1 << 19)
    counts = t["point_counts"]
    total = t["pair_count"]
    assert total == counts.sum() and t["tile_offsets"][-1] == total
    tiles = (-(-W // tw)) * (-(-H // th))
    ids = t["gaussian_ids"][:total]
    tile_of = np.repeat(np.arange(tiles), np.diff(t["tile_offsets"]))
    # ranges == searchsorted of the sorted tile keys (tests/test_cute.py:102)
    np.testing.assert_array_equal(t["tile_offsets"], np.searchsorted(tile_of, np.arange(tiles + 1)))
    # every Gaussian appears exactly point_counts times, pairs unique
    np.testing.assert_array_equal(np.bincount(ids, minlength=len(counts)), counts)
    assert np.unique(ids.astype(np.int64) * tiles + tile_of).size == total
    # (tile, depth, id) order inside each tile
    same = tile_of[1:] == tile_of[:-1]
    d = proj["depth"][ids]
    assert (np.diff(d)[same] >= 0).all()
    tie = same & (np.diff(d) == 0)
    assert (np.diff(ids)[tie] > 0).all()
    # the per-Gaussian tile lists agree with the sequential walk
    for g in np.flatnonzero(counts)[:200]:
        keys, n = O.gaussian_tiles(*proj["mean"][2 * g:2 * g + 2], proj["conic"][4 * g],
                                   proj["conic"][4 * g + 1], proj["conic"][4 * g + 3],
                                   proj["alpha"][g], tw, th, -(-W // tw), -(-H // th))
        assert n == counts[g]
        assert set(keys.tolist()) == set(tile_of[ids == g].tolist())


def test_oracle_keeps_the_reference_tile_range_formula():
    """AccuTile's last tile row/column is int((max + tile - 1) / tile)
    (kernels/sorted_visibility.py:96-97), an integer ceiling applied to a
    fractional extent: an ellipse that reaches less than one pixel past a tile
    boundary does not bin into the next tile even when a pixel centre there
    has alpha >= 1/255.  Bit-exact binning keeps that behaviour."""
    rng = np.random.default_rng(5)
    proj = splats(rng, 300, 96, 64, radius=(0.5, 12.0), alpha=(0.01, 0.99))
    g = 5
    m, c, a = proj["mean"][2 * g:2 * g + 2], proj["conic"][4 * g:4 * g + 4], proj["alpha"][g]
    keys, n = O.gaussian_tiles(m[0], m[1], c[0], c[1], c[3], a, 16, 8, 6, 8)
    assert sorted(keys.tolist()) == [4, 9, 10] and n == 3
    ys, xs = np.mgrid[16:24, 48:64]
    d = np.stack([xs + 0.5 - m[0], ys + 0.5 - m[1]], -1).astype(np.float64)
    q = np.einsum("...i,ij,...j->...", d, c.astype(np.float64).reshape(2, 2), d)
    assert (a * np.exp(-0.5 * q)).max() > 1.0 / 255  # tile 15 holds such a pixel


# ---------------------------------------------------------------------------
# 4. Golden fixtures of the oracle
# ---------------------------------------------------------------------------
def test_oracle_matches_committed_golden_fixtures():
    from tests.golden.make_golden import compute

    data = np.load(GOLDEN / "oracle_small.npz")
    now = compute()
    for key in data.files:
        if data[key].dtype.kind in "iub":
            np.testing.assert_array_equal(now[key], data[key], err_msg=key)
        else:
            np.testing.assert_allclose(now[key], data[key], rtol=1e-5, atol=1e-6, err_msg=key)


def test_oracle_whole_chain_matches_finite_differences():
    """tests/test_cute.py:328-355: the gradient of a weighted sum of the
    rendered image (weights arange(size) / size) through projection,
    binning and fp32 compositing, against central differences, within
    rtol 0.04 / atol 0.003 as there.  For the 12 Gaussians with the largest
    opacity gradient, log_scale, rotation, opacity and an SH coefficient
    all match with a step of 1e-4.  Positions use a 2e-5 step and at least
    90% of them match: a 1e-3 move carries some pixel's alpha across the
    1/256 cut, or a tile across the binning level, and no difference quotient
    sees past that jump; a smaller step makes such a crossing rare, while
    float32 rounding still leaves the quotient accurate."""
    pool, cam, _ = _small_pool(300, seed=1)
    W, H = cam.width, cam.height
    weights = (np.arange(H * W * 3, dtype=np.float64) / (H * W * 3)).astype(np.float32)

    def render(p):
        proj = O.project_fwd(p, cam, degree=3, sh_dim=16)
        table = O.bin(proj, W, H, 16, 8, 300 * 96)
        return proj, table, O.raster_fwd(proj, table, W, H, 16, 8)

    def loss(p):
        return float(np.sum(render(p)[2]["rgb"].astype(np.float64) * weights))

    proj, table, fwd = render(pool)
    cot = O.raster_bwd(proj, table, fwd, weights, W, H, 16, 8)
    cot["radius"] = np.zeros(300, np.float32)
    grads = O.project_bwd(pool, cam, proj["color"], cot, degree=3, sh_dim=16)
    names = ("xyz", "log_scale", "rotation", "opacity", "sh")

    def check(name, index, h):
        analytic = grads[names.index(name)].reshape(pool[name].shape)[index]
        plus = {k: v.copy() for k, v in pool.items()}
        minus = {k: v.copy() for k, v in pool.items()}
        plus[name][index] += h
        minus[name][index] -= h
        numeric = (loss(plus) - loss(minus)) / (2 * h)
        return abs(analytic - numeric) <= 0.003 + 0.04 * abs(numeric)

    top = np.argsort(-np.abs(grads[3]))[:12]
    for g in top:
        for name, index in (("log_scale", (g, 1)), ("rotation", (g, 2)), ("opacity", (g, 0)),
                            ("sh", (g, 1, 0))):
            assert check(name, index, 1e-4), (name, index)
    positions = [check("xyz", (g, c), 2e-5) for g in top for c in range(3)]
    assert np.mean(positions) >= 0.9, positions


def _autograd_projection(pool, cam, degree, weights_fn):
    """Gradients of weights_fn(projected fields) through the torch
    restatement of render/projection.py, in float64."""
    params = [torch.tensor(pool[k], dtype=torch.float64, requires_grad=True)
              for k in ("xyz", "log_scale", "rotation", "opacity", "sh")]
    out = R.project(*params, torch.as_tensor(pool["alive"]), cam, degree)
    weights_fn(*out[:6]).backward()
    return [p.grad.numpy() for p in params]


def test_oracle_projection_pullback_zero_and_individual_cotangents():
    """tests/test_cute.py:356-390: one cotangent per Gaussian (depth, radius,
    mean, conic, colour, alpha on Gaussians 1-6) reaches only its own
    Gaussian's parameters, matching autodiff of the reference projection;
    Gaussians 0, 7 and 8 get exact zeros."""
    from jaxgs_b200.scene import Camera, CapacityConfig, create_gaussians, seed_gaussians

    config = CapacityConfig(9, 1, 16, 16, 3)
    cam = Camera.from_colmap([1, 0, 0, 0], [0, 0, 0], 20, 20, 16, 16, 32, 32)
    pool = seed_gaussians(create_gaussians(config), np.tile([[0.1, 0.2, 2.0]], (9, 1)),
                          np.full((9, 3), 0.4), scale=np.tile([[0.1, 0.2, 0.3]], (9, 1)),
                          opacity=0.3)
    pool["sh"][:, 1:] = 0.02

    def weighted(mean, depth, conic, radius, color, alpha):
        return (depth[1] + radius[2] * 0.01 + mean[3].sum() + conic[4].sum() + color[5].sum()
                + alpha[6])

    expected = _autograd_projection(pool, cam, 3, weighted)
    cot = {"mean": np.zeros((9, 2), np.float32), "depth": np.zeros(9, np.float32),
           "conic": np.zeros((9, 4), np.float32), "radius": np.zeros(9, np.float32),
           "color": np.zeros((9, 3), np.float32), "alpha": np.zeros(9, np.float32)}
    cot["depth"][1] = 1
    cot["radius"][2] = 0.01
    cot["mean"][3] = 1
    cot["conic"][4] = 1
    cot["color"][5] = 1
    cot["alpha"][6] = 1
    proj = O.project_fwd(pool, cam, degree=3, sh_dim=16)
    grads = O.project_bwd(pool, cam, proj["color"], {k: v.reshape(-1) for k, v in cot.items()},
                          degree=3, sh_dim=16)
    for name, got, ref in zip(("xyz", "log_scale", "rotation", "opacity", "sh"), grads, expected):
        got = got.reshape(ref.shape)
        np.testing.assert_allclose(got, ref, rtol=2e-4, atol=2e-5, err_msg=name)
        np.testing.assert_array_equal(got[[0, 7, 8]], 0)


@pytest.mark.parametrize("degree", [0, 2])
def test_oracle_projection_pullback_clipped_color_and_near_plane(degree):
    """tests/test_cute.py:439-476: a Gaussian in front of the near plane
    (depth clamped in the Jacobian) whose colour is clipped to zero, beside
    an ordinary one; the pullback of squared means and conics plus radii,
    depths, colours and alphas matches autodiff (rtol 3e-3, atol 3e-4)."""
    from jaxgs_b200.scene import Camera, CapacityConfig, create_gaussians

    config = CapacityConfig(2, 2, 2, 4, degree)
    cam = Camera.from_colmap([1, 0, 0, 0], [0, 0, 0], 8, 8, 4, 4, 8, 8)
    pool = create_gaussians(config)
    pool["xyz"][:] = [[0.005, -0.003, 0.1], [0.1, 0.2, 2.0]]
    pool["log_scale"][:] = np.log([[0.1, 0.2, 0.3], [0.2, 0.15, 0.1]])
    pool["rotation"][:] = [[0.9, 0.2, -0.1, 0.15], [0.8, -0.1, 0.25, 0.2]]
    pool["opacity"][:] = [[0.1], [-0.2]]
    pool["sh"][:] = 0.1
    pool["sh"][0, 0, 0] = -3.0
    pool["alive"][:] = True
    sh_dim = (degree + 1) ** 2
    proj = O.project_fwd(pool, cam, degree=degree, sh_dim=sh_dim)
    assert proj["color"][0] == 0.0

    def weighted(mean, depth, conic, radius, color, alpha):
        return ((mean ** 2).sum() + (conic ** 2).sum() + radius.sum() + depth.sum()
                + color.sum() + alpha.sum())

    expected = _autograd_projection(pool, cam, degree, weighted)
    cot = {"mean": 2 * proj["mean"], "depth": np.ones(2, np.float32),
           "conic": 2 * proj["conic"], "radius": np.ones(2, np.float32),
           "color": np.ones(6, np.float32), "alpha": np.ones(2, np.float32)}
    grads = O.project_bwd(pool, cam, proj["color"], cot, degree=degree, sh_dim=sh_dim)
    for name, got, ref in zip(("xyz", "log_scale", "rotation", "opacity", "sh"), grads, expected):
        np.testing.assert_allclose(got.reshape(ref.shape), ref, rtol=3e-3, atol=3e-4,
                                   err_msg=name)


@pytest.mark.parametrize("degree", [0, 1, 3])
@pytest.mark.parametrize("empty", [False, True])
@pytest.mark.parametrize("cluster_size", [65, 128])
def test_oracle_active_sh_and_color_only_pullbacks_match_the_full_one(degree, empty,
                                                                       cluster_size):
    """tests/test_packed.py:14-78: in compact order, the active-bands SH
    gradient is the prefix of the full one and every other field is the
    same; the colour-only pullback's [C, 1, 3] cotangent times the SH DC
    constant is the full DC gradient."""
    from jaxgs_b200.scene import Camera, CapacityConfig, create_gaussians, seed_gaussians

    capacity = 257
    config = CapacityConfig(capacity, cluster_size, 16, 16, 3, 4096, tile_height=8)
    cam = Camera.from_colmap([1, 0, 0, 0], [0, 0, 0], 20, 20, 9, 8, 19, 17)
    visible = (np.zeros(capacity, bool) if empty
               else (np.arange(capacity) // cluster_size) % 2 == 0)
    pool = seed_gaussians(create_gaussians(config), np.tile([[0.1, -0.2, 2.0]], (capacity, 1)),
                          np.full((capacity, 3), 0.4), scale=0.1)
    pool["alive"] = visible.copy()
    pool["sh"] = (np.random.default_rng(5).normal(0, 0.2, pool["sh"].shape)).astype(np.float32)
    listed = np.unique(np.nonzero(visible)[0] // cluster_size).astype(np.int32)
    n_clusters = -(-capacity // cluster_size)
    clusters = (np.pad(listed, (0, n_clusters - len(listed))), len(listed))
    proj = O.project_fwd(pool, cam, degree=degree, sh_dim=16, clusters=clusters,
                         cluster_size=cluster_size)
    cot = {"mean": np.ones(capacity * 2, np.float32), "conic": np.full(capacity * 4, 0.01, np.float32),
           "color": np.ones(capacity * 3, np.float32), "alpha": np.ones(capacity, np.float32),
           "depth": np.zeros(capacity, np.float32), "radius": np.zeros(capacity, np.float32)}
    common = dict(degree=degree, sh_dim=16, clusters=clusters, cluster_size=cluster_size,
                  compact_gradients=True, rgb_only=True)
    full = O.project_bwd(pool, cam, proj["color"], cot, **common)
    sh_dim = (degree + 1) ** 2
    narrow = O.project_bwd(pool, cam, proj["color"], cot, sh_gradient_dim=sh_dim, **common)
    color = O.project_bwd(pool, cam, proj["color"], cot, sh_color_only=True, **common)
    rows = int(visible.sum())
    widths = (3, 3, 4, 1)
    for a, b, c, w in zip(narrow[:4], full[:4], color[:4], widths):
        np.testing.assert_allclose(a.reshape(capacity, w)[:rows], b.reshape(capacity, w)[:rows],
                                   rtol=2e-5, atol=2e-6)
        np.testing.assert_allclose(c.reshape(capacity, w)[:rows], b.reshape(capacity, w)[:rows],
                                   rtol=2e-5, atol=2e-6)
    full_sh = full[4].reshape(capacity, 16, 3)[:rows]
    np.testing.assert_allclose(narrow[4].reshape(capacity, sh_dim, 3)[:rows], full_sh[:, :sh_dim],
                               rtol=2e-5, atol=2e-6)
    np.testing.assert_allclose(color[4].reshape(capacity, 1, 3)[:rows] * 0.28209479177387814,
                               full_sh[:, :1], rtol=2e-5, atol=2e-6)
    if not empty:
        assert np.abs(full_sh[:, 0]).max() > 0


def test_every_reference_case_names_existing_tests():
    """tests/golden/known_answers.json lists each reference test that pins
    this path's values and the tests here that re-express it: each named
    test function exists, and every case says how the reference obtains its
    expectation."""
    import ast
    import json
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    cases = json.loads((root / "tests/golden/known_answers.json").read_text())["reference_cases"]
    defined = {}
    for case in cases["cases"]:
        assert case["expectation"] in ("fixed", "jax", "rule"), case
        for name in case["repo"]:
            path, func = name.split("::")
            if path not in defined:
                tree = ast.parse((root / path).read_text())
                defined[path] = {n.name for n in ast.walk(tree) if isinstance(n, ast.FunctionDef)}
            assert func in defined[path], name
