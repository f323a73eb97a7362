"""The synthetic workloads against BASELINE.json's config descriptions (the
stand-ins for MipNeRF360 bicycle, which is absent here): sizes, seeds,
value distributions and cameras, so the benchmark and the parity tests
run on the scenes the configs name."""

import numpy as np
import pytest

from jaxgs_b200 import scene as S


def _check_pool(pool, n, sh_dim=16):
    assert pool["xyz"].shape == (n, 3) and pool["log_scale"].shape == (n, 3)
    assert pool["rotation"].shape == (n, 4) and pool["opacity"].shape == (n, 1)
    assert pool["sh"].shape == (n, sh_dim, 3) and pool["alive"].all()
    for k in ("xyz", "log_scale", "rotation", "opacity", "sh"):
        assert pool[k].dtype == np.float32, k
    np.testing.assert_allclose(np.linalg.norm(pool["rotation"], axis=1), 1, atol=1e-5)
    sh = pool["sh"]
    assert abs(sh[:, 0].std() - 0.5) < 0.02 and abs(sh[:, 1:].std() - 0.05) < 0.002


def test_config0_scene_matches_its_description():
    """4,096 Gaussians (seed 0): means uniform in [-1, 1]^3, log-scales
    N(-3.5, 0.3), opacity logits N(0, 1); camera at (0, 0, -4) looking at
    the origin, 128x96, fx = fy = 110, centred principal point, near 0.01,
    far 100; uint8 target uniform on [0, 255] (seed 1)."""
    pool, cam, target = S.config0_scene()
    _check_pool(pool, 4096)
    assert pool["xyz"].min() >= -1 and pool["xyz"].max() <= 1
    assert abs(pool["log_scale"].mean() + 3.5) < 0.02 and abs(pool["log_scale"].std() - 0.3) < 0.02
    assert abs(pool["opacity"].mean()) < 0.05 and abs(pool["opacity"].std() - 1) < 0.05
    assert (cam.width, cam.height, cam.fx, cam.fy, cam.cx, cam.cy) == (128, 96, 110, 110, 64, 48)
    assert (cam.near, cam.far) == (0.01, 100.0)
    np.testing.assert_allclose(cam.center, [0, 0, -4], atol=1e-6)
    assert target.shape == (96, 128, 3) and target.dtype == np.uint8
    np.testing.assert_array_equal(
        target, np.random.default_rng(1).integers(0, 256, (96, 128, 3), dtype=np.uint8))
    again = S.config0_scene()[0]
    for k in pool:
        np.testing.assert_array_equal(pool[k], again[k])


def test_config1_scene_matches_its_description():
    """1,000,000 Gaussians (seed 2): 70% on a 20x20 ground patch at y = 0
    with N(0, 0.05) jitter, 30% uniform in a radius-10 sphere; log-scales
    N(-4, 0.6) with a per-axis jitter; opacity logits N(-1, 1.5); camera
    1237x822, fx = fy = 1040, eye (0, 1.5, -6) looking at the origin."""
    pool = S.config1_scene()
    n = 1_000_000
    _check_pool(pool, n)
    xyz = pool["xyz"]
    plane = xyz[:700_000]
    assert np.abs(plane[:, [0, 2]]).max() <= 10 and abs(plane[:, 1].std() - 0.05) < 0.002
    assert np.linalg.norm(xyz[700_000:], axis=1).max() <= 10
    per_point = pool["log_scale"].mean(axis=1)
    assert abs(per_point.mean() + 4) < 0.01 and abs(per_point.std() - 0.6) < 0.02
    assert abs(pool["opacity"].mean() + 1) < 0.01 and abs(pool["opacity"].std() - 1.5) < 0.01
    cam = S.config1_camera()
    assert (cam.width, cam.height, cam.fx, cam.fy) == (1237, 822, 1040, 1040)
    np.testing.assert_allclose(cam.center, [0, 1.5, -6], atol=1e-5)
    np.testing.assert_array_equal(S.config1_scene(n=1000)["xyz"], S.config1_scene(n=1000)["xyz"])


@pytest.mark.parametrize("radius", [6.0, 8.0])
def test_ring_cameras_look_at_the_origin(radius):
    """Configs 3-4: eight pinhole cameras on a ring of the given radius at
    height 1.5, 1237x822, fx = fy = 1040, each looking at the origin."""
    cams = S.ring_cameras(8, radius=radius)
    assert len(cams) == 8
    centres = np.array([c.center for c in cams])
    np.testing.assert_allclose(np.linalg.norm(centres[:, [0, 2]], axis=1), radius, rtol=1e-5)
    np.testing.assert_allclose(centres[:, 1], 1.5, atol=1e-5)
    for cam in cams:
        assert (cam.width, cam.height, cam.fx) == (1237, 822, 1040)
        origin = cam.world_to_camera @ np.array([0, 0, 0, 1.0])
        assert origin[2] > 0 and np.allclose(origin[:2], 0, atol=1e-4)


@pytest.mark.parametrize("qvec,tvec", [([1, 0, 0], [0, 0, 0]), ([1, 0, 0, 0], [0, 0])])
def test_camera_rejects_malformed_extrinsics(qvec, tvec):
    """tests/test_chex_contracts.py:31-34."""
    with pytest.raises(ValueError, match="quaternion"):
        S.Camera.from_colmap(qvec, tvec, 4, 4, 2, 2, 4, 4)
