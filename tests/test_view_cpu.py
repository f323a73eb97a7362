"""Inference host logic without a GPU (tests/test_viewer.py:23-62):
resize_camera keeps the pose and scales the intrinsics; ViewRenderer
refuses a model with no active Gaussians or an unsupported SH width before
touching the device."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def test_resize_camera_keeps_pose_and_scales_intrinsics():
    from jaxgs_b200.scene import Camera
    from jaxgs_b200.view import RESOLUTIONS, resize_camera

    camera = Camera.from_colmap([0.97, 0.1, -0.08, 0.18], [0.3, -0.2, 1.5], 500.0, 480.0,
                                320.0, 180.0, 640, 360)
    resized = resize_camera(camera, *RESOLUTIONS["1920x1080"])
    assert (resized.width, resized.height) == (1920, 1080)
    np.testing.assert_array_equal(resized.world_to_camera, camera.world_to_camera)
    np.testing.assert_allclose([resized.fx, resized.fy, resized.cx, resized.cy],
                               np.array([camera.fx, camera.fy, camera.cx, camera.cy]) * 3)


@pytest.mark.parametrize("invalid", ["empty", "sh"])
def test_renderer_rejects_invalid_models(invalid):
    from jaxgs_b200.scene import CapacityConfig, create_gaussians, seed_gaussians
    from jaxgs_b200.types import GaussianArrays
    from jaxgs_b200.view import ViewRenderer

    pool_np = seed_gaussians(create_gaussians(CapacityConfig(4, sh_degree=1)),
                             np.array([[0.0, 0.0, 2.0], [0.3, 0.1, 3.0]]),
                             np.array([[0.8, 0.2, 0.1], [0.2, 0.8, 0.3]]), scale=0.06, opacity=0.7)
    if invalid == "empty":
        pool_np["alive"][:] = False
    else:
        pool_np["sh"] = np.zeros((4, 2, 3), np.float32)
    pool = GaussianArrays.from_numpy(pool_np, device="cpu")
    with pytest.raises(ValueError, match="active Gaussians|SH dimension"):
        ViewRenderer(pool)
