"""Inference rendering: the RGB-only raster forward (no backward state)
and ViewRenderer (render/view.py:37-80)."""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import torch_proj

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("tile_h,tile_w", [(8, 16), (12, 16), (16, 16)])
def test_rgb_only_forward_equals_the_recording_forward(tile_h, tile_w):
    """record=False composites exactly as the training forward: the same
    image, depth and alpha bit for bit, and no cache."""
    from jaxgs_b200 import kernels as K
    from jaxgs_b200.scene import CapacityConfig
    from jaxgs_b200.types import DeviceCamera, SortedVisibilityTable
    from tests.test_gpu_parity import _raster_case

    W, H = 67, 45
    proj, table = _raster_case(41, W, H, tw=tile_w, th=tile_h)
    c = len(proj["alpha"])
    config = CapacityConfig(c, 128, 1, tile_w, 0, len(table["gaussian_ids"]), tile_height=tile_h)
    t_table = SortedVisibilityTable(*(torch.as_tensor(table[k], device="cuda") for k in
                                      ("gaussian_ids", "tile_offsets", "point_counts")),
                                    torch.tensor([table["pair_count"]], device="cuda"),
                                    torch.tensor([0], device="cuda"))
    cam = DeviceCamera(None, None, None, None, W, H)
    projected = torch_proj(proj)
    bg = torch.tensor([0.2, 0.1, 0.3], device="cuda")
    full, cache = K.rasterize_forward(projected, t_table, cam, config, bg)
    rgb_only, none = K.rasterize_forward(projected, t_table, cam, config, bg, record=False)
    torch.cuda.synchronize()
    assert cache is not None and none is None
    for a, b in ((full.rgb, rgb_only.rgb), (full.depth, rgb_only.depth),
                 (full.alpha, rgb_only.alpha)):
        assert torch.equal(a, b)
    exp = O.raster_fwd(proj, table, W, H, tile_w, tile_h, bg.cpu().numpy())
    ok = exp["ambiguous"] == 0
    np.testing.assert_allclose(rgb_only.rgb.cpu().numpy().reshape(-1, 3)[ok],
                               exp["rgb"].reshape(-1, 3)[ok], atol=1e-4)


def test_view_renderer_frames():
    """ViewRenderer's uint8 frame is rint(clip(rgb) * 255) of the training
    forward for that view; a graph replay with another camera of the same
    resolution equals an eager frame of that camera; presets render."""
    from jaxgs_b200 import kernels as K
    from jaxgs_b200.scene import Camera, CapacityConfig, config0_scene
    from jaxgs_b200.types import DeviceCamera, GaussianArrays
    from jaxgs_b200.view import ViewRenderer, resize_camera

    pool_np, cam, _ = config0_scene()
    pool = GaussianArrays.from_numpy(pool_np)
    renderer = ViewRenderer(pool, pair_capacity=1 << 20)
    image, overflow = renderer(cam)
    torch.cuda.synchronize()
    assert image.dtype == torch.uint8 and tuple(image.shape) == (cam.height, cam.width, 3)
    assert int(overflow.item()) == 0
    # The training forward of the same view.
    config = renderer.config
    dcam = DeviceCamera.from_camera(cam)
    clusters, _ = K.compact_visible_clusters(renderer.bounds, dcam, config, want_slots=False)
    projected = K.project_cute(pool, dcam, config, config.sh_degree, clusters)
    table = K.build_sorted_visibility_table_cute(projected, dcam, config)
    full, _ = K.rasterize_forward(projected, table, dcam, config, want_depth=False,
                                  want_alpha=False)
    expected = torch.round(full.rgb.clamp(0, 1) * 255).to(torch.uint8)
    assert torch.equal(image, expected)
    assert image.float().mean().item() > 1.0
    other = Camera.look_at((1.0, 0.3, -3.2), (0.2, 0.0, 0.0), cam.fx, cam.fy, cam.width,
                           cam.height, near=cam.near, far=cam.far)
    replayed, _ = renderer(other)
    replayed = replayed.clone()
    eager = ViewRenderer(pool, pair_capacity=1 << 20, graphs=False)(other)[0]
    torch.cuda.synchronize()
    assert torch.equal(replayed, eager)
    assert not torch.equal(replayed, image)
    small = resize_camera(cam, 64, 48)
    assert (small.fx, small.cx) == (float(np.float32(cam.fx) * np.float32(0.5)),
                                    float(np.float32(cam.cx) * np.float32(0.5)))
    img_small, _ = renderer(small)
    torch.cuda.synchronize()
    assert tuple(img_small.shape) == (48, 64, 3)
