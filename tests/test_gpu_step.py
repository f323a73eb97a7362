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
