"""jaxgs_b200.autograd on the GPU: loss = fused_loss(render(pool)[0], target,
clip_input=True); loss.backward() gives the fp32 step's loss and, on every
parameter tensor, its gradient in pool order -- checked against the
oracle's step with the fp32 conventions (rasterize_loss_and_grad, loss on
clip(rgb, 0, 1)) at the north-star bars: loss 1e-5 relative, gradients 1e-3
relative L2; rows of culled clusters are zero.  The counterpart of the
reference's custom_vjp rules (kernels/projector.py:152-224,
kernels/sorted_rasterizer.py:165-236, kernels/fused_loss.py:333-352).
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

NAMES = ("xyz", "log_scale", "rotation", "opacity", "sh")


def test_autograd_render_and_loss_match_the_oracle_step():
    from jaxgs_b200 import kernels as K
    from jaxgs_b200.autograd import fused_loss, render
    from jaxgs_b200.scene import CapacityConfig, config0_scene, world_cluster_bounds
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    pool_np, cam, target = config0_scene()
    n = pool_np["xyz"].shape[0]
    # Some dead slots: their rows stay zero.
    pool_np = dict(pool_np)
    pool_np["alive"] = pool_np["alive"].copy()
    pool_np["alive"][::17] = False
    config = CapacityConfig(n, 128, 16, 16, 3, n * 64, tile_height=8)
    bounds = tuple(torch.as_tensor(a, device="cuda") for a in world_cluster_bounds(pool_np, 128))
    bounds = (bounds[0], bounds[1], bounds[2].to(torch.uint8))
    params = {k: torch.as_tensor(np.ascontiguousarray(pool_np[k]), device="cuda").requires_grad_()
              for k in NAMES}
    alive = torch.as_tensor(pool_np["alive"].astype(np.uint8), device="cuda")
    pool = GaussianArrays(**params, alive=alive)
    dcam = DeviceCamera.from_camera(cam)
    rgb, overflow = render(pool, bounds, dcam, config, 3)
    loss = fused_loss(rgb, torch.as_tensor(target, device="cuda"), clip_input=True)
    loss.backward()
    clusters, _ = K.compact_visible_clusters(bounds, dcam, config, want_slots=False)
    torch.cuda.synchronize()
    assert not bool(overflow.item())
    ids = clusters[0].cpu().numpy()
    count = int(clusters[1].item())
    exp = O.training_step(pool_np, cam, target, degree=3, sh_dim=16, tile_w=16, tile_h=8,
                          max_pairs=n * 64, clusters=(ids, count), packed=False)
    assert abs(float(loss) - exp["loss"]) <= 1e-5 * abs(exp["loss"]), (float(loss), exp["loss"])
    slots = (ids[:count, None] * 128 + np.arange(128)).reshape(-1)
    listed = np.zeros(n, bool)
    listed[slots] = True
    for name in NAMES:
        g = params[name].grad.detach().cpu().numpy().reshape(n, -1)
        r = exp["grads"][NAMES.index(name)].reshape(n, -1)[: count * 128]
        err = rel_l2(g[slots], r)
        assert err < 1e-3, (name, err)
        assert not g[~listed].any(), name
