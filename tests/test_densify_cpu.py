"""refresh_cluster_bounds (torch, any device) against the host
scene.world_cluster_bounds (scene/cluster.py:15-37): the same boxes,
written into the existing tensors."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("capacity,cluster_size", [(1000, 128), (257, 65), (128, 128)])
def test_refresh_cluster_bounds_matches_host_bounds(capacity, cluster_size):
    from jaxgs_b200.densify import refresh_cluster_bounds
    from jaxgs_b200.scene import world_cluster_bounds
    from jaxgs_b200.types import GaussianArrays

    rng = np.random.default_rng(capacity)
    pool_np = {
        "xyz": rng.normal(0, 2, (capacity, 3)).astype(np.float32),
        "log_scale": rng.normal(-3, 0.5, (capacity, 3)).astype(np.float32),
        "rotation": rng.normal(0, 1, (capacity, 4)).astype(np.float32),
        "opacity": np.zeros((capacity, 1), np.float32),
        "sh": np.zeros((capacity, 1, 3), np.float32),
        "alive": rng.random(capacity) < 0.7,
    }
    pool_np["alive"][:cluster_size] = False  # a cluster with nothing alive
    pool = GaussianArrays.from_numpy(pool_np, device="cpu")
    n = -(-capacity // cluster_size)
    bounds = (torch.full((n, 3), 7.0), torch.full((n, 3), 7.0), torch.full((n,), 9, dtype=torch.uint8))
    keep = [t.data_ptr() for t in bounds]
    refresh_cluster_bounds(pool, bounds, cluster_size)
    assert [t.data_ptr() for t in bounds] == keep
    center, extent, valid = world_cluster_bounds(pool_np, cluster_size)
    np.testing.assert_array_equal(bounds[2].numpy(), valid.astype(np.uint8))
    assert not valid[0]
    np.testing.assert_allclose(bounds[0].numpy(), center, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(bounds[1].numpy(), extent, rtol=1e-6, atol=1e-6)
    with pytest.raises(ValueError, match="clusters"):
        refresh_cluster_bounds(pool, (bounds[0][: n - 1], bounds[1], bounds[2]), cluster_size)
