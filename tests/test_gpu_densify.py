"""Density-control consumers on the GPU (gsb_densify_scores,
gsb_decay_opacity) against the oracle's float64 restatements."""

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_densification_scores_and_decay_match_oracle():
    from jaxgs_b200.densify import compute_densification_scores, decay_opacity
    from jaxgs_b200.scene import CapacityConfig, create_gaussians, seed_gaussians
    from jaxgs_b200.types import GaussianArrays

    rng = np.random.default_rng(4)
    config = CapacityConfig(5000, 128, 2, 16, 3)
    pool_np = seed_gaussians(create_gaussians(config), rng.normal(0, 1, (4000, 3)),
                             rng.random((4000, 3)), scale=0.1, opacity=0.3)
    pool_np["opacity"] = rng.normal(0, 2, (5000, 1)).astype(np.float32)
    stats = np.stack([rng.integers(0, 50, 5000).astype(np.float32),
                      rng.random(5000).astype(np.float32) * (rng.random(5000) < 0.8),
                      rng.normal(0, 1, 5000).astype(np.float32),
                      rng.random(5000).astype(np.float32) * 5], 1)
    stats[7] = [np.inf, 1.0, 0.0, 1.0]  # a non-finite score is zeroed
    pool = GaussianArrays.from_numpy(pool_np)
    scores, prune = compute_densification_scores(pool, torch.as_tensor(stats, device="cuda"))
    torch.cuda.synchronize()
    exp_scores, exp_prune = O.densification_scores(pool_np["opacity"], pool_np["alive"], stats)
    # float32 against float64: the variance cancels, so the bound is absolute
    # at the scores' scale as well as relative.
    np.testing.assert_allclose(scores.cpu().numpy(), exp_scores, rtol=1e-5, atol=1e-7)
    np.testing.assert_array_equal(prune.cpu().numpy(), exp_prune)
    assert scores[7].item() == 0.0 and exp_prune.sum() > 0
    _, state = decay_opacity(pool)
    torch.cuda.synchronize()
    np.testing.assert_allclose(pool.opacity.cpu().numpy().reshape(-1),
                               O.decay_opacity(pool_np["opacity"], pool_np["alive"]),
                               rtol=1e-5, atol=1e-5)
    assert all(float(m.abs().sum()) == 0 for m in state.m)
