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


def _seeded(capacity, points, cluster_size=1, scale=0.2, opacity=0.5):
    from jaxgs_b200.scene import CapacityConfig, create_gaussians, seed_gaussians
    from jaxgs_b200.types import GaussianArrays

    config = CapacityConfig(capacity, cluster_size, 4, 4, 0)
    pool_np = seed_gaussians(create_gaussians(config), np.asarray(points, np.float64),
                             np.ones((len(points), 3)), scale=scale, opacity=opacity)
    return GaussianArrays.from_numpy(pool_np), pool_np


def test_densify_step_prunes_and_appends_children():
    """tests/test_training_protocol.py:11-50: one budget plus the pruned
    slot's replacement gives two children; the parent is unchanged, the
    split child's scale is the parent's / 1.6, and the children's Adam
    state is zero."""
    from jaxgs_b200.densify import densify_step
    from jaxgs_b200.optimizer import create_adam_state

    pool, pool_np = _seeded(4, [[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]])
    state = create_adam_state(pool)
    for m in state.m:
        m.fill_(1.0)
    stats = torch.tensor([[3.0, 1.0, 2.0, 4.0], [0.0] * 4, [0.0] * 4, [0.0] * 4], device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(1)
    pool, state, born, removed = densify_step(pool, state, stats, gen, 1, 1.0, cluster_size=1)
    assert born == 2 and removed == 1
    np.testing.assert_array_equal(pool.xyz[0].cpu().numpy(), pool_np["xyz"][0])
    np.testing.assert_array_equal(pool.log_scale[0].cpu().numpy(), pool_np["log_scale"][0])
    np.testing.assert_allclose(pool.log_scale[1].cpu().numpy(),
                               pool_np["log_scale"][0] - np.log(1.6), rtol=1e-6)
    for m in state.m:
        assert float(m[1:3].abs().sum()) == 0
    assert pool.alive.cpu().numpy().tolist() == [1, 1, 1, 0]


def test_densify_step_percent_dense_splits_or_clones():
    """tests/test_training_protocol.py:53-78."""
    from jaxgs_b200.densify import densify_step
    from jaxgs_b200.optimizer import create_adam_state

    stats = torch.tensor([[3.0, 1.0, 2.0, 4.0], [0.0] * 4], device="cuda")
    for percent_dense, split in ((0.01, True), (1.0, False)):
        pool, pool_np = _seeded(2, [[1.0, 2.0, 3.0]], opacity=0.1)
        gen = torch.Generator(device="cuda").manual_seed(5)
        pool, _, born, _ = densify_step(pool, create_adam_state(pool), stats, gen, 2, 1.0,
                                        cluster_size=1, percent_dense=percent_dense)
        assert born == 1
        np.testing.assert_allclose(pool.log_scale[1].cpu().numpy(),
                                   pool_np["log_scale"][0] - (np.log(1.6) if split else 0),
                                   rtol=1e-6)
        same = np.array_equal(pool.xyz[1].cpu().numpy(), pool_np["xyz"][0])
        assert same != split


@pytest.mark.parametrize("pattern", ["split", "clone", "mixed"])
@pytest.mark.parametrize("capacity,active,target,cluster_size",
                         [(1, 0, 0, 1), (9, 9, 9, 2), (17, 7, 10, 1),
                          (257, 129, 257, 128)])
def test_densify_step_children_follow_the_sampled_parent_order(pattern, capacity, active,
                                                               target, cluster_size):
    """tests/test_training_protocol.py:81-147 with this generator's draws:
    children fill the first free slots in sampled order, splits before
    clones, and start with zero Adam state; live slots are unchanged."""
    from jaxgs_b200.densify import compute_densification_scores, densify_step
    from jaxgs_b200.optimizer import create_adam_state

    pool, pool_np = _seeded(capacity, np.zeros((active, 3)), cluster_size=cluster_size,
                            opacity=0.1)
    idx = np.arange(capacity)
    split = (idx % 2 == 0) if pattern == "mixed" else np.full(capacity, pattern == "split")
    pool.log_scale.copy_(torch.as_tensor(np.repeat(np.log(np.where(split, 0.2, 0.001))[:, None],
                                                   3, axis=1), dtype=torch.float32))
    pool.sh[:, 0, 0] = torch.arange(capacity, dtype=torch.float32)
    before = {k: getattr(pool, k).clone() for k in ("xyz", "log_scale", "sh")}
    stats = torch.tensor([3.0, 1.0, 2.0, 4.0], device="cuda").repeat(capacity, 1)
    state = create_adam_state(pool)
    for t in (*state.m, *state.v):
        t.fill_(1.0)
    gen = torch.Generator(device="cuda").manual_seed(23)
    replay = torch.Generator(device="cuda").manual_seed(23)
    scores, _ = compute_densification_scores(pool, stats)
    u = torch.rand(capacity, generator=replay, device="cuda")
    gumbel = -torch.log(-torch.log(torch.clamp(u, min=1e-20)))
    alive = pool.alive.bool()
    priorities = torch.where(alive, torch.log(torch.clamp(scores, min=1e-30)) + gumbel,
                             torch.full_like(scores, -np.inf))
    candidates = min(max(target - active, 1), active)
    sampled = torch.argsort(-priorities, stable=True)[:candidates].cpu().numpy()
    parents = np.concatenate((sampled[split[sampled]], sampled[~split[sampled]]))
    births = min(candidates // cluster_size * cluster_size,
                 (capacity - active) // cluster_size * cluster_size)
    pool, state, born, pruned = densify_step(pool, state, stats, gen, target, 1.0,
                                             cluster_size=cluster_size)
    assert born == births and pruned == 0
    children = slice(active, active + births)
    np.testing.assert_array_equal(pool.sh[children, 0, 0].cpu().numpy(), parents[:births])
    np.testing.assert_allclose(
        pool.log_scale[children].cpu().numpy(),
        before["log_scale"].cpu().numpy()[parents[:births]]
        - np.where(split[parents[:births], None], np.log(1.6), 0), atol=2e-7)
    assert torch.equal(pool.xyz[:active], before["xyz"][:active])
    for t in (*state.m, *state.v, state.step):
        assert float(t[children].abs().sum()) == 0
