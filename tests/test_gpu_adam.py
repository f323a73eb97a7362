"""Visible-cluster sparse Adam on the GPU (gsb_sparse_adam) against the
oracle's restatement of kernels/sparse_adam.py:16-54, bit for bit: both
round every operation to float32 in the same order."""

import numpy as np
import pytest

from oracle import oracle as O
from tests.test_oracle_cpu import ADAM_RATES

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

NAMES = ("xyz", "log_scale", "rotation", "opacity", "sh")


def _dev(a, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a), device="cuda")
    return t if dtype is None else t.to(dtype)


def test_known_answer_sparse_adam_on_gpu():
    """tests/test_training_protocol.py:201-224 through sparse_adam_update."""
    from jaxgs_b200.optimizer import create_adam_state, sparse_adam_update
    from jaxgs_b200.scene import CapacityConfig, create_gaussians, seed_gaussians
    from jaxgs_b200.types import GaussianArrays

    config = CapacityConfig(2, 1, 2, 4, 1)
    pool_np = seed_gaussians(create_gaussians(config), np.ones((2, 3)), np.ones((2, 3)))
    pool = GaussianArrays.from_numpy(pool_np)
    state = create_adam_state(pool)
    grads = tuple(torch.ones_like(getattr(pool, n)) for n in NAMES)
    clusters = (_dev(np.array([0, 1], np.int32)), _dev(np.array([1], np.int32)))
    visible = _dev(np.array([True, False]))
    sparse_adam_update(pool, state, grads, visible, 0, 2.0, compacted_clusters=clusters,
                       cluster_size=1)
    torch.cuda.synchronize()
    for name, rate in zip(NAMES[:4], (0.00032, 0.005, 0.001, 0.025)):
        got = getattr(pool, name).cpu().numpy()
        np.testing.assert_allclose(got[0], pool_np[name][0] - rate * 0.1 / np.sqrt(0.001),
                                   atol=1e-6)
        np.testing.assert_array_equal(got[1], pool_np[name][1])
    sh = pool.sh.cpu().numpy()
    np.testing.assert_allclose(sh[0, 0], pool_np["sh"][0, 0] - 0.0025 * np.sqrt(10), atol=1e-6)
    np.testing.assert_allclose(sh[0, 1], pool_np["sh"][0, 1] - 0.00025 * np.sqrt(10), atol=1e-6)
    np.testing.assert_array_equal(sh[1], pool_np["sh"][1])
    np.testing.assert_array_equal(state.step.cpu().numpy(), [1, 0])


@pytest.mark.parametrize("cluster_size,compact", [(128, False), (128, True), (3, False), (5, True)])
def test_sparse_adam_fields_match_oracle_bit_exact(cluster_size, compact):
    """Random values, moments and gradients on 1000 slots (the last cluster
    partial), holes in the alive mask, a subset of clusters listed: every
    field (3, 3, 4, 1 and 48 channels) equals the oracle exactly, and every
    element outside the listed alive slots is unchanged."""
    from jaxgs_b200.optimizer import update_field

    rng = np.random.default_rng(cluster_size * 7 + compact)
    capacity = 1000
    n_clusters = -(-capacity // cluster_size)
    listed = np.sort(rng.choice(n_clusters, size=max(1, n_clusters // 2), replace=False))
    ids = np.zeros(n_clusters, np.int32)
    ids[:len(listed)] = listed
    count = len(listed)
    alive = (rng.random(capacity) < 0.9).astype(np.uint8)
    rates = O.parameter_learning_rates(77, 1.5, 30000, **ADAM_RATES)
    for name, ch, rate in zip(NAMES, (3, 3, 4, 1, 48), rates):
        value = rng.normal(0, 1, capacity * ch).astype(np.float32)
        mean = rng.normal(0, 0.1, capacity * ch).astype(np.float32)
        var = rng.random(capacity * ch).astype(np.float32) * 0.01
        grad_pool = rng.normal(0, 0.3, capacity * ch).astype(np.float32)
        if compact:
            slots = (ids[:count, None] * cluster_size + np.arange(cluster_size)).reshape(-1)
            grad = np.zeros(count * cluster_size * ch, np.float32)
            ok = slots < capacity
            grad.reshape(-1, ch)[ok] = grad_pool.reshape(-1, ch)[slots[ok]]
        else:
            grad = grad_pool
        exp = O.sparse_adam(value, mean, var, grad, alive, ids, count, rate,
                            cluster_size=cluster_size, is_sh=name == "sh",
                            compact_gradients=compact)
        x, m, v = _dev(value), _dev(mean), _dev(var)
        update_field(x, m, v, _dev(grad), _dev(alive), (_dev(ids), _dev(np.array([count], np.int32))),
                     float(rate), cluster_size, name == "sh", compact)
        torch.cuda.synchronize()
        for got, ref in zip((x, m, v), exp):
            np.testing.assert_array_equal(got.cpu().numpy(), ref, err_msg=name)
        touched = np.zeros(capacity, bool)
        for c in listed:
            touched[c * cluster_size:(c + 1) * cluster_size] = True
        touched &= alive.astype(bool)
        untouched = np.repeat(~touched, ch)
        np.testing.assert_array_equal(x.cpu().numpy()[untouched], value[untouched])
        assert np.mean(x.cpu().numpy()[~untouched] != value[~untouched]) > 0.99


def test_sparse_adam_after_the_training_step():
    """The step's compact gradients feed sparse_adam_update directly
    (training/step.py:110-122 order): pool and moments equal the oracle's
    update of the same gradients."""
    from jaxgs_b200.optimizer import create_adam_state, sparse_adam_update
    from jaxgs_b200.scene import CapacityConfig, config0_scene, world_cluster_bounds
    from jaxgs_b200.step import compute_training_step
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    pool_np, cam, target = config0_scene()
    n = pool_np["xyz"].shape[0]
    config = CapacityConfig(n, 128, 16, 16, 3, n * 64, tile_height=8)
    c, e, v = world_cluster_bounds(pool_np, 128)
    bounds = (_dev(c), _dev(e), _dev(v.astype(np.uint8)))
    pool = GaussianArrays.from_numpy(pool_np)
    out = compute_training_step(pool, bounds, DeviceCamera.from_camera(cam), _dev(target), config, 3)
    state = create_adam_state(pool)
    ids = out.visible_clusters[0].cpu().numpy()
    count = int(out.visible_clusters[1].item())
    grads_np = [g.cpu().numpy().reshape(-1) for g in out.gradients]
    visible = torch.zeros(n, dtype=torch.bool, device="cuda")
    for cl in ids[:count]:
        visible[cl * 128:(cl + 1) * 128] = True
    sparse_adam_update(pool, state, out.gradients, visible, 10, 3.0,
                       compacted_clusters=out.visible_clusters, compact_gradients=True)
    torch.cuda.synchronize()
    rates = O.parameter_learning_rates(10, 3.0, 30000, **ADAM_RATES)
    for i, name in enumerate(NAMES):
        field = pool_np[name].reshape(-1)
        exp = O.sparse_adam(field, np.zeros_like(field), np.zeros_like(field), grads_np[i],
                            pool_np["alive"], ids, count, rates[i], cluster_size=128,
                            is_sh=name == "sh", compact_gradients=True)
        np.testing.assert_array_equal(getattr(pool, name).cpu().numpy().reshape(-1), exp[0])
        np.testing.assert_array_equal(state.m[i].cpu().numpy().reshape(-1), exp[1])
    assert int(state.step.sum().item()) == int((visible.cpu().numpy() & pool_np["alive"]).sum())


@pytest.mark.parametrize("degree,views,cluster_size,compact",
                         [(3, 1, 128, True), (3, 3, 128, False), (1, 2, 5, True), (0, 1, 128, False),
                          (2, 1, 200, True)])
def test_sh_adam_from_colours_equals_expansion_then_update(degree, views, cluster_size, compact):
    """gsb_sparse_adam_sh (SH gradient rebuilt inside the update) against the
    unfused pair it replaces, gsb_sh_from_colors (training/sh_pullback.py:18-53)
    then gsb_sparse_adam on the materialised [C, 16, 3] gradient: value and
    both moments bit for bit, with dead slots, zero colour rows, a partial
    last cluster and clusters of more than one block of slots."""
    from jaxgs_b200 import kernels as K
    from jaxgs_b200.optimizer import update_field, update_sh_from_colors

    rng = np.random.default_rng(degree * 31 + views * 7 + cluster_size)
    capacity, sh_dim = 1000, 16
    n_clusters = -(-capacity // cluster_size)
    listed = np.sort(rng.choice(n_clusters, size=max(1, n_clusters // 2), replace=False))
    ids = np.zeros(n_clusters, np.int32)
    ids[:len(listed)] = listed
    count = len(listed)
    clusters = (_dev(ids), _dev(np.array([count], np.int32)))
    alive = (rng.random(capacity) < 0.9).astype(np.uint8)
    xyz = rng.normal(0, 3, (capacity, 3)).astype(np.float32)
    centers = rng.normal(0, 6, (views, 3)).astype(np.float32)
    colors = rng.normal(0, 0.2, (views, capacity, 3)).astype(np.float32)
    colors[:, rng.random(capacity) < 0.3] = 0.0  # slots a view does not see
    value = rng.normal(0, 1, (capacity, sh_dim, 3)).astype(np.float32)
    mean = rng.normal(0, 0.1, value.shape).astype(np.float32)
    var = (rng.random(value.shape) * 0.01).astype(np.float32)
    rate = float(O.parameter_learning_rates(5, 1.0, 30000, **ADAM_RATES)[4])

    gsh = K.sh_from_colors(_dev(xyz), _dev(centers), _dev(colors), degree, sh_dim)
    x0, m0, v0 = _dev(value), _dev(mean), _dev(var)
    update_field(x0, m0, v0, gsh, _dev(alive), clusters, rate, cluster_size, True, False)

    if compact:
        # The listed clusters' rows in list order; ids are sorted, so only
        # the last listed cluster can be partial and the prefix fits in C
        # rows.  Rows past it are NaN: they must never be read.
        slots = (ids[:count, None] * cluster_size + np.arange(cluster_size)).reshape(-1)
        slots = slots[slots < capacity]
        given = np.full((views, capacity, 3), np.nan, np.float32)
        given[:, :len(slots)] = colors[:, slots]
    else:
        given = colors
    x1, m1, v1 = _dev(value), _dev(mean), _dev(var)
    update_sh_from_colors(x1, m1, v1, _dev(xyz), _dev(centers), _dev(given), _dev(alive),
                          clusters, rate, cluster_size, degree, compact)
    torch.cuda.synchronize()
    for got, ref, what in ((x1, x0, "value"), (m1, m0, "mean"), (v1, v0, "variance")):
        assert torch.equal(got, ref), what
    assert not torch.equal(x1, _dev(value))


def test_sparse_adam_update_with_sh_pullback_center_equals_the_unfused_update():
    """sparse_adam_update(..., sh_pullback_center=camera centre) on the
    step's sh_color_only gradients (training/step.py:55-66 and :95-111, the
    reference's deferred SH update) equals the unfused update of the same
    gradients: the colour cotangent expanded by gsb_sh_from_colors at the
    positions before the update, then gsb_sparse_adam on every field; all
    fields and moments bit for bit, and the step counts alike."""
    from jaxgs_b200 import kernels as K
    from jaxgs_b200.optimizer import (create_adam_state, parameter_learning_rates,
                                      sparse_adam_update, update_field)
    from jaxgs_b200.scene import CapacityConfig, config0_scene, world_cluster_bounds
    from jaxgs_b200.step import compute_training_step
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    pool_np, cam, target = config0_scene()
    n = pool_np["xyz"].shape[0]
    config = CapacityConfig(n, 128, 16, 16, 3, n * 64, tile_height=8)
    c, e, v = world_cluster_bounds(pool_np, 128)
    bounds = (_dev(c), _dev(e), _dev(v.astype(np.uint8)))
    dcam = DeviceCamera.from_camera(cam)
    pool = GaussianArrays.from_numpy(pool_np)
    out = compute_training_step(pool, bounds, dcam, _dev(target), config, 2, sh_color_only=True)
    assert out.gradients[4].numel() == n * 3
    count = int(out.visible_clusters[1].item())
    listed = out.visible_clusters[0][:count].long()
    slots = (listed[:, None] * 128 + torch.arange(128, device="cuda")).reshape(-1)
    slots = slots[slots < n]
    visible = torch.zeros(n, dtype=torch.bool, device="cuda")
    visible[slots] = True

    state = create_adam_state(pool)
    sparse_adam_update(pool, state, out.gradients, visible, 10, 3.0,
                       compacted_clusters=out.visible_clusters, compact_gradients=True,
                       sh_pullback_center=dcam.center, active_degree=2)

    ref = GaussianArrays.from_numpy(pool_np)
    ref_state = create_adam_state(ref)
    colors = torch.zeros(n, 3, device="cuda")
    colors[slots] = out.gradients[4].reshape(-1, 3)[:slots.numel()]
    gsh = K.sh_from_colors(ref.xyz, dcam.center.reshape(1, 3), colors[None], 2, 16)
    rates = parameter_learning_rates(10, 3.0)
    for i, name in enumerate(NAMES):
        grad = gsh if name == "sh" else out.gradients[i]
        update_field(getattr(ref, name), ref_state.m[i], ref_state.v[i], grad.contiguous(),
                     ref.alive, out.visible_clusters, rates[i], 128, name == "sh",
                     name != "sh")
    torch.cuda.synchronize()
    for i, name in enumerate(NAMES):
        assert torch.equal(getattr(pool, name), getattr(ref, name)), name
        assert torch.equal(state.m[i], ref_state.m[i]) and torch.equal(state.v[i],
                                                                      ref_state.v[i]), name
    assert not torch.equal(pool.sh, GaussianArrays.from_numpy(pool_np).sh)
    assert int(state.step.sum().item()) == int((visible & pool.alive.bool()).sum().item())
