"""sparse_adam_update refuses an incompatible call before any launch
(tests/test_chex_contracts.py:57-76): a mask that is not one flag per
slot, moments of another shape, a gradient of another dtype or size (in
pool or compact order); the pool and the state stay as they were."""

import dataclasses

import numpy as np
import pytest

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("invalid", ["mask", "moment_shape", "gradient_dtype", "gradient_rows",
                                     "compact_short"])
def test_sparse_adam_update_rejects_incompatible_state(invalid):
    from jaxgs_b200.optimizer import create_adam_state, sparse_adam_update
    from jaxgs_b200.scene import CapacityConfig, create_gaussians, seed_gaussians
    from jaxgs_b200.types import GaussianArrays

    pool_np = seed_gaussians(create_gaussians(CapacityConfig(2, sh_degree=1)), np.ones((1, 3)),
                             np.full((1, 3), 0.5))
    pool = GaussianArrays.from_numpy(pool_np, device="cpu")
    state = create_adam_state(pool)
    names = ("xyz", "log_scale", "rotation", "opacity", "sh")
    gradients = [torch.ones_like(getattr(pool, n)) for n in names]
    visible = pool.alive.to(torch.bool)
    message = {"mask": "one flag per pool slot", "moment_shape": "moments",
               "gradient_dtype": "float32", "gradient_rows": "field's size",
               "compact_short": "field's size"}[invalid]
    if invalid == "mask":
        visible = visible[:, None]
    elif invalid == "moment_shape":
        state = dataclasses.replace(state, m=(torch.zeros(1, 3), *state.m[1:]))
    elif invalid == "gradient_dtype":
        gradients[4] = gradients[4].double()
    elif invalid == "gradient_rows":
        gradients[4] = torch.ones(2, 1, 3)
    else:
        # A compact gradient shorter than the field: the listed clusters'
        # rows (known only on the device) could reach past it.
        gradients[0] = torch.ones(1, 3)
    before = [getattr(pool, n).clone() for n in names]
    clusters = (torch.zeros(2, dtype=torch.int32), torch.ones(1, dtype=torch.int32))
    with pytest.raises(ValueError, match=message):
        sparse_adam_update(pool, state, gradients, visible, 0, 1.0, compacted_clusters=clusters,
                           cluster_size=1, compact_gradients=invalid == "compact_short")
    for n, b in zip(names, before):
        assert torch.equal(getattr(pool, n), b)
    assert int(state.step.sum()) == 0


@pytest.mark.parametrize("invalid", ["center_and_rows", "center_size", "colour_size", "degree",
                                     "rows_shape"])
def test_deferred_sh_arguments_are_checked_before_any_update(invalid):
    """The deferred-SH forms of sparse_adam_update (sh_pullback_center: the
    colour cotangent of one view; sh_pullback_rows: the gathered rows of the
    view-sharded exchange) refuse inconsistent arguments on the host, with
    the pool and the state untouched."""
    from jaxgs_b200.optimizer import create_adam_state, sparse_adam_update
    from jaxgs_b200.scene import CapacityConfig, create_gaussians, seed_gaussians
    from jaxgs_b200.types import GaussianArrays

    pool_np = seed_gaussians(create_gaussians(CapacityConfig(2, sh_degree=1)), np.ones((1, 3)),
                             np.full((1, 3), 0.5))
    pool = GaussianArrays.from_numpy(pool_np, device="cpu")
    state = create_adam_state(pool)
    names = ("xyz", "log_scale", "rotation", "opacity", "sh")
    gradients = [torch.ones_like(getattr(pool, n)) for n in names]
    gradients[4] = torch.ones(2, 1, 3)  # colour cotangents
    center, rows, degree = torch.zeros(3), None, 1
    message = {"center_and_rows": "not both", "center_size": "one camera centre",
               "colour_size": "3 floats per slot", "degree": "does not fit",
               "rows_shape": "colour rows"}[invalid]
    if invalid == "center_and_rows":
        rows = torch.zeros(1, 4 + 6)
    elif invalid == "center_size":
        center = torch.zeros(2)
    elif invalid == "colour_size":
        gradients[4] = torch.ones(2, 2, 3)
    elif invalid == "degree":
        degree = 2  # 9 coefficients in a pool of 4
    else:
        center, rows = None, torch.zeros(2, 4 + 5)  # one float short of C * 3
    before = [getattr(pool, n).clone() for n in names]
    clusters = (torch.zeros(2, dtype=torch.int32), torch.ones(1, dtype=torch.int32))
    with pytest.raises(ValueError, match=message):
        sparse_adam_update(pool, state, gradients, pool.alive.to(torch.bool), 0, 1.0,
                           compacted_clusters=clusters, cluster_size=1, compact_gradients=False,
                           sh_pullback_center=center, sh_pullback_rows=rows,
                           active_degree=degree)
    for n, b in zip(names, before):
        assert torch.equal(getattr(pool, n), b)
    assert all(float(m.abs().sum()) == 0.0 for m in state.m)
