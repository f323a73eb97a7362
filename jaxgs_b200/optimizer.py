"""Visible-cluster sparse Adam, the consumer of the step's gradients.

Mirrors training/optimizer.py:18-27 (AdamState, create_adam_state),
:93-120 (the per-field learning rates) and :276-341 (sparse_adam_update
with compacted clusters), each field updated in place by one
gsb_sparse_adam launch (kernels/sparse_adam.py:16-136).  LiteGS Adam: no
bias correction, eps 1e-15, moments frozen in slots that are not updated.

With sh_pullback_center (training/optimizer.py:180-261), the SH gradient is
the step's colour cotangent (the sh_color_only pullback) and the SH field's
update rebuilds the coefficient gradients itself (gsb_sparse_adam_sh, the
deferred pullback of training/sh_pullback.py:18-53 fused into the update).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib as L
from .types import GaussianArrays

PARAMETER_NAMES = ("xyz", "log_scale", "rotation", "opacity", "sh")


@dataclass(frozen=True)
class OptimizationConfig:
    """The optimisation rates of config/training.py:33-44 with the values of
    config/default.toml:24-30."""

    position_lr_init: float = 0.00016
    position_lr_final: float = 0.0000016
    position_lr_max_steps: int = 30000
    feature_lr: float = 0.0025
    opacity_lr: float = 0.025
    scaling_lr: float = 0.005
    rotation_lr: float = 0.001


@dataclass
class AdamState:
    """training/optimizer.py:18-21: first and second moments per field and
    the per-slot count of updates."""

    m: tuple
    v: tuple
    step: torch.Tensor  # [C] int32


def create_adam_state(pool: GaussianArrays) -> AdamState:
    """Zero moments shaped like the pool's fields (training/optimizer.py:24-27)."""
    fields = [getattr(pool, name) for name in PARAMETER_NAMES]
    return AdamState(tuple(torch.zeros_like(f) for f in fields),
                     tuple(torch.zeros_like(f) for f in fields),
                     torch.zeros(pool.xyz.shape[0], dtype=torch.int32, device=pool.xyz.device))


def reset_adam_slots(state: AdamState, slot_mask: torch.Tensor) -> AdamState:
    """training/optimizer.py:78-90: zero both moments and the update count
    of the masked slots, in place."""
    mask = slot_mask.to(torch.bool)
    for moments in (state.m, state.v):
        for t in moments:
            t[mask] = 0
    state.step[mask] = 0
    return state


def parameter_learning_rates(step: float, spatial_scale: float, max_steps: int | None = None,
                             optimization: OptimizationConfig = OptimizationConfig()):
    """training/optimizer.py:93-120: rates of (xyz, log_scale, rotation,
    opacity, sh).  The position rate decays log-linearly from init to final
    over max_steps (position_lr_max_steps by default), scaled by the scene's
    spatial scale; the SH rate is feature_lr / 10, the DC coefficient's x10
    being applied per channel by the update."""
    o = optimization
    frac = min(max(float(step) / float(max_steps or o.position_lr_max_steps), 0.0), 1.0)
    if o.position_lr_init == o.position_lr_final == 0:
        position = 0.0
    else:
        position = float(spatial_scale) * math.exp(math.log(o.position_lr_init) * (1 - frac)
                                                   + math.log(o.position_lr_final) * frac)
    return position, o.scaling_lr, o.rotation_lr, o.opacity_lr, o.feature_lr / 10


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def update_field(value: torch.Tensor, mean: torch.Tensor, variance: torch.Tensor,
                 gradient: torch.Tensor, alive: torch.Tensor, clusters, rate,
                 cluster_size: int, is_sh: bool, compact_gradients: bool):
    """kernels/sparse_adam.py:98-136: one field's update, in place on value,
    mean and variance (contiguous float32 on the GPU).  rate: a float or a
    device float tensor of one element; clusters: (ids, count) on the device.
    Returns (value, mean, variance)."""
    if value.shape != mean.shape or value.shape != variance.shape:
        raise ValueError("value and moments must have one shape")
    if gradient.dim() > 1 and tuple(gradient.shape[1:]) != tuple(value.shape[1:]):
        raise ValueError("gradient rows must have the field's shape (every SH coefficient)")
    capacity = int(alive.shape[0])
    if capacity == 0:
        return value, mean, variance
    channels = value.numel() // capacity
    if channels * capacity != value.numel():
        raise ValueError("field size must be capacity x channels")
    for t in (value, mean, variance, gradient):
        if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("sparse Adam needs contiguous float32 CUDA tensors")
    ids, count = clusters
    if not torch.is_tensor(rate):
        rate = torch.full((1,), float(rate), dtype=torch.float32, device=value.device)
    if alive.dtype == torch.int8:
        alive8 = alive
    elif alive.dtype == torch.uint8:
        alive8 = alive.view(torch.int8)
    else:
        alive8 = alive.to(torch.int8)
    p = L.AdamParams(capacity, channels, int(cluster_size), int(is_sh), int(compact_gradients))
    ptr = lambda t: t.data_ptr()
    L.check(L.lib.gsb_sparse_adam(_stream(), L.ref(p), ptr(value), ptr(mean), ptr(variance),
                                  ptr(gradient), ptr(alive8.contiguous()),
                                  ptr(ids.to(torch.int32).contiguous()),
                                  ptr(count.to(torch.int32).contiguous()),
                                  ptr(rate.to(torch.float32).contiguous())),
            "sparse Adam")
    return value, mean, variance


def update_sh_from_colors(sh: torch.Tensor, mean: torch.Tensor, variance: torch.Tensor,
                          xyz: torch.Tensor, centers: torch.Tensor, colors: torch.Tensor,
                          alive: torch.Tensor, clusters, rate, cluster_size: int, degree: int,
                          compact_colors: bool):
    """The SH field's sparse Adam with its gradient rebuilt from colour
    cotangents (gsb_sparse_adam_sh): for every alive slot of the listed
    clusters, g[k][c] = sum over views of Y_k(direction from the view's
    centre) * colour[c] for k < (degree + 1)^2 and 0 above, then the update of
    update_field(..., is_sh=True) on every coefficient, in place.
    colors: [V, C, 3] (or [C, 3], [C, 1, 3] for one view) masked colour
    cotangents, in pool order or (compact_colors) the visible-cluster prefix;
    centers: [V, 3] (or [3]) camera centres.  Returns (sh, mean, variance)."""
    if sh.dim() != 3 or sh.shape[2] != 3:
        raise ValueError("sh must be [C, sh_dim, 3]")
    if sh.shape != mean.shape or sh.shape != variance.shape:
        raise ValueError("sh and moments must have one shape")
    capacity, sh_dim = int(sh.shape[0]), int(sh.shape[1])
    if int(alive.shape[0]) != capacity or tuple(xyz.shape) != (capacity, 3):
        raise ValueError("xyz and alive must have one row per SH row")
    if not 0 <= degree <= 3 or (degree + 1) ** 2 > sh_dim:
        raise ValueError(f"degree {degree} needs (degree + 1)^2 <= {sh_dim} coefficients")
    centers = centers.reshape(-1, 3)
    views = int(centers.shape[0])
    if colors.numel() != views * capacity * 3:
        raise ValueError("colors must hold C x 3 cotangents per view (pool or compact order)")
    for t in (sh, mean, variance, xyz, centers, colors):
        if not t.is_cuda or t.dtype != torch.float32:
            raise ValueError("sparse Adam needs float32 CUDA tensors")
    for t in (sh, mean, variance):
        if not t.is_contiguous():
            raise ValueError("sh and moments must be contiguous")
    if capacity == 0:
        return sh, mean, variance
    ids, count = clusters
    if not torch.is_tensor(rate):
        rate = torch.full((1,), float(rate), dtype=torch.float32, device=sh.device)
    alive8 = alive if alive.dtype == torch.int8 else (
        alive.view(torch.int8) if alive.dtype == torch.uint8 else alive.to(torch.int8))
    colors = colors.contiguous()
    centers = centers.contiguous()
    p = L.AdamShParams(capacity, sh_dim, int(degree), int(cluster_size), views,
                       int(compact_colors), 0, 0)
    ptr = lambda t: t.data_ptr()
    L.check(L.lib.gsb_sparse_adam_sh(_stream(), L.ref(p), ptr(sh), ptr(mean), ptr(variance),
                                     ptr(xyz.contiguous()), ptr(centers), ptr(colors),
                                     ptr(alive8.contiguous()),
                                     ptr(ids.to(torch.int32).contiguous()),
                                     ptr(count.to(torch.int32).contiguous()),
                                     ptr(rate.to(torch.float32).contiguous())),
            "sparse Adam (SH from colours)")
    return sh, mean, variance


def update_sh_from_rows(sh: torch.Tensor, mean: torch.Tensor, variance: torch.Tensor,
                        xyz: torch.Tensor, rows: torch.Tensor, alive: torch.Tensor, clusters,
                        rate, cluster_size: int, degree: int):
    """update_sh_from_colors for the view-sharded exchange's gathered rows:
    rows [V, >= 4 + C*3], each a view's camera centre (3 floats and a pad)
    followed by its masked colour cotangents in pool order
    (NvlsExchange(deferred_sh=True).exchange() returns them), read in
    place."""
    capacity = int(sh.shape[0])
    if rows.dim() != 2 or rows.shape[1] < 4 + capacity * 3 or not rows.is_contiguous():
        raise ValueError("colour rows must be [V, >= 4 + C*3] contiguous")
    if not rows.is_cuda or rows.dtype != torch.float32:
        raise ValueError("sparse Adam needs float32 CUDA tensors")
    if sh.dim() != 3 or sh.shape[2] != 3 or sh.shape != mean.shape or sh.shape != variance.shape:
        raise ValueError("sh and moments must be [C, sh_dim, 3] of one shape")
    if int(alive.shape[0]) != capacity or tuple(xyz.shape) != (capacity, 3):
        raise ValueError("xyz and alive must have one row per SH row")
    sh_dim = int(sh.shape[1])
    if not 0 <= degree <= 3 or (degree + 1) ** 2 > sh_dim:
        raise ValueError(f"degree {degree} needs (degree + 1)^2 <= {sh_dim} coefficients")
    for t in (sh, mean, variance):
        if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("sh and moments must be contiguous float32 CUDA tensors")
    if capacity == 0:
        return sh, mean, variance
    ids, count = clusters
    if not torch.is_tensor(rate):
        rate = torch.full((1,), float(rate), dtype=torch.float32, device=sh.device)
    alive8 = alive if alive.dtype == torch.int8 else (
        alive.view(torch.int8) if alive.dtype == torch.uint8 else alive.to(torch.int8))
    row = int(rows.shape[1])
    p = L.AdamShParams(capacity, sh_dim, int(degree), int(cluster_size), int(rows.shape[0]), 0,
                       row, row)
    ptr = lambda t: t.data_ptr()
    L.check(L.lib.gsb_sparse_adam_sh(_stream(), L.ref(p), ptr(sh), ptr(mean), ptr(variance),
                                     ptr(xyz.contiguous()), ptr(rows), ptr(rows) + 16,
                                     ptr(alive8.contiguous()),
                                     ptr(ids.to(torch.int32).contiguous()),
                                     ptr(count.to(torch.int32).contiguous()),
                                     ptr(rate.to(torch.float32).contiguous())),
            "sparse Adam (SH from gathered colour rows)")
    return sh, mean, variance


def sparse_adam_update(pool: GaussianArrays, state: AdamState, gradients, visible: torch.Tensor,
                       step: float, spatial_scale: float, max_steps: int | None = None, *,
                       compacted_clusters, cluster_size: int = 128,
                       compact_gradients: bool = False,
                       optimization: OptimizationConfig = OptimizationConfig(),
                       sh_pullback_center: torch.Tensor | None = None,
                       active_degree: int | None = None,
                       sh_pullback_rows: torch.Tensor | None = None):
    """training/optimizer.py:276-341 with compacted clusters: LiteGS Adam on
    every field of the listed clusters' alive slots, in place on the pool and
    the state; state.step counts the update in every slot of `visible` that
    is alive.  gradients: (xyz, log_scale, rotation, opacity, sh) in pool
    order, or the visible-cluster prefix with compact_gradients; the SH
    gradient carries every coefficient of the pool, or, with
    sh_pullback_center (the camera centre [3]), it is the sh_color_only
    pullback's colour cotangent [C, 1, 3] from which the update rebuilds the
    gradients of the first (active_degree + 1)^2 coefficients (zero above;
    active_degree defaults to the pool's full degree).  Every field, moment
    and gradient is checked before the first launch, so a rejected call
    leaves the pool and the state untouched (the reference's trace-time
    checks, tests/test_chex_contracts.py:57-76).  sh_pullback_rows: the
    view-sharded form, the gathered rows of every view (camera centre, pad,
    pool-order colour cotangents; NvlsExchange(deferred_sh=True)); the SH
    gradient argument is then ignored.  Returns (pool, state)."""
    capacity = int(pool.alive.shape[0])
    if tuple(visible.shape) != (capacity,):
        raise ValueError("visible must hold one flag per pool slot")
    if len(gradients) != len(PARAMETER_NAMES):
        raise ValueError("gradients must be (xyz, log_scale, rotation, opacity, sh)")
    for i, (name, gradient) in enumerate(zip(PARAMETER_NAMES, gradients)):
        value = getattr(pool, name)
        if tuple(state.m[i].shape) != tuple(value.shape) or \
                tuple(state.v[i].shape) != tuple(value.shape):
            raise ValueError(f"{name} moments must have the field's shape")
        if gradient.dtype != torch.float32:
            raise ValueError(f"{name} gradient must be float32")
        if name == "sh" and sh_pullback_rows is not None:
            continue
        if name == "sh" and sh_pullback_center is not None:
            if gradient.numel() != capacity * 3:
                raise ValueError("with sh_pullback_center the sh gradient is the colour "
                                 "cotangent, 3 floats per slot (compact or pool order)")
            continue
        # Compact gradients also have the pool's shape (the visible-cluster
        # prefix, tail undefined): the kernel reads up to the listed
        # clusters' rows, which only the device knows, and never past C rows.
        if gradient.numel() != value.numel():
            raise ValueError(f"{name} gradient must have the field's size "
                             f"({value.numel()} floats, compact or pool order)")
        if gradient.dim() > 1 and tuple(gradient.shape[1:]) != tuple(value.shape[1:]):
            raise ValueError(f"{name} gradient rows must have the field's shape "
                             "(every SH coefficient)")
    sh_dim = int(pool.sh.shape[1])
    degree = int(round(sh_dim ** 0.5)) - 1 if active_degree is None else int(active_degree)
    if sh_pullback_rows is not None and sh_pullback_center is not None:
        raise ValueError("give sh_pullback_center or sh_pullback_rows, not both")
    if sh_pullback_rows is not None and not (0 <= degree <= 3 and (degree + 1) ** 2 <= sh_dim):
        raise ValueError(f"active_degree {degree} does not fit {sh_dim} SH coefficients")
    if sh_pullback_center is not None:
        if sh_pullback_center.numel() != 3:
            raise ValueError("sh_pullback_center must be one camera centre (3 floats)")
        if not 0 <= degree <= 3 or (degree + 1) ** 2 > sh_dim:
            raise ValueError(f"active_degree {degree} does not fit {sh_dim} SH coefficients")
    rates = parameter_learning_rates(step, spatial_scale, max_steps, optimization)
    dev = pool.xyz.device
    rate_t = torch.tensor(rates, dtype=torch.float32, device=dev)
    order = list(enumerate(zip(PARAMETER_NAMES, gradients)))
    if sh_pullback_center is not None or sh_pullback_rows is not None:
        # The SH directions use the positions before this update (the
        # reference's transform sees the parameters it updates), so the SH
        # field goes first; the fields are otherwise independent.
        order = order[-1:] + order[:-1]
    for i, (name, gradient) in order:
        value = getattr(pool, name)
        if name == "sh" and sh_pullback_rows is not None:
            update_sh_from_rows(value, state.m[i], state.v[i], pool.xyz, sh_pullback_rows,
                                pool.alive, compacted_clusters, rate_t[i:i + 1], cluster_size,
                                degree)
            continue
        if name == "sh" and sh_pullback_center is not None:
            update_sh_from_colors(value, state.m[i], state.v[i], pool.xyz,
                                  sh_pullback_center.to(dev, torch.float32), gradient,
                                  pool.alive, compacted_clusters, rate_t[i:i + 1], cluster_size,
                                  degree, compact_gradients)
            continue
        update_field(value, state.m[i], state.v[i], gradient.contiguous(), pool.alive,
                     compacted_clusters, rate_t[i:i + 1], cluster_size, name == "sh",
                     compact_gradients)
    state.step += (visible.to(torch.bool) & pool.alive.to(torch.bool)).to(torch.int32)
    return pool, state
