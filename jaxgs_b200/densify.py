"""Density control fed by the fragment statistics (training/densify.py):
compute_densification_scores (:20-35) and decay_opacity (:158-165), one
elementwise kernel each, and densify_step (:38-155), the pool management
around them (prune, weighted sampling of parents, split/clone children into
free slots), written with torch operations on the pool's device, and
refresh_cluster_bounds (scene/cluster.py:15-37), which recomputes the
culling bounds of the changed pool in place."""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib as L
from .optimizer import AdamState, create_adam_state, reset_adam_slots
from .types import GaussianArrays


def _alive8(alive: torch.Tensor) -> torch.Tensor:
    if alive.dtype == torch.int8:
        return alive
    if alive.dtype == torch.uint8:
        return alive.view(torch.int8)
    return alive.to(torch.int8)


def compute_densification_scores(pool: GaussianArrays, fragment_stats: torch.Tensor):
    """training/densify.py:20-35: (scores [C] float32, prune [C] bool) from the
    [C, 4] fragment statistics (count, compositing weight, alpha cotangent
    sum, squared sum): the opacity-weighted variance of the per-fragment
    opacity gradient, and the alive slots that composited nothing."""
    C = int(pool.xyz.shape[0])
    if tuple(fragment_stats.shape) != (C, 4):
        raise ValueError("fragment statistics must be [C, 4]")
    stats = fragment_stats.detach().to(torch.float32).contiguous()
    scores = torch.empty(C, dtype=torch.float32, device=stats.device)
    prune = torch.empty(C, dtype=torch.int8, device=stats.device)
    L.check(L.lib.gsb_densify_scores(
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), C,
        ctypes.c_void_p(stats.data_ptr()),
        ctypes.c_void_p(pool.opacity.contiguous().data_ptr()),
        ctypes.c_void_p(_alive8(pool.alive).contiguous().data_ptr()),
        ctypes.c_void_p(scores.data_ptr()), ctypes.c_void_p(prune.data_ptr())),
        "densification scores")
    return scores, prune.bool()


def decay_opacity(pool: GaussianArrays, state: AdamState | None = None):
    """training/densify.py:158-165: halve every alive slot's alpha (not
    below 1/128), in place on pool.opacity, and return fresh Adam moments."""
    C = int(pool.xyz.shape[0])
    if not pool.opacity.is_contiguous():
        raise ValueError("pool.opacity must be contiguous")
    L.check(L.lib.gsb_decay_opacity(
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), C,
        ctypes.c_void_p(pool.opacity.data_ptr()),
        ctypes.c_void_p(_alive8(pool.alive).contiguous().data_ptr())), "opacity decay")
    return pool, create_adam_state(pool)


def prune_step(pool: GaussianArrays, state: AdamState, remove: torch.Tensor):
    """training/pool_ops.py:11-20: release the masked live slots (in place)
    and reset their Adam state; returns the released mask."""
    alive = pool.alive.to(torch.bool)
    remove = remove.to(torch.bool) & alive
    pool.alive.copy_((alive & ~remove).to(pool.alive.dtype))
    reset_adam_slots(state, remove)
    return remove


def _rotation_matrices(q: torch.Tensor) -> torch.Tensor:
    """render/projection.py:20-30: wxyz quaternions (normalised, 1e-8 floor)
    to rotation matrices."""
    q = q / torch.clamp(torch.linalg.norm(q, dim=-1, keepdim=True), min=1e-8)
    w, x, y, z = q.unbind(-1)
    return torch.stack([
        torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1),
        torch.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1),
        torch.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1),
    ], -2)


def densify_step(pool: GaussianArrays, state: AdamState, fragment_stats: torch.Tensor,
                 generator: torch.Generator, target_count: int, scene_radius: float,
                 cluster_size: int = 128, percent_dense: float = 0.01):
    """training/densify.py:38-155, in place on the pool and the Adam state.

    Prunes alive slots that composited nothing (whole clusters' worth of
    them), samples up to the growth budget of parents without replacement
    with probability proportional to their scores (Gumbel top-k, the
    distribution of torch.multinomial; zero-score live slots come last),
    splits parents larger than percent_dense * scene_radius (child moved by
    a rotated Gaussian jitter of the parent's scale, scale / 1.6) and clones
    the others, writing children into the lowest free slots; parents are
    left unchanged and the children's Adam state is zeroed.  Randomness
    comes from `generator` (on the pool's device), so the draws differ from
    the reference's JAX key stream; the budget arithmetic, ordering and
    child formulas are the reference's.  Returns (pool, state, born,
    pruned); the cluster bounds are stale afterwards (refresh_cluster_bounds)."""
    capacity = int(pool.xyz.shape[0])
    dev = pool.xyz.device
    scores, prune_mask = compute_densification_scores(pool, fragment_stats)
    alive0 = pool.alive.to(torch.bool).clone()
    n_active = int(alive0.sum().item())
    prune_candidates = int(prune_mask.sum().item())
    candidate_count = min(max(int(target_count) - n_active, 1) + prune_candidates, n_active)
    prune_count = prune_candidates // cluster_size * cluster_size
    prune_mask = prune_mask & (torch.cumsum(prune_mask.to(torch.int64), 0) <= prune_count)
    prune_step(pool, state, prune_mask)
    n_after = n_active - int(prune_mask.sum().item())
    max_births = min(candidate_count // cluster_size * cluster_size,
                     (capacity - n_after) // cluster_size * cluster_size)
    # Exponential race: log(score) + Gumbel noise, largest first.
    u = torch.rand(capacity, generator=generator, device=dev, dtype=torch.float32)
    gumbel = -torch.log(-torch.log(torch.clamp(u, min=1e-20)))
    priorities = torch.where(alive0, torch.log(torch.clamp(scores, min=1e-30)) + gumbel,
                             torch.full_like(scores, -math.inf))
    candidates = torch.argsort(-priorities, stable=True)
    parents = candidates[:candidate_count]
    split = torch.exp(pool.log_scale[parents]).amax(dim=1) > percent_dense * scene_radius
    # Stable partition of the sampled parents: splits first, then clones.
    order = torch.cat([torch.nonzero(split).flatten(), torch.nonzero(~split).flatten()])
    parents, split = parents[order][:max_births], split[order][:max_births]
    free = ~pool.alive.to(torch.bool)
    free_slots = torch.nonzero(free).flatten()
    width = min(max_births, int(free_slots.numel()))
    parents, split = parents[:width], split[:width]
    valid = alive0[parents]
    child_slots = free_slots[:width][valid]
    parents, split = parents[valid], split[valid]
    jitter = torch.randn(parents.numel(), 3, generator=generator, device=dev,
                         dtype=torch.float32) * torch.exp(pool.log_scale[parents])
    offsets = torch.einsum("nij,nj->ni", _rotation_matrices(pool.rotation[parents]), jitter)
    # Gather every parent value before any child is written.
    child = {
        "xyz": pool.xyz[parents] + torch.where(split[:, None], offsets, torch.zeros_like(offsets)),
        "log_scale": pool.log_scale[parents] - torch.where(
            split[:, None], torch.full_like(offsets, math.log(1.6)), torch.zeros_like(offsets)),
        "rotation": pool.rotation[parents].clone(),
        "opacity": pool.opacity[parents].clone(),
        "sh": pool.sh[parents].clone(),
    }
    for name, value in child.items():
        getattr(pool, name)[child_slots] = value
    newborn = torch.zeros(capacity, dtype=torch.bool, device=dev)
    newborn[child_slots] = True
    pool.alive.copy_((pool.alive.to(torch.bool) | newborn).to(pool.alive.dtype))
    reset_adam_slots(state, newborn)
    return pool, state, int(newborn.sum().item()), prune_count


def refresh_cluster_bounds(pool: GaussianArrays, bounds, cluster_size: int = 128):
    """scene/cluster.py:15-37 on the pool's device, written in place into
    the (center [N, 3], extent [N, 3], valid [N]) tensors of `bounds`: the
    axis-aligned box of every cluster's alive Gaussians, each grown by its
    rotated and scaled 1/255-level half extents (sqrt(2 ln 255) sigma).
    Call it after densify_step, prune_step or an optimizer step that moved
    Gaussians; updating in place keeps the tensors a captured
    GraphedTrainingStep reads.  Same formulas as
    scene.world_cluster_bounds, in float64."""
    center, extent, valid = bounds
    capacity = int(pool.xyz.shape[0])
    n_clusters = -(-capacity // cluster_size)
    if tuple(center.shape) != (n_clusters, 3) or tuple(extent.shape) != (n_clusters, 3) \
            or tuple(valid.shape) != (n_clusters,):
        raise ValueError(f"bounds must hold {n_clusters} clusters of {cluster_size} slots")
    f64 = torch.float64
    transform = _rotation_matrices(pool.rotation.to(f64)) * torch.exp(pool.log_scale.to(f64))[:, None, :]
    half = transform.abs().sum(-1) * math.sqrt(2 * math.log(255.0))
    alive = pool.alive.to(torch.bool)[:, None]
    xyz = pool.xyz.to(f64)
    pad = n_clusters * cluster_size - capacity
    lower = torch.nn.functional.pad(torch.where(alive, xyz - half, math.inf), (0, 0, 0, pad),
                                    value=math.inf)
    upper = torch.nn.functional.pad(torch.where(alive, xyz + half, -math.inf), (0, 0, 0, pad),
                                    value=-math.inf)
    lower = lower.reshape(n_clusters, cluster_size, 3).amin(dim=1)
    upper = upper.reshape(n_clusters, cluster_size, 3).amax(dim=1)
    ok = torch.isfinite(lower[:, 0])
    zero = torch.zeros((), dtype=f64, device=xyz.device)
    center.copy_(torch.where(ok[:, None], (lower + upper) / 2, zero).to(center.dtype))
    extent.copy_(torch.where(ok[:, None], (upper - lower) / 2, zero).to(extent.dtype))
    valid.copy_(ok.to(valid.dtype))
    return bounds
