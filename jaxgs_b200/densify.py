"""Density-control consumers of the fragment statistics
(training/densify.py:20-35 compute_densification_scores, :158-165
decay_opacity), one elementwise kernel each.  The sampling, split/clone and
slot allocation of densify_step (:38-155) are not part of this package."""

from __future__ import annotations

import ctypes

import torch

from . import _lib as L
from .optimizer import AdamState, create_adam_state
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
