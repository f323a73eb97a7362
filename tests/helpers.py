"""Shared test utilities: scene generators, tensor <-> numpy conversion and
the oracle-side restatements of whole pipeline stages."""

from __future__ import annotations

import numpy as np

from jaxgs_b200.scene import Camera, CapacityConfig, create_gaussians, seed_gaussians


def np_proj(projected) -> dict:
    """ProjectedGaussians (torch) -> flat numpy dict in the oracle's layout."""
    return {
        "mean": projected.mean.detach().cpu().numpy().reshape(-1),
        "depth": projected.depth.detach().cpu().numpy().reshape(-1),
        "conic": projected.conic.detach().cpu().numpy().reshape(-1),
        "radius": projected.radius.detach().cpu().numpy().reshape(-1),
        "color": projected.color.detach().cpu().numpy().reshape(-1),
        "alpha": projected.alpha.detach().cpu().numpy().reshape(-1),
        "visible": projected.visible.detach().cpu().numpy().astype(np.int8).reshape(-1),
    }


def torch_proj(d: dict, device="cuda"):
    import torch

    from jaxgs_b200.types import ProjectedGaussians

    c = len(d["alpha"])
    t = lambda a, shape, dt=torch.float32: torch.as_tensor(np.ascontiguousarray(a), device=device).reshape(shape).to(dt)
    return ProjectedGaussians(t(d["mean"], (c, 2)), t(d["depth"], (c,)), t(d["conic"], (c, 2, 2)),
                              t(d.get("radius", np.zeros(c, np.float32)), (c,)), t(d["color"], (c, 3)),
                              t(d["alpha"], (c,)), t(d["visible"], (c,), torch.int8))


def splats(rng, count, width, height, radius=(0.4, 40.0), alpha=(0.005, 0.99), huge=0):
    """Small, large, thin and nearly degenerate screen-space ellipses with depth
    ties (the generator of the reference's tests/test_work_balance.py:59-86)."""
    mean = rng.uniform((-0.1 * width, -0.1 * height), (1.1 * width, 1.1 * height), (count, 2))
    scale = np.exp(rng.uniform(np.log(radius[0]), np.log(radius[1]), (count, 2)))
    scale[:huge] = rng.uniform(0.3, 0.6, (huge, 2)) * max(width, height)
    thin = (rng.random(count) < 0.25) & (np.arange(count) >= huge)
    scale[thin, 1] = scale[thin, 0] * rng.uniform(0.005, 0.05, thin.sum())
    angle = rng.uniform(0, np.pi, count)
    rot = np.stack([np.stack([np.cos(angle), -np.sin(angle)], -1),
                    np.stack([np.sin(angle), np.cos(angle)], -1)], -2)
    cov = rot @ (scale[:, :, None] ** 2 * np.eye(2)) @ rot.transpose(0, 2, 1)
    conic = np.linalg.inv(cov)
    conic = (conic + conic.transpose(0, 2, 1)) / 2
    depth = rng.integers(1, max(2, count // 3), count).astype(np.float32)
    return {
        "mean": mean.astype(np.float32).reshape(-1),
        "depth": depth,
        "conic": conic.astype(np.float32).reshape(-1),
        "radius": (3 * scale.max(1)).astype(np.float32),
        "color": rng.uniform(0.05, 0.95, (count, 3)).astype(np.float32).reshape(-1),
        "alpha": rng.uniform(*alpha, count).astype(np.float32),
        "visible": (rng.random(count) < 0.9).astype(np.int8),
    }


def known_answer_three():
    """tests/test_cute.py:141-159: 3 Gaussians, 8x8 image, 4x4 tiles."""
    config = CapacityConfig(4, 2, 1, 4, 0, 16)
    camera = Camera.from_colmap([1, 0, 0, 0], [0, 0, 0], 8, 8, 4, 4, 8, 8)
    pool = seed_gaussians(create_gaussians(config), np.array([[0, 0, 3.0], [0.1, 0, 2], [0, 0.1, 2]]),
                          np.ones((3, 3)) * 0.5, scale=0.2, opacity=0.5)
    return config, camera, pool


def rel_l2(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))
