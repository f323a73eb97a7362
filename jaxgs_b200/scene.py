"""Host-side scene data: camera, capacity config, Gaussian pool, synthetic scenes.

Layouts follow the reference exactly so that pools and cameras are drop-in:

* ``Camera`` — column-vector world-to-camera 4x4, camera looks along +Z,
  OpenCV axes (scene/camera.py:6-65); ``center = -R^T t``.
* ``CapacityConfig`` — config/capacity.py:4-41 (tile_size is the tile width,
  tile_height defaults to tile_size).
* Pool — xyz[C,3], log_scale[C,3], rotation[C,4] (wxyz), opacity[C,1]
  (logit), sh[C,(deg+1)^2,3], alive[C] bool (scene/point.py:12-23).

Synthetic scenes stand in for MipNeRF360 bicycle (absent here); their
distributions are the ones BASELINE.json's configs state, seeded with
``numpy.random.default_rng``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

SH_C0 = 0.28209479177387814


@dataclass(frozen=True)
class CapacityConfig:
    """config/capacity.py:4-41."""

    max_gaussians: int = 1 << 20
    cluster_size: int = 128
    max_gaussians_per_tile: int = 128
    tile_size: int = 16
    sh_degree: int = 3
    max_visibility_pairs: int | None = None
    tile_height: int | None = None

    def __post_init__(self) -> None:
        if min(self.max_gaussians, self.cluster_size, self.max_gaussians_per_tile, self.tile_size) <= 0:
            raise ValueError("capacities and tile_size must be positive")
        if not 0 <= self.sh_degree <= 3:
            raise ValueError("sh_degree must be between 0 and 3")
        if self.max_visibility_pairs is not None and self.max_visibility_pairs <= 0:
            raise ValueError("max_visibility_pairs must be positive")
        if self.tile_height is not None and self.tile_height <= 0:
            raise ValueError("tile_height must be positive")

    @property
    def raster_tile_height(self) -> int:
        return self.tile_height or self.tile_size

    @property
    def sh_dim(self) -> int:
        return (self.sh_degree + 1) ** 2

    @property
    def num_clusters(self) -> int:
        return (self.max_gaussians + self.cluster_size - 1) // self.cluster_size

    @property
    def visibility_capacity(self) -> int:
        return self.max_visibility_pairs or self.max_gaussians * 16


def quaternion_to_matrix(q: np.ndarray) -> np.ndarray:
    """render/projection.py:20-30 (wxyz, normalised with a 1e-8 floor)."""
    q = np.asarray(q, np.float64)
    q = q / np.maximum(np.linalg.norm(q, axis=-1, keepdims=True), 1e-8)
    w, x, y, z = np.moveaxis(q, -1, 0)
    return np.stack(
        [
            np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1),
            np.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1),
            np.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1),
        ],
        -2,
    )


@dataclass
class Camera:
    """scene/camera.py:6-65: world_to_camera [4,4] float32, intrinsics."""

    world_to_camera: np.ndarray
    fx: float
    fy: float
    cx: float
    cy: float
    width: int
    height: int
    near: float = 0.2
    far: float = 1000.0

    @classmethod
    def from_colmap(cls, qvec, tvec, fx, fy, cx, cy, width, height, near=0.2, far=1000.0):
        """scene/camera.py:19-56 (quaternion normalised in float32)."""
        q = np.asarray(qvec, np.float32)
        if q.shape != (4,) or np.asarray(tvec).shape != (3,):
            raise ValueError("COLMAP extrinsics are a wxyz quaternion [4] and a translation [3]")
        q = q / np.linalg.norm(q)
        w, x, y, z = q
        rotation = np.array(
            [
                [1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)],
            ],
            np.float32,
        )
        transform = np.eye(4, dtype=np.float32)
        transform[:3, :3] = rotation
        transform[:3, 3] = np.asarray(tvec, np.float32)
        return cls(transform, float(np.float32(fx)), float(np.float32(fy)), float(np.float32(cx)),
                   float(np.float32(cy)), int(width), int(height), float(near), float(far))

    @classmethod
    def look_at(cls, eye, target, fx, fy, width, height, cx=None, cy=None, near=0.2,
                far=1000.0, up=(0.0, 1.0, 0.0)):
        """OpenCV axes (x right, y down, z forward) with world up +y."""
        eye = np.asarray(eye, np.float64)
        forward = np.asarray(target, np.float64) - eye
        forward /= np.linalg.norm(forward)
        right = np.cross(forward, np.asarray(up, np.float64))
        right /= np.linalg.norm(right)
        down = np.cross(forward, right)
        rotation = np.stack([right, down, forward])
        transform = np.eye(4, dtype=np.float64)
        transform[:3, :3] = rotation
        transform[:3, 3] = -rotation @ eye
        return cls(transform.astype(np.float32), float(fx), float(fy),
                   float(width / 2 if cx is None else cx), float(height / 2 if cy is None else cy),
                   int(width), int(height), float(near), float(far))

    @property
    def center(self) -> np.ndarray:
        r = self.world_to_camera[:3, :3].astype(np.float32)
        return (-(r.T @ self.world_to_camera[:3, 3].astype(np.float32))).astype(np.float32)

    @property
    def intrinsics(self) -> np.ndarray:
        return np.array([self.fx, self.fy, self.cx, self.cy], np.float32)

    def frustum_planes(self) -> np.ndarray:
        """Six (a, b, c, d) planes of scene/cluster.py:40-63 (LiteGS near 0.01, far 5000)."""
        near, far = 0.01, 5000.0
        projection = np.array(
            [
                [2 * self.fx / self.width, 0, 2 * self.cx / self.width - 1, 0],
                [0, 2 * self.fy / self.height, 2 * self.cy / self.height - 1, 0],
                [0, 0, far / (far - near), -far * near / (far - near)],
                [0, 0, 1, 0],
            ],
            np.float32,
        )
        m = projection @ self.world_to_camera.astype(np.float32)
        return np.stack((m[3] + m[0], m[3] - m[0], m[3] + m[1], m[3] - m[1], m[2], m[3] - m[2])).astype(np.float32)


def create_gaussians(config: CapacityConfig) -> dict:
    """scene/point.py:61-72."""
    c = config.max_gaussians
    return {
        "xyz": np.zeros((c, 3), np.float32),
        "log_scale": np.zeros((c, 3), np.float32),
        "rotation": np.tile(np.array([1.0, 0.0, 0.0, 0.0], np.float32), (c, 1)),
        "opacity": np.zeros((c, 1), np.float32),
        "sh": np.zeros((c, config.sh_dim, 3), np.float32),
        "alive": np.zeros((c,), bool),
    }


def seed_gaussians(pool: dict, xyz, rgb, scale=0.01, opacity=0.1) -> dict:
    """scene/point.py:75-104 (log of scale, logit of opacity, SH0 from RGB)."""
    xyz = np.asarray(xyz, np.float32)
    n = xyz.shape[0]
    scale = np.asarray(scale, np.float32)
    if scale.ndim == 0:
        scale = np.broadcast_to(scale, (n, 3))
    elif scale.shape == (n,):
        scale = np.broadcast_to(scale[:, None], (n, 3))
    pool = {k: v.copy() for k, v in pool.items()}
    pool["sh"][:n, 0, :] = (np.asarray(rgb, np.float32) - 0.5) / np.float32(SH_C0)
    pool["xyz"][:n] = xyz
    pool["log_scale"][:n] = np.log(scale)
    pool["opacity"][:n] = np.float32(math.log(opacity / (1 - opacity)))
    pool["alive"][:n] = True
    return pool


def world_cluster_bounds(pool: dict, cluster_size: int):
    """scene/cluster.py:15-37: per-cluster AABB centre/half extent/valid."""
    transform = quaternion_to_matrix(pool["rotation"]) * np.exp(pool["log_scale"].astype(np.float64))[:, None, :]
    extent = np.sum(np.abs(transform), axis=-1) * math.sqrt(2 * math.log(255.0))
    alive = pool["alive"][:, None]
    n = pool["xyz"].shape[0]
    padding = (-n) % cluster_size
    lower = np.pad(np.where(alive, pool["xyz"] - extent, np.inf), ((0, padding), (0, 0)), constant_values=np.inf)
    upper = np.pad(np.where(alive, pool["xyz"] + extent, -np.inf), ((0, padding), (0, 0)), constant_values=-np.inf)
    lower = lower.reshape(-1, cluster_size, 3).min(axis=1)
    upper = upper.reshape(-1, cluster_size, 3).max(axis=1)
    valid = np.isfinite(lower[:, 0])
    with np.errstate(invalid="ignore"):  # empty clusters: inf + -inf, replaced below
        center = np.where(valid[:, None], (lower + upper) / 2, 0).astype(np.float32)
        half = np.where(valid[:, None], (upper - lower) / 2, 0).astype(np.float32)
    return center, half, valid


# --------------------------------------------------------------------------
# Synthetic scenes of BASELINE.json configs 0-4.
# --------------------------------------------------------------------------
def _random_quaternions(rng, n):
    q = rng.normal(0, 1, (n, 4)).astype(np.float32)
    return q / np.linalg.norm(q, axis=1, keepdims=True)


def _sh(rng, n, degree=3):
    sh = np.empty((n, (degree + 1) ** 2, 3), np.float32)
    sh[:, 0] = rng.normal(0, 0.5, (n, 3))
    sh[:, 1:] = rng.normal(0, 0.05, (n, (degree + 1) ** 2 - 1, 3))
    return sh


def _pool(xyz, log_scale, rotation, opacity, sh):
    return {"xyz": np.ascontiguousarray(xyz, np.float32),
            "log_scale": np.ascontiguousarray(log_scale, np.float32),
            "rotation": np.ascontiguousarray(rotation, np.float32),
            "opacity": np.ascontiguousarray(opacity, np.float32).reshape(-1, 1),
            "sh": np.ascontiguousarray(sh, np.float32),
            "alive": np.ones(xyz.shape[0], bool)}


def config0_scene():
    """4,096 Gaussians (seed 0), 128x96 camera at (0,0,-4)."""
    rng = np.random.default_rng(0)
    n = 4096
    xyz = rng.uniform(-1, 1, (n, 3))
    log_scale = rng.normal(-3.5, 0.3, (n, 3))
    rotation = _random_quaternions(rng, n)
    opacity = rng.normal(0, 1, (n, 1))
    sh = _sh(rng, n)
    camera = Camera.look_at((0.0, 0.0, -4.0), (0.0, 0.0, 0.0), 110.0, 110.0, 128, 96,
                            near=0.01, far=100.0)
    target = np.random.default_rng(1).integers(0, 256, (96, 128, 3), dtype=np.uint8)
    return _pool(xyz, log_scale, rotation, opacity, sh), camera, target


def _plane_sphere_means(rng, n, plane, sphere_radius=10.0, plane_fraction=0.7):
    n_plane = int(round(plane_fraction * n))
    plane_xyz = np.stack(
        [rng.uniform(-plane / 2, plane / 2, n_plane), rng.normal(0, 0.05, n_plane),
         rng.uniform(-plane / 2, plane / 2, n_plane)], 1)
    m = n - n_plane
    direction = rng.normal(0, 1, (m, 3))
    direction /= np.linalg.norm(direction, axis=1, keepdims=True)
    radius = sphere_radius * rng.uniform(0, 1, m) ** (1.0 / 3.0)
    return np.concatenate([plane_xyz, direction * radius[:, None]], 0)


def config1_scene(n=1_000_000, seed=2, plane=20.0):
    """plane/sphere mixture, log-scales N(-4, 0.6) with a
    small per-axis jitter, random rotations, opacity logits N(-1, 1.5)."""
    rng = np.random.default_rng(seed)
    xyz = _plane_sphere_means(rng, n, plane)
    log_scale = rng.normal(-4.0, 0.6, (n, 1)) + rng.normal(0, 0.1, (n, 3))
    rotation = _random_quaternions(rng, n)
    opacity = rng.normal(-1.0, 1.5, (n, 1))
    sh = _sh(rng, n)
    return _pool(xyz, log_scale, rotation, opacity, sh)


def config1_camera():
    """1237x822, fx=fy=1040, eye (0, 1.5, -6) looking at the origin."""
    return Camera.look_at((0.0, 1.5, -6.0), (0.0, 0.0, 0.0), 1040.0, 1040.0, 1237, 822)


def ring_cameras(count=8, radius=8.0, height=1.5, width=1237, height_px=822, focal=1040.0):
    """cameras on a ring looking at the origin."""
    cams = []
    for k in range(count):
        angle = 2 * math.pi * k / count
        eye = (radius * math.sin(angle), height, -radius * math.cos(angle))
        cams.append(Camera.look_at(eye, (0.0, 0.0, 0.0), focal, focal, width, height_px))
    return cams


def config3_scene():
    return config1_scene(n=3_000_000, seed=4, plane=40.0)


def config4_scene(n=6_000_000, seed=5):
    rng = np.random.default_rng(seed)
    xyz = _plane_sphere_means(rng, n, 60.0, sphere_radius=30.0)
    large = rng.random(n) < 0.05
    base = np.where(large, rng.normal(-1.0, 0.5, n), rng.normal(-4.5, 0.5, n))
    log_scale = base[:, None] + rng.normal(0, 0.3, (n, 3))
    rotation = _random_quaternions(rng, n)
    opacity = rng.normal(0, 2, (n, 1))
    sh = _sh(rng, n)
    return _pool(xyz, log_scale, rotation, opacity, sh)


def capacity_for(pool: dict, tile_size=16, tile_height=8, max_pairs=None, cluster_size=128,
                 sh_degree=3) -> CapacityConfig:
    return CapacityConfig(max_gaussians=pool["xyz"].shape[0], cluster_size=cluster_size,
                          tile_size=tile_size, sh_degree=sh_degree,
                          max_visibility_pairs=max_pairs, tile_height=tile_height)
