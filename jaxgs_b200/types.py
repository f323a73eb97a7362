"""Fixed-shape device data shared by the stages (torch tensors on CUDA).

Mirrors render/types.py:7-63 and scene/types.py:6-31 of the reference:
field names, shapes and dtypes are the reference's, so values convert
one-to-one to the JAX pytrees.
"""

from __future__ import annotations

from dataclasses import dataclass, fields, replace

import numpy as np
import torch

from .scene import Camera

PARAMETER_NAMES = ("xyz", "log_scale", "rotation", "opacity", "sh")


@dataclass
class GaussianArrays:
    """scene/point.py:12-23 (free_mask / n_active are not read by the hot path)."""

    xyz: torch.Tensor        # [C, 3]
    log_scale: torch.Tensor  # [C, 3]
    rotation: torch.Tensor   # [C, 4] wxyz
    opacity: torch.Tensor    # [C, 1] logits
    sh: torch.Tensor         # [C, SH_DIM, 3]
    alive: torch.Tensor      # [C] bool or uint8 (uint8 avoids a per-call conversion)

    @classmethod
    def from_numpy(cls, pool: dict, device="cuda") -> "GaussianArrays":
        arrays = [torch.as_tensor(np.ascontiguousarray(pool[k]), device=device)
                  for k in ("xyz", "log_scale", "rotation", "opacity", "sh")]
        alive = torch.as_tensor(np.ascontiguousarray(pool["alive"], np.uint8), device=device)
        return cls(*arrays, alive)

    @property
    def capacity(self) -> int:
        return int(self.xyz.shape[0])

    def replace(self, **kwargs) -> "GaussianArrays":
        return replace(self, **kwargs)


@dataclass
class DeviceCamera:
    """scene/camera.py:6-65 with the traced arrays on the device."""

    world_to_camera: torch.Tensor  # [4, 4] float32
    intrinsics: torch.Tensor       # [4] fx, fy, cx, cy
    center: torch.Tensor           # [3]
    planes: torch.Tensor           # [6, 4] frustum planes of scene/cluster.py:40-63
    width: int
    height: int
    near: float = 0.2
    far: float = 1000.0

    @classmethod
    def from_camera(cls, camera: Camera, device="cuda") -> "DeviceCamera":
        def t(a):
            return torch.as_tensor(np.ascontiguousarray(a, np.float32), device=device)

        return cls(t(camera.world_to_camera), t(camera.intrinsics), t(camera.center),
                   t(camera.frustum_planes()), camera.width, camera.height, camera.near,
                   camera.far)

    # Packed layout (floats): planes [0, 24), world_to_camera [24, 40),
    # intrinsics [40, 44), center [44, 47), one pad; every field starts on a
    # 16-byte boundary, so the arrays of one camera move in one copy.
    PACKED_FLOATS = 48

    @classmethod
    def packed_views(cls, flat: torch.Tensor, width: int, height: int, near: float = 0.2,
                     far: float = 1000.0) -> "DeviceCamera":
        """A DeviceCamera whose arrays are views of one packed [48] buffer."""
        if flat.numel() != cls.PACKED_FLOATS or flat.dtype != torch.float32:
            raise ValueError("a packed camera is 48 float32 values")
        return cls(flat[24:40].view(4, 4), flat[40:44], flat[44:47], flat[0:24].view(6, 4),
                   width, height, near, far)

    def pack(self, out: torch.Tensor | None = None) -> torch.Tensor:
        """This camera's arrays in the packed layout (a new tensor on the
        arrays' device, or copied into `out`)."""
        flat = torch.zeros(self.PACKED_FLOATS, dtype=torch.float32,
                           device=self.world_to_camera.device) if out is None else out
        view = DeviceCamera.packed_views(flat, self.width, self.height, self.near, self.far)
        for dst, src in ((view.planes, self.planes), (view.world_to_camera, self.world_to_camera),
                         (view.intrinsics, self.intrinsics), (view.center, self.center)):
            dst.copy_(src.reshape(dst.shape))
        return flat


@dataclass
class ProjectedGaussians:
    """render/types.py:7-16."""

    mean: torch.Tensor     # [C, 2]
    depth: torch.Tensor    # [C]
    conic: torch.Tensor    # [C, 2, 2]
    radius: torch.Tensor   # [C]
    color: torch.Tensor    # [C, 3]
    alpha: torch.Tensor    # [C]
    visible: torch.Tensor  # [C] int8 (0/1)

    def replace(self, **kwargs) -> "ProjectedGaussians":
        return replace(self, **kwargs)


@dataclass
class SortedVisibilityTable:
    """render/types.py:29-37.  gaussian_ids' valid prefix ends at pair_count."""

    gaussian_ids: torch.Tensor  # [P_MAX] int32
    tile_offsets: torch.Tensor  # [T + 1] int32
    point_counts: torch.Tensor  # [C] int32
    pair_count: torch.Tensor    # [1] int32
    overflow: torch.Tensor      # [1] int32 (bool)


@dataclass
class RenderResult:
    """render/types.py:40-45."""

    rgb: torch.Tensor    # [H, W, 3]
    depth: torch.Tensor  # [H, W]
    alpha: torch.Tensor  # [H, W]


@dataclass
class RasterCache:
    """State the forward hands to the backward (splat records, per-pixel final
    transmittance and last pair, per-tile backward work)."""

    splats: torch.Tensor             # [C, 12] float32
    final_t: torch.Tensor            # [H * W]
    last: torch.Tensor               # [H * W] int32
    backward_work: torch.Tensor      # [T] int32
    contribution_bits: torch.Tensor  # [gsb_raster_bit_words] int32 (uint32 words)


def tree_fields(obj):
    return {f.name: getattr(obj, f.name) for f in fields(obj)}
