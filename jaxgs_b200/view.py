"""Inference rendering of a fixed model (render/view.py:17-80).

ViewRenderer keeps the pool and its cluster bounds on the device; a frame is
cluster culling -> compact projection -> binning -> the RGB-only raster
forward (no backward state, kernels/packed_rasterizer.py:219-232) ->
rint(clip(rgb) * 255) as uint8, with the arena overflow flag.  Each
resolution's frame is captured once as a CUDA graph and replayed with the
new camera's arrays copied into its static inputs, so a frame costs no
host launches.  The image stays a device buffer (no window or graphics
API); callers copy it out or write it to a file.
"""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import torch

from . import kernels as K
from .scene import Camera, CapacityConfig, world_cluster_bounds
from .step import render
from .types import DeviceCamera, GaussianArrays

RESOLUTIONS = {
    "640x360": (640, 360),
    "640x480": (640, 480),
    "1280x720": (1280, 720),
    "1920x1080": (1920, 1080),
}


def resize_camera(camera: Camera, width: int, height: int) -> Camera:
    """render/view.py:24-34: the same viewing rays sampled at another
    resolution (intrinsics scaled in float32)."""
    f = np.float32
    sx, sy = f(width / camera.width), f(height / camera.height)
    return replace(camera, width=int(width), height=int(height),
                   fx=float(f(camera.fx) * sx), fy=float(f(camera.fy) * sy),
                   cx=float(f(camera.cx) * sx), cy=float(f(camera.cy) * sy))


class _Frame:
    """One resolution's frame captured as a CUDA graph."""

    def __init__(self, renderer: "ViewRenderer", camera: DeviceCamera):
        self.camera = DeviceCamera(camera.world_to_camera.clone(), camera.intrinsics.clone(),
                                   camera.center.clone(), camera.planes.clone(), camera.width,
                                   camera.height, camera.near, camera.far)
        side = torch.cuda.Stream(device=renderer.device)
        side.wait_stream(torch.cuda.current_stream(renderer.device))
        with torch.cuda.stream(side):
            renderer._frame(self.camera)  # allocations and library state before capture
        torch.cuda.current_stream(renderer.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.image, self.overflow = renderer._frame(self.camera)

    def __call__(self, camera: DeviceCamera):
        for dst, src in ((self.camera.world_to_camera, camera.world_to_camera),
                         (self.camera.intrinsics, camera.intrinsics),
                         (self.camera.center, camera.center), (self.camera.planes, camera.planes)):
            dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.image, self.overflow


class ViewRenderer:
    """render/view.py:37-80: keep the model on the device; only the camera
    changes between frames.  __call__(camera) returns (uint8 [H, W, 3]
    device image, overflow [1] device flag), fresh tensors (copy=False
    returns the graph's own output buffers instead, which the next frame at
    that resolution overwrites); warmup(camera) renders every preset
    resolution once and returns the first-call seconds."""

    def __init__(self, pool: GaussianArrays, *, pair_capacity: int = 8_000_000,
                 graphs: bool = True):
        sh_dims = (1, 4, 9, 16)
        if int(pool.sh.shape[1]) not in sh_dims:
            raise ValueError("model SH dimension must be 1, 4, 9 or 16")
        if int(pool.alive.to(torch.int64).sum().item()) == 0:
            raise ValueError("model has no active Gaussians")
        self.pool = pool
        self.device = pool.xyz.device
        self.config = CapacityConfig(max_gaussians=int(pool.xyz.shape[0]), cluster_size=128,
                                     tile_size=16, sh_degree=sh_dims.index(int(pool.sh.shape[1])),
                                     max_visibility_pairs=int(pair_capacity), tile_height=8)
        host = {k: getattr(pool, k).detach().cpu().numpy()
                for k in ("xyz", "log_scale", "rotation", "alive")}
        host["alive"] = host["alive"].astype(bool)
        center, extent, valid = world_cluster_bounds(host, self.config.cluster_size)
        self.bounds = (torch.as_tensor(center, device=self.device),
                       torch.as_tensor(extent, device=self.device),
                       torch.as_tensor(valid.astype(np.uint8), device=self.device))
        self.graphs = graphs
        self._frames: dict = {}

    def _frame(self, camera: DeviceCamera):
        # The compact projection reads only the listed clusters, whose alive
        # mask is the pool's, so the culled pool is not materialised.
        clusters, _ = K.compact_visible_clusters(self.bounds, camera, self.config, want_slots=False)
        image, _, overflow = render(camera, self.pool, clusters, self.config.sh_degree,
                                    self.config)
        return torch.round(image * 255.0).to(torch.uint8), overflow

    def __call__(self, camera: Camera | DeviceCamera, copy: bool = True):
        dcam = camera if isinstance(camera, DeviceCamera) else DeviceCamera.from_camera(
            camera, device=self.device)
        if not self.graphs:
            return self._frame(dcam)
        key = (dcam.width, dcam.height, dcam.near, dcam.far)
        if key not in self._frames:
            self._frames[key] = _Frame(self, dcam)
        image, overflow = self._frames[key](dcam)
        return (image.clone(), overflow.clone()) if copy else (image, overflow)

    def warmup(self, camera: Camera) -> dict:
        """Render every preset once (capturing its graph); first-call seconds."""
        import time

        times = {}
        for name, (width, height) in RESOLUTIONS.items():
            start = time.perf_counter()
            _, overflow = self(resize_camera(camera, width, height))
            torch.cuda.synchronize(self.device)
            if bool(overflow.item()):
                raise RuntimeError(f"{name}: visibility overflow; increase pair_capacity")
            times[name] = time.perf_counter() - start
        return times
