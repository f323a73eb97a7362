"""Torch-facing entry points of the hot path, one per reference binding.

Each function keeps the reference binding's name, argument meaning and error
behaviour (ValueError / RuntimeError before launch) and calls the C ABI of
libgsb200.so on the current CUDA stream.  Outputs are allocated with torch;
nothing synchronises with the host.

Reference bindings mirrored (src/jaxgs/...):
  project_cute / project_with_compact_pullback   kernels/projector.py:103-395
  compact_visible_clusters                        kernels/cluster_compact.py:31-44
  build_sorted_visibility_table_cute              kernels/sorted_binning.py:9-117
  rasterize_forward / rasterize_loss_and_grad     kernels/sorted_rasterizer.py:15-236
  fused_loss_and_grad(_with_scale)                kernels/fused_loss.py:333-352
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib as L
from .scene import CapacityConfig
from .types import (DeviceCamera, GaussianArrays, ProjectedGaussians, RasterCache, RenderResult,
                    SortedVisibilityTable)

_f32 = torch.float32
_i32 = torch.int32


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what} requires CUDA tensors (the sm_100a path has no CPU fallback)")


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


_ZEROS = {}


def _zeros(n: int, device) -> torch.Tensor:
    """Cached read-only zeros (background, absent cotangents)."""
    key = (str(device), n)
    if key not in _ZEROS:
        _ZEROS[key] = torch.zeros(n, dtype=_f32, device=device)
    return _ZEROS[key]


def _c(t: torch.Tensor, dtype=None) -> torch.Tensor:
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t if t.is_contiguous() else t.contiguous()


# ---------------------------------------------------------------------------
# Cluster culling (render/pipeline.py:18-44)
# ---------------------------------------------------------------------------
def compact_visible_clusters(bounds, camera: DeviceCamera, config: CapacityConfig,
                             want_slots: bool = True):
    """frustum_cluster_mask + compact_visible_clusters.

    bounds: (center [N,3], extent [N,3], valid [N] bool/uint8) device tensors.
    Returns ((ids [N] int32, count [1] int32), visible_slots [C] bool or None).
    """
    center, extent, valid = bounds
    _require_cuda(center, "compact_visible_clusters")
    n = int(valid.shape[0])
    ids = torch.empty(max(n, 1), dtype=_i32, device=center.device)
    count = torch.empty(1, dtype=_i32, device=center.device)
    slots = (torch.empty(config.max_gaussians, dtype=torch.uint8, device=center.device)
             if want_slots else None)
    p = L.ClusterParams(n, config.cluster_size, config.max_gaussians)
    ws = _workspace(L.lib.gsb_cluster_compact_workspace_size(L.ref(p)), center.device)
    L.check(L.lib.gsb_cluster_compact(_stream(), L.ref(p), _ptr(ws), ws.numel(),
                                      _ptr(_c(center, _f32)), _ptr(_c(extent, _f32)),
                                      _ptr(_c(valid, torch.uint8)), _ptr(_c(camera.planes, _f32)),
                                      _ptr(ids), _ptr(count), _ptr(slots)),
            "compact_visible_clusters")
    return (ids[:n] if n else ids[:0], count), (slots.bool() if want_slots else None)


def render_preprocess(cluster_bounds, camera: DeviceCamera, gaussians: GaussianArrays,
                      pp: CapacityConfig):
    """render/pipeline.py:18-44: visible clusters, slot mask, culled pool view."""
    clusters, slots = compact_visible_clusters(cluster_bounds, camera, pp)
    return clusters, slots, gaussians.replace(alive=gaussians.alive & slots)


# ---------------------------------------------------------------------------
# Projection (kernels/projector.py)
# ---------------------------------------------------------------------------
def _project(pool: GaussianArrays, camera: DeviceCamera, config: CapacityConfig,
             active_degree: int | None, clusters, clear_invisible: bool,
             visible_color_only: bool) -> ProjectedGaussians:
    _require_cuda(pool.xyz, "projection")
    C = config.max_gaussians
    if pool.capacity != C:
        raise ValueError("pool capacity must equal config.max_gaussians")
    degree = config.sh_degree if active_degree is None else active_degree
    if not 0 <= degree <= config.sh_degree:
        raise ValueError("active_degree must fit the pool's SH coefficients")
    dev = pool.xyz.device
    mean = torch.empty(C, 2, dtype=_f32, device=dev)
    depth = torch.empty(C, dtype=_f32, device=dev)
    conic = torch.empty(C, 2, 2, dtype=_f32, device=dev)
    radius = torch.empty(C, dtype=_f32, device=dev)
    color = torch.empty(C, 3, dtype=_f32, device=dev)
    alpha = torch.empty(C, dtype=_f32, device=dev)
    visible = torch.empty(C, dtype=torch.int8, device=dev)
    ids, count = (None, None) if clusters is None else clusters
    p = L.ProjectParams(C, int(pool.sh.shape[1]), degree, camera.width, camera.height, camera.near,
                        camera.far, config.cluster_size, int(clusters is not None),
                        int(clear_invisible), int(visible_color_only))
    L.check(L.lib.gsb_project_fwd(
        _stream(), L.ref(p), _ptr(_c(pool.xyz, _f32)), _ptr(_c(pool.log_scale, _f32)),
        _ptr(_c(pool.rotation, _f32)), _ptr(_c(pool.opacity, _f32)), _ptr(_c(pool.sh, _f32)),
        _ptr(_c(pool.alive, torch.uint8)), _ptr(_c(camera.world_to_camera, _f32)),
        _ptr(_c(camera.intrinsics, _f32)), _ptr(_c(camera.center, _f32)),
        _ptr(None if ids is None else _c(ids, _i32)), _ptr(None if count is None else _c(count, _i32)),
        _ptr(mean), _ptr(depth), _ptr(conic), _ptr(radius), _ptr(color), _ptr(alpha),
        _ptr(visible)), "projection")
    return ProjectedGaussians(mean, depth, conic, radius, color, alpha, visible)


def project_cute(pool: GaussianArrays, camera: DeviceCamera, config: CapacityConfig,
                 active_degree: int | None = None, compacted_clusters=None,
                 clear_invisible: bool = True) -> ProjectedGaussians:
    """kernels/projector.py:103-127 (plus the compact options of :17-100)."""
    return _project(pool, camera, config, active_degree, compacted_clusters, clear_invisible, False)


project = project_cute


def compute_projection_gradients(parameters, camera: DeviceCamera, projected_color,
                                 cotangents: ProjectedGaussians, config: CapacityConfig,
                                 active_degree: int | None, visible_clusters,
                                 compact_gradients: bool, rgb_only: bool = False,
                                 active_sh_only: bool = False, sh_color_only: bool = False,
                                 out=None):
    """kernels/projector.py:240-307: parameter gradients from cotangents.

    out: optional (xyz, log_scale, rotation, opacity, sh) gradient tensors to
    write (contiguous float32 of the output shapes), e.g. views of one flat
    buffer that a collective reduces in place."""
    xyz, log_scale, rotation, opacity, sh = parameters
    _require_cuda(xyz, "projection pullback")
    C = config.max_gaussians
    degree = config.sh_degree if active_degree is None else active_degree
    sh_dim = int(sh.shape[1])
    shg = 1 if sh_color_only else ((degree + 1) ** 2 if active_sh_only else sh_dim)
    dev = xyz.device
    shapes = ((C, 3), (C, 3), (C, 4), (C, 1), (C, shg, 3))
    if out is None:
        out = [torch.empty(shape, dtype=_f32, device=dev) for shape in shapes]
    else:
        out = list(out)[:len(shapes)]
        for o, shape in zip(out, shapes):
            if tuple(o.shape) != shape or o.dtype != _f32 or not o.is_contiguous():
                raise ValueError(f"gradient output must be contiguous float32 {shape}")
    ids, count = (None, None) if visible_clusters is None else visible_clusters
    p = L.ProjectBwdParams(C, sh_dim, shg, degree, camera.near, config.cluster_size,
                           int(visible_clusters is not None), int(compact_gradients),
                           int(rgb_only), int(sh_color_only))
    gdepth, gradius = cotangents.depth, cotangents.radius
    if rgb_only:
        gdepth = gradius = None
    args = (_stream(), L.ref(p), _ptr(_c(xyz, _f32)), _ptr(_c(log_scale, _f32)),
            _ptr(_c(rotation, _f32)), _ptr(_c(opacity, _f32)), _ptr(_c(sh, _f32)),
            _ptr(_c(camera.world_to_camera, _f32)), _ptr(_c(camera.intrinsics, _f32)),
            _ptr(_c(camera.center, _f32)), _ptr(_c(projected_color, _f32)),
            _ptr(None if ids is None else _c(ids, _i32)),
            _ptr(None if count is None else _c(count, _i32)),
            _ptr(_c(cotangents.mean, _f32)), _ptr(None if gdepth is None else _c(gdepth, _f32)),
            _ptr(_c(cotangents.conic, _f32)), _ptr(None if gradius is None else _c(gradius, _f32)),
            _ptr(_c(cotangents.color, _f32)), _ptr(_c(cotangents.alpha, _f32)),
            *[_ptr(o) for o in out])
    L.check(L.lib.gsb_project_bwd(*args), "projection pullback")
    return tuple(out)


def sh_from_colors(xyz: torch.Tensor, centers: torch.Tensor, colors: torch.Tensor,
                   degree: int, sh_dim: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """training/sh_pullback.py:18-53 summed over views: SH coefficient
    cotangents [C, sh_dim, 3] from per-view masked colour cotangents (the
    sh_color_only pullback output of each view, pool order) and the views'
    camera centres.  colors: [V, C, 3], or [V, >= 4 + C*3] rows holding a
    view's centre (3 floats and a pad) followed by its C*3 cotangents (then
    centers is None)."""
    _require_cuda(xyz, "SH reconstruction")
    C = int(xyz.shape[0])
    views = int(colors.shape[0])
    if centers is None:
        if colors.ndim != 2 or colors.shape[1] < C * 3 + 4 or not colors.is_contiguous():
            raise ValueError("packed colour rows must be [V, >= 4 + C*3] contiguous")
        row = int(colors.shape[1])
        p = L.ShParams(C, sh_dim, degree, views, row, row)
        centers_ptr = colors.data_ptr()
        colors_ptr = colors.data_ptr() + 4 * 4
    else:
        if tuple(colors.reshape(views, -1).shape) != (views, C * 3) or tuple(centers.shape) != (views, 3):
            raise ValueError("colors must be [V, C, 3] with centers [V, 3]")
        centers = _c(centers, _f32)
        colors = _c(colors, _f32)
        p = L.ShParams(C, sh_dim, degree, views, 0, 0)
        centers_ptr = centers.data_ptr()
        colors_ptr = colors.data_ptr()
    if out is None:
        out = torch.empty(C, sh_dim, 3, dtype=_f32, device=xyz.device)
    L.check(L.lib.gsb_sh_from_colors(_stream(), L.ref(p), _ptr(_c(xyz, _f32)),
                                     ctypes.c_void_p(centers_ptr), ctypes.c_void_p(colors_ptr),
                                     _ptr(out)),
            "SH reconstruction")
    return out


def project_with_compact_pullback(pool: GaussianArrays, camera: DeviceCamera,
                                  config: CapacityConfig, active_degree: int, clusters, *,
                                  rgb_only: bool = False, active_sh_only: bool = False,
                                  sh_color_only: bool = False, visible_color_only: bool = False):
    """kernels/projector.py:310-395: projection and a pullback producing
    gradients in visible-cluster order (only clusters[0][:count] rows valid)."""
    if not 0 <= active_degree <= config.sh_degree:
        raise ValueError("active_degree must fit the pool's SH coefficients")
    parameters = (pool.xyz, pool.log_scale, pool.rotation, pool.opacity, pool.sh)
    projected = _project(pool, camera, config, active_degree, clusters, False, visible_color_only)

    def pullback(cotangents: ProjectedGaussians, out=None, compact: bool = True):
        """Gradients in visible-cluster order, or (compact=False) in pool
        order with the unlisted clusters' rows zeroed; out as in
        compute_projection_gradients."""
        return compute_projection_gradients(parameters, camera, projected.color, cotangents,
                                            config, active_degree, clusters, compact, rgb_only,
                                            active_sh_only, sh_color_only, out=out)

    return projected, pullback


# ---------------------------------------------------------------------------
# Binning (kernels/sorted_binning.py:9-117)
# ---------------------------------------------------------------------------
def build_sorted_visibility_table_cute(projected: ProjectedGaussians, camera: DeviceCamera,
                                       config: CapacityConfig) -> SortedVisibilityTable:
    """LiteGS count / depth sort / scan / emit / tile sort / ranges."""
    _require_cuda(projected.mean, "binning")
    C = config.max_gaussians
    dev = projected.mean.device
    tw, th = config.tile_size, config.raster_tile_height
    tiles = (-(-camera.width // tw)) * (-(-camera.height // th))
    max_pairs = config.visibility_capacity
    counts = torch.empty(C, dtype=_i32, device=dev)
    ids = torch.empty(max_pairs, dtype=_i32, device=dev)
    offsets = torch.empty(tiles + 1, dtype=_i32, device=dev)
    pair_count = torch.empty(1, dtype=_i32, device=dev)
    overflow = torch.empty(1, dtype=_i32, device=dev)
    p = L.BinParams(C, camera.width, camera.height, tw, th, max_pairs)
    ws = _workspace(L.lib.gsb_bin_workspace_size(L.ref(p)), dev)
    L.check(L.lib.gsb_bin(_stream(), L.ref(p), _ptr(ws), ws.numel(),
                          _ptr(_c(projected.mean, _f32)), _ptr(_c(projected.conic, _f32)),
                          _ptr(_c(projected.alpha, _f32)), _ptr(_c(projected.depth, _f32)),
                          _ptr(_c(projected.visible, torch.int8)), _ptr(counts), _ptr(ids),
                          _ptr(offsets), _ptr(pair_count), _ptr(overflow)), "binning")
    return SortedVisibilityTable(ids, offsets, counts, pair_count, overflow)


build_sorted_visibility_table = build_sorted_visibility_table_cute


# ---------------------------------------------------------------------------
# fp32 rasterization (kernels/sorted_rasterizer.py)
# ---------------------------------------------------------------------------
def _tiles(camera: DeviceCamera, config: CapacityConfig) -> int:
    return (-(-camera.width // config.tile_size)) * (-(-camera.height // config.raster_tile_height))


def _raster_params(camera: DeviceCamera, config: CapacityConfig, max_pairs: int, flags: int = 0):
    return L.RasterParams(config.max_gaussians, camera.width, camera.height, config.tile_size,
                          config.raster_tile_height, int(max_pairs), flags)


def pack_splats(projected: ProjectedGaussians, camera: DeviceCamera, config: CapacityConfig,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """The first stage of rasterize_forward on its own (gsb_raster_pack): the
    48-byte splat records of the visible Gaussians.  It needs only the
    projection, so it can run on a second stream while the table is built;
    pass the result to rasterize_forward(splats=...)."""
    _require_cuda(projected.mean, "splat packing")
    dev = projected.mean.device
    splats = torch.empty(config.max_gaussians, 12, dtype=_f32, device=dev) if out is None else out
    p = _raster_params(camera, config, 0)
    L.check(L.lib.gsb_raster_pack(
        _stream(), L.ref(p), _ptr(_c(projected.mean, _f32)), _ptr(_c(projected.conic, _f32)),
        _ptr(_c(projected.color, _f32)), _ptr(_c(projected.alpha, _f32)),
        _ptr(_c(projected.visible, torch.int8)), _ptr(splats)), "splat packing")
    return splats


def rasterize_forward(projected: ProjectedGaussians, table: SortedVisibilityTable,
                      camera: DeviceCamera, config: CapacityConfig, background=None,
                      want_depth: bool = True, want_alpha: bool = True,
                      splats: torch.Tensor | None = None, record: bool = True,
                      clamp_rgb: bool = False, fragment_stats: torch.Tensor | None = None):
    """sorted_rasterizer.py:15-70: returns (RenderResult, RasterCache).

    The table may reference only visible Gaussians (others are not staged).
    splats: records already written by pack_splats (the packing stage is
    then skipped).  record=False is the inference forward
    (packed_rasterizer.py:219-232, record_contributions=False): the same
    image with no backward state, and the cache is None.  clamp_rgb writes
    min(rgb, 1), the packed rasterizer's output (packed_rasterize.py:396).
    fragment_stats: a [C * 2] float32 tensor that receives the forward's
    fragment statistics (count, weight per Gaussian, interleaved;
    packed_rasterize.py:363-377); recording forward only.
    """
    _require_cuda(projected.mean, "rasterization")
    C = config.max_gaussians
    dev = projected.mean.device
    W, H = camera.width, camera.height
    if background is None:
        background = _zeros(3, dev)
    rgb = torch.empty(H, W, 3, dtype=_f32, device=dev)
    out_depth = torch.empty(H, W, dtype=_f32, device=dev) if want_depth else None
    out_alpha = torch.empty(H, W, dtype=_f32, device=dev) if want_alpha else None
    final_t = torch.empty(H * W, dtype=_f32, device=dev) if record else None
    last = torch.empty(H * W, dtype=_i32, device=dev) if record else None
    work = torch.empty(_tiles(camera, config), dtype=_i32, device=dev) if record else None
    packed = splats is not None
    if not packed:
        splats = torch.empty(C, 12, dtype=_f32, device=dev)
    if fragment_stats is not None and (not record or fragment_stats.numel() != 2 * C):
        raise ValueError("fragment_stats needs the recording forward and C * 2 floats")
    p = _raster_params(camera, config, table.gaussian_ids.shape[0],
                       (L.RASTER_SPLATS_READY if packed else 0) | (0 if record else L.RASTER_RGB_ONLY)
                       | (L.RASTER_CLAMP_RGB if clamp_rgb else 0))
    bits = (torch.empty(max(int(L.lib.gsb_raster_bit_words(L.ref(p))), 1), dtype=_i32, device=dev)
            if record else None)
    ws = _workspace(L.lib.gsb_raster_workspace_size(L.ref(p)), dev)
    L.check(L.lib.gsb_raster_fwd(
        _stream(), L.ref(p), _ptr(ws), ws.numel(), _ptr(_c(projected.mean, _f32)),
        _ptr(_c(projected.conic, _f32)), _ptr(_c(projected.depth, _f32)),
        _ptr(_c(projected.color, _f32)), _ptr(_c(projected.alpha, _f32)),
        _ptr(_c(projected.visible, torch.int8)), _ptr(table.gaussian_ids),
        _ptr(table.tile_offsets), _ptr(_c(background, _f32)), _ptr(rgb), _ptr(out_depth),
        _ptr(out_alpha), _ptr(final_t), _ptr(last), _ptr(work), _ptr(splats), _ptr(bits),
        _ptr(None if fragment_stats is None else _c(fragment_stats, _f32))),
        "rasterization forward")
    cache = RasterCache(splats, final_t, last, work, bits) if record else None
    return RenderResult(rgb, out_depth, out_alpha), cache


class BackwardBuffers:
    """Outputs and workspace of one rasterize_backward call, allocated up
    front so that prepare_rasterize_backward can fill them on another stream.
    collect_stats: also gather the fragment statistics (statistics())."""

    def __init__(self, table: SortedVisibilityTable, camera: DeviceCamera, config: CapacityConfig,
                 visible_clusters=None, collect_stats: bool = False,
                 symmetric_conic: bool = False):
        C = config.max_gaussians
        dev = table.gaussian_ids.device
        self.gmean = torch.empty(C, 2, dtype=_f32, device=dev)
        self.gconic = torch.empty(C, 2, 2, dtype=_f32, device=dev)
        self.gdepth = torch.empty(C, dtype=_f32, device=dev)
        self.gcolor = torch.empty(C, 3, dtype=_f32, device=dev)
        self.galpha = torch.empty(C, dtype=_f32, device=dev)
        self.fragments = torch.empty(C * 3, dtype=_f32, device=dev) if collect_stats else None
        self.visible_clusters = visible_clusters
        self.symmetric_conic = symmetric_conic
        self.max_pairs = int(table.gaussian_ids.shape[0])
        rp = _raster_params(camera, config, self.max_pairs)
        self.workspace = _workspace(L.lib.gsb_raster_workspace_size(L.ref(rp)), dev)
        self.prepared = False

    def params(self, camera: DeviceCamera, config: CapacityConfig, flags: int = 0):
        if self.symmetric_conic:
            flags |= L.RASTER_BWD_SYMMETRIC_CONIC
        return L.RasterBwdParams(config.max_gaussians, camera.width, camera.height,
                                 config.tile_size, config.raster_tile_height, config.cluster_size,
                                 self.max_pairs, flags)

    def statistics(self) -> torch.Tensor:
        """[C, 4] fragment statistics of the backward: composited fragment
        count, compositing weight sum, alpha cotangent, squared opacity
        cotangent sum (kernels/sorted_rasterizer.py:227-235)."""
        if self.fragments is None:
            raise ValueError("these backward buffers do not collect fragment statistics")
        f = self.fragments.view(-1, 3)
        return torch.stack((f[:, 0], f[:, 1], self.galpha, f[:, 2]), dim=1)

    def clusters(self):
        ids, count = (None, None) if self.visible_clusters is None else self.visible_clusters
        return (_ptr(None if ids is None else _c(ids, _i32)),
                _ptr(None if count is None else _c(count, _i32)))


def prepare_rasterize_backward(cache: RasterCache, camera: DeviceCamera, config: CapacityConfig,
                               buffers: BackwardBuffers) -> BackwardBuffers:
    """The preparation stages of rasterize_backward on their own
    (gsb_raster_bwd_prepare): zero the cotangents and order the tiles by the
    forward's backward work.  Needs only the forward, so it can overlap the
    loss on a second stream."""
    p = buffers.params(camera, config)
    ids, count = buffers.clusters()
    L.check(L.lib.gsb_raster_bwd_prepare(
        _stream(), L.ref(p), _ptr(buffers.workspace), buffers.workspace.numel(),
        _ptr(cache.backward_work), ids, count, _ptr(buffers.gmean), _ptr(buffers.gconic),
        _ptr(buffers.gdepth), _ptr(buffers.gcolor), _ptr(buffers.galpha),
        _ptr(buffers.fragments)),
        "rasterization backward preparation")
    buffers.prepared = True
    return buffers


def rasterize_backward(projected: ProjectedGaussians, table: SortedVisibilityTable,
                       cache: RasterCache, drgb: torch.Tensor, camera: DeviceCamera,
                       config: CapacityConfig, background=None, ddepth=None, dalpha=None,
                       visible_clusters=None, buffers: BackwardBuffers | None = None,
                       collect_stats: bool = False) -> ProjectedGaussians:
    """sorted_rasterize.py:91-236: projected-field cotangents (mean, conic,
    depth, color, alpha).  With visible_clusters only those clusters' rows
    are zeroed and defined, and depth cotangents are left undefined.
    buffers: from BackwardBuffers (and prepare_rasterize_backward, which then
    replaces the zeroing and ordering stages); its visible_clusters and
    collect_stats are used.  With fragment statistics (collect_stats, or
    buffers made with it) the result is (cotangents, [C, 4] statistics), as
    kernels/packed_rasterizer.py:96-175 returns a pair."""
    _require_cuda(drgb, "rasterization backward")
    C = config.max_gaussians
    dev = drgb.device
    if background is None:
        background = _zeros(3, dev)
    if buffers is None:
        buffers = BackwardBuffers(table, camera, config, visible_clusters, collect_stats)
    elif collect_stats and buffers.fragments is None:
        raise ValueError("collect_stats needs BackwardBuffers made with collect_stats")
    if ddepth is not None and buffers.visible_clusters is not None:
        raise ValueError("depth cotangents are not defined with visible_clusters")
    p = buffers.params(camera, config, L.RASTER_BWD_PREPARED if buffers.prepared else 0)
    ids, count = buffers.clusters()
    L.check(L.lib.gsb_raster_bwd(
        _stream(), L.ref(p), _ptr(buffers.workspace), buffers.workspace.numel(),
        _ptr(cache.splats), _ptr(_c(projected.depth, _f32)), _ptr(table.gaussian_ids),
        _ptr(table.tile_offsets), _ptr(_c(background, _f32)), _ptr(cache.final_t),
        _ptr(cache.last), _ptr(cache.backward_work), _ptr(cache.contribution_bits),
        _ptr(_c(drgb, _f32)), _ptr(None if ddepth is None else _c(ddepth, _f32)),
        _ptr(None if dalpha is None else _c(dalpha, _f32)), ids, count,
        _ptr(buffers.gmean), _ptr(buffers.gconic), _ptr(buffers.gdepth), _ptr(buffers.gcolor),
        _ptr(buffers.galpha), _ptr(buffers.fragments)),
        "rasterization backward")
    # The radius cotangent of a rasterizer is zero (sorted_rasterizer.py:224).
    radius = _zeros(1, dev).expand(C)
    cot = projected.replace(mean=buffers.gmean, conic=buffers.gconic, depth=buffers.gdepth,
                            color=buffers.gcolor, alpha=buffers.galpha, radius=radius)
    if buffers.fragments is not None:
        return cot, buffers.statistics()
    return cot


# ---------------------------------------------------------------------------
# Fused loss (kernels/fused_loss.py:333-352)
# ---------------------------------------------------------------------------
def _fused_loss(prediction: torch.Tensor, target: torch.Tensor, with_scale: bool,
                clip_input: bool = False):
    if prediction.ndim != 3 or prediction.shape[2] != 3 or tuple(target.shape) != tuple(prediction.shape):
        raise ValueError("L1+SSIM expects matching HWC RGB images")
    _require_cuda(prediction, "fused loss")
    H, W, _ = prediction.shape
    dev = prediction.device
    u8 = target.dtype == torch.uint8
    grad = torch.empty(H, W, 3, dtype=_f32, device=dev)
    loss = torch.empty(1, dtype=_f32, device=dev)
    scale = torch.empty(1, dtype=_f32, device=dev) if with_scale else None
    p = L.LossParams(W, H, int(u8), int(clip_input))
    ws = _workspace(L.lib.gsb_loss_workspace_size(L.ref(p)), dev)
    L.check(L.lib.gsb_loss(_stream(), L.ref(p), _ptr(ws), ws.numel(),
                           _ptr(_c(prediction, _f32)), _ptr(_c(target, None if u8 else _f32)),
                           _ptr(loss), _ptr(grad), _ptr(scale)), "fused loss")
    return loss[0], grad, scale


def fused_loss_and_grad(prediction: torch.Tensor, target: torch.Tensor):
    """Mean L1(0.8)+SSIM(0.2) and its image gradient; uint8 or float target."""
    loss, grad, _ = _fused_loss(prediction, target, False)
    return loss, grad


def fused_loss_and_grad_with_scale(prediction: torch.Tensor, target: torch.Tensor):
    """Also the floored max |grad| (the packed rasterizer's gradient scale)."""
    return _fused_loss(prediction, target, True)


def rasterize_loss_and_grad(projected: ProjectedGaussians, table: SortedVisibilityTable,
                            camera: DeviceCamera, config: CapacityConfig, target: torch.Tensor,
                            collect_stats: bool = False, visible_clusters=None):
    """kernels/sorted_rasterizer.py:165-236: fp32 forward, loss on
    clip(rgb, 0, 1) with the clip's VJP, fp32 backward.  Returns
    (loss, cotangents, stats): stats is the [C, 4] fragment statistics
    (count, weight, alpha cotangent, squared opacity cotangent) with
    collect_stats, else zeros, as sorted_rasterizer.py:227-235 returns."""
    result, cache = rasterize_forward(projected, table, camera, config, want_depth=False,
                                      want_alpha=False)
    loss, drgb, _ = _fused_loss(result.rgb, target, False, clip_input=True)
    cot = rasterize_backward(projected, table, cache, drgb, camera, config,
                             visible_clusters=visible_clusters, collect_stats=collect_stats)
    if collect_stats:
        return loss, cot[0], cot[1]
    return loss, cot, torch.zeros(config.max_gaussians, 4, dtype=_f32, device=drgb.device)


# ---------------------------------------------------------------------------
# The packed rasterizer's entry points (kernels/packed_rasterizer.py:23-216),
# the ones the reference's training step calls for 8- and 16-pixel-wide
# tiles (training/step.py:74-80).
# ---------------------------------------------------------------------------
PACKED_TILES = ((8, 8), (8, 16), (12, 16), (16, 16))  # (tile_height, tile_size)


def _check_packed_tiles(config: CapacityConfig) -> None:
    if (config.raster_tile_height, config.tile_size) not in PACKED_TILES:
        raise ValueError("Packed rasterizer supports tiles 8x8, 8x16, 12x16 and 16x16")


def packed_forward(projected: ProjectedGaussians, table: SortedVisibilityTable,
                   camera: DeviceCamera, config: CapacityConfig, collect_stats: bool = False):
    """kernels/packed_rasterizer.py:23-95: (rgb [H, W, 3], cache, stats).

    The same interface and output convention as the reference: rgb =
    min(colour, 1) over no background; cache holds what packed_backward
    needs (this backend's RasterCache: 48-byte splat records, final
    transmittance, last index, backward work, contribution words, in place
    of the reference's 32-byte half2 records); stats is the [C * 2]
    (fragment count, compositing weight) pairs with collect_stats, else a
    one-element placeholder, as the reference's output shapes are.  The
    compositing is float32 (fp32 fragments and transmittance; the reference
    packs them as half2), so images meet the 1e-4 fp32 bar.  The table may
    reference only visible Gaussians."""
    _check_packed_tiles(config)
    _require_cuda(projected.mean, "packed rasterization")
    C = config.max_gaussians
    dev = projected.mean.device
    stats = torch.empty(C * 2 if collect_stats else 1, dtype=_f32, device=dev)
    result, cache = rasterize_forward(projected, table, camera, config, want_depth=False,
                                      want_alpha=False, clamp_rgb=True,
                                      fragment_stats=stats if collect_stats else None)
    if not collect_stats:
        stats.zero_()
    return result.rgb, cache, stats


def packed_backward(projected: ProjectedGaussians, table: SortedVisibilityTable,
                    cache: RasterCache, image_grad: torch.Tensor, camera: DeviceCamera,
                    config: CapacityConfig, collect_stats: bool = False, *,
                    symmetric_conic: bool = False, visible_clusters=None,
                    image_grad_scale: torch.Tensor | None = None,
                    buffers: BackwardBuffers | None = None):
    """kernels/packed_rasterizer.py:98-177: (cotangents, alpha_grad_sq_sum).

    Field cotangents of the packed forward, with the reference's
    conventions: the image gradient is taken as given (the forward's clamp
    at 1 is not differentiated); symmetric_conic puts both off-diagonal
    contributions into conic[0, 1] and leaves conic[1, 0] zero (the
    analytic pullback reads their sum); with visible_clusters (which must
    hold every Gaussian of the table) mean, conic and colour cotangents are
    defined only in those clusters and depth cotangents nowhere, alpha
    cotangents everywhere when collecting statistics; the radius cotangent
    is zero.  alpha_grad_sq_sum is the per-Gaussian sum of squared opacity
    cotangents ([C]) with collect_stats, else a one-element zero.
    image_grad_scale is accepted for the reference's signature and not
    needed: the float32 backward does no range scaling.  buffers: from
    BackwardBuffers(..., symmetric_conic=...), optionally prepared on a
    second stream."""
    _check_packed_tiles(config)
    del image_grad_scale
    if buffers is None:
        buffers = BackwardBuffers(table, camera, config, visible_clusters, collect_stats,
                                  symmetric_conic=symmetric_conic)
    elif buffers.symmetric_conic != symmetric_conic:
        raise ValueError("buffers were made for the other conic convention")
    out = rasterize_backward(projected, table, cache, image_grad.reshape(camera.height,
                                                                         camera.width, 3),
                             camera, config, buffers=buffers, collect_stats=collect_stats)
    if collect_stats:
        cot, stats = out
        return cot, stats[:, 3].contiguous()
    return out, _zeros(1, image_grad.device)


def packed_loss_and_grad(projected: ProjectedGaussians, table: SortedVisibilityTable,
                         camera: DeviceCamera, config: CapacityConfig, target: torch.Tensor,
                         collect_stats: bool, *, symmetric_conic: bool = False,
                         visible_clusters=None):
    """kernels/packed_rasterizer.py:180-216: (loss, cotangents, stats).

    packed_forward -> fused L1+SSIM on its (clamped) image -> packed_backward;
    stats is the detached [C, 4] (fragment count, compositing weight, alpha
    cotangent, squared opacity cotangent) with collect_stats, else zeros.
    visible_clusters limits the defined cotangents as in packed_backward."""
    image, cache, fragments = packed_forward(projected, table, camera, config, collect_stats)
    loss, image_grad, scale = fused_loss_and_grad_with_scale(image, target)
    gradients, square = packed_backward(projected, table, cache, image_grad, camera, config,
                                        collect_stats, symmetric_conic=symmetric_conic,
                                        visible_clusters=visible_clusters, image_grad_scale=scale)
    if collect_stats:
        stats = torch.stack((fragments[0::2], fragments[1::2], gradients.alpha, square), dim=1)
    else:
        stats = torch.zeros(config.max_gaussians, 4, dtype=_f32, device=image.device)
    return loss, gradients, stats
