"""The north-star training step: cluster cull -> compact projection -> binning
-> raster forward -> fused L1+SSIM -> raster backward -> projection pullback,
with no host synchronisation (one stream, plus a second one for the stages
that can overlap).

Mirrors training/step.py:32-132 (compute_training_step) up to, not including,
the optimizer: the result is the loss, the parameter gradients in compact
visible-cluster order and the binning metrics.  Like the reference
(step.py:74-80), the packed tile shapes (kernels.PACKED_TILES: 8x8, 8x16,
12x16, 16x16) take packed_loss_and_grad's conventions -- image min(rgb, 1),
loss on it with the gradient taken as given, symmetric conic cotangents --
and other shapes take rasterize_loss_and_grad's (loss on clip(rgb, 0, 1)
with the clip's VJP); both run this backend's float32 compositing, which
meets the 1e-4 / 1e-3 parity bars (the reference packs the former as half2).

``GraphedTrainingStep`` captures the whole step once as a CUDA graph and
replays it: every size the kernels need is static (device-side counts bound
the work), so a replay issues the ~40 launches without host involvement.

Multi-GPU (view sharding): each rank renders its views and writes its
gradients in pool order; the ranks sum them with this library's own
NVLink collectives (NvlsExchange, captured into the step's graph) or with
NCCL (ViewShardedExchange).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch

from . import kernels as K
from .scene import CapacityConfig
from .types import DeviceCamera, GaussianArrays


_SIDE_STREAMS: dict = {}


def _side_stream(device) -> torch.cuda.Stream:
    key = torch.device(device).index
    if key not in _SIDE_STREAMS:
        _SIDE_STREAMS[key] = torch.cuda.Stream(device=device)
    return _SIDE_STREAMS[key]


@dataclass
class StepOutput:
    loss: torch.Tensor            # [] float32 (device)
    gradients: tuple              # (xyz, log_scale, rotation, opacity, sh) compact order
    visible_clusters: tuple       # (ids, count)
    pair_count: torch.Tensor      # [1] int32
    overflow: torch.Tensor        # [1] int32
    point_counts: torch.Tensor | None = None  # [C] int32 pairs per Gaussian
    image: torch.Tensor | None = None
    stats: torch.Tensor | None = None  # [C, 4] fragment statistics (collect_stats)


def compute_training_step(pool: GaussianArrays, bounds, camera: DeviceCamera, target: torch.Tensor,
                          config: CapacityConfig, active_degree: int, *,
                          active_sh_only: bool = True, sh_color_only: bool = False,
                          keep_image: bool = False, stage_events: dict | None = None,
                          overlap: bool = True, pool_grads=None, collect_stats: bool = False,
                          stats: torch.Tensor | None = None,
                          packed: bool | None = None) -> StepOutput:
    """training/step.py:32-89 without the optimizer update.

    bounds: world cluster bounds (center, extent, valid) on the device.
    target: uint8 [H, W, 3] (normalised in the loss kernel) or float [0, 1].
    The culled pool's alive mask (render/pipeline.py:44, alive & slots) equals
    the pool's alive mask on every listed cluster, which is all the compact
    projection reads, so it is not materialised.
    stage_events: optional dict; receives (start, end) CUDA events recorded on
    the current stream around each stage (cull, project, bin, raster_fwd,
    loss, raster_bwd, project_bwd).
    overlap: run the splat packing and the backward preparation on a second
    stream (joined back before their consumers); False keeps one stream.
    pool_grads: optional (xyz, log_scale, rotation, opacity, sh) tensors; the
    gradients are then written there in pool order (rows of culled clusters
    zero), ready to be summed across view-sharded ranks in place.
    collect_stats: also gather this view's [C, 4] fragment statistics (count,
    compositing weight, alpha cotangent, squared opacity cotangent); with
    stats given they are added into it in place (step.py:125-126,
    stats = stats + fragment_stats), and StepOutput.stats is that tensor.
    packed: the packed_loss_and_grad conventions (see the module docstring);
    None picks them for the packed tile shapes, as training/step.py:74-80
    does (shapes it would reject take the fp32 conventions here).
    """
    if packed is None:
        packed = (config.raster_tile_height, config.tile_size) in K.PACKED_TILES
    stream = torch.cuda.current_stream()

    def mark(name):
        if stage_events is None:
            return None
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record(stream)
        stage_events[name] = ev
        return ev

    def done(ev):
        if ev is not None:
            ev[1].record(stream)

    # Work that depends on fewer inputs than its position in the chain runs on
    # a second stream, joined back before its consumer: the splat records
    # (need the projection) overlap the binning, and the cotangent zeroing and
    # backward tile order (need the forward) overlap the loss.
    side = _side_stream(stream.device) if overlap else None
    ev = mark("cull")
    clusters, _ = K.compact_visible_clusters(bounds, camera, config, want_slots=False)
    done(ev)
    ev = mark("project")
    projected, pullback = K.project_with_compact_pullback(
        pool, camera, config, active_degree, clusters, rgb_only=True,
        active_sh_only=active_sh_only, sh_color_only=sh_color_only, visible_color_only=True)
    done(ev)
    splats = None
    if side is not None:
        splats = torch.empty(config.max_gaussians, 12, dtype=torch.float32, device=stream.device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            K.pack_splats(projected, camera, config, out=splats)
    ev = mark("bin")
    table = K.build_sorted_visibility_table_cute(projected, camera, config)
    done(ev)
    if side is not None:
        stream.wait_stream(side)
    ev = mark("raster_fwd")
    result, cache = K.rasterize_forward(projected, table, camera, config, want_depth=False,
                                        want_alpha=False, splats=splats, clamp_rgb=packed)
    done(ev)
    buffers = K.BackwardBuffers(table, camera, config, visible_clusters=clusters,
                                collect_stats=collect_stats, symmetric_conic=packed)
    if side is not None:
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            K.prepare_rasterize_backward(cache, camera, config, buffers)
    ev = mark("loss")
    loss, drgb, _ = K._fused_loss(result.rgb, target, False, clip_input=not packed)
    done(ev)
    if side is not None:
        stream.wait_stream(side)
    ev = mark("raster_bwd")
    cot = K.rasterize_backward(projected, table, cache, drgb, camera, config, buffers=buffers)
    fragment_stats = None
    if collect_stats:
        cot, fragment_stats = cot
        if stats is not None:
            fragment_stats = stats.add_(fragment_stats)
    done(ev)
    ev = mark("project_bwd")
    grads = pullback(cot) if pool_grads is None else pullback(cot, out=pool_grads, compact=False)
    done(ev)
    return StepOutput(loss, grads, clusters, table.pair_count, table.overflow,
                      table.point_counts, result.rgb if keep_image else None, fragment_stats)


def required_pairs(pool: GaussianArrays, bounds, camera: DeviceCamera, config: CapacityConfig,
                   active_degree: int) -> int:
    """The (tile, Gaussian) pairs one view needs: the binning's pair count,
    which is not clamped to config.max_visibility_pairs (a view that
    overflows the arena still reports its total, sorted_binning.py:78 and
    :116).  Culls, projects and bins the view once; reads the count back
    to the host."""
    clusters, _ = K.compact_visible_clusters(bounds, camera, config, want_slots=False)
    projected, _ = K.project_with_compact_pullback(pool, camera, config, active_degree, clusters,
                                                   rgb_only=True, visible_color_only=True)
    table = K.build_sorted_visibility_table_cute(projected, camera, config)
    return int(table.pair_count.item())


def size_pair_arena(pool: GaussianArrays, bounds, cameras, config: CapacityConfig,
                    active_degree: int, margin: float = 1.25,
                    granule: int = 1 << 20) -> CapacityConfig:
    """config with max_visibility_pairs sized from the count pass: the
    largest required_pairs over `cameras` times `margin`, rounded up to a
    multiple of `granule` (a fixed default such as the reference's 8M can
    overflow a dense view; an oversized one costs memory and the sort
    grids' idle blocks)."""
    need = max(required_pairs(pool, bounds, cam, config, active_degree) for cam in cameras)
    pairs = max(granule, -(-int(math.ceil(need * margin)) // granule) * granule)
    if pairs >= 1 << 31:
        raise ValueError(f"{need} pairs per view exceed the 2^31 arena limit")
    return replace(config, max_visibility_pairs=pairs)


def render(camera: DeviceCamera, gaussians: GaussianArrays, visible_clusters, active_degree: int,
           pp: CapacityConfig):
    """render/pipeline.py:47-93 (fp32 compositing, the RGB-only forward):
    (image clipped to [0,1], primitive_visible, overflow)."""
    projected = K.project_cute(gaussians, camera, pp, active_degree, visible_clusters)
    table = K.build_sorted_visibility_table_cute(projected, camera, pp)
    result, _ = K.rasterize_forward(projected, table, camera, pp, want_depth=False,
                                    want_alpha=False, record=False)
    return result.rgb.clamp(0, 1), table.point_counts > 0, table.overflow


def pool_gradient_buffer(pool: GaussianArrays, config: CapacityConfig, active_degree: int,
                         active_sh_only: bool = True):
    """One flat float32 buffer and its (xyz, log_scale, rotation, opacity,
    sh) views in pool order: the view-sharded step writes its gradients there
    and the ranks sum the whole buffer with a single all-reduce."""
    C = config.max_gaussians
    shg = (active_degree + 1) ** 2 if active_sh_only else int(pool.sh.shape[1])
    sizes = (C * 3, C * 3, C * 4, C, C * shg * 3)
    flat = torch.empty(sum(sizes), dtype=torch.float32, device=pool.xyz.device)
    views, at = [], 0
    for n, shape in zip(sizes, ((C, 3), (C, 3), (C, 4), (C, 1), (C, shg, 3))):
        views.append(flat[at:at + n].view(shape))
        at += n
    return flat, tuple(views)


class ViewShardedExchange:
    """The gradient sum of the view-sharded step (one view per rank).

    Each rank's step writes, in pool order, its geometric gradients (xyz,
    log_scale, rotation, opacity: 11 floats per Gaussian) into one flat buffer
    and its masked colour cotangents (3 floats, the sh_color_only pullback)
    into a row that also carries its camera centre.  exchange() all-gathers
    the rows, sums the geometric buffer with one all-reduce and, while that
    runs, expands every view's colour cotangents into the summed SH gradients
    (training/sh_pullback.py:18-53 summed over the views).  The result equals
    the all-reduced per-view gradients with SH, while 12 instead of 192
    bytes per Gaussian and view cross NVLink for the SH part.
    """

    def __init__(self, pool: GaussianArrays, config: CapacityConfig, active_degree: int,
                 group=None, active_sh_only: bool = True):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.degree = active_degree
        self.sh_dim = (active_degree + 1) ** 2 if active_sh_only else int(pool.sh.shape[1])
        self.xyz = pool.xyz
        C = config.max_gaussians
        dev = pool.xyz.device
        self.geometric = torch.empty(C * 11, dtype=torch.float32, device=dev)
        at, views = 0, []
        for n, shape in ((C * 3, (C, 3)), (C * 3, (C, 3)), (C * 4, (C, 4)), (C, (C, 1))):
            views.append(self.geometric[at:at + n].view(shape))
            at += n
        # [camera centre 3 | pad 1 | colour cotangents C*3] per rank.
        self.row = torch.zeros(4 + C * 3, dtype=torch.float32, device=dev)
        self.center = self.row[:3]
        self.colors = self.row[4:].view(C, 1, 3)
        self.rows = torch.empty(self.world, 4 + C * 3, dtype=torch.float32, device=dev)
        self.sh = torch.empty(C, self.sh_dim, 3, dtype=torch.float32, device=dev)
        self.pool_grads = (*views, self.colors)
        self.step_kwargs = dict(pool_grads=self.pool_grads, sh_color_only=True)

    def exchange(self, camera_center: torch.Tensor):
        """Sum the ranks' gradients; returns (xyz, log_scale, rotation,
        opacity, sh) in pool order, identical on every rank."""
        self.center.copy_(camera_center.reshape(3))
        self.dist.all_gather_into_tensor(self.rows, self.row, group=self.group)
        work = self.dist.all_reduce(self.geometric, group=self.group, async_op=True)
        K.sh_from_colors(self.xyz, None, self.rows, self.degree, self.sh_dim, out=self.sh)
        work.wait()
        return (*self.pool_grads[:4], self.sh)


class NvlsExchange:
    """ViewShardedExchange's sum with collectives written for NVLink /
    NVSwitch multicast (include/gsb200.h, gsb_exchange_barrier,
    gsb_nvls_allreduce, gsb_multicast_nonzero).

    The geometric gradients and a table of colour rows live in symmetric
    memory.  The step's pullback writes the geometric gradients and this
    rank's colour cotangents (row r of the table: [camera centre | pad |
    colours]) locally.  exchange() stores the camera centre into the row,
    pushes the row's non-zero 16-byte chunks (most of a view is zero)
    through the multicast address into every GPU's copy, passes a cross-GPU
    barrier, sums shard r of the geometric gradients (allreduce="p2p": peer
    loads of every copy's shard r, added in rank order, stored into every
    copy; "nvls": multimem.ld_reduce in the switch and multimem.st) while a
    second stream expands the gathered colours into the summed SH
    gradients and clears the table, and passes a second barrier.  No NCCL
    call is made per step and every launch can be captured in a CUDA graph.
    Build it only when NvlsExchange.available(group) says the GPUs share
    multicast.

    deferred_sh: the SH gradients stay in the reference's deferred form
    (training/step.py:55-66): exchange() gathers every view's colour row
    and camera centre into dense rows and returns them instead of expanding
    them, and the optimizer rebuilds the SH gradients
    (sparse_adam_update(..., sh_pullback_rows=rows)).  The dense rows are
    cleared by begin_step() (call it before the step's work, after the
    previous rows' consumer) or at the start of exchange().
    colour_push says how the rows travel:
      "compact" (default): this rank appends (id, r, g, b) for every
        Gaussian with a non-zero colour cotangent to its row of a symmetric
        table through the multicast address, whole lines through the switch
        (gsb_colour_push_compact), and after the second barrier every rank
        scatters the entries into its local dense rows (gsb_colour_expand).
        Two tables alternate by a device word, so the push leaves right
        after the step, beside the first barrier: a peer still expanding
        the previous step's entries reads the other table.
      "sparse": the dense rows themselves are the symmetric table; the
        dense row's non-zero 16-byte chunks are stored into every copy
        after the first barrier (a peer must not push into rows this rank
        has not consumed yet), beside the all-reduce.
    """

    @staticmethod
    def available(group=None) -> bool:
        try:
            import torch.distributed as dist
            import torch.distributed._symmetric_memory as symm_mem

            probe = symm_mem.empty(4, dtype=torch.float32, device=torch.cuda.current_device())
            handle = symm_mem.rendezvous(probe, group or dist.group.WORLD)
            return int(handle.multicast_ptr) != 0
        except Exception:
            return False

    def __init__(self, pool: GaussianArrays, config: CapacityConfig, active_degree: int,
                 group=None, active_sh_only: bool = True, allreduce: str = "auto",
                 deferred_sh: bool = False, colour_push: str = "compact"):
        import ctypes

        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        from . import _lib

        self.L = _lib
        group = group or dist.group.WORLD
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.degree = active_degree
        self.sh_dim = (active_degree + 1) ** 2 if active_sh_only else int(pool.sh.shape[1])
        self.xyz = pool.xyz
        C = config.max_gaussians
        dev = pool.xyz.device
        self.params = _lib.ExchangeParams(self.world, self.rank)
        self.geo_count = -(-(C * 11) // 4) * 4
        self.geometric = symm_mem.empty(self.geo_count, dtype=torch.float32, device=dev)
        # Row r = [camera centre 3 | pad 1 | colour cotangents C*3 | pad].
        self.row_floats = 4 + -(-(C * 3) // 4) * 4
        self.table = symm_mem.empty(self.world * self.row_floats, dtype=torch.float32, device=dev)
        if colour_push not in ("compact", "sparse"):
            raise ValueError("colour_push must be 'compact' or 'sparse'")
        self.compact_push = bool(deferred_sh) and colour_push == "compact"
        if self.compact_push:
            # Two tables of rows [centre 3 | entry count | C entries of
            # (id, r, g, b)], alternating by a device word.
            self.compact_floats = 4 + 4 * C
            self.compact = symm_mem.empty(2 * self.world * self.compact_floats,
                                          dtype=torch.float32, device=dev)
            self.compact.zero_()
            self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
            self.slot = torch.zeros(1, dtype=torch.int32, device=dev)
        self.flags = symm_mem.empty(self.world, dtype=torch.int32, device=dev)
        self.flags.zero_()
        self.geometric.zero_()
        self.table.zero_()
        h_geo = symm_mem.rendezvous(self.geometric, group)
        h_tab = symm_mem.rendezvous(self.table, group)
        h_flags = symm_mem.rendezvous(self.flags, group)
        if not (int(h_geo.multicast_ptr) and int(h_tab.multicast_ptr)):
            raise RuntimeError("NVLS multicast is not available for this group")
        self._handles = (h_geo, h_tab, h_flags)
        if self.compact_push:
            h_cmp = symm_mem.rendezvous(self.compact, group)
            if not int(h_cmp.multicast_ptr):
                raise RuntimeError("NVLS multicast is not available for this group")
            self._handles += (h_cmp,)
            table_bytes = self.world * self.compact_floats * 4
            self.mc_compact = [int(h_cmp.multicast_ptr) + t * table_bytes
                               + self.rank * self.compact_floats * 4 for t in (0, 1)]
            self.compact_tables = [self.compact.data_ptr() + t * table_bytes for t in (0, 1)]
        self.mc_geo = int(h_geo.multicast_ptr)
        # allreduce: "p2p" (plain peer loads/stores, up to 8 ranks), "nvls"
        # (multimem reduction in the switch) or "auto".  Per GPU and direction
        # P2P moves 2 (N-1)/N of the buffer over NVLink and the switch form
        # about (N+1)/N of it, so P2P is chosen for up to 3 ranks (at 2 it
        # took 77 us against 131 us for the 44 MB buffer).
        if allreduce not in ("p2p", "nvls", "auto"):
            raise ValueError("allreduce must be 'p2p', 'nvls' or 'auto'")
        if allreduce == "auto":
            allreduce = "p2p" if self.world <= 3 else "nvls"
        self.allreduce = "nvls" if self.world > 8 else allreduce
        self.geo_peers = (ctypes.c_void_p * self.world)(*[int(x) for x in h_geo.buffer_ptrs])
        self.mc_row = int(h_tab.multicast_ptr) + self.rank * self.row_floats * 4
        self.peer_flags = torch.tensor(list(h_flags.buffer_ptrs), dtype=torch.int64, device=dev)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.error = torch.zeros(1, dtype=torch.int32, device=dev)
        self.rows = self.table.view(self.world, self.row_floats)
        self.sh = torch.empty(C, self.sh_dim, 3, dtype=torch.float32, device=dev)
        at, views = 0, []
        for n, shape in ((C * 3, (C, 3)), (C * 3, (C, 3)), (C * 4, (C, 4)), (C, (C, 1))):
            views.append(self.geometric[at:at + n].view(shape))
            at += n
        # The pullback's colour-only output [C, 1, 3] is this rank's row: row
        # r of the table itself, or (deferred, where the table is cleared
        # while the step runs) a local row that the push copies into it.
        self.deferred_sh = bool(deferred_sh)
        if self.deferred_sh:
            self.own_row = torch.zeros(self.row_floats, dtype=torch.float32, device=dev)
        else:
            self.own_row = self.rows[self.rank]
        colours = self.own_row[4:4 + C * 3].view(C, 1, 3)
        self.pool_grads = (*views, colours)
        self.step_kwargs = dict(pool_grads=self.pool_grads, sh_color_only=True)
        self.side = torch.cuda.Stream(device=dev)
        self._cleared = False
        torch.cuda.synchronize(dev)
        dist.barrier(group)

    def _barrier(self):
        import ctypes

        L = self.L
        L.check(L.lib.gsb_exchange_barrier(
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), L.ref(self.params),
            ctypes.c_void_p(self.peer_flags.data_ptr()), ctypes.c_void_p(self.flags.data_ptr()),
            ctypes.c_void_p(self.epoch.data_ptr()), ctypes.c_void_p(self.error.data_ptr())),
            "exchange barrier")

    def begin_step(self) -> None:
        """Deferred mode: clear the colour table on the side stream, after
        everything queued so far on the current stream (the consumer of the
        previous rows); exchange() waits for it before its first barrier.
        Lets the clearing overlap the step's work; optional."""
        if not self.deferred_sh:
            return
        self.side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.side):
            self.table.zero_()
        self._cleared = True

    def _allreduce(self, stream, err) -> None:
        import ctypes

        L = self.L
        if self.allreduce == "p2p":
            L.check(L.lib.gsb_p2p_allreduce(ctypes.c_void_p(stream.cuda_stream), L.ref(self.params),
                                            self.geo_peers, self.geo_count, err), "P2P all-reduce")
        else:
            L.check(L.lib.gsb_nvls_allreduce(ctypes.c_void_p(stream.cuda_stream),
                                             L.ref(self.params), ctypes.c_void_p(self.mc_geo),
                                             self.geo_count, err), "NVLS all-reduce")

    def _exchange_compact(self, main, err):
        """Deferred SH, compact colour push: the push goes out at once (into
        the table the device slot picks; a peer may still be expanding the
        other one), then barrier -> geometric all-reduce -> barrier ->
        expand into the dense rows (cleared by begin_step) and advance the
        slot; returns the dense rows."""
        import ctypes

        L = self.L
        if not self._cleared:
            self.begin_step()
        self._cleared = False
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            L.check(L.lib.gsb_colour_push_compact(
                ctypes.c_void_p(self.side.cuda_stream), ctypes.c_void_p(self.own_row.data_ptr()),
                self.xyz.shape[0], ctypes.c_void_p(self.mc_compact[0]),
                ctypes.c_void_p(self.mc_compact[1]), ctypes.c_void_p(self.slot.data_ptr()),
                ctypes.c_void_p(self.counter.data_ptr()), err), "compact colour push")
        self._barrier()
        self._allreduce(main, err)
        main.wait_stream(self.side)
        self._barrier()
        L.check(L.lib.gsb_colour_expand(ctypes.c_void_p(main.cuda_stream),
                                        ctypes.c_void_p(self.compact_tables[0]),
                                        ctypes.c_void_p(self.compact_tables[1]),
                                        ctypes.c_void_p(self.slot.data_ptr()), self.world,
                                        self.xyz.shape[0], ctypes.c_void_p(self.table.data_ptr()),
                                        self.row_floats, err), "colour expand")
        return (*self.pool_grads[:4], self.rows)

    def _exchange_deferred(self, main, err):
        """Clear (unless begin_step did) -> barrier -> colour push beside the
        geometric all-reduce -> barrier; returns the gathered rows."""
        import ctypes

        L = self.L
        if self.compact_push:
            return self._exchange_compact(main, err)
        if not self._cleared:
            self.begin_step()
        self._cleared = False
        main.wait_stream(self.side)
        self._barrier()
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            L.check(L.lib.gsb_multicast_nonzero(ctypes.c_void_p(self.side.cuda_stream),
                                                ctypes.c_void_p(self.own_row.data_ptr()),
                                                ctypes.c_void_p(self.mc_row), self.row_floats,
                                                err), "colour row all-gather")
        self._allreduce(main, err)
        main.wait_stream(self.side)
        self._barrier()
        return (*self.pool_grads[:4], self.rows)

    def exchange(self, camera_center: torch.Tensor | None = None):
        """Sum the ranks' gradients after a step run with step_kwargs;
        returns (xyz, log_scale, rotation, opacity, sh) in pool order,
        identical on every rank -- with deferred_sh the last item is the
        gathered colour rows [world, row_floats] (each: camera centre, pad,
        C*3 masked colour cotangents) instead of SH gradients.
        camera_center: this rank's camera centre [3] on the device (it
        travels with the colour row)."""
        import ctypes

        L = self.L
        main = torch.cuda.current_stream()
        if camera_center is None:
            raise ValueError("NvlsExchange.exchange needs this rank's camera centre")
        self.own_row[:3].copy_(camera_center.reshape(3))
        err = ctypes.c_void_p(self.error.data_ptr())
        if self.deferred_sh:
            return self._exchange_deferred(main, err)
        L.check(L.lib.gsb_multicast_nonzero(ctypes.c_void_p(main.cuda_stream),
                                            ctypes.c_void_p(self.own_row.data_ptr()),
                                            ctypes.c_void_p(self.mc_row), self.row_floats, err),
                "colour row all-gather")
        self._barrier()
        self.side.wait_stream(main)
        self._allreduce(main, err)
        with torch.cuda.stream(self.side):
            K.sh_from_colors(self.xyz, None, self.rows, self.degree, self.sh_dim, out=self.sh)
            # The all-gather skips all-zero chunks, so the table must be zero
            # before the next step's rows arrive (they come after the next
            # barrier, which this rank reaches only after clearing).
            self.table.zero_()
        main.wait_stream(self.side)
        self._barrier()
        return (*self.pool_grads[:4], self.sh)

    def failed(self) -> bool:
        """Did a barrier give up waiting for a peer (host read, synchronises)?
        Once it did, the collectives return without touching their buffers,
        so the sums are stale: check this (or a StepMonitor) before an
        optimizer consumes them."""
        return bool(self.error.item())


class StepMonitor:
    """The trainer's failure checks (training/trainer.py:175-231) without a
    host synchronisation per step: record(out) folds each step's overflow
    word and pair count into device accumulators and keeps its loss;
    check(epoch) reads them once and raises RuntimeError, in the trainer's
    order, when a step overflowed the pair arena (bit 0 of the overflow
    word), when a binning look-back wait gave up (bit 1), or when the last
    recorded loss is not finite.  Returns {"epoch", "loss", "peak_pairs"}
    and clears the accumulators."""

    def __init__(self, pair_capacity: int, device=None):
        self.capacity = int(pair_capacity)
        self.overflow = torch.zeros(1, dtype=torch.int32, device=device)
        self.peak_pairs = torch.zeros(1, dtype=torch.int32, device=device)
        self.loss = torch.zeros((), dtype=torch.float32, device=device)

    def record(self, out: StepOutput) -> None:
        torch.bitwise_or(self.overflow, out.overflow.view(1), out=self.overflow)
        torch.maximum(self.peak_pairs, out.pair_count.view(1), out=self.peak_pairs)
        self.loss.copy_(out.loss.reshape(()))

    def check(self, epoch: int = 0) -> dict:
        overflow = int(self.overflow.item())
        peak = int(self.peak_pairs.item())
        loss = float(self.loss.item())
        self.overflow.zero_()
        self.peak_pairs.zero_()
        self.loss.zero_()
        if overflow & 2:
            raise RuntimeError(f"epoch {epoch}: a binning scan gave up waiting for its "
                               "predecessor; the table is incomplete")
        if overflow & 1:
            raise RuntimeError(f"epoch {epoch}: {peak} pairs exceed {self.capacity}")
        if not math.isfinite(loss):
            raise RuntimeError("non-finite training loss")
        return {"epoch": epoch, "loss": loss, "peak_pairs": peak}


def scatter_compact(grads, clusters, config: CapacityConfig, out=None):
    """Compact visible-cluster rows -> pool order (rows of unlisted clusters 0).

    Used by the view-sharded step to make per-view gradients summable.
    """
    ids, count = clusters
    n = int(count.item()) if count.numel() else 0
    cs = config.cluster_size
    slots = (ids[:n, None].long() * cs + torch.arange(cs, device=ids.device)).reshape(-1)
    keep = slots < config.max_gaussians
    rows = torch.arange(n * cs, device=ids.device)[keep]
    slots = slots[keep]
    outs = []
    for i, g in enumerate(grads):
        dst = torch.zeros_like(g) if out is None else out[i]
        dst.index_add_(0, slots, g[rows])
        outs.append(dst)
    return outs


class GraphedTrainingStep:
    """compute_training_step captured as CUDA graphs, then replayed.

    The pool, cluster bounds and the returned buffers keep their device
    addresses across replays (an in-place optimizer update of the pool is
    seen by the next replay).  Inputs are double-buffered: the step is
    captured once per input buffer (the captures share one memory pool and
    replay in order on the current stream), so that upload() can write the
    next step's camera and target straight into the buffer the next replay
    reads while the current one runs -- a loader's prefetch with no
    device-to-device copy.  A call with camera/target copies them into the
    next buffer first (host or device tensors; host tensors should be pinned
    for asynchronous copies); a call with neither replays the last inputs.
    With pool_grads the gradients land there in pool order on every replay.
    exchange: an NvlsExchange built for this step (its step_kwargs passed
    here too); its exchange() is captured after the step (and, deferred,
    its begin_step() before it), so each replay also sums the ranks'
    gradients with no host launch (every rank must replay in step).  The
    sums are self.gradients.
    """

    BUFFERS = 2

    def __init__(self, pool: GaussianArrays, bounds, camera: DeviceCamera, target: torch.Tensor,
                 config: CapacityConfig, active_degree: int, *, active_sh_only: bool = True,
                 sh_color_only: bool = False, warmup: int = 2, pool_grads=None,
                 collect_stats: bool = False,
                 stats: torch.Tensor | None = None, exchange=None):
        dev = pool.xyz.device
        # Each buffer's camera arrays are views of one packed buffer, so a new
        # camera arrives in one copy (DeviceCamera.pack).
        self.camera_flats, self.cameras, self.targets = [], [], []
        for _ in range(self.BUFFERS):
            flat = camera.pack().to(dev)
            self.camera_flats.append(flat)
            self.cameras.append(DeviceCamera.packed_views(flat, camera.width, camera.height,
                                                          camera.near, camera.far))
            buf = torch.empty_like(target, device=dev)
            buf.copy_(target)
            self.targets.append(buf)
        kwargs = dict(active_sh_only=active_sh_only, sh_color_only=sh_color_only,
                      pool_grads=pool_grads, collect_stats=collect_stats)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        self.exchange = exchange
        begin = getattr(exchange, "begin_step", None)
        with torch.cuda.stream(side):
            for _ in range(max(warmup, 1)):
                if begin is not None:
                    begin()
                compute_training_step(pool, bounds, self.cameras[0], self.targets[0], config,
                                      active_degree, **kwargs)
                if exchange is not None:
                    exchange.exchange(self.cameras[0].center)
        torch.cuda.current_stream(dev).wait_stream(side)
        # Statistics accumulate across replays into `stats` (the warm-up steps
        # above do not touch it): the captured step adds into it in place.
        if collect_stats:
            kwargs["stats"] = stats if stats is not None else torch.zeros(
                config.max_gaussians, 4, dtype=torch.float32, device=dev)
        from . import _lib

        mempool = torch.cuda.graph_pool_handle()
        self.graphs, self.outs, self.sums = [], [], []
        before = _lib.launch_count()
        for b in range(self.BUFFERS):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, pool=mempool):
                if begin is not None:
                    begin()
                out = compute_training_step(pool, bounds, self.cameras[b], self.targets[b],
                                            config, active_degree, **kwargs)
                sums = exchange.exchange(self.cameras[b].center) if exchange is not None else None
            self.graphs.append(graph)
            self.outs.append(out)
            self.sums.append(sums)
        self.launches_per_step = (_lib.launch_count() - before) // self.BUFFERS
        # Replay b has finished reading buffer b once done[b] has passed.
        self._done = [torch.cuda.Event() for _ in range(self.BUFFERS)]
        for ev in self._done:
            ev.record(torch.cuda.current_stream(dev))
        self._last = 0
        self._staged = None
        self._copy = None
        self._readback = None
        self._read_done = [None] * self.BUFFERS

    @property
    def out(self) -> StepOutput:
        """The latest replay's output buffers."""
        return self.outs[self._last]

    @property
    def camera(self) -> DeviceCamera:
        """The latest replay's camera arrays (device views)."""
        return self.cameras[self._last]

    @property
    def target(self) -> torch.Tensor:
        return self.targets[self._last]

    @property
    def gradients(self):
        """The latest replay's cross-rank gradient sums (with an exchange)."""
        return self.sums[self._last]

    def _check_inputs(self, camera, target) -> None:
        """The graphs keep the captured camera's image size and clip planes
        and the target's shape; a camera or target that differs would be
        replayed with the captured values, so it is refused."""
        ref_cam, ref_target = self.cameras[0], self.targets[0]
        if isinstance(camera, DeviceCamera):
            got = (camera.width, camera.height, float(camera.near), float(camera.far))
            want = (ref_cam.width, ref_cam.height, float(ref_cam.near), float(ref_cam.far))
            if got != want:
                raise ValueError(f"camera (width, height, near, far) {got} differs from the "
                                 f"captured {want}; capture another GraphedTrainingStep")
        elif camera is not None and camera.numel() != self.camera_flats[0].numel():
            raise ValueError(f"packed camera has {camera.numel()} values, expected "
                             f"{self.camera_flats[0].numel()}")
        if target is not None and (tuple(target.shape) != tuple(ref_target.shape)
                                   or target.dtype != ref_target.dtype):
            raise ValueError(f"target {tuple(target.shape)} {target.dtype} differs from the "
                             f"captured {tuple(ref_target.shape)} {ref_target.dtype}")

    def _write_inputs(self, b: int, camera, target) -> None:
        """Copy camera/target into buffer b on the current stream; inputs not
        given are carried over from the latest buffer."""
        last = self._last
        if isinstance(camera, DeviceCamera):
            dst = self.cameras[b]
            for d, src in ((dst.planes, camera.planes), (dst.world_to_camera, camera.world_to_camera),
                           (dst.intrinsics, camera.intrinsics), (dst.center, camera.center)):
                d.copy_(src.reshape(d.shape), non_blocking=True)
        elif camera is not None:
            self.camera_flats[b].copy_(camera.reshape(-1), non_blocking=True)
        elif b != last:
            self.camera_flats[b].copy_(self.camera_flats[last], non_blocking=True)
        if target is not None:
            self.targets[b].copy_(target, non_blocking=True)
        elif b != last:
            self.targets[b].copy_(self.targets[last], non_blocking=True)

    def upload(self, camera=None, target: torch.Tensor | None = None):
        """Write the next step's inputs (pinned host tensors, not modified
        until that step has run) into the next input buffer on a copy stream,
        so that their transfer overlaps the step in flight; the next call
        without arguments replays with them.  A data loader's prefetch: each
        step still moves its own inputs.  camera: a DeviceCamera or its
        packed [48] form (DeviceCamera.pack), which moves in one copy.  A
        camera of another image size or other clip planes, or a target of
        another shape or dtype, raises ValueError: only the captured ones can
        be replayed."""
        self._check_inputs(camera, target)
        dev = self.targets[0].device
        if self._copy is None:
            self._copy = torch.cuda.Stream(device=dev)
        if self._staged is not None:
            # A second upload before the staged one was consumed replaces it.
            torch.cuda.current_stream(dev).wait_event(self._staged[1])
            self._staged = None
        b = (self._last + 1) % self.BUFFERS
        # The replay that last read buffer b must be done with it (inputs not
        # given are copied over from the latest buffer, which the replay in
        # flight only reads).
        self._copy.wait_event(self._done[b])
        with torch.cuda.stream(self._copy):
            self._write_inputs(b, camera, target)
        ready = torch.cuda.Event()
        ready.record(self._copy)
        self._staged = (b, ready)

    def __call__(self, camera: DeviceCamera | None = None, target: torch.Tensor | None = None) -> StepOutput:
        self._check_inputs(camera, target)
        stream = torch.cuda.current_stream(self.targets[0].device)
        staged = self._staged
        if staged is not None:
            b, ready = staged
            stream.wait_event(ready)
            self._staged = None
            if camera is not None or target is not None:
                self._write_inputs(b, camera, target)
        elif camera is not None or target is not None:
            b = (self._last + 1) % self.BUFFERS
            self._write_inputs(b, camera, target)
        else:
            b = self._last
        if self._read_done[b] is not None:
            # A loss readback of this buffer's previous replay must finish
            # before the replay overwrites it.
            stream.wait_event(self._read_done[b])
            self._read_done[b] = None
        self.graphs[b].replay()
        self._done[b].record(stream)
        self._last = b
        return self.outs[b]

    def read_loss(self, dst: torch.Tensor) -> torch.cuda.Event:
        """Copy the latest replay's loss into dst (one float, pinned host
        memory) without holding up the next replay: the copy runs on a side
        stream after the step, and the replay that next overwrites this loss
        waits for the copy.  Returns the event that marks the copy done (dst
        is valid once it has passed)."""
        b = self._last
        dev = self.targets[0].device
        if self._readback is None:
            self._readback = torch.cuda.Stream(device=dev)
        step_done = torch.cuda.Event()
        step_done.record(torch.cuda.current_stream(dev))
        self._readback.wait_event(step_done)
        with torch.cuda.stream(self._readback):
            dst.copy_(self.outs[b].loss, non_blocking=True)
        copied = torch.cuda.Event()
        copied.record(self._readback)
        self._read_done[b] = copied
        return copied
