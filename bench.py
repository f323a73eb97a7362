"""Benchmark of the north-star hot path: train views/sec (fwd+bwd+loss).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: 1,000,000-Gaussian pool (config-1 scene,
seed 2, all slots active, SH degree 3), 1237x822 pinhole camera fx=fy=1040 at
(0, 1.5, -6) looking at the origin, 8x16 tiles, uint8 target rendered from a
second random scene (seed 3).  One step = cluster cull + compact projection +
binning + fp32 raster forward + fused L1+SSIM + raster backward + projection
pullback to xyz/log_scale/rotation/opacity/SH (degree 3).  Synthetic data.

Multi-GPU (torchrun, one rank per GPU): every rank renders one view per step
(ring camera r of BASELINE config 3's ring, radius 6) and the ranks sum the
per-view gradients inside the step's CUDA graph (jaxgs_b200.step.NvlsExchange:
peer or NVLS all-reduce of the geometric gradients, multicast all-gather of
the non-zero colour cotangents, SH expansion of all views on every rank;
GSB_EXCHANGE=nccl takes ViewShardedExchange's NCCL collectives instead);
value = views of all ranks / max-over-ranks time.  stage_ms.exchange is the
exchange's own time in the eager steps.

--impl reference times the reference path's CPU restatement (oracle/, the
reference being JAX code that is not installed here) on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "train views/sec (fwd+bwd+loss) at 1M Gaussians, 1237x822"
UNIT = "views/s"


def _config():
    """Config 2's capacities; run_ours sizes the pair arena from the count
    pass (the 8M here, the reference's default, is only the probe's)."""
    from jaxgs_b200.scene import CapacityConfig

    return CapacityConfig(max_gaussians=1_000_000, cluster_size=128, tile_size=16, sh_degree=3,
                          max_visibility_pairs=8_000_000, tile_height=8)


def _workload(rank: int):
    """(pool dict, camera, target uint8) of config 2; rank picks its ring camera."""
    import numpy as np

    from jaxgs_b200.scene import config1_scene, ring_cameras

    pool = config1_scene()
    camera = ring_cameras(8, radius=6.0, height=1.5)[rank % 8]
    return pool, camera


def _target(camera, device):
    """uint8 render of the seed-3 scene from the same camera (GPU forward)."""
    import torch

    from jaxgs_b200 import kernels as K
    from jaxgs_b200.scene import config1_scene
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    config = _config()
    other = GaussianArrays.from_numpy(config1_scene(seed=3), device=device)
    cam = DeviceCamera.from_camera(camera, device=device)
    projected = K.project_cute(other, cam, config)
    table = K.build_sorted_visibility_table_cute(projected, cam, config)
    result, _ = K.rasterize_forward(projected, table, cam, config, want_depth=False,
                                    want_alpha=False)
    target = (result.rgb.clamp(0, 1) * 255.0 + 0.5).to(torch.uint8)
    del other, projected, table, result
    return target


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "10"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def run_ours(args) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    from jaxgs_b200 import _lib
    from jaxgs_b200 import kernels as K
    from jaxgs_b200.scene import world_cluster_bounds
    from jaxgs_b200.step import (GraphedTrainingStep, NvlsExchange, ViewShardedExchange,
                                 compute_training_step)
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        # NCCL may print its version banner on stdout; keep stdout for the
        # one JSON line.
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=device)
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    config = _config()
    pool_np, camera = _workload(rank)
    pool = GaussianArrays.from_numpy(pool_np, device=device)
    center, extent, valid = world_cluster_bounds(pool_np, 128)
    bounds = (torch.as_tensor(center, device=device), torch.as_tensor(extent, device=device),
              torch.as_tensor(valid.astype(np.uint8), device=device))
    dcam = DeviceCamera.from_camera(camera, device=device)
    # The pair arena from the count pass over the ring's eight views (the
    # same on every rank), not a fixed default.
    from jaxgs_b200.scene import ring_cameras
    from jaxgs_b200.step import size_pair_arena

    ring = [DeviceCamera.from_camera(c, device=device)
            for c in ring_cameras(8, radius=6.0, height=1.5)]
    config = size_pair_arena(pool, bounds, ring, config, 3)
    del ring
    target = _target(camera, device)
    target_host = target.cpu().pin_memory()
    cam_host = [t.cpu().pin_memory() for t in (dcam.world_to_camera, dcam.intrinsics,
                                               dcam.center, dcam.planes)]
    degree = 3
    exch = None
    if world > 1:
        use_nvls = os.environ.get("GSB_EXCHANGE", "nvls") == "nvls" and NvlsExchange.available()
        if use_nvls:
            # GSB_ALLREDUCE: "auto" (default), "p2p" or "nvls" sum of the geometric gradients.
            exch = NvlsExchange(pool, config, degree,
                                allreduce=os.environ.get("GSB_ALLREDUCE", "auto"),
                                deferred_sh=args.sh == "deferred",
                                colour_push=os.environ.get("GSB_COLOUR_PUSH", "compact"))
        else:
            exch = ViewShardedExchange(pool, config, degree)
    # The reference's default step (optimizer "optax", config/default.toml:54)
    # defers the SH pullback to the optimizer (training/step.py:55-66): the
    # pullback gives the masked colour cotangent and the update rebuilds the
    # SH gradients.  --sh materialized writes all 16 SH gradients instead.
    deferred_sh = args.sh == "deferred" and not isinstance(exch, ViewShardedExchange)
    sharded = exch.step_kwargs if exch is not None else {"sh_color_only": deferred_sh}
    stream = torch.cuda.current_stream()
    stage_events = []
    current_center = [dcam.center]

    def eager_step(cam, tgt, record=False):
        events = {} if record else None
        out = compute_training_step(pool, bounds, cam, tgt, config, degree, stage_events=events,
                                    **sharded)
        if record:
            stage_events.append(events)
        return out

    def exchange(out):
        """View-sharded gradient sum (ViewShardedExchange: one all-reduce of
        the geometric gradients, all-gathers of the colour cotangents and
        camera centres, SH expansion)."""
        if exch is not None:
            exch.exchange(current_center[0])

    # Eager warm-up and the per-stage breakdown (events around each stage on
    # the launching stream; the dominant kernel's time comes from here).
    for _ in range(max(args.warmup, 0)):
        out = eager_step(dcam, target)
        exchange(out)
    for _ in range(args.steps):
        out = eager_step(dcam, target, record=True)
        if exch is not None:
            # The exchange as its own stage: barrier, gradient sum, colour
            # all-gather and SH expansion, on the launching stream.
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record(stream)
            exchange(out)
            ev[1].record(stream)
            stage_events[-1]["exchange"] = ev
    torch.cuda.synchronize()
    stage_ms = {}
    for events in stage_events:
        for name, (a, b) in events.items():
            stage_ms.setdefault(name, []).append(a.elapsed_time(b))
    stage_ms = {k: statistics.mean(v) for k, v in stage_ms.items()}
    pairs = int(out.pair_count.item())
    overflow = bool(out.overflow.item())
    visible_clusters = int(out.visible_clusters[1].item())
    binned = int((out.point_counts > 0).sum().item())
    # Every rank counts its own view's visits (only rank 0's is reported), so
    # no rank reaches the exchange's barriers while another is still here.
    visits = _backward_visits(pool, bounds, dcam, config, degree)

    # The product step: captured as CUDA graphs (one per input buffer),
    # replayed per view.  NvlsExchange's launches are captured into the
    # step's graphs as well.
    captured = isinstance(exch, NvlsExchange)
    graphed = GraphedTrainingStep(pool, bounds, dcam, target, config, degree, **sharded,
                                  exchange=exch if captured else None)
    if captured:
        def exchange(out):
            return None
    else:
        def exchange(out):
            """The NCCL exchange after the replay, with the replayed camera."""
            if exch is not None:
                exch.exchange(graphed.camera.center)
    for _ in range(max(args.warmup, 0)):
        out = graphed()
        exchange(out)
    torch.cuda.synchronize()

    # Device-resident timed region.
    sampler = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    launches0 = _lib.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        out = graphed()
        exchange(out)
    end.record(stream)
    torch.cuda.synchronize()
    eager_launches = _lib.launch_count() - launches0
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    elapsed = start.elapsed_time(end) / 1e3
    launches = eager_launches + graphed.launches_per_step * args.steps

    # End-to-end through the public API from pinned host buffers: each step
    # copies the camera arrays and the uint8 target to the device and reads
    # the loss back.
    e2e_loss = torch.empty(max(args.steps, 1), dtype=torch.float32).pin_memory()
    host_cam = DeviceCamera(cam_host[0], cam_host[1], cam_host[2], cam_host[3], camera.width,
                            camera.height, camera.near, camera.far)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    n_e2e = 0 if args.no_e2e else args.steps
    # The camera in its packed form (one 192-byte copy per step).
    cam_packed = host_cam.pack().pin_memory()
    if n_e2e:
        graphed.upload(cam_packed, target_host)
    for i in range(n_e2e):
        # Each step's inputs are uploaded from pinned host memory while the
        # previous step runs (a loader's prefetch); every step moves its own.
        out = graphed()
        if i + 1 < n_e2e:
            graphed.upload(cam_packed, target_host)
        exchange(out)
        # The step's loss to the host on a side stream (GraphedTrainingStep
        # makes the next replay of these buffers wait for the copy).
        read = graphed.read_loss(e2e_loss[i])
    if n_e2e:
        # The last readback is part of the timed region.
        stream.wait_event(read)
    e_end.record(stream)
    torch.cuda.synchronize()
    e2e_elapsed = e_start.elapsed_time(e_end) / 1e3 if not args.no_e2e else float("nan")
    h2d = target.numel() + DeviceCamera.PACKED_FLOATS * 4
    # Inference of the same view (RGB-only forward, uint8 frame), then the
    # consumer of the gradients (it updates the pool in place): visible-
    # cluster sparse Adam over the step's compact gradients.
    inference = _time_inference(pool, camera, stream) if world == 1 else None
    # The optimizer timings below update the pool; every measurement starts
    # from the benchmark's scene.
    fields = ("xyz", "log_scale", "rotation", "opacity", "sh")
    snapshot = [getattr(pool, f).clone() for f in fields]

    def restore():
        for f, saved in zip(fields, snapshot):
            getattr(pool, f).copy_(saved)

    optimizer = deferred = materialized = None
    if world == 1:
        # The step with the other SH form (all 16 SH gradients written by the
        # pullback, or deferred), on the same scene.
        materialized = _time_step_variant(pool, bounds, dcam, target, config, degree, stream,
                                          args.steps, sh_color_only=not deferred_sh)
        # Both forms of the update: rebuilding SH gradients from the colour
        # cotangent (the reference's default) and reading materialised ones.
        colour_out = compute_training_step(pool, bounds, dcam, target, config, degree,
                                           sh_color_only=True)
        deferred = _time_optimizer(pool, colour_out, stream, center=dcam.center)
        restore()
        full_out = compute_training_step(pool, bounds, dcam, target, config, degree)
        optimizer = _time_optimizer(pool, full_out, stream)
        restore()
        del colour_out, full_out
    # The whole training iteration (step, exchange, optimizer update) on the
    # same graph, every rank; it trains the scene as it goes.
    iteration = None
    if world == 1 or captured:
        iteration = _time_iteration(graphed, pool, stream, args.steps, world, deferred_sh,
                                    dcam.center)
        restore()
    if iteration is not None and world > 1:
        iteration["ms_per_step"] = _max_over_ranks(iteration["ms_per_step"], device)
        iteration["views_per_s"] = round(world * 1e3 / iteration["ms_per_step"], 1)
    del snapshot
    heavy = _time_config4(stream) if world == 1 and not args.no_config4 else None
    d2h = 4

    if world > 1:
        t = torch.tensor([elapsed, e2e_elapsed], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed, e2e_elapsed = float(t[0]), float(t[1])

    if rank == 0:
        views = world * args.steps
        value = views / elapsed
        peak, peak_kind = _peaks()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(elapsed / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "BASELINE config 2: 1M-Gaussian training step, 1237x822, 8x16 tiles, SH3",
                       "gaussians": 1_000_000, "width": 1237, "height": 822, "tile": "8x16",
                       "views_per_gpu_per_step": 1, "pairs": pairs, "overflow": overflow,
                       "pair_arena": config.max_visibility_pairs,
                       "visible_clusters": visible_clusters, "binned_gaussians": binned,
                       "l2": "inputs larger than L2 (236 MB pool)",
                       "launch": "CUDA graph replay of the whole step",
                       "parallelism": f"view-sharded dp{world}" if world > 1 else "single view",
                       "sh_gradients": ("deferred to the optimizer update as in the reference's "
                                        "default step (masked colour cotangents, SH rebuilt by "
                                        "gsb_sparse_adam_sh)" if deferred_sh else
                                        "all 16 coefficients written by the pullback"),
                       "exchange": _exchange_text(exch, config) if exch is not None else None},
            "e2e": {"value": None if args.no_e2e else round(world * args.steps / e2e_elapsed, 2),
                    "unit": UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches),
            "clocks": clocks,
            "stage_ms": {k: round(v, 4) for k, v in stage_ms.items()},
        }
        # Nine reductions per visit under the packed conventions (two mean,
        # three conic with the off-diagonal once, three colour, opacity).
        line["roofline"] = _roofline(stage_ms, peak, peak_kind, pairs, binned, visits,
                                     clocks.get("sm_mhz") or 1965.0, 9)
        if inference is not None:
            line["inference"] = inference
        line["iteration"] = iteration
        if materialized is not None:
            line["other_sh_form"] = materialized
        for key, entry in (("optimizer", optimizer), ("optimizer_deferred_sh", deferred)):
            if entry is not None:
                entry["frac"] = round(entry["achieved_gbs"] / peak, 4)
                entry["peak_gbs"] = peak
                line[key] = entry
        if heavy is not None:
            line["config4"] = heavy
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(pool_np, camera, target.cpu().numpy())
        print(json.dumps(line), flush=True)
    if world > 1:
        del graphed
        dist.destroy_process_group()


def _exchange_text(exch, config) -> str:
    """What the view-sharded exchange moves per step, for the JSON line."""
    from jaxgs_b200.step import NvlsExchange

    geo = exch.geometric.numel() * 4 / 1e6
    colours = config.max_gaussians * 12 / 1e6
    if isinstance(exch, NvlsExchange) and exch.deferred_sh:
        form = ("compact (id, rgb) entries of the Gaussians with a non-zero colour cotangent"
                if exch.compact_push else
                f"the non-zero 16-byte chunks of {colours:.0f} MB colour cotangents")
        return (f"per step, own kernels in the step's CUDA graph: {exch.allreduce.upper()} "
                f"all-reduce of {geo:.0f} MB geometric gradients beside the NVLS multicast "
                f"all-gather of every rank's colour row as {form}, scattered into dense rows; "
                "SH gradients rebuilt by the optimizer update")
    if isinstance(exch, NvlsExchange):
        return (f"per step, own kernels in the step's CUDA graph: {exch.allreduce.upper()} "
                f"all-reduce of {geo:.0f} MB geometric gradients, NVLS multicast all-gather of "
                f"the non-zero part of {colours:.0f} MB colour cotangents per rank, SH "
                "expansion of all views")
    return (f"per step, NCCL: all-reduce of {geo:.0f} MB geometric gradients, all-gather of "
            f"{colours:.0f} MB colour cotangents per rank, SH expansion of all views")


def _time_inference(pool, camera, stream, iters: int = 30) -> dict:
    """ViewRenderer frames (cull, project, bin, RGB-only raster, uint8) of
    the bench view, graph replays timed with CUDA events."""
    import torch

    from jaxgs_b200.view import ViewRenderer

    renderer = ViewRenderer(pool)
    for _ in range(3):
        renderer(camera, copy=False)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(iters):
        image, overflow = renderer(camera, copy=False)
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    return {"what": "ViewRenderer frame (uint8 1237x822, CUDA graph replay)",
            "ms_per_frame": round(ms, 4), "frames_per_s": round(1e3 / ms, 1),
            "overflow": bool(overflow.item())}


def _time_optimizer(pool, out, stream, iters: int = 20, center=None) -> dict:
    """sparse_adam_update's field launches over the step's compact
    gradients, CUDA events on the launching stream.  Algorithmic bytes: per
    element of an alive listed slot, value, both moments and the gradient
    read (16 B) and value and moments written (12 B); 59 elements per
    Gaussian at SH degree 3.  With `center` the SH gradient is the step's
    colour cotangent and the SH field's update rebuilds it
    (gsb_sparse_adam_sh): 24 B per SH element plus the colour cotangent and
    position read (24 B per slot)."""
    import torch

    from jaxgs_b200.optimizer import (PARAMETER_NAMES, create_adam_state,
                                      parameter_learning_rates, update_field,
                                      update_sh_from_colors)

    state = create_adam_state(pool)
    rates = torch.tensor(parameter_learning_rates(100, 1.0), dtype=torch.float32,
                         device=pool.xyz.device)

    def update():
        for i, name in enumerate(PARAMETER_NAMES):
            if name == "sh" and center is not None:
                update_sh_from_colors(pool.sh, state.m[i], state.v[i], pool.xyz, center,
                                      out.gradients[i], pool.alive, out.visible_clusters,
                                      rates[i:i + 1], 128, 3, True)
                continue
            update_field(getattr(pool, name), state.m[i], state.v[i], out.gradients[i],
                         pool.alive, out.visible_clusters, rates[i:i + 1], 128, name == "sh",
                         True)

    for _ in range(3):
        update()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(iters):
        update()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    count = int(out.visible_clusters[1].item())
    ids = out.visible_clusters[0][:count].long()
    slots = (ids[:, None] * 128 + torch.arange(128, device=ids.device)).reshape(-1)
    slots = slots[slots < pool.alive.shape[0]]
    alive = int(pool.alive[slots].to(torch.int64).sum().item())
    other = sum(getattr(pool, n)[0].numel() for n in PARAMETER_NAMES[:4])
    sh = pool.sh[0].numel()
    if center is None:
        nbytes = alive * (other + sh) * 28
        what = "sparse Adam, 5 fields (gsb_sparse_adam)"
    else:
        nbytes = alive * (other * 28 + sh * 24 + 24)
        what = ("sparse Adam, 4 fields (gsb_sparse_adam) + SH rebuilt from the colour "
                "cotangent inside its update (gsb_sparse_adam_sh)")
    return {"kernel": what, "ms": round(ms, 4), "slots": alive, "bytes": nbytes,
            "achieved_gbs": round(nbytes / ms / 1e6, 1), "unit": "GB/s"}


def _max_over_ranks(x: float, device) -> float:
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(x)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return round(float(t), 4)


def _time_iteration(graphed, pool, stream, steps: int, world: int, deferred_sh: bool,
                    center) -> dict:
    """The whole training iteration: the graph replay (step and, with
    several ranks, the exchange) followed by the sparse Adam update of every
    field from its output (deferred SH: rebuilt from the colour cotangent
    or, view-sharded, from the gathered colour rows of every view).  CUDA
    events around `steps` iterations after three untimed ones."""
    import torch

    from jaxgs_b200.optimizer import (PARAMETER_NAMES, create_adam_state,
                                      parameter_learning_rates, update_field,
                                      update_sh_from_colors, update_sh_from_rows)

    state = create_adam_state(pool)
    rates = torch.tensor(parameter_learning_rates(100, 1.0), dtype=torch.float32,
                         device=pool.xyz.device)
    n_clusters = -(-pool.xyz.shape[0] // 128)
    all_clusters = (torch.arange(n_clusters, dtype=torch.int32, device=pool.xyz.device),
                    torch.tensor([n_clusters], dtype=torch.int32, device=pool.xyz.device))

    def one():
        out = graphed()
        if world > 1:
            grads, clusters, compact = graphed.gradients, all_clusters, False
        else:
            grads, clusters, compact = out.gradients, out.visible_clusters, True
        # SH first: its directions use the positions before the xyz update.
        i = len(PARAMETER_NAMES) - 1
        if deferred_sh and world > 1:
            update_sh_from_rows(pool.sh, state.m[i], state.v[i], pool.xyz, grads[i], pool.alive,
                                clusters, rates[i:i + 1], 128, 3)
        elif deferred_sh:
            update_sh_from_colors(pool.sh, state.m[i], state.v[i], pool.xyz, center, grads[i],
                                  pool.alive, clusters, rates[i:i + 1], 128, 3, compact)
        else:
            update_field(pool.sh, state.m[i], state.v[i], grads[i], pool.alive, clusters,
                         rates[i:i + 1], 128, True, compact)
        for i, name in enumerate(PARAMETER_NAMES[:-1]):
            update_field(getattr(pool, name), state.m[i], state.v[i], grads[i], pool.alive,
                         clusters, rates[i:i + 1], 128, False, compact)

    for _ in range(3):
        one()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        one()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    return {"what": "graph replay of the step (and exchange) + sparse Adam on every field",
            "ms_per_step": round(ms, 4), "views_per_s": round(world * 1e3 / ms, 1)}


def _time_step_variant(pool, bounds, camera, target, config, degree, stream, steps: int,
                       sh_color_only: bool) -> dict:
    """The single-view step in the other SH form (graph replays, CUDA
    events), to show what the choice costs."""
    import torch

    from jaxgs_b200.step import GraphedTrainingStep

    graphed = GraphedTrainingStep(pool, bounds, camera, target, config, degree,
                                  sh_color_only=sh_color_only)
    for _ in range(3):
        graphed()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        graphed()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    return {"sh_gradients": "deferred (colour cotangent)" if sh_color_only else
            "all 16 coefficients written by the pullback",
            "ms_per_step": round(ms, 4), "views_per_s": round(1e3 / ms, 2)}


def _time_config4(stream, steps: int = 24, warmup: int = 3) -> dict:
    """BASELINE config 4 on one GPU: the heavy-tailed 6M-Gaussian scene, its
    eight 1600x1067 ring cameras (radius 8, fx = fy = 1350), synthetic uint8
    targets, 8x16 tiles, the pair arena sized from the count pass over the
    eight views.  Each step is one view's whole training step, the graph
    replayed with the next camera and target copied in from the device;
    CUDA events around `steps` replays."""
    import numpy as np
    import torch

    from jaxgs_b200.scene import CapacityConfig, config4_scene, ring_cameras, world_cluster_bounds
    from jaxgs_b200.step import GraphedTrainingStep, required_pairs, size_pair_arena
    from jaxgs_b200.types import DeviceCamera, GaussianArrays

    pool_np = config4_scene()
    n = pool_np["xyz"].shape[0]
    device = torch.device("cuda", torch.cuda.current_device())
    pool = GaussianArrays.from_numpy(pool_np, device=device)
    center, extent, valid = world_cluster_bounds(pool_np, 128)
    del pool_np
    bounds = (torch.as_tensor(center, device=device), torch.as_tensor(extent, device=device),
              torch.as_tensor(valid.astype(np.uint8), device=device))
    cams = [DeviceCamera.from_camera(c, device=device) for c in
            ring_cameras(8, radius=8.0, height=1.5, width=1600, height_px=1067, focal=1350.0)]
    rng = np.random.default_rng(8)
    targets = [torch.as_tensor(rng.integers(0, 256, (1067, 1600, 3), dtype=np.uint8),
                               device=device) for _ in cams]
    default = CapacityConfig(n, 128, 16, 16, 3, 8_000_000, tile_height=8)
    pairs = [required_pairs(pool, bounds, c, default, 3) for c in cams]
    config = size_pair_arena(pool, bounds, cams, default, 3)
    graphed = GraphedTrainingStep(pool, bounds, cams[0], targets[0], config, 3)
    for i in range(warmup):
        graphed(cams[i % 8], targets[i % 8])
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(steps):
        out = graphed(cams[i % 8], targets[i % 8])
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    return {"workload": "BASELINE config 4: 6M-Gaussian heavy-tailed scene, 1600x1067, 8 ring "
                        "cameras cycled, one view per step, 8x16 tiles, SH3",
            "views_per_s": round(1e3 / ms, 1), "ms_per_view": round(ms, 4),
            "pairs_per_view": {"min": min(pairs), "max": max(pairs),
                               "mean": int(sum(pairs) / len(pairs))},
            "arena": config.max_visibility_pairs, "reference_default_arena": 8_000_000,
            "overflow": bool(out.overflow.item())}


# DRAM traffic of one raster_bwd_kernel launch on this workload
# (dram__bytes_read.sum + dram__bytes_write.sum, one-kernel ncu capture of
# `python bench.py --steps 1 --warmup 1 --no-cpu-baseline --no-e2e`, the
# launch after the first): 87.37 MB read + 4.76 MB written.
RASTER_BWD_DRAM_BYTES = 92_134_400
# FP32 work per backward fragment evaluation (one splat at one pixel): the
# alpha, transmittance, colour and moment arithmetic of the reverse pass.
BWD_FLOP_PER_FRAGMENT = 35
SM_COUNT, FP32_LANES_PER_SM = 148, 128


def _backward_visits(pool, bounds, camera, config, degree) -> int:
    """Contributing (splat, warp) visits of the raster backward on the bench
    view, counted from the forward's contribution words exactly as
    raster_bwd_kernel walks them: for each warp (8x8 pixels of a tile), the
    words of the batches up to its last composited pair, the top word masked
    above that pair.  Each visit evaluates the splat at the warp's 64
    pixels.  Runs outside every timed region."""
    from jaxgs_b200 import kernels as K

    clusters, _ = K.compact_visible_clusters(bounds, camera, config, want_slots=False)
    projected, _ = K.project_with_compact_pullback(pool, camera, config, degree, clusters,
                                                   rgb_only=True, visible_color_only=True)
    table = K.build_sorted_visibility_table_cute(projected, camera, config)
    _, cache = K.rasterize_forward(projected, table, camera, config, want_depth=False,
                                   want_alpha=False, clamp_rgb=True)
    return count_visits(cache.last, table.tile_offsets, cache.contribution_bits, camera.width,
                        camera.height, config.tile_size, config.raster_tile_height)


def count_visits(last, tile_offsets, bits, W: int, H: int, tw: int, th: int) -> int:
    """Set contribution bits that raster_bwd_kernel visits, from the
    per-pixel last pair (last), the tile offsets and the contribution words
    (torch tensors on any device)."""
    import torch

    rows = 2 if th % 8 == 0 else 1
    blocks_x, block_h = tw // 8, 4 * rows
    warps = blocks_x * (th // block_h)
    tiles_x = -(-W // tw)
    dev = last.device
    y = torch.arange(H, device=dev)[:, None].expand(H, W).reshape(-1)
    x = torch.arange(W, device=dev)[None, :].expand(H, W).reshape(-1)
    tile = (y // th) * tiles_x + x // tw
    warp = (x % tw) // 8 + ((y % th) // block_h) * blocks_x
    offsets = tile_offsets.long()
    T = offsets.numel() - 1
    start = offsets[:-1].repeat_interleave(warps)
    top = start.clone().scatter_reduce_(0, tile * warps + warp, last.long(), "amax")
    n_batches = torch.where(top > start, ((top - 1 - start) >> 5) + 1, torch.zeros_like(top))
    owner = torch.arange(T * warps, device=dev).repeat_interleave(n_batches)
    first = torch.cumsum(n_batches, 0) - n_batches
    batch = torch.arange(owner.numel(), device=dev) - first[owner]
    t_idx, w_idx = owner // warps, owner % warps
    word_at = ((start[owner] >> 5) + t_idx + batch) * warps + w_idx
    words = bits.long()[word_at] & 0xFFFFFFFF
    is_top = batch == n_batches[owner] - 1
    k_max = (top[owner] - 1 - start[owner]) & 31
    words = torch.where(is_top, words & ((2 << k_max) - 1), words)
    bytes_ = torch.stack([(words >> s) & 255 for s in (0, 8, 16, 24)])
    table8 = torch.tensor([bin(i).count("1") for i in range(256)], device=dev)
    return int(table8[bytes_].sum().item())


def _roofline(stage_ms, peak, peak_kind, pairs, binned, visits, sm_mhz, atomics_per_visit):
    """Roofline of the dominant kernel, the fp32 raster backward.

    The kernel is bound by SIMT issue, so the roofline is fragment
    evaluations per second against the FP32 SIMT ceiling: 148 SMs x 128 FP32
    lanes x the SM clock sampled during the timed region, divided by the
    35 flop a fragment costs (packed f32x2 instructions can take it past
    1.0).  A fragment is one splat at one pixel of a contributing
    (splat, warp) visit (64 pixels).  The bytes are reported beside it:
    per pixel final T, last index and dL/drgb (20 B); per pair of the table
    its id and 48-byte splat record (52 B); per binned Gaussian the ten f32
    cotangents it accumulates (40 B); traffic is the DRAM figure of the
    committed one-kernel capture.
    """
    ms = stage_ms.get("raster_bwd")
    if not ms or not visits:
        return None
    seconds = ms * 1e-3
    fragments = visits * 64
    achieved = fragments / seconds / 1e9
    ceiling = SM_COUNT * FP32_LANES_PER_SM * sm_mhz * 1e6 / BWD_FLOP_PER_FRAGMENT / 1e9
    algo = 1237 * 822 * 20 + pairs * 52 + binned * 40
    gbs = algo / seconds / 1e9
    return {"kernel": "raster_bwd (zero + order + main kernel, one call)", "bound": "simt",
            "achieved": round(achieved, 1), "peak": round(ceiling, 1), "unit": "Gfragment/s",
            "frac": round(achieved / ceiling, 4), "traffic": RASTER_BWD_DRAM_BYTES,
            "fragments": fragments, "visits": visits,
            "atomics_per_s": round(visits * atomics_per_visit / seconds / 1e9, 2),
            "peak_source": f"FP32 SIMT: {SM_COUNT} SMs x {FP32_LANES_PER_SM} lanes x "
                           f"{sm_mhz:.0f} MHz / {BWD_FLOP_PER_FRAGMENT} flop per fragment",
            "bytes": {"algorithmic": int(algo), "achieved_gbs": round(gbs, 1), "peak_gbs": peak,
                      "frac": round(gbs / peak, 4), "peak_source": peak_kind}}


def cpu_baseline(pool_np, camera, target, budget_s: float = 30.0) -> dict:
    """The oracle (CPU restatement) on the host cores: one full config-2 step."""
    from oracle import oracle as O

    config = _config()
    timings = {}
    t0 = time.perf_counter()
    O.training_step(pool_np, camera, target, degree=3, sh_dim=16, tile_w=16, tile_h=8,
                    max_pairs=config.visibility_capacity, timings=timings)
    dt = time.perf_counter() - t0
    return {"value": round(1.0 / dt, 5), "unit": UNIT, "cores": O.num_threads(), "kind": "port",
            "sample": "one full config-2 view (1M Gaussians, 1237x822): oracle/ C restatement, "
                      "OpenMP over the host cores",
            "stage_s": {k: round(v, 3) for k, v in timings.items()}}


def run_reference(args) -> None:
    """CPU restatement of the reference path (JAX is not installed) on rank 0."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle import oracle as O

    # A launcher sets OMP_NUM_THREADS=1 per rank; this rank is the only one
    # working, so it takes every host thread it may run on.
    O.set_num_threads(len(os.sched_getaffinity(0)))

    config = _config()
    pool_np, camera = _workload(0)
    import numpy as np

    rng = np.random.default_rng(3)
    target = rng.integers(0, 256, (camera.height, camera.width, 3), dtype=np.uint8)
    steps = max(1, min(args.steps, 3))
    for _ in range(min(args.warmup, 1)):
        O.training_step(pool_np, camera, target, degree=3, sh_dim=16, tile_w=16, tile_h=8,
                        max_pairs=config.visibility_capacity)
    t0 = time.perf_counter()
    for _ in range(steps):
        O.training_step(pool_np, camera, target, degree=3, sh_dim=16, tile_w=16, tile_h=8,
                        max_pairs=config.visibility_capacity)
    dt = time.perf_counter() - t0
    value = steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": UNIT,
        "n_gpus": world, "steps": steps, "warmup": min(args.warmup, 1),
        "ms_per_step": round(dt / steps * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "BASELINE config 2: 1M-Gaussian training step, 1237x822, 8x16 tiles, SH3",
                   "note": "reference is JAX (not installed); its CPU path is restated in oracle/"},
        "cpu_baseline": {"value": round(value, 5), "unit": UNIT, "cores": O.num_threads(),
                         "kind": "port", "sample": f"{steps} full config-2 views"},
        "e2e": {"value": round(value, 5), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=100)
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--no-cpu-baseline", action="store_true",
                        help="skip the oracle timing (profiling runs)")
    parser.add_argument("--no-e2e", action="store_true",
                        help="skip the host-buffer end-to-end loop (profiling runs)")
    parser.add_argument("--sh", choices=["deferred", "materialized"], default="deferred",
                        help="SH gradients of the step: the reference's deferred form (default) "
                             "or all 16 coefficients from the pullback")
    parser.add_argument("--no-config4", action="store_true",
                        help="skip the config-4 (6M Gaussians, 1600x1067) throughput figure")
    args = parser.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
