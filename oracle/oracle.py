"""ctypes/numpy front end of the CPU oracle (oracle/gs_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py to check and time the CUDA path.  The product
package never imports it.

Each function restates a reference entry point (cited per function) on numpy
arrays laid out exactly like the reference's flat buffers.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_vp = ctypes.c_void_p
_int = ctypes.c_int
_flt = ctypes.c_float


def build() -> Path:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    env = dict(os.environ)
    if Path("/usr/bin/gcc").exists():
        env["CC"] = "/usr/bin/gcc"
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True, env=env)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(_LIB_PATH))
        _lib.gs_logf.argtypes = [_flt]
        _lib.gs_logf.restype = _flt
        _lib.orc_project_fwd.restype = None
        _lib.orc_project_bwd.restype = None
        _lib.orc_count.restype = None
        _lib.orc_gaussian_tiles.restype = ctypes.c_int32
        _lib.orc_gaussian_tiles.argtypes = [_flt] * 6 + [_int] * 4 + [_i64p]
        _lib.orc_bin.restype = ctypes.c_int64
        _lib.orc_raster_fwd.restype = None
        _lib.orc_raster_bwd.restype = None
        _lib.orc_loss.restype = ctypes.c_double
        _lib.orc_cluster_compact.restype = _int
        _lib.orc_num_threads.restype = _int
        _lib.orc_set_num_threads.argtypes = [_int]
        _lib.orc_set_num_threads.restype = None
    return _lib


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_vp)


def gs_logf(x: float) -> float:
    return float(lib().gs_logf(ctypes.c_float(x)))


def num_threads() -> int:
    return int(lib().orc_num_threads())


def set_num_threads(n: int) -> None:
    """Threads of the oracle's parallel loops from here on."""
    lib().orc_set_num_threads(_int(int(n)))


def project_fwd(pool, camera, *, degree, sh_dim, clusters=None, cluster_size=128,
                visible_color_only=False):
    """kernels/projection.py:6-175 (+ compact mapping :42-47).

    pool: dict of numpy arrays xyz[C,3], log_scale[C,3], rotation[C,4],
    opacity[C,1], sh[C,sh_dim,3], alive[C] (bool).  camera: scene.Camera.
    clusters: (ids int32[N], count) or None.  Returns a dict of the seven
    projected fields (flat layouts as the reference's outputs).
    """
    capacity = pool["xyz"].shape[0]
    out = {
        "mean": np.zeros(capacity * 2, np.float32),
        "depth": np.full(capacity, np.inf, np.float32),
        "conic": np.zeros(capacity * 4, np.float32),
        "radius": np.zeros(capacity, np.float32),
        "color": np.zeros(capacity * 3, np.float32),
        "alpha": np.zeros(capacity, np.float32),
        "visible": np.zeros(capacity, np.int8),
    }
    ids, count = (None, 0) if clusters is None else (np.ascontiguousarray(clusters[0], np.int32), int(clusters[1]))
    args = [_f(pool["xyz"]), _f(pool["log_scale"]), _f(pool["rotation"]), _f(pool["opacity"]),
            _f(pool["sh"]), np.ascontiguousarray(pool["alive"], np.uint8),
            _f(camera.world_to_camera), _f(camera.intrinsics), _f(camera.center)]
    lib().orc_project_fwd(
        *[_ptr(a) for a in args], _ptr(ids), _int(count), _int(capacity), _int(sh_dim),
        _int(degree), _int(camera.width), _int(camera.height), _flt(camera.near),
        _flt(camera.far), _int(cluster_size), _int(int(visible_color_only)),
        *[_ptr(out[k]) for k in ("mean", "depth", "conic", "radius", "color", "alpha", "visible")])
    return out


def project_bwd(pool, camera, color, cot, *, degree, sh_dim, sh_gradient_dim=None,
                clusters=None, cluster_size=128, compact_gradients=False, rgb_only=False,
                sh_color_only=False):
    """kernels/projection_backward.py:7-367.  cot: dict of flat cotangents
    mean, depth, conic, radius, color, alpha.  Returns (xyz, log_scale,
    rotation, opacity, sh) flat gradient arrays of capacity rows."""
    capacity = pool["xyz"].shape[0]
    if sh_gradient_dim is None:
        sh_gradient_dim = 1 if sh_color_only else sh_dim
    outs = [np.zeros(capacity * 3, np.float32), np.zeros(capacity * 3, np.float32),
            np.zeros(capacity * 4, np.float32), np.zeros(capacity, np.float32),
            np.zeros(capacity * sh_gradient_dim * 3, np.float32)]
    ids, count = (None, 0) if clusters is None else (np.ascontiguousarray(clusters[0], np.int32), int(clusters[1]))
    args = [_f(pool["xyz"]), _f(pool["log_scale"]), _f(pool["rotation"]), _f(pool["opacity"]),
            _f(pool["sh"]), _f(camera.world_to_camera), _f(camera.intrinsics),
            _f(camera.center), _f(color)]
    cots = [_f(cot["mean"]), _f(cot["depth"]), _f(cot["conic"]), _f(cot["radius"]),
            _f(cot["color"]), _f(cot["alpha"])]
    lib().orc_project_bwd(
        *[_ptr(a) for a in args], _ptr(ids), _int(count), _int(capacity), _int(sh_dim),
        _int(sh_gradient_dim), _int(degree), _flt(camera.near), _int(cluster_size),
        _int(int(compact_gradients)), _int(int(rgb_only)), _int(int(sh_color_only)),
        *[_ptr(a) for a in cots], *[_ptr(a) for a in outs])
    return tuple(outs)


def count_pairs(proj, width, height, tile_w, tile_h):
    """_count, kernels/sorted_visibility.py:307-370: (counts, depth keys)."""
    capacity = proj["alpha"].shape[0]
    tiles_x = -(-width // tile_w)
    tiles_y = -(-height // tile_h)
    counts = np.zeros(capacity, np.int32)
    keys = np.zeros(capacity, np.uint32)
    lib().orc_count(_ptr(_f(proj["mean"])), _ptr(_f(proj["conic"])), _ptr(_f(proj["alpha"])),
                    _ptr(_f(proj["depth"])), _ptr(np.ascontiguousarray(proj["visible"], np.int8)),
                    _int(capacity), _int(tile_w), _int(tile_h), _int(tiles_x), _int(tiles_y),
                    _int(width), _int(height), _ptr(counts), _ptr(keys))
    return counts, keys


def gaussian_tiles(mx, my, c00, c01, c11, alpha, tile_w, tile_h, tiles_x, tiles_y):
    """Tile keys of one Gaussian in the reference's emission order."""
    buf = np.zeros(max(1, tiles_x * tiles_y), np.int64)
    n = lib().orc_gaussian_tiles(mx, my, c00, c01, c11, alpha, tile_w, tile_h, tiles_x, tiles_y, buf)
    return buf[:max(0, n)].copy(), n


def bin(proj, width, height, tile_w, tile_h, max_pairs):
    """build_sorted_visibility_table_cute, kernels/sorted_binning.py:9-117.

    Returns dict(gaussian_ids[max_pairs] (-1 past the pairs), tile_offsets
    [T+1], point_counts[C], pair_count (unclamped), overflow (bool)).
    """
    capacity = proj["alpha"].shape[0]
    tiles = (-(-width // tile_w)) * (-(-height // tile_h))
    counts = np.zeros(capacity, np.int32)
    ids = np.zeros(max_pairs, np.int32)
    offsets = np.zeros(tiles + 1, np.int32)
    overflow = np.zeros(1, np.int32)
    total = lib().orc_bin(
        _ptr(_f(proj["mean"])), _ptr(_f(proj["conic"])), _ptr(_f(proj["alpha"])),
        _ptr(_f(proj["depth"])), _ptr(np.ascontiguousarray(proj["visible"], np.int8)),
        _int(capacity), _int(width), _int(height), _int(tile_w), _int(tile_h),
        ctypes.c_int64(max_pairs), _ptr(counts), _ptr(ids), _ptr(offsets), _ptr(overflow))
    return {"gaussian_ids": ids, "tile_offsets": offsets, "point_counts": counts,
            "pair_count": int(total), "overflow": bool(overflow[0])}


def raster_fwd(proj, table, width, height, tile_w, tile_h, background=(0.0, 0.0, 0.0)):
    """fp32 compositing, kernels/sorted_rasterize.py:28-88 (rectangular tiles).

    proj needs mean, conic, depth, color, alpha.  Returns dict rgb[H*W*3],
    depth, alpha, final_t, last, ambiguous (uint8 per pixel).
    """
    n = width * height
    out = {"rgb": np.zeros(n * 3, np.float32), "depth": np.zeros(n, np.float32),
           "alpha": np.zeros(n, np.float32), "final_t": np.zeros(n, np.float32),
           "last": np.zeros(n, np.int32), "ambiguous": np.zeros(n, np.uint8)}
    lib().orc_raster_fwd(
        _int(width), _int(height), _int(tile_w), _int(tile_h), _ptr(_f(proj["mean"])),
        _ptr(_f(proj["conic"])), _ptr(_f(proj["depth"])), _ptr(_f(proj["color"])),
        _ptr(_f(proj["alpha"])), _ptr(np.ascontiguousarray(table["gaussian_ids"], np.int32)),
        _ptr(np.ascontiguousarray(table["tile_offsets"], np.int32)),
        _ptr(_f(np.asarray(background))), *[_ptr(out[k]) for k in
                                            ("rgb", "depth", "alpha", "final_t", "last", "ambiguous")])
    return out


def raster_bwd(proj, table, fwd, drgb, width, height, tile_w, tile_h, background=(0.0, 0.0, 0.0),
               ddepth=None, dalpha=None):
    """fp32 compositing pullback, kernels/sorted_rasterize.py:91-236.

    Returns dict of flat cotangents mean[C*2], conic[C*4], depth, color, alpha,
    and "stats" [C, 4]: the fragment statistics (count, compositing weight,
    alpha cotangent, squared opacity cotangent) that
    kernels/sorted_rasterizer.py:227-235 stacks from the collect_stats outputs.
    """
    capacity = proj["alpha"].shape[0]
    out = {"mean": np.zeros(capacity * 2, np.float32), "conic": np.zeros(capacity * 4, np.float32),
           "depth": np.zeros(capacity, np.float32), "color": np.zeros(capacity * 3, np.float32),
           "alpha": np.zeros(capacity, np.float32)}
    fragments = np.zeros(capacity * 3, np.float32)
    lib().orc_raster_bwd(
        _int(width), _int(height), _int(tile_w), _int(tile_h), _int(capacity),
        _ptr(_f(proj["mean"])), _ptr(_f(proj["conic"])), _ptr(_f(proj["depth"])),
        _ptr(_f(proj["color"])), _ptr(_f(proj["alpha"])),
        _ptr(np.ascontiguousarray(table["gaussian_ids"], np.int32)),
        _ptr(np.ascontiguousarray(table["tile_offsets"], np.int32)),
        _ptr(_f(np.asarray(background))), _ptr(_f(fwd["final_t"])),
        _ptr(np.ascontiguousarray(fwd["last"], np.int32)), _ptr(_f(drgb)),
        _ptr(None if ddepth is None else _f(ddepth)), _ptr(None if dalpha is None else _f(dalpha)),
        *[_ptr(out[k]) for k in ("mean", "conic", "depth", "color", "alpha")], _ptr(fragments))
    out["stats"] = np.stack((fragments[0::3], fragments[1::3], out["alpha"], fragments[2::3]),
                            axis=1)
    return out


def loss(image, target, want_grad=True):
    """L1(0.8)+SSIM(0.2): reference/loss.py:6-43 with kernels/fused_loss.py's
    per-pixel gradient (:229-288).  image [H,W,3] float; target float [0,1]
    or uint8.  Returns (loss, grad [H,W,3] or None)."""
    image = _f(image)
    H, W, _ = image.shape
    grad = np.zeros_like(image) if want_grad else None
    if np.asarray(target).dtype == np.uint8:
        value = lib().orc_loss(_int(H), _int(W), _ptr(image), None,
                               _ptr(np.ascontiguousarray(target, np.uint8)), _ptr(grad))
    else:
        value = lib().orc_loss(_int(H), _int(W), _ptr(image), _ptr(_f(target)), None, _ptr(grad))
    return float(value), grad


def cluster_compact(center, extent, valid, planes):
    """frustum_cluster_mask + compact_visible_clusters (scene/cluster.py:40-67,
    kernels/cluster_compact.py:31-44).  Returns (ids, count, cluster_visible)."""
    n = int(np.asarray(valid).shape[0])
    ids = np.zeros(max(n, 1), np.int32)
    vis = np.zeros(max(n, 1), np.uint8)
    count = lib().orc_cluster_compact(_int(n), _ptr(_f(center)), _ptr(_f(extent)),
                                      _ptr(np.ascontiguousarray(valid, np.uint8)),
                                      _ptr(_f(planes)), _ptr(ids), _ptr(vis))
    return ids[:n], int(count), vis[:n].astype(bool)


def clip_grad(image):
    """d clip(x, 0, 1)/dx with jnp.maximum/minimum tie semantics (1/2 at a bound)."""
    image = np.asarray(image, np.float32)
    g = ((image > 0) & (image < 1)).astype(np.float32)
    g[(image == 0) | (image == 1)] = 0.5
    return g


PACKED_TILES = ((8, 8), (8, 16), (12, 16), (16, 16))  # (tile_h, tile_w)


def training_step(pool, camera, target, *, degree, sh_dim, tile_w, tile_h, max_pairs,
                  cluster_size=128, bounds=None, timings=None, clusters=None, packed=None):
    """Whole hot path of training/step.py:32-89: cluster cull -> compact
    projection -> binning -> raster -> loss -> raster pullback -> projection
    pullback (compact, rgb_only, active SH only).  The loss follows the
    step's dispatch (training/step.py:74-80): for the packed tile shapes
    packed_loss_and_grad's (kernels/packed_rasterizer.py:180-216: image
    min(rgb, 1) over no background, its image gradient passed on as is,
    packed_rasterize.py:396,440-463), else rasterize_loss_and_grad's
    (kernels/sorted_rasterizer.py:165-236: loss on clip(rgb, 0, 1) with the
    clip's VJP); compositing is fp32 either way.  packed overrides the choice.

    Returns dict(loss, grads (xyz, log_scale, rotation, opacity, sh) in
    compact order, clusters (ids, count), table, fwd, proj, stats (the [C, 4]
    fragment statistics of this view)).  timings, if a
    dict, receives per-stage seconds; clusters overrides the culled list."""
    import time

    from jaxgs_b200.scene import world_cluster_bounds

    W, H = camera.width, camera.height
    clock = time.perf_counter
    t0 = clock()
    if bounds is None:
        bounds = world_cluster_bounds(pool, cluster_size)
    if clusters is None:
        ids, count, _ = cluster_compact(*bounds, camera.frustum_planes())
    else:
        ids, count = np.asarray(clusters[0], np.int32), int(clusters[1])
    t1 = clock()
    proj = project_fwd(pool, camera, degree=degree, sh_dim=sh_dim, clusters=(ids, count),
                       cluster_size=cluster_size, visible_color_only=True)
    t2 = clock()
    table = bin(proj, W, H, tile_w, tile_h, max_pairs)
    t3 = clock()
    fwd = raster_fwd(proj, table, W, H, tile_w, tile_h)
    t4 = clock()
    image = fwd["rgb"].reshape(H, W, 3)
    if packed is None:
        packed = (tile_h, tile_w) in PACKED_TILES
    if packed:
        value, grad = loss(np.minimum(image, np.float32(1.0)), target)
    else:
        value, grad = loss(np.clip(image, 0.0, 1.0), target)
        grad = grad * clip_grad(image)
    t5 = clock()
    cot = raster_bwd(proj, table, fwd, grad.reshape(-1), W, H, tile_w, tile_h)
    t6 = clock()
    capacity = pool["xyz"].shape[0]
    cot_full = dict(cot)
    cot_full["depth"] = np.zeros(capacity, np.float32)
    cot_full["radius"] = np.zeros(capacity, np.float32)
    grads = project_bwd(pool, camera, proj["color"], cot_full, degree=degree, sh_dim=sh_dim,
                        sh_gradient_dim=(degree + 1) ** 2, clusters=(ids, count),
                        cluster_size=cluster_size, compact_gradients=True, rgb_only=True)
    t7 = clock()
    if timings is not None:
        timings.update(cull=t1 - t0, project=t2 - t1, bin=t3 - t2, raster_fwd=t4 - t3,
                       loss=t5 - t4, raster_bwd=t6 - t5, project_bwd=t7 - t6, total=t7 - t0)
    return {"loss": value, "grads": grads, "clusters": (ids, count), "table": table, "fwd": fwd,
            "proj": proj, "stats": cot["stats"]}


def sparse_adam(value, mean, variance, gradient, alive, ids, count, rate, *, cluster_size,
                is_sh, compact_gradients):
    """Visible-cluster LiteGS Adam on one field, kernels/sparse_adam.py:16-54
    (as called by training/optimizer.py:310-325): for every channel of every
    alive slot of the first `count` listed clusters,
        m = 0.9 m + 0.1 g;  v = 0.999 v + 0.001 g g;  x -= lr m / (sqrt(v) + 1e-15)
    with lr = rate (times 10 for the first three channels of an SH row), each
    operation rounded to float32 in that order.  gradient is in pool order,
    or (compact_gradients) the visible-cluster prefix.  Returns new
    (value, mean, variance) flat float32 arrays; other elements unchanged."""
    f = np.float32
    x = np.array(value, np.float32).reshape(-1)
    m = np.array(mean, np.float32).reshape(-1)
    v = np.array(variance, np.float32).reshape(-1)
    g_all = np.asarray(gradient, np.float32).reshape(-1)
    alive = np.asarray(alive).reshape(-1).astype(bool)
    capacity = alive.size
    ch = x.size // capacity
    lr0 = f(rate)
    channel_rate = np.full(ch, lr0, np.float32)
    if is_sh:
        channel_rate[:3] = lr0 * f(10.0)
    for c in range(int(count)):
        slots = int(ids[c]) * cluster_size + np.arange(cluster_size)
        in_pool = slots < capacity
        keep = np.zeros(cluster_size, bool)
        keep[in_pool] = alive[slots[in_pool]]
        elems = (slots[:, None] * ch + np.arange(ch)).reshape(-1)
        gidx = (c * cluster_size * ch + np.arange(cluster_size * ch)) if compact_gradients else elems
        mask = np.repeat(keep, ch)
        e, gi = elems[mask], gidx[mask]
        g = g_all[gi]
        lr = np.tile(channel_rate, cluster_size)[mask]
        mm = f(0.9) * m[e] + f(0.1) * g
        vv = f(0.999) * v[e] + (f(0.001) * g) * g
        x[e] = x[e] - (lr * mm) / (np.sqrt(vv) + f(1e-15))
        m[e], v[e] = mm, vv
    return x, m, v


def parameter_learning_rates(step, spatial_scale, max_steps, position_lr_init,
                             position_lr_final, feature_lr, opacity_lr, scaling_lr, rotation_lr):
    """training/optimizer.py:93-120: (xyz, log_scale, rotation, opacity, sh)
    rates of sparse_adam_update, the SH one being feature_lr / 10 (the DC
    coefficient's x10 is applied per channel).  float64 host arithmetic."""
    import math

    frac = min(max(step / max_steps, 0.0), 1.0)
    if position_lr_init == position_lr_final == 0:
        position = 0.0
    else:
        position = spatial_scale * math.exp(math.log(position_lr_init) * (1 - frac)
                                            + math.log(position_lr_final) * frac)
    return position, scaling_lr, rotation_lr, opacity_lr, feature_lr / 10


def densification_scores(opacity, alive, stats):
    """training/densify.py:20-35 in float64: opacity-weighted variance of the
    per-fragment opacity gradient, zero for dead slots and non-finite values,
    and the prune mask alive & (compositing weight == 0)."""
    n, w, s, q = np.asarray(stats, np.float64).T
    alive = np.asarray(alive).astype(bool)
    variance = np.maximum(q / (n + 1) - (s / (n + 1)) ** 2, 0)
    a = 1.0 / (1.0 + np.exp(-np.asarray(opacity, np.float64).reshape(-1)))
    with np.errstate(all="ignore"):
        scores = np.nan_to_num(variance * n * a ** 2, nan=0, posinf=0, neginf=0)
    return np.where(alive, scores, 0), alive & (w == 0)


def decay_opacity(opacity, alive):
    """training/densify.py:158-165 (float64): alive logits -> logit(max(sigmoid/2, 1/128))."""
    o = np.asarray(opacity, np.float64).reshape(-1)
    a = np.maximum(0.5 / (1.0 + np.exp(-o)), 1 / 128)
    return np.where(np.asarray(alive).astype(bool), np.log(a / (1 - a)), o)
