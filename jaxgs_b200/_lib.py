"""ctypes binding of libgsb200.so (include/gsb200.h).

The product path has no fallback: if the library (built for sm_100a by
jaxgs_b200.build) is missing or fails to load, importing this module raises.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libgsb200.so"

GSB_OK = 0
_ERRORS = {1: "invalid parameters", 2: "workspace too small or misaligned", 3: "CUDA launch error",
           4: "required pointer is NULL"}


class ClusterParams(ctypes.Structure):
    _fields_ = [("num_clusters", ctypes.c_int), ("cluster_size", ctypes.c_int),
                ("capacity", ctypes.c_int)]


class ProjectParams(ctypes.Structure):
    _fields_ = [("capacity", ctypes.c_int), ("sh_dim", ctypes.c_int), ("degree", ctypes.c_int),
                ("width", ctypes.c_int), ("height", ctypes.c_int),
                ("near_plane", ctypes.c_float), ("far_plane", ctypes.c_float),
                ("cluster_size", ctypes.c_int), ("compacted", ctypes.c_int),
                ("clear_invisible", ctypes.c_int), ("visible_color_only", ctypes.c_int)]


class ProjectBwdParams(ctypes.Structure):
    _fields_ = [("capacity", ctypes.c_int), ("sh_dim", ctypes.c_int),
                ("sh_gradient_dim", ctypes.c_int), ("degree", ctypes.c_int),
                ("near_plane", ctypes.c_float), ("cluster_size", ctypes.c_int),
                ("compacted", ctypes.c_int), ("compact_gradients", ctypes.c_int),
                ("rgb_only", ctypes.c_int), ("sh_color_only", ctypes.c_int)]


class ShParams(ctypes.Structure):
    _fields_ = [("capacity", ctypes.c_int), ("sh_dim", ctypes.c_int), ("degree", ctypes.c_int),
                ("views", ctypes.c_int), ("view_stride", ctypes.c_int64),
                ("center_stride", ctypes.c_int64)]


class ExchangeParams(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int)]


class BinParams(ctypes.Structure):
    _fields_ = [("capacity", ctypes.c_int), ("width", ctypes.c_int), ("height", ctypes.c_int),
                ("tile_w", ctypes.c_int), ("tile_h", ctypes.c_int), ("max_pairs", ctypes.c_int64)]


class RasterParams(ctypes.Structure):
    _fields_ = [("capacity", ctypes.c_int), ("width", ctypes.c_int), ("height", ctypes.c_int),
                ("tile_w", ctypes.c_int), ("tile_h", ctypes.c_int), ("max_pairs", ctypes.c_int64),
                ("flags", ctypes.c_int)]


RASTER_SPLATS_READY = 1
RASTER_RGB_ONLY = 2
RASTER_CLAMP_RGB = 4
RASTER_BWD_PREPARED = 1
RASTER_BWD_SYMMETRIC_CONIC = 2


class RasterBwdParams(ctypes.Structure):
    _fields_ = [("capacity", ctypes.c_int), ("width", ctypes.c_int), ("height", ctypes.c_int),
                ("tile_w", ctypes.c_int), ("tile_h", ctypes.c_int), ("cluster_size", ctypes.c_int),
                ("max_pairs", ctypes.c_int64), ("flags", ctypes.c_int)]


class AdamParams(ctypes.Structure):
    _fields_ = [("capacity", ctypes.c_int), ("channels", ctypes.c_int),
                ("cluster_size", ctypes.c_int), ("is_sh", ctypes.c_int),
                ("compact_gradients", ctypes.c_int)]


class AdamShParams(ctypes.Structure):
    _fields_ = [("capacity", ctypes.c_int), ("sh_dim", ctypes.c_int), ("degree", ctypes.c_int),
                ("cluster_size", ctypes.c_int), ("views", ctypes.c_int),
                ("compact_colors", ctypes.c_int), ("view_stride", ctypes.c_int64),
                ("center_stride", ctypes.c_int64)]


class LossParams(ctypes.Structure):
    _fields_ = [("width", ctypes.c_int), ("height", ctypes.c_int), ("target_u8", ctypes.c_int),
                ("clip_input", ctypes.c_int)]


# Symbols declared by include/gsb200.h.
SYMBOLS = (
    "gsb_abi_version", "gsb_last_error", "gsb_launch_count",
    "gsb_cluster_compact_workspace_size", "gsb_cluster_compact",
    "gsb_project_fwd", "gsb_project_bwd", "gsb_sh_from_colors",
    "gsb_bin_workspace_size", "gsb_tile_sort_plan", "gsb_bin",
    "gsb_raster_workspace_size", "gsb_raster_bit_words", "gsb_raster_fwd", "gsb_raster_bwd",
    "gsb_raster_pack", "gsb_raster_bwd_prepare",
    "gsb_loss_workspace_size", "gsb_loss", "gsb_loss_noalloc",
    "gsb_exchange_barrier", "gsb_nvls_allreduce", "gsb_multicast_nonzero", "gsb_p2p_allreduce",
    "gsb_colour_push_compact", "gsb_colour_expand",
    "gsb_sparse_adam", "gsb_sparse_adam_sh", "gsb_densify_scores", "gsb_decay_opacity",
)


def _load():
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build the sm_100a kernels with `python -m jaxgs_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    vp, sz = ctypes.c_void_p, ctypes.c_size_t
    lib.gsb_abi_version.restype = ctypes.c_int
    lib.gsb_abi_version.argtypes = []
    lib.gsb_last_error.restype = ctypes.c_char_p
    lib.gsb_last_error.argtypes = []
    lib.gsb_launch_count.restype = ctypes.c_ulonglong
    lib.gsb_launch_count.argtypes = []
    for name in ("gsb_cluster_compact_workspace_size", "gsb_bin_workspace_size",
                 "gsb_raster_workspace_size", "gsb_raster_bit_words", "gsb_loss_workspace_size"):
        getattr(lib, name).restype = sz
        getattr(lib, name).argtypes = [vp]
    lib.gsb_tile_sort_plan.restype = ctypes.c_int
    lib.gsb_tile_sort_plan.argtypes = [ctypes.c_int64, vp, vp]
    lib.gsb_cluster_compact.restype = ctypes.c_int
    lib.gsb_cluster_compact.argtypes = [vp, vp, vp, sz] + [vp] * 7
    lib.gsb_project_fwd.restype = ctypes.c_int
    lib.gsb_project_fwd.argtypes = [vp, vp] + [vp] * 18
    lib.gsb_project_bwd.restype = ctypes.c_int
    lib.gsb_project_bwd.argtypes = [vp, vp] + [vp] * 22
    lib.gsb_sh_from_colors.restype = ctypes.c_int
    lib.gsb_sh_from_colors.argtypes = [vp, vp] + [vp] * 4
    lib.gsb_bin.restype = ctypes.c_int
    lib.gsb_bin.argtypes = [vp, vp, vp, sz] + [vp] * 10
    lib.gsb_raster_fwd.restype = ctypes.c_int
    lib.gsb_raster_fwd.argtypes = [vp, vp, vp, sz] + [vp] * 18
    lib.gsb_raster_bwd.restype = ctypes.c_int
    lib.gsb_raster_bwd.argtypes = [vp, vp, vp, sz] + [vp] * 20
    lib.gsb_raster_pack.restype = ctypes.c_int
    lib.gsb_raster_pack.argtypes = [vp, vp] + [vp] * 6
    lib.gsb_raster_bwd_prepare.restype = ctypes.c_int
    lib.gsb_raster_bwd_prepare.argtypes = [vp, vp, vp, sz] + [vp] * 9
    lib.gsb_loss.restype = ctypes.c_int
    lib.gsb_loss.argtypes = [vp, vp, vp, sz] + [vp] * 5
    for name, n in (("gsb_exchange_barrier", 4),):
        getattr(lib, name).restype = ctypes.c_int
        getattr(lib, name).argtypes = [vp, vp] + [vp] * n
    lib.gsb_nvls_allreduce.restype = ctypes.c_int
    lib.gsb_nvls_allreduce.argtypes = [vp, vp, vp, ctypes.c_int64, vp]
    lib.gsb_multicast_nonzero.restype = ctypes.c_int
    lib.gsb_multicast_nonzero.argtypes = [vp, vp, vp, ctypes.c_int64, vp]
    lib.gsb_p2p_allreduce.restype = ctypes.c_int
    lib.gsb_p2p_allreduce.argtypes = [vp, vp, vp, ctypes.c_int64, vp]
    lib.gsb_colour_push_compact.restype = ctypes.c_int
    lib.gsb_colour_push_compact.argtypes = [vp, vp, ctypes.c_int64, vp, vp, vp, vp, vp]
    lib.gsb_colour_expand.restype = ctypes.c_int
    lib.gsb_colour_expand.argtypes = [vp, vp, vp, vp, ctypes.c_int, ctypes.c_int64, vp,
                                      ctypes.c_int64, vp]
    lib.gsb_sparse_adam.restype = ctypes.c_int
    lib.gsb_sparse_adam.argtypes = [vp, vp] + [vp] * 8
    lib.gsb_sparse_adam_sh.restype = ctypes.c_int
    lib.gsb_sparse_adam_sh.argtypes = [vp, vp] + [vp] * 10
    lib.gsb_densify_scores.restype = ctypes.c_int
    lib.gsb_densify_scores.argtypes = [vp, ctypes.c_int64] + [vp] * 5
    lib.gsb_decay_opacity.restype = ctypes.c_int
    lib.gsb_decay_opacity.argtypes = [vp, ctypes.c_int64, vp, vp]
    lib.gsb_loss_noalloc.restype = ctypes.c_int
    lib.gsb_loss_noalloc.argtypes = [vp, vp] + [vp] * 5
    return lib


lib = _load()
if lib.gsb_abi_version() != 11:
    raise RuntimeError("libgsb200.so ABI version mismatch; rebuild with `python -m jaxgs_b200.build`")


def check(code: int, what: str) -> None:
    """Raise like the reference's pre-launch checks (ValueError for bad shapes)."""
    if code == GSB_OK:
        return
    detail = _ERRORS.get(code, f"error {code}")
    if code == 3:
        raise RuntimeError(f"{what}: {detail}: {lib.gsb_last_error().decode()}")
    raise ValueError(f"{what}: {detail}")


def ref(struct) -> ctypes.c_void_p:
    return ctypes.cast(ctypes.pointer(struct), ctypes.c_void_p)


def launch_count() -> int:
    """Kernels launched by libgsb200.so so far in this process."""
    return int(lib.gsb_launch_count())


def tile_sort_plan(num_tiles: int) -> tuple[int, int]:
    """(passes, digit bits) of the stable tile sort (kernels/pair_sort.py:33-37)."""
    passes, bits = ctypes.c_int(0), ctypes.c_int(0)
    check(lib.gsb_tile_sort_plan(num_tiles, ctypes.byref(passes), ctypes.byref(bits)), "tile_sort_plan")
    return passes.value, bits.value
