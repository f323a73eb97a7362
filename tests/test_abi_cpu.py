"""libgsb200.so loads without a GPU, exports every symbol include/gsb200.h
declares, and rejects bad parameters before any CUDA call (the reference
raises ValueError before launch: kernels/projector.py:46-47,
packed_rasterizer.py:52-53, fused_loss.py:361-362)."""

import ctypes
import re
from pathlib import Path

import pytest

from jaxgs_b200 import _lib as L

HEADER = Path(__file__).resolve().parents[1] / "include" / "gsb200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"GSB_API\s+[\w\s\*]+?\b(gsb_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    names = declared_symbols()
    assert len(names) >= 14
    for name in names:
        assert hasattr(L.lib, name), name
    assert set(names) == set(L.SYMBOLS)


def test_abi_version_and_launch_counter():
    assert L.lib.gsb_abi_version() == 11
    assert L.launch_count() >= 0


def _code(fn, *args):
    return fn(*args)


def test_invalid_parameters_are_rejected_before_launch():
    vp = None
    bad_bin = L.BinParams(10, 64, 48, 0, 8, 100)  # tile_w 0
    assert L.lib.gsb_bin(vp, L.ref(bad_bin), vp, 0, *([vp] * 10)) == 1
    big = L.BinParams(10, 64, 48, 16, 8, 1 << 31)  # arena >= 2^31
    assert L.lib.gsb_bin(vp, L.ref(big), vp, 0, *([vp] * 10)) == 1
    ok = L.BinParams(10, 64, 48, 16, 8, 100)
    assert L.lib.gsb_bin_workspace_size(L.ref(ok)) > 0
    assert L.lib.gsb_bin(vp, L.ref(ok), vp, 0, *([vp] * 10)) == 2  # no workspace
    proj = L.ProjectParams(10, 16, 4, 64, 48, 0.2, 1000.0, 128, 0, 1, 0)  # degree 4
    assert L.lib.gsb_project_fwd(vp, L.ref(proj), *([vp] * 18)) == 1
    proj = L.ProjectParams(10, 4, 2, 64, 48, 0.2, 1000.0, 128, 0, 1, 0)  # (2+1)^2 > sh_dim
    assert L.lib.gsb_project_fwd(vp, L.ref(proj), *([vp] * 18)) == 1
    proj = L.ProjectParams(10, 16, 3, 64, 48, 0.2, 1000.0, 128, 0, 1, 0)
    assert L.lib.gsb_project_fwd(vp, L.ref(proj), *([vp] * 18)) == 4  # NULL pointers
    bwd = L.ProjectBwdParams(10, 16, 2, 3, 0.2, 128, 1, 1, 1, 1)  # colour-only needs 1
    assert L.lib.gsb_project_bwd(vp, L.ref(bwd), *([vp] * 22)) == 1
    rast = L.RasterParams(10, 64, 48, 12, 8, 100)  # tile width not a multiple of 8
    assert L.lib.gsb_raster_fwd(vp, L.ref(rast), vp, 0, *([vp] * 18)) == 1
    assert L.lib.gsb_raster_bit_words(L.ref(rast)) == 0
    rast = L.RasterParams(10, 64, 48, 16, 8, 100)
    assert L.lib.gsb_raster_bit_words(L.ref(rast)) == (100 // 32 + 4 * 6 + 1) * 2
    rast = L.RasterParams(10, 64, 48, 16, 8, 100, 8)  # unknown flag
    assert L.lib.gsb_raster_fwd(vp, L.ref(rast), vp, 0, *([vp] * 18)) == 1
    assert L.lib.gsb_raster_pack(vp, L.ref(rast), *([vp] * 6)) == 1
    # Forward statistics are gathered only by the recording forward.
    rast = L.RasterParams(10, 64, 48, 16, 8, 100, L.RASTER_RGB_ONLY | L.RASTER_CLAMP_RGB)
    stats = ctypes.c_void_p(16)
    assert L.lib.gsb_raster_fwd(vp, L.ref(rast), vp, 0, *([vp] * 17), stats) == 1
    rast = L.RasterParams(10, 64, 48, 16, 8, 100, L.RASTER_SPLATS_READY)
    assert L.lib.gsb_raster_pack(vp, L.ref(rast), *([vp] * 6)) == 4  # NULL pointers
    rbwd = L.RasterBwdParams(10, 64, 48, 16, 8, 128, 100, 4)  # unknown flag (1, 2 are known)
    assert L.lib.gsb_raster_bwd_prepare(vp, L.ref(rbwd), vp, 0, *([vp] * 9)) == 1
    rbwd = L.RasterBwdParams(10, 64, 48, 16, 8, 128, 100, L.RASTER_BWD_PREPARED)
    assert L.lib.gsb_raster_bwd_prepare(vp, L.ref(rbwd), vp, 0, *([vp] * 9)) == 2  # no workspace
    loss = L.LossParams(0, 5, 1, 0)
    assert L.lib.gsb_loss(vp, L.ref(loss), vp, 0, *([vp] * 5)) == 1
    assert L.lib.gsb_bin(vp, None, vp, 0, *([vp] * 10)) == 4


def test_python_bindings_refuse_cpu_tensors():
    torch = pytest.importorskip("torch")
    from jaxgs_b200 import kernels as K

    with pytest.raises(RuntimeError, match="no CPU fallback"):
        K.fused_loss_and_grad(torch.zeros(4, 4, 3), torch.zeros(4, 4, 3))
    with pytest.raises(ValueError, match="HWC"):
        # shape errors come first, as in kernels/fused_loss.py:361-362
        K.fused_loss_and_grad(torch.zeros(4, 4, 2), torch.zeros(4, 4, 2))


def test_optimizer_density_and_exchange_entry_points_validate_before_launch():
    """The newer entry points refuse bad shapes (1), NULL pointers (4) and
    misaligned buffers (1) on the host, before any launch."""
    import ctypes

    vp = None
    adam = L.AdamParams(10, 0, 128, 0, 0)  # zero channels
    assert L.lib.gsb_sparse_adam(vp, L.ref(adam), *([vp] * 8)) == 1
    adam = L.AdamParams(10, 48, 1 << 21, 1, 0)  # run past the grid's reach
    assert L.lib.gsb_sparse_adam(vp, L.ref(adam), *([vp] * 8)) == 1
    adam = L.AdamParams(10, 3, 128, 0, 0)
    assert L.lib.gsb_sparse_adam(vp, L.ref(adam), *([vp] * 8)) == 4
    assert L.lib.gsb_sparse_adam(vp, L.ref(L.AdamParams(0, 3, 128, 0, 0)), *([vp] * 8)) == 0
    sh = L.AdamShParams(10, 17, 3, 128, 1, 1, 0, 0)  # more than 16 coefficients
    assert L.lib.gsb_sparse_adam_sh(vp, L.ref(sh), *([vp] * 10)) == 1
    sh = L.AdamShParams(10, 4, 2, 128, 1, 1, 0, 0)  # (2+1)^2 > sh_dim
    assert L.lib.gsb_sparse_adam_sh(vp, L.ref(sh), *([vp] * 10)) == 1
    sh = L.AdamShParams(10, 16, 3, 128, 1, 1, 0, 2)  # centre stride below 3
    assert L.lib.gsb_sparse_adam_sh(vp, L.ref(sh), *([vp] * 10)) == 1
    sh = L.AdamShParams(10, 16, 3, 128, 1, 1, 0, 0)
    assert L.lib.gsb_sparse_adam_sh(vp, L.ref(sh), *([vp] * 10)) == 4
    sh = L.AdamShParams(0, 16, 3, 128, 1, 1, 0, 0)
    assert L.lib.gsb_sparse_adam_sh(vp, L.ref(sh), *([vp] * 10)) == 0
    assert L.lib.gsb_densify_scores(vp, -1, *([vp] * 5)) == 1
    assert L.lib.gsb_densify_scores(vp, 10, *([vp] * 5)) == 4
    assert L.lib.gsb_densify_scores(vp, 0, *([vp] * 5)) == 0
    assert L.lib.gsb_decay_opacity(vp, 10, vp, vp) == 4
    assert L.lib.gsb_multicast_nonzero(vp, vp, vp, 6, vp) == 1  # not a multiple of 4
    assert L.lib.gsb_multicast_nonzero(vp, ctypes.c_void_p(8), ctypes.c_void_p(16), 8, vp) == 1
    assert L.lib.gsb_multicast_nonzero(vp, vp, vp, 0, vp) == 0
    nine = L.ExchangeParams(9, 0)  # more ranks than the P2P form takes
    buffers = (ctypes.c_void_p * 9)(*([16] * 9))
    assert L.lib.gsb_p2p_allreduce(vp, L.ref(nine), buffers, 8, vp) == 1
    two = L.ExchangeParams(2, 0)
    assert L.lib.gsb_p2p_allreduce(vp, L.ref(two), (ctypes.c_void_p * 2)(16, 24), 8, vp) == 1
    assert L.lib.gsb_p2p_allreduce(vp, L.ref(two), (ctypes.c_void_p * 2)(16, None), 8, vp) == 4
    assert L.lib.gsb_p2p_allreduce(vp, L.ref(L.ExchangeParams(2, 2)), buffers, 8, vp) == 1
    a16, a8 = ctypes.c_void_p(16), ctypes.c_void_p(8)
    assert L.lib.gsb_colour_push_compact(vp, vp, -1, vp, vp, vp, vp, vp) == 1
    assert L.lib.gsb_colour_push_compact(vp, vp, 10, vp, vp, vp, vp, vp) == 4
    assert L.lib.gsb_colour_push_compact(vp, a8, 10, a16, a16, a16, a16, vp) == 1  # misaligned row
    assert L.lib.gsb_colour_push_compact(vp, a16, 10, a16, a8, a16, a16, vp) == 1  # misaligned table
    assert L.lib.gsb_colour_expand(vp, a16, a16, a16, 2, 10, a16, 33, vp) == 1  # dense row < 4 + 3C
    assert L.lib.gsb_colour_expand(vp, vp, vp, vp, 2, 10, vp, 34, vp) == 4


def test_sparse_adam_python_checks_refuse_mismatched_rows():
    """update_field refuses SH gradients narrower than the field (an
    active-bands gradient), on the host."""
    import torch

    from jaxgs_b200.optimizer import update_field

    sh = torch.zeros(4, 16, 3)
    narrow = torch.zeros(4, 4, 3)
    with pytest.raises(ValueError, match="every SH coefficient"):
        update_field(sh, sh.clone(), sh.clone(), narrow, torch.ones(4, dtype=torch.uint8),
                     (torch.zeros(1, dtype=torch.int32), torch.ones(1, dtype=torch.int32)),
                     0.1, 1, True, False)
