"""The raster forward's splat-versus-block tests (pack_record, block_hit and
the exact ellipse_hit of jaxgs_b200/csrc/raster.cu), compiled for the host
(tests/host/raster_block_harness.cu): a splat they reject must not
composite at any pixel centre of the block.  The brute force evaluates each
splat's power at every pixel centre in the kernel's operation order (the
conic scaled by -1/2, fused dy terms) and applies the compositing test of
kernels/sorted_rasterize.py:28-90 (power <= 0 and alpha >= 1/256).  Thin,
large, small, nearly transparent and non-positive-definite splats around
the block."""

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
f32 = np.float32


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    if not Path(NVCC).exists():
        pytest.skip("nvcc is not installed")
    out = tmp_path_factory.mktemp("raster_block") / "raster_block_harness"
    cmd = [NVCC, "-gencode=arch=compute_100a,code=sm_100a", "-O1", "-std=c++17",
           "--expt-relaxed-constexpr", "-I", str(ROOT / "include"),
           "-I", str(ROOT / "jaxgs_b200" / "csrc"), "-o", str(out),
           str(ROOT / "tests" / "host" / "raster_block_harness.cu")]
    subprocess.run(cmd, check=True, capture_output=True)
    return out


def _splats(rng, n):
    s1 = np.exp(rng.uniform(np.log(0.3), np.log(80.0), n))
    s2 = s1 * np.exp(rng.uniform(np.log(0.01), 0.0, n))
    th = rng.uniform(0.0, np.pi, n)
    cs, sn = np.cos(th), np.sin(th)
    a11 = cs ** 2 * s1 ** 2 + sn ** 2 * s2 ** 2
    a22 = sn ** 2 * s1 ** 2 + cs ** 2 * s2 ** 2
    a12 = cs * sn * (s1 ** 2 - s2 ** 2)
    det = a11 * a22 - a12 ** 2
    c00, c01, c11 = a22 / det, -a12 / det, a11 / det
    o = rng.uniform(1.0 / 256.0, 1.0, n)
    o[: n // 10] = rng.uniform(1.0 / 256.0, 1.02 / 256.0, n // 10)  # at the alpha cut
    mx = rng.uniform(-90.0, 98.0, n)
    my = rng.uniform(-90.0, 98.0, n)
    out = np.stack([mx, my, c00, c01, c01, c11, o], 1).astype(f32)
    bad = rng.random(n) < 0.02  # not positive definite
    out[bad, 3] = out[bad, 4] = (np.sqrt(out[bad, 2] * out[bad, 5]) * 1.5).astype(f32)
    return out


def _composites(s, rows):
    """Any pixel centre of the 8 x (4 rows) block composites the splat."""
    f = lambda a, b, c: (a.astype(np.float64) * b + c).astype(f32)  # fma of float32 inputs
    mx, my = s[:, 0], s[:, 1]
    c00, c01, c10, c11 = (f32(-0.5) * s[:, k] for k in (2, 3, 4, 5))
    o = s[:, 6]
    hit = np.zeros(len(s), bool)
    for py in range(4 * rows):
        for px in range(8):
            dx = (f32(px + 0.5) + (-mx)).astype(f32)
            dy = (f32(py + 0.5) + (-my)).astype(f32)
            t1 = f(c01, dy, (c00 * dx).astype(f32))
            t2 = f(c11, dy, (c10 * dx).astype(f32))
            power = f(dy, t2, (dx * t1).astype(f32))
            with np.errstate(over="ignore"):
                alpha = (o * np.exp(power.astype(np.float64))).astype(f32)
            hit |= (power <= 0) & (alpha >= f32(1.0 / 256.0))
    return hit


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_block_tests_never_reject_a_compositing_splat(harness, tmp_path, seed):
    rng = np.random.default_rng(seed)
    s = _splats(rng, 100_000)
    (tmp_path / "s.f32").write_bytes(s.tobytes())
    subprocess.run([str(harness), str(tmp_path / "s.f32"), str(tmp_path / "o.u8")], check=True)
    flags = np.fromfile(tmp_path / "o.u8", np.uint8).reshape(-1, 4).astype(bool)
    for rows, (bbox, exact) in ((1, (0, 1)), (2, (2, 3))):
        comp = _composites(s, rows)
        assert comp.sum() > 1000
        assert not np.any(comp & ~flags[:, bbox]), "bounding box rejected a compositing splat"
        assert not np.any(comp & ~flags[:, exact]), "ellipse test rejected a compositing splat"
        # The exact test is tighter than the box on this mix.
        assert flags[:, exact].sum() < 0.9 * flags[:, bbox].sum()
