"""Gaussian model files (jaxgs_b200.io) against the behaviour pinned by the
reference's tests/test_checkpoint.py:10-61: the PLY holds only the active
Gaussians, in the standard 3DGS layout (channel-major SH rest
coefficients), and reads back exactly; unsupported SH widths are refused;
an NPZ keeps the whole fixed-capacity pool."""

import numpy as np
import pytest

from jaxgs_b200.io import _read_vertices, load_gaussians, save_gaussians
from jaxgs_b200.types import GaussianArrays

NAMES = ("xyz", "log_scale", "rotation", "opacity", "sh")


def _pool(degree, alive, seed=8):
    rng = np.random.default_rng(seed)
    n = len(alive)
    shapes = {"xyz": (n, 3), "log_scale": (n, 3), "rotation": (n, 4), "opacity": (n, 1),
              "sh": (n, (degree + 1) ** 2, 3)}
    arrays = {}
    for name in NAMES:
        value = rng.normal(size=shapes[name]).astype(np.float32)
        value[~alive] = np.nan  # unused slots must never reach the exported model
        arrays[name] = value
    arrays["alive"] = alive
    return GaussianArrays.from_numpy(arrays, device="cpu"), arrays


@pytest.mark.parametrize("degree", range(4))
@pytest.mark.parametrize("empty", [False, True])
def test_ply_keeps_active_parameters_and_standard_sh_layout(tmp_path, degree, empty):
    alive = np.zeros(7, bool) if empty else np.array([True, False, False, True, False, True, False])
    pool, arrays = _pool(degree, alive)
    output = tmp_path / "nested" / "model.ply"
    save_gaussians(output, pool)
    assert output.read_bytes().startswith(b"ply\nformat binary_little_endian 1.0\n")
    vertices = _read_vertices(output)
    count = int(alive.sum())
    assert len(vertices) == count
    for name in ("nx", "ny", "nz"):
        np.testing.assert_array_equal(vertices[name], 0)
    for i in range(3):
        np.testing.assert_array_equal(vertices[f"f_dc_{i}"], arrays["sh"][alive, 0, i])
        np.testing.assert_array_equal(vertices[f"scale_{i}"], arrays["log_scale"][alive, i])
    np.testing.assert_array_equal(vertices["opacity"], arrays["opacity"][alive, 0])
    rest = 3 * (arrays["sh"].shape[1] - 1)
    expected = arrays["sh"][alive, 1:].transpose(0, 2, 1).reshape(count, rest)
    for i in range(rest):
        np.testing.assert_array_equal(vertices[f"f_rest_{i}"], expected[:, i])
    restored = load_gaussians(output, device="cpu")
    for name in NAMES:
        np.testing.assert_array_equal(getattr(restored, name).numpy(), arrays[name][alive])
    np.testing.assert_array_equal(restored.alive.numpy(), np.ones(count, np.uint8))


def _write_raw_ply(path, fields, count=1):
    header = ["ply", "format binary_little_endian 1.0", f"element vertex {count}"]
    header += [f"property float {f}" for f in fields] + ["end_header"]
    path.write_bytes(("\n".join(header) + "\n").encode() + np.zeros(count * len(fields), "<f4").tobytes())


@pytest.mark.parametrize("rest_count", [3, 48])
def test_ply_rejects_unsupported_sh_dimension(tmp_path, rest_count):
    path = tmp_path / "invalid.ply"
    _write_raw_ply(path, [f"f_rest_{i}" for i in range(rest_count)])
    with pytest.raises(ValueError, match="PLY SH dimension"):
        load_gaussians(path, device="cpu")


def test_ascii_ply_and_npz_pool(tmp_path):
    """An ASCII PLY with an extra colour property reads the same values; an
    NPZ restores every slot, the dead ones included."""
    alive = np.array([True, True, False])
    pool, arrays = _pool(1, alive, seed=3)
    binary = tmp_path / "m.ply"
    save_gaussians(binary, pool)
    vertices = _read_vertices(binary)
    names = list(vertices.dtype.names) + ["red"]
    lines = ["ply", "format ascii 1.0", "comment written by a test",
             f"element vertex {len(vertices)}"]
    lines += [f"property float {n}" for n in names[:-1]] + ["property uchar red", "end_header"]
    for row in vertices:
        lines.append(" ".join(repr(float(v)) for v in row) + " 255")
    text = tmp_path / "m_ascii.ply"
    text.write_text("\n".join(lines) + "\n")
    a, b = load_gaussians(binary, device="cpu"), load_gaussians(text, device="cpu")
    for name in NAMES:
        np.testing.assert_array_equal(getattr(a, name).numpy(), getattr(b, name).numpy())
    npz = tmp_path / "pool.npz"
    save_gaussians(npz, pool)
    restored = load_gaussians(npz, device="cpu")
    for name in NAMES:
        np.testing.assert_array_equal(getattr(restored, name).numpy(), arrays[name])
    np.testing.assert_array_equal(restored.alive.numpy(), alive.astype(np.uint8))
