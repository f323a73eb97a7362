"""Gaussian models on disk (io_manager/checkpoint.py:13-99).

save_gaussians writes the active Gaussians of a pool as a standard 3D
Gaussian Splatting PLY (binary little endian, float properties x y z, nx ny
nz, f_dc_0..2, f_rest_* channel-major, opacity, scale_0..2, rot_0..3), or the
whole fixed-capacity pool as an NPZ; load_gaussians reads either back.  The
PLY reader parses the header itself (no plyfile dependency) and accepts any
binary little-endian or ASCII vertex element that carries those properties.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from .types import GaussianArrays

PARAMETER_NAMES = ("xyz", "log_scale", "rotation", "opacity", "sh")
_PLY_TYPES = {
    "char": "i1", "int8": "i1", "uchar": "u1", "uint8": "u1", "short": "i2", "int16": "i2",
    "ushort": "u2", "uint16": "u2", "int": "i4", "int32": "i4", "uint": "u4", "uint32": "u4",
    "float": "f4", "float32": "f4", "double": "f8", "float64": "f8",
}


def _host(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def save_gaussians(path, pool: GaussianArrays) -> None:
    """io_manager/checkpoint.py:13-28: PLY of the active Gaussians for a
    .ply path, else an NPZ holding every pool array."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    if path.suffix.lower() == ".ply":
        _save_ply(path, pool)
        return
    with path.open("wb") as stream:
        np.savez_compressed(stream, **{name: _host(getattr(pool, name))
                                       for name in PARAMETER_NAMES + ("alive",)})


def load_gaussians(path, device="cuda") -> GaussianArrays:
    """io_manager/checkpoint.py:31-38: a PLY becomes a compact pool with every
    slot alive; an NPZ restores the saved pool."""
    if Path(path).suffix.lower() == ".ply":
        arrays = _load_ply(path)
    else:
        with np.load(path, allow_pickle=False) as saved:
            arrays = {name: saved[name] for name in PARAMETER_NAMES + ("alive",)}
    tensors = [torch.as_tensor(np.ascontiguousarray(arrays[name], np.float32), device=device)
               for name in PARAMETER_NAMES]
    alive = torch.as_tensor(np.ascontiguousarray(arrays["alive"]).astype(np.uint8), device=device)
    return GaussianArrays(*tensors, alive)


def _save_ply(path: Path, pool: GaussianArrays) -> None:
    """io_manager/checkpoint.py:41-64: one float property per value, SH rest
    coefficients channel-major (all red, then green, then blue)."""
    alive = _host(pool.alive).astype(bool)
    xyz, scale, rotation, opacity, sh = (_host(getattr(pool, n)).astype(np.float32)[alive]
                                         for n in PARAMETER_NAMES)
    count = len(xyz)
    columns = {name: xyz[:, i] for i, name in enumerate(("x", "y", "z"))}
    columns.update({name: np.zeros(count, np.float32) for name in ("nx", "ny", "nz")})
    columns.update({f"f_dc_{i}": sh[:, 0, i] for i in range(3)})
    rest = sh.shape[1] - 1
    columns.update({f"f_rest_{channel * rest + k}": sh[:, k + 1, channel]
                    for channel in range(3) for k in range(rest)})
    columns["opacity"] = opacity[:, 0]
    columns.update({f"scale_{i}": scale[:, i] for i in range(3)})
    columns.update({f"rot_{i}": rotation[:, i] for i in range(4)})
    records = np.empty(count, dtype=[(name, "<f4") for name in columns])
    for name, values in columns.items():
        records[name] = values
    header = ["ply", "format binary_little_endian 1.0", f"element vertex {count}"]
    header += [f"property float {name}" for name in columns]
    header.append("end_header")
    with path.open("wb") as stream:
        stream.write(("\n".join(header) + "\n").encode("ascii"))
        stream.write(records.tobytes())


def _read_vertices(path) -> np.ndarray:
    """The vertex element of a PLY file as a numpy structured array."""
    data = Path(path).read_bytes()
    end = data.find(b"end_header")
    if not data.startswith(b"ply") or end < 0:
        raise ValueError("not a PLY file")
    body = data.index(b"\n", end) + 1
    fmt, elements, current = None, [], None
    for line in data[:end].decode("ascii").splitlines()[1:]:
        words = line.split()
        if not words or words[0] in ("comment", "obj_info"):
            continue
        if words[0] == "format":
            fmt = words[1]
        elif words[0] == "element":
            current = [words[1], int(words[2]), []]
            elements.append(current)
        elif words[0] == "property":
            if words[1] == "list":
                raise ValueError("PLY list properties are not supported")
            current[2].append((words[2], _PLY_TYPES[words[1]]))
    if fmt not in ("binary_little_endian", "ascii"):
        raise ValueError(f"unsupported PLY format {fmt}")
    offset = body
    text = data[body:].decode("ascii").split() if fmt == "ascii" else None
    position = 0
    for name, count, props in elements:
        dtype = np.dtype([(p, "<" + t) for p, t in props])
        if fmt == "binary_little_endian":
            array = np.frombuffer(data, dtype=dtype, count=count, offset=offset)
            offset += count * dtype.itemsize
        else:
            values = np.array(text[position:position + count * len(props)], np.float64)
            position += count * len(props)
            array = np.empty(count, dtype=dtype)
            for i, (p, _) in enumerate(props):
                array[p] = values[i::len(props)]
        if name == "vertex":
            return array
    raise ValueError("PLY file has no vertex element")


def _load_ply(path) -> dict:
    """io_manager/checkpoint.py:67-99."""
    vertices = _read_vertices(path)
    names = vertices.dtype.names
    count = len(vertices)
    rest_count = sum(name.startswith("f_rest_") for name in names)
    if rest_count not in (0, 9, 24, 45):
        raise ValueError("PLY SH dimension must be 1, 4, 9 or 16")

    def fields(keys):
        return np.stack([vertices[k] for k in keys], axis=-1).astype(np.float32)

    sh = np.empty((count, rest_count // 3 + 1, 3), np.float32)
    sh[:, 0] = fields([f"f_dc_{i}" for i in range(3)])
    if rest_count:
        sh[:, 1:] = (fields([f"f_rest_{i}" for i in range(rest_count)])
                     .reshape(count, 3, rest_count // 3).transpose(0, 2, 1))
    return {"xyz": fields(["x", "y", "z"]), "log_scale": fields([f"scale_{i}" for i in range(3)]),
            "rotation": fields([f"rot_{i}" for i in range(4)]), "opacity": fields(["opacity"]),
            "sh": sh, "alive": np.ones(count, bool)}
