"""COLMAP scenes (io_manager/colmap.py, data.py:13-27) for the training
and inference paths: undistorted PINHOLE / SIMPLE_PINHOLE cameras and
registered images from sparse/0 (or sparse) in text or binary form, the
sparse points, and image decoding to the camera's size.  Host code; the
images feed GraphedTrainingStep as uint8 targets."""

from __future__ import annotations

import struct
from dataclasses import dataclass, replace
from pathlib import Path

import numpy as np

from .scene import Camera

try:  # image decoding only; the reconstructions themselves need no PIL
    from PIL import Image
    _LANCZOS = Image.Resampling.LANCZOS
    _BICUBIC = Image.Resampling.BICUBIC
except ImportError:  # pragma: no cover
    Image = None
    _LANCZOS = _BICUBIC = None


@dataclass(frozen=True)
class Frame:
    """data.py:13-27: an image file and the camera that took it."""

    image_path: Path
    camera: Camera
    resample: int | None = _LANCZOS

    def load_rgb(self) -> np.ndarray:
        """uint8 [H, W, 3] at the camera's size (resized with `resample`)."""
        if Image is None:
            raise RuntimeError("decoding images needs PIL")
        with Image.open(self.image_path) as image:
            image = image.convert("RGB")
            if image.size != (self.camera.width, self.camera.height):
                image = image.resize((self.camera.width, self.camera.height), self.resample)
            return np.asarray(image, dtype=np.uint8)

    def load_image(self) -> np.ndarray:
        """float32 [H, W, 3] in [0, 1]."""
        return self.load_rgb().astype(np.float32) / 255.0


def _records(path: Path):
    return [line.strip() for line in path.read_text().splitlines()
            if line.strip() and not line.lstrip().startswith("#")]


def _sparse_dir(scene_dir: Path) -> Path:
    nested = scene_dir / "sparse" / "0"
    return nested if nested.exists() else scene_dir / "sparse"


def _intrinsics(model: str, width: int, height: int, params, downsample: int):
    """Pinhole intrinsics scaled to round(size / downsample)."""
    if model == "PINHOLE":
        fx, fy, cx, cy = params
    elif model == "SIMPLE_PINHOLE":
        f, cx, cy = params
        fx = fy = f
    else:
        raise ValueError(f"use an undistorted PINHOLE model, got {model}")
    w, h = max(1, round(width / downsample)), max(1, round(height / downsample))
    sx, sy = w / width, h / height
    return w, h, fx * sx, fy * sy, cx * sx, cy * sy


def _frame(scene_dir: Path, name: str, qvec, tvec, camera_id: int, intrinsics) -> Frame:
    w, h, fx, fy, cx, cy = intrinsics[camera_id]
    return Frame(scene_dir / "images" / name, Camera.from_colmap(qvec, tvec, fx, fy, cx, cy, w, h))


def _unpack(stream, fmt: str):
    record = struct.Struct("<" + fmt)
    data = stream.read(record.size)
    if len(data) != record.size:
        raise ValueError("truncated COLMAP binary file")
    return record.unpack(data)


def _name(stream) -> str:
    out = bytearray()
    while True:
        c = stream.read(1)
        if not c:
            raise ValueError("truncated COLMAP image name")
        if c == b"\0":
            return out.decode("utf-8")
        out += c


def load_colmap_text(scene_dir, downsample: int = 1) -> list[Frame]:
    """cameras.txt and images.txt (two lines per image), frames sorted by name."""
    if downsample < 1:
        raise ValueError("downsample must be at least 1")
    scene_dir = Path(scene_dir)
    sparse = _sparse_dir(scene_dir)
    intrinsics = {}
    for line in _records(sparse / "cameras.txt"):
        parts = line.split()
        intrinsics[int(parts[0])] = _intrinsics(parts[1], int(parts[2]), int(parts[3]),
                                                [float(x) for x in parts[4:]], downsample)
    lines = [line.strip() for line in (sparse / "images.txt").read_text().splitlines()
             if not line.lstrip().startswith("#")]
    if len(lines) % 2:
        raise ValueError("COLMAP images.txt must contain two lines per image")
    frames = []
    for line in lines[::2]:
        parts = line.split(maxsplit=9)
        frames.append(_frame(scene_dir, parts[9], [float(x) for x in parts[1:5]],
                             [float(x) for x in parts[5:8]], int(parts[8]), intrinsics))
    return sorted(frames, key=lambda f: f.image_path.name)


def load_colmap_binary(scene_dir, downsample: int = 1) -> list[Frame]:
    """cameras.bin and images.bin, frames sorted by name."""
    if downsample < 1:
        raise ValueError("downsample must be at least 1")
    scene_dir = Path(scene_dir)
    sparse = _sparse_dir(scene_dir)
    models = {0: ("SIMPLE_PINHOLE", 3), 1: ("PINHOLE", 4)}
    intrinsics = {}
    with (sparse / "cameras.bin").open("rb") as stream:
        for _ in range(_unpack(stream, "Q")[0]):
            camera_id, model_id, width, height = _unpack(stream, "iiQQ")
            if model_id not in models:
                raise ValueError(f"camera {camera_id}: unsupported COLMAP model ID {model_id}; "
                                 "undistort first")
            model, n = models[model_id]
            intrinsics[camera_id] = _intrinsics(model, width, height, _unpack(stream, "d" * n),
                                                downsample)
    frames = []
    with (sparse / "images.bin").open("rb") as stream:
        for _ in range(_unpack(stream, "Q")[0]):
            record = _unpack(stream, "idddddddi")
            name = _name(stream)
            stream.seek(24 * _unpack(stream, "Q")[0], 1)  # the image's 2D points
            frames.append(_frame(scene_dir, name, record[1:5], record[5:8], record[8],
                                 intrinsics))
    return sorted(frames, key=lambda f: f.image_path.name)


def load_colmap(scene_dir, downsample: int = 1) -> list[Frame]:
    """Binary reconstruction when both .bin files exist, else text."""
    sparse = _sparse_dir(Path(scene_dir))
    if (sparse / "cameras.bin").exists() and (sparse / "images.bin").exists():
        return load_colmap_binary(scene_dir, downsample)
    return load_colmap_text(scene_dir, downsample)


def load_colmap_images(scene_dir, images: str = "images", *, resolution: int = 1) -> list[Frame]:
    """Frames whose cameras take the size of the files under `images`, then
    the native training resolution rule: 1, 2, 4, 8 divide the size; -1
    caps the width at 1600; another positive value is the target width."""
    if resolution != -1 and resolution <= 0:
        raise ValueError("resolution must be -1 or positive")
    if Image is None:
        raise RuntimeError("reading image sizes needs PIL")
    scene_dir = Path(scene_dir)
    out = []
    for frame in load_colmap(scene_dir):
        path = scene_dir / images / frame.image_path.relative_to(scene_dir / "images")
        with Image.open(path) as image:
            width, height = image.size
        if resolution in (1, 2, 4, 8):
            width, height = round(width / resolution), round(height / resolution)
        else:
            scale = (width / 1600 if width > 1600 else 1) if resolution == -1 else width / resolution
            width, height = int(width / scale), int(height / scale)
        width, height = max(1, width), max(1, height)
        c = frame.camera
        sx, sy = width / c.width, height / c.height
        camera = replace(c, width=width, height=height, fx=c.fx * sx, fy=c.fy * sy,
                         cx=c.cx * sx, cy=c.cy * sy)
        out.append(replace(frame, image_path=path, camera=camera, resample=_BICUBIC))
    return out


def load_colmap_points(scene_dir):
    """The sparse points: (xyz [N, 3], rgb [N, 3] in [0, 1]) float32."""
    sparse = _sparse_dir(Path(scene_dir))
    binary = sparse / "points3D.bin"
    if binary.exists():
        with binary.open("rb") as stream:
            count = _unpack(stream, "Q")[0]
            xyz = np.empty((count, 3), np.float32)
            rgb = np.empty((count, 3), np.float32)
            for i in range(count):
                record = _unpack(stream, "QdddBBBd")
                xyz[i] = record[1:4]
                rgb[i] = np.array(record[4:7], np.float64) / 255.0
                stream.seek(8 * _unpack(stream, "Q")[0], 1)  # the point's track
        return xyz, rgb
    records = _records(sparse / "points3D.txt")
    xyz = np.empty((len(records), 3), np.float32)
    rgb = np.empty((len(records), 3), np.float32)
    for i, line in enumerate(records):
        parts = line.split()
        xyz[i] = [float(v) for v in parts[1:4]]
        rgb[i] = np.array([int(v) for v in parts[4:7]], np.float64) / 255.0
    return xyz, rgb
