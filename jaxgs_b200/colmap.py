"""COLMAP reconstructions for the training and inference paths.

Reads an undistorted reconstruction -- a `sparse/0` (or flat `sparse`)
directory of cameras, images and points in COLMAP's text or binary format
-- into Frames (an image file and the Camera that took it, data.py:13-27)
and the sparse point cloud that seeds a pool.  Only pinhole cameras are
accepted (the rasterizer has no distortion model).  Host code: the images
feed GraphedTrainingStep as uint8 targets.

The file layouts follow COLMAP's documented formats:
  text   -- '#' comment lines; cameras.txt "ID MODEL WIDTH HEIGHT PARAMS...";
            images.txt two lines per image, the pose line
            "ID QW QX QY QZ TX TY TZ CAMERA_ID NAME" and a (possibly empty)
            line of 2D points; points3D.txt "ID X Y Z R G B ERROR TRACK...".
  binary -- little-endian; each file starts with a u64 record count.
            cameras.bin: i32 id, i32 model id, u64 width, u64 height,
            f64 params[n(model)].  images.bin: i32 id, f64 qvec[4],
            f64 tvec[3], i32 camera id, NUL-terminated name, u64 point
            count, then (f64 x, f64 y, i64 point id) per point.
            points3D.bin: u64 id, f64 xyz[3], u8 rgb[3], f64 error,
            u64 track length, then (i32 image id, i32 point index) each.
"""

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

# COLMAP's camera models: id -> (name, parameter count).
CAMERA_MODELS = {
    0: ("SIMPLE_PINHOLE", 3), 1: ("PINHOLE", 4), 2: ("SIMPLE_RADIAL", 4), 3: ("RADIAL", 5),
    4: ("OPENCV", 8), 5: ("OPENCV_FISHEYE", 8), 6: ("FULL_OPENCV", 12), 7: ("FOV", 5),
    8: ("SIMPLE_RADIAL_FISHEYE", 4), 9: ("RADIAL_FISHEYE", 5), 10: ("THIN_PRISM_FISHEYE", 12),
}


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


@dataclass(frozen=True)
class CameraRecord:
    id: int
    model: str
    width: int
    height: int
    params: tuple


@dataclass(frozen=True)
class ImageRecord:
    id: int
    qvec: tuple  # world-to-camera rotation, (w, x, y, z)
    tvec: tuple
    camera_id: int
    name: str


class _Cursor:
    """Sequential little-endian reads over a whole binary file in memory."""

    def __init__(self, path: Path):
        self.data = path.read_bytes()
        self.at = 0
        self.path = path

    def take(self, fmt: str):
        layout = struct.Struct("<" + fmt)
        if self.at + layout.size > len(self.data):
            raise ValueError(f"truncated COLMAP binary file {self.path.name}")
        values = layout.unpack_from(self.data, self.at)
        self.at += layout.size
        return values

    def skip(self, nbytes: int) -> None:
        if self.at + nbytes > len(self.data):
            raise ValueError(f"truncated COLMAP binary file {self.path.name}")
        self.at += nbytes

    def cstring(self) -> str:
        end = self.data.find(b"\0", self.at)
        if end < 0:
            raise ValueError(f"truncated COLMAP image name in {self.path.name}")
        text = self.data[self.at:end].decode("utf-8")
        self.at = end + 1
        return text


def _content_lines(path: Path, keep_blank: bool = False) -> list[str]:
    """The lines of a COLMAP text file without its '#' comments (blank
    lines kept when asked: images.txt's empty 2D-point lines count)."""
    out = []
    for line in path.read_text().splitlines():
        if line.lstrip().startswith("#"):
            continue
        if line.strip() or keep_blank:
            out.append(line.strip())
    return out


def sparse_dir(scene_dir) -> Path:
    """`sparse/0` when present, else `sparse`."""
    scene_dir = Path(scene_dir)
    nested = scene_dir / "sparse" / "0"
    return nested if nested.exists() else scene_dir / "sparse"


def read_cameras(sparse: Path, binary: bool) -> dict[int, CameraRecord]:
    cameras = {}
    if binary:
        cur = _Cursor(sparse / "cameras.bin")
        (count,) = cur.take("Q")
        for _ in range(count):
            cam_id, model_id, width, height = cur.take("iiQQ")
            if model_id not in CAMERA_MODELS:
                raise ValueError(f"camera {cam_id}: model id {model_id} is not a COLMAP camera "
                                 "model")
            name, n = CAMERA_MODELS[model_id]
            cameras[cam_id] = CameraRecord(cam_id, name, width, height, cur.take("d" * n))
        return cameras
    for line in _content_lines(sparse / "cameras.txt"):
        fields = line.split()
        cam_id = int(fields[0])
        cameras[cam_id] = CameraRecord(cam_id, fields[1], int(fields[2]), int(fields[3]),
                                       tuple(float(v) for v in fields[4:]))
    return cameras


def read_images(sparse: Path, binary: bool) -> list[ImageRecord]:
    images = []
    if binary:
        cur = _Cursor(sparse / "images.bin")
        (count,) = cur.take("Q")
        for _ in range(count):
            image_id, qw, qx, qy, qz, tx, ty, tz, cam_id = cur.take("i4d3di")
            name = cur.cstring()
            (points,) = cur.take("Q")
            cur.skip(points * struct.calcsize("<ddq"))
            images.append(ImageRecord(image_id, (qw, qx, qy, qz), (tx, ty, tz), cam_id, name))
        return images
    lines = _content_lines(sparse / "images.txt", keep_blank=True)
    # A final newline leaves one blank line past the last points line.
    while len(lines) % 2 and lines and not lines[-1]:
        lines.pop()
    if len(lines) % 2:
        raise ValueError("images.txt holds a pose line and a points line per image; "
                         "found an odd number of lines")
    for pose in lines[0::2]:
        fields = pose.split(maxsplit=9)  # the name may contain spaces
        images.append(ImageRecord(int(fields[0]), tuple(float(v) for v in fields[1:5]),
                                  tuple(float(v) for v in fields[5:8]), int(fields[8]),
                                  fields[9]))
    return images


def read_points(sparse: Path) -> tuple[np.ndarray, np.ndarray]:
    """(xyz [N, 3], rgb [N, 3] in [0, 1]) float32 from points3D.bin or .txt."""
    path = sparse / "points3D.bin"
    xyz, rgb = [], []
    if path.exists():
        cur = _Cursor(path)
        (count,) = cur.take("Q")
        for _ in range(count):
            values = cur.take("Q3d3Bd")
            xyz.append(values[1:4])
            rgb.append(values[4:7])
            (track,) = cur.take("Q")
            cur.skip(track * struct.calcsize("<ii"))
    else:
        for line in _content_lines(sparse / "points3D.txt"):
            fields = line.split()
            xyz.append([float(v) for v in fields[1:4]])
            rgb.append([int(v) for v in fields[4:7]])
    xyz_a = np.asarray(xyz, np.float64).reshape(-1, 3).astype(np.float32)
    rgb_a = (np.asarray(rgb, np.float64).reshape(-1, 3) / 255.0).astype(np.float32)
    return xyz_a, rgb_a


def pinhole_intrinsics(camera: CameraRecord) -> tuple[float, float, float, float]:
    """(fx, fy, cx, cy) of a pinhole camera; any other model is refused."""
    if camera.model == "PINHOLE":
        return tuple(camera.params[:4])
    if camera.model == "SIMPLE_PINHOLE":
        f, cx, cy = camera.params[:3]
        return f, f, cx, cy
    raise ValueError(f"camera {camera.id}: {camera.model} is not an undistorted pinhole model; "
                     "undistort the reconstruction first")


def _frames(scene_dir: Path, binary: bool, downsample: int) -> list[Frame]:
    if downsample < 1:
        raise ValueError(f"downsample factor {downsample} is below 1")
    sparse = sparse_dir(scene_dir)
    cameras = read_cameras(sparse, binary)
    scaled = {}
    frames = []
    for image in read_images(sparse, binary):
        if image.camera_id not in scaled:
            # Only the cameras that images use must be pinholes.
            if image.camera_id not in cameras:
                raise ValueError(f"image {image.name}: camera {image.camera_id} is not in the "
                                 "reconstruction's cameras")
            cam = cameras[image.camera_id]
            fx, fy, cx, cy = pinhole_intrinsics(cam)
            # The image shrinks to round(size / downsample); intrinsics follow.
            width = max(1, round(cam.width / downsample))
            height = max(1, round(cam.height / downsample))
            sx, sy = width / cam.width, height / cam.height
            scaled[image.camera_id] = (width, height, fx * sx, fy * sy, cx * sx, cy * sy)
        width, height, fx, fy, cx, cy = scaled[image.camera_id]
        camera = Camera.from_colmap(image.qvec, image.tvec, fx, fy, cx, cy, width, height)
        frames.append(Frame(scene_dir / "images" / image.name, camera))
    frames.sort(key=lambda f: f.image_path.name)
    return frames


def load_colmap_text(scene_dir, downsample: int = 1) -> list[Frame]:
    """Frames of a text reconstruction, sorted by image name."""
    return _frames(Path(scene_dir), False, downsample)


def load_colmap_binary(scene_dir, downsample: int = 1) -> list[Frame]:
    """Frames of a binary reconstruction, sorted by image name."""
    return _frames(Path(scene_dir), True, downsample)


def load_colmap(scene_dir, downsample: int = 1) -> list[Frame]:
    """The binary reconstruction when both cameras.bin and images.bin exist,
    else the text one."""
    sparse = sparse_dir(scene_dir)
    binary = (sparse / "cameras.bin").exists() and (sparse / "images.bin").exists()
    return _frames(Path(scene_dir), binary, downsample)


def training_size(width: int, height: int, resolution: int) -> tuple[int, int]:
    """The reference trainer's image size rule: a resolution of 1, 2, 4 or 8
    divides the size (rounded); -1 keeps the size up to 1600 pixels of width
    and scales wider images down to 1600; any other positive value is the
    target width."""
    if resolution in (1, 2, 4, 8):
        w, h = round(width / resolution), round(height / resolution)
    else:
        if resolution == -1:
            factor = width / 1600 if width > 1600 else 1.0
        else:
            factor = width / resolution
        w, h = int(width / factor), int(height / factor)
    return max(1, w), max(1, h)


def load_colmap_images(scene_dir, images: str = "images", *, resolution: int = 1) -> list[Frame]:
    """Frames whose images come from the `images` folder, with cameras at the
    training size of those files (training_size) and the bicubic resize the
    reference's trainer applies when it loads them."""
    if resolution != -1 and resolution <= 0:
        raise ValueError(f"resolution {resolution}: use -1 or a positive factor or width")
    if Image is None:
        raise RuntimeError("reading image sizes needs PIL")
    scene_dir = Path(scene_dir)
    out = []
    for frame in load_colmap(scene_dir):
        path = scene_dir / images / frame.image_path.relative_to(scene_dir / "images")
        with Image.open(path) as image:
            width, height = training_size(*image.size, resolution)
        c = frame.camera
        sx, sy = width / c.width, height / c.height
        camera = replace(c, width=width, height=height, fx=c.fx * sx, fy=c.fy * sy,
                         cx=c.cx * sx, cy=c.cy * sy)
        out.append(replace(frame, image_path=path, camera=camera, resample=_BICUBIC))
    return out


def load_colmap_points(scene_dir) -> tuple[np.ndarray, np.ndarray]:
    """The sparse points: (xyz [N, 3], rgb [N, 3] in [0, 1]) float32."""
    return read_points(sparse_dir(scene_dir))
