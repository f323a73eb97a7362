"""COLMAP scenes (jaxgs_b200.colmap) against the cases of the reference's
tests/test_dataset.py:19-61 and :110-185: text and binary reconstructions,
downsampling, SIMPLE_PINHOLE and a flat sparse directory, the refusals,
and the training resolution rule; also image names in subfolders and the
whole camera-model table of the binary format."""

import struct

import numpy as np
import pytest
from PIL import Image

from jaxgs_b200.colmap import (load_colmap, load_colmap_binary, load_colmap_images,
                               load_colmap_points, load_colmap_text)


def test_colmap_text_dataset(tmp_path):
    sparse = tmp_path / "sparse" / "0"
    sparse.mkdir(parents=True)
    (tmp_path / "images").mkdir()
    (sparse / "cameras.txt").write_text("# cameras\n1 PINHOLE 4 4 4 4 2 2\n")
    (sparse / "images.txt").write_text("# images\n1 1 0 0 0 0 0 0 1 frame.png\n\n")
    (sparse / "points3D.txt").write_text("1 0 0 2 255 0 0 0.1\n")
    Image.fromarray(np.full((4, 4, 3), 255, np.uint8)).save(tmp_path / "images" / "frame.png")
    frames = load_colmap_text(tmp_path, downsample=2)
    assert len(frames) == 1
    assert frames[0].camera.width == frames[0].camera.height == 2
    assert frames[0].load_image().shape == (2, 2, 3)
    xyz, rgb = load_colmap_points(tmp_path)
    np.testing.assert_allclose(xyz, [[0, 0, 2]])
    np.testing.assert_allclose(rgb, [[1, 0, 0]])


def test_colmap_binary_dataset(tmp_path):
    sparse = tmp_path / "sparse" / "0"
    sparse.mkdir(parents=True)
    (tmp_path / "images").mkdir()
    (sparse / "cameras.bin").write_bytes(struct.pack("<QiiQQdddd", 1, 1, 1, 4, 4, 4, 4, 2, 2))
    (sparse / "images.bin").write_bytes(struct.pack("<Qidddddddi", 1, 1, 1, 0, 0, 0, 0, 0, 0, 1)
                                        + b"frame.png\0" + struct.pack("<Q", 0))
    (sparse / "points3D.bin").write_bytes(struct.pack("<QQdddBBBdQ", 1, 1, 0, 0, 2, 255, 0, 0,
                                                      0.1, 0))
    Image.fromarray(np.full((4, 4, 3), 255, np.uint8)).save(tmp_path / "images" / "frame.png")
    frames = load_colmap(tmp_path, downsample=2)
    assert len(frames) == 1
    assert frames[0].camera.width == frames[0].camera.height == 2
    np.testing.assert_allclose(frames[0].camera.fx, 2)
    assert frames[0].load_image().shape == (2, 2, 3)
    xyz, rgb = load_colmap_points(tmp_path)
    np.testing.assert_allclose(xyz, [[0, 0, 2]])
    np.testing.assert_allclose(rgb, [[1, 0, 0]])


@pytest.mark.parametrize("loader", [load_colmap_text, load_colmap_binary])
def test_colmap_rejects_invalid_downsample(tmp_path, loader):
    with pytest.raises(ValueError, match="downsample"):
        loader(tmp_path, downsample=0)


def test_simple_pinhole_and_sparse_without_subdirectory(tmp_path):
    sparse = tmp_path / "sparse"
    sparse.mkdir()
    (sparse / "cameras.txt").write_text("1 SIMPLE_PINHOLE 9 5 6 4.5 2.5\n")
    (sparse / "images.txt").write_text("1 1 0 0 0 0 0 0 1 image with spaces.png\n\n")
    (sparse / "points3D.txt").write_text("# empty reconstruction\n")
    (frame,) = load_colmap(tmp_path, downsample=2)
    assert frame.image_path.name == "image with spaces.png"
    assert (frame.camera.width, frame.camera.height) == (4, 2)
    np.testing.assert_allclose([frame.camera.fx, frame.camera.fy], [6 * 4 / 9, 6 * 2 / 5],
                               rtol=1e-6)
    assert all(points.shape == (0, 3) for points in load_colmap_points(tmp_path))
    (sparse / "images.txt").write_text("1 1 0 0 0 0 0 0 1 incomplete.png\n")
    with pytest.raises(ValueError, match="a pose line and a points line"):
        load_colmap(tmp_path)
    (sparse / "images.txt").write_text("1 1 0 0 0 0 0 0 1 image with spaces.png\n\n")
    (sparse / "cameras.txt").write_text("1 OPENCV 9 5 6 6 4.5 2.5 0.1 0 0 0\n")
    with pytest.raises(ValueError, match="undistorted"):
        load_colmap(tmp_path)
    (sparse / "cameras.txt").write_text("2 PINHOLE 9 5 6 6 4.5 2.5\n")
    with pytest.raises(ValueError, match="camera 1 is not in"):
        load_colmap(tmp_path)


@pytest.mark.parametrize("damage", ["header", "model", "name"])
def test_colmap_rejects_truncated_or_unsupported_binary(tmp_path, damage):
    sparse = tmp_path / "sparse"
    sparse.mkdir()
    cameras = struct.pack("<QiiQQddd", 1, 1, 0, 4, 4, 4, 2, 2)
    images = struct.pack("<Qidddddddi", 1, 1, 1, 0, 0, 0, 0, 0, 0, 1)
    expected = "truncated COLMAP image name"
    if damage == "header":
        cameras = b"\x01"
        expected = "truncated COLMAP binary"
    elif damage == "model":
        cameras = struct.pack("<QiiQQ", 1, 1, 99, 4, 4)
        expected = "not a COLMAP camera model"
    (sparse / "cameras.bin").write_bytes(cameras)
    (sparse / "images.bin").write_bytes(images + b"missing terminator")
    with pytest.raises(ValueError, match=expected):
        load_colmap(tmp_path)


@pytest.mark.parametrize("width,height,resolution,expected",
                         [(2000, 1000, -1, (1600, 800)), (31, 17, -1, (31, 17)),
                          (31, 17, 2, (16, 8)), (32, 16, 10, (10, 5))])
def test_training_resolution_matches_native_resize(tmp_path, width, height, resolution,
                                                   expected):
    sparse = tmp_path / "sparse"
    sparse.mkdir()
    (tmp_path / "pyramid").mkdir()
    (sparse / "cameras.txt").write_text(
        f"1 PINHOLE {width * 2} {height * 2} {width} {height} {width} {height}\n")
    (sparse / "images.txt").write_text("1 1 0 0 0 0 0 0 1 frame.png\n\n")
    pixels = np.random.default_rng(0).integers(0, 256, (height, width, 3), dtype=np.uint8)
    path = tmp_path / "pyramid" / "frame.png"
    Image.fromarray(pixels).save(path)
    (frame,) = load_colmap_images(tmp_path, "pyramid", resolution=resolution)
    assert (frame.camera.width, frame.camera.height) == expected
    np.testing.assert_allclose([frame.camera.fx, frame.camera.fy], np.array(expected) / 2,
                               rtol=1e-6)
    with Image.open(path) as original:
        resized = np.asarray(original.resize(expected))  # PIL's default filter: bicubic
    np.testing.assert_array_equal(frame.load_rgb(), resized)
    with pytest.raises(ValueError, match="resolution"):
        load_colmap_images(tmp_path, "pyramid", resolution=0)


def test_binary_cameras_of_every_model_parse_and_only_pinholes_are_used(tmp_path):
    """Every COLMAP model's parameter count is known, so a reconstruction
    that mixes models parses; a frame of a distorted camera is refused."""
    from jaxgs_b200.colmap import CAMERA_MODELS, read_cameras

    sparse = tmp_path / "sparse"
    sparse.mkdir()
    blob = struct.pack("<Q", len(CAMERA_MODELS))
    for model_id, (_, n) in CAMERA_MODELS.items():
        blob += struct.pack("<iiQQ", model_id + 1, model_id, 8, 6) + struct.pack(
            f"<{n}d", *[float(k + 1) for k in range(n)])
    (sparse / "cameras.bin").write_bytes(blob)
    cameras = read_cameras(sparse, binary=True)
    assert [cameras[i + 1].model for i in range(len(CAMERA_MODELS))] == [
        name for name, _ in CAMERA_MODELS.values()]
    assert cameras[2].params == (1.0, 2.0, 3.0, 4.0)
    images = struct.pack("<Qi4d3di", 1, 1, 1, 0, 0, 0, 0, 0, 0, 5) + b"a/b.png\0" + \
        struct.pack("<Q", 2) + struct.pack("<ddq", 1, 2, -1) * 2
    (sparse / "images.bin").write_bytes(images)
    with pytest.raises(ValueError, match="not an undistorted pinhole"):
        load_colmap(tmp_path)
    images = images[:8] + struct.pack("<i4d3di", 1, 1, 0, 0, 0, 0, 0, 0, 2) + images[72:]
    (sparse / "images.bin").write_bytes(images)
    (frame,) = load_colmap(tmp_path)
    assert frame.image_path == tmp_path / "images" / "a" / "b.png"
    assert (frame.camera.width, frame.camera.height) == (8, 6)
