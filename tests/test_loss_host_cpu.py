"""The fused loss kernel's stage and pass bodies, compiled for the host
(tests/host/loss_harness.cu, -fsanitize=bounds) and run thread by thread
over the whole launch grid, against the oracle's L1+SSIM loss and gradient
(reference/loss.py:6-43, kernels/fused_loss.py:229-288).  Checks the
row-streaming ring-buffer indexing (every shared-memory index in range, no
unstaged row read: the shared state starts as NaN) without a GPU; the GPU
parity tests check the same kernel on the device."""

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

ROOT = Path(__file__).resolve().parents[1]
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    if not Path(NVCC).exists():
        pytest.skip("nvcc is not installed")
    out = tmp_path_factory.mktemp("loss_harness") / "loss_harness"
    cmd = [NVCC, "-gencode=arch=compute_100a,code=sm_100a", "-O1", "-std=c++17",
           "--expt-relaxed-constexpr", "-I", str(ROOT / "include"),
           "-I", str(ROOT / "jaxgs_b200" / "csrc"), "-Xcompiler", "-fsanitize=bounds",
           "-Xcompiler", "-fsanitize=undefined", "-Xcompiler", "-fno-sanitize-recover=all",
           "-o", str(out), str(ROOT / "tests" / "host" / "loss_harness.cu"), "-Xlinker", "-lubsan"]
    subprocess.run(cmd, check=True, capture_output=True)
    return out


def _run(harness, tmp_path, image, target, clip):
    h, w, _ = image.shape
    paths = {k: tmp_path / k for k in ("image", "target", "grad", "out")}
    image.astype(np.float32).tofile(paths["image"])
    target.tofile(paths["target"])
    subprocess.run([str(harness), str(w), str(h), str(int(target.dtype == np.uint8)),
                    str(int(clip)), *(str(paths[k]) for k in ("image", "target", "grad", "out"))],
                   check=True, capture_output=True)
    out = np.fromfile(paths["out"], np.float32)
    return float(out[0]), np.fromfile(paths["grad"], np.float32).reshape(h, w, 3), \
        float(out[1]), int(out[2])


@pytest.mark.parametrize("shape", [(1, 1, 3), (17, 31, 3), (96, 128, 3), (480, 640, 3)])
@pytest.mark.parametrize("u8", [False, True])
@pytest.mark.parametrize("clip", [False, True])
def test_host_run_of_the_loss_kernel_matches_oracle(harness, tmp_path, shape, u8, clip):
    rng = np.random.default_rng(hash((shape, u8, clip)) % 2**32)
    image = (rng.uniform(-0.1, 1.1, shape) if clip else rng.uniform(0.02, 0.98, shape)).astype(np.float32)
    target = (rng.integers(0, 256, shape, dtype=np.uint8) if u8
              else rng.uniform(0.02, 0.98, shape).astype(np.float32))
    loss, grad, scale, seg_rows = _run(harness, tmp_path, image, target, clip)
    exp_loss, exp_grad = O.loss(np.clip(image, 0, 1) if clip else image, target)
    if clip:
        exp_grad = exp_grad * O.clip_grad(image)
    assert np.isfinite(grad).all()
    np.testing.assert_allclose(loss, exp_loss, rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(grad, exp_grad, rtol=2e-4, atol=2e-7)
    assert scale == float(np.abs(grad).max())
    if shape[0] == 480:
        assert seg_rows > 16  # several chunks per CTA: the rings wrap


@pytest.mark.parametrize("shape", [(1, 1, 3), (3, 5, 3), (17, 31, 3), (64, 49, 3)])
def test_host_run_uint8_target_equals_normalised_float(harness, tmp_path, shape):
    """tests/test_loss.py:35-51: a uint8 target and the same target divided
    by 255 in float32 give bit-identical loss, gradient and |grad| maximum,
    for a random prediction and for the normalised target itself (where the
    L1 subgradient is zero and the loss vanishes)."""
    rng = np.random.default_rng(42 + shape[0])
    target = rng.integers(0, 256, shape, dtype=np.uint8)
    target[0, 0] = [0, 128, 255]
    normalised = target.astype(np.float32) * np.float32(1.0 / 255.0)
    for prediction in (rng.uniform(0, 1, shape).astype(np.float32), normalised):
        a = _run(harness, tmp_path, prediction, target, False)
        b = _run(harness, tmp_path, prediction, normalised, False)
        assert a[0] == b[0] and a[2] == b[2]
        np.testing.assert_array_equal(a[1], b[1])
    loss, grad, _, _ = _run(harness, tmp_path, normalised, target, False)
    assert abs(loss) < 2e-6 and float(np.abs(grad).max()) < 2e-7


@pytest.mark.parametrize("value", [0.0, np.nan, np.inf])
def test_host_run_gradient_maximum_propagates_nan(harness, tmp_path, value):
    """tests/test_loss.py:70-77: the |grad| maximum is taken over the float
    bits, so a NaN anywhere in the gradient (from a NaN or infinite
    prediction) makes it NaN, and it equals max |grad| otherwise."""
    prediction = np.zeros((17, 31, 3), np.float32)
    prediction[0, 0, 0] = value
    _, grad, scale, _ = _run(harness, tmp_path, prediction, np.zeros_like(prediction), False)
    expected = float(np.max(np.abs(grad)))
    if np.isnan(expected):
        assert np.isnan(scale)
    else:
        assert scale == expected
    assert np.isnan(scale) == (not np.isfinite(value))
