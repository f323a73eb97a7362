"""PyTorch (CPU, autograd) restatement of the reference's JAX numerics.

Independent of the C oracle: used to check the oracle's forward values and
its analytic gradients.  Each function restates one reference function:

  project          render/projection.py:33-74 (+ reference/sh.py:8-36)
  dense_composite  tests/test_cute.py:244-264 (front-to-back compositing with
                   the T >= 1/8192 early stop, over every splat in depth order)
  dense_fragment_statistics  kernels/sorted_rasterize.py:155-203 on the
                   same dense compositing
  photometric_loss reference/loss.py:6-43
"""

from __future__ import annotations

import math

import torch

C0 = 0.28209479177387814
C1 = 0.4886025119029199


def quaternion_to_matrix(q):
    q = q / torch.clamp(torch.linalg.norm(q, dim=-1, keepdim=True), min=1e-8)
    w, x, y, z = q.unbind(-1)
    return torch.stack(
        [
            torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1),
            torch.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1),
            torch.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1),
        ],
        -2,
    )


def eval_sh(sh, direction, degree):
    x, y, z = direction[..., 0:1], direction[..., 1:2], direction[..., 2:3]
    result = C0 * sh[..., 0, :]
    if degree >= 1:
        result = result - C1 * y * sh[..., 1, :] + C1 * z * sh[..., 2, :] - C1 * x * sh[..., 3, :]
    if degree >= 2:
        xx, yy, zz = x * x, y * y, z * z
        result = (result + 1.0925484305920792 * x * y * sh[..., 4, :]
                  - 1.0925484305920792 * y * z * sh[..., 5, :]
                  + 0.31539156525252005 * (2 * zz - xx - yy) * sh[..., 6, :]
                  - 1.0925484305920792 * x * z * sh[..., 7, :]
                  + 0.5462742152960396 * (xx - yy) * sh[..., 8, :])
    if degree >= 3:
        xx, yy, zz = x * x, y * y, z * z
        result = (result - 0.5900435899266435 * y * (3 * xx - yy) * sh[..., 9, :]
                  + 2.890611442640554 * x * y * z * sh[..., 10, :]
                  - 0.4570457994644658 * y * (4 * zz - xx - yy) * sh[..., 11, :]
                  + 0.3731763325901154 * z * (2 * zz - 3 * xx - 3 * yy) * sh[..., 12, :]
                  - 0.4570457994644658 * x * (4 * zz - xx - yy) * sh[..., 13, :]
                  + 1.445305721320277 * z * (xx - yy) * sh[..., 14, :]
                  - 0.5900435899266435 * x * (xx - 3 * yy) * sh[..., 15, :])
    return torch.clamp(result + 0.5, min=0.0)


def project(xyz, log_scale, rotation, opacity, sh, alive, camera, degree):
    """render/projection.py:33-74; camera is a jaxgs_b200.scene.Camera."""
    dt = xyz.dtype
    w2c = torch.as_tensor(camera.world_to_camera, dtype=dt)
    rot = w2c[:3, :3]
    points = xyz @ rot.T + w2c[:3, 3]
    x, y, z = points[:, 0], points[:, 1], points[:, 2]
    safe_z = torch.clamp(z, min=camera.near)
    mean = torch.stack([camera.fx * x / safe_z + camera.cx, camera.fy * y / safe_z + camera.cy], -1)
    scales = torch.exp(log_scale)
    local = quaternion_to_matrix(rotation) * scales[:, None, :]
    world_cov = local @ local.transpose(-1, -2)
    view_cov = rot[None] @ world_cov @ rot.T
    zeros = torch.zeros_like(z)
    jac = torch.stack([
        torch.stack([camera.fx / safe_z, zeros, -camera.fx * x / safe_z ** 2], -1),
        torch.stack([zeros, camera.fy / safe_z, -camera.fy * y / safe_z ** 2], -1)], -2)
    cov = jac @ view_cov @ jac.transpose(-1, -2) + 0.3 * torch.eye(2, dtype=dt)
    a, b, d = cov[:, 0, 0], cov[:, 0, 1], cov[:, 1, 1]
    det = torch.clamp(a * d - b * b, min=1e-8)
    conic = torch.stack([torch.stack([d, -b], -1), torch.stack([-b, a], -1)], -2) / det[:, None, None]
    radius = 3.0 * torch.sqrt(0.5 * (a + d + torch.sqrt(torch.clamp((a - d) ** 2 + 4 * b * b, min=1e-12))))
    center = torch.as_tensor(camera.center, dtype=dt)
    direction = xyz - center
    direction = direction / torch.clamp(torch.linalg.norm(direction, dim=-1, keepdim=True), min=1e-8)
    color = eval_sh(sh, direction, degree)
    alpha = torch.sigmoid(opacity[:, 0])
    visible = (alive & (z > camera.near) & (z < camera.far) & (alpha >= 1.0 / 255)
               & (mean[:, 0] >= -0.15 * camera.width) & (mean[:, 0] <= 1.15 * camera.width)
               & (mean[:, 1] >= -0.15 * camera.height) & (mean[:, 1] <= 1.15 * camera.height))
    return mean, z, conic, radius, color, alpha, visible


def dense_composite(mean, conic, color, alpha, depth, order, width, height, background=None):
    """tests/test_cute.py:244-264: every splat (in `order`) at every pixel,
    alpha cutoff 1/256, cap 255/256, power <= 0, T >= 1/8192 early stop.
    Returns rgb [H,W,3], depth [H,W], alpha [H,W]."""
    dt = mean.dtype
    ys, xs = torch.meshgrid(torch.arange(height, dtype=dt), torch.arange(width, dtype=dt), indexing="ij")
    pix = torch.stack([xs + 0.5, ys + 0.5], -1)
    m, c, col, a, dep = mean[order], conic[order], color[order], alpha[order], depth[order]
    delta = pix[:, :, None, :] - m
    power = -0.5 * torch.einsum("hwgi,gij,hwgj->hwg", delta, c, delta)
    raw = a * torch.exp(power)
    keep = (power <= 0) & (raw >= 1.0 / 256)
    al = torch.where(keep, torch.clamp(raw, max=255.0 / 256), torch.zeros_like(raw))
    prefix = torch.cumprod(1 - al, -1)
    before = torch.cat([torch.ones_like(prefix[..., :1]), prefix[..., :-1]], -1)
    active = before >= 1.0 / 8192
    al = torch.where(active, al, torch.zeros_like(al))
    weight = before * al
    final_t = torch.prod(1 - al, -1)
    rgb = torch.einsum("hwg,gc->hwc", weight, col)
    if background is not None:
        rgb = rgb + final_t[:, :, None] * torch.as_tensor(background, dtype=dt)
    return rgb, (weight * dep).sum(-1), 1 - final_t


def dense_fragment_statistics(mean, conic, color, opacity, width, height, drgb, background=None):
    """The fragment statistics of kernels/sorted_rasterize.py:155-203 from the
    dense compositing above (splats in index order), float64: per Gaussian
    the composited fragment count, the compositing weight sum, the opacity
    cotangent of sum(rgb * drgb) and the sum over pixels of its squared
    per-pixel part.  The per-pixel part comes from autograd through one
    opacity leaf per (pixel, Gaussian).  Returns [C, 4]."""
    dt = mean.dtype
    ys, xs = torch.meshgrid(torch.arange(height, dtype=dt), torch.arange(width, dtype=dt), indexing="ij")
    pix = torch.stack([xs + 0.5, ys + 0.5], -1)
    delta = pix[:, :, None, :] - mean
    power = -0.5 * torch.einsum("hwgi,gij,hwgj->hwg", delta, conic, delta)
    per_pixel = opacity.detach().expand(height, width, -1).clone().requires_grad_(True)
    raw = per_pixel * torch.exp(power)
    keep = (power <= 0) & (raw >= 1.0 / 256)
    al = torch.where(keep, torch.clamp(raw, max=255.0 / 256), torch.zeros_like(raw))
    prefix = torch.cumprod(1 - al, -1)
    before = torch.cat([torch.ones_like(prefix[..., :1]), prefix[..., :-1]], -1)
    active = (before >= 1.0 / 8192).detach()
    al = torch.where(active, al, torch.zeros_like(al))
    weight = before * al
    rgb = torch.einsum("hwg,gc->hwc", weight, color)
    if background is not None:
        rgb = rgb + torch.prod(1 - al, -1)[:, :, None] * torch.as_tensor(background, dtype=dt)
    (rgb * drgb).sum().backward()
    go = per_pixel.grad
    count = (keep & active).to(dt).sum((0, 1))
    return torch.stack([count, weight.detach().sum((0, 1)), go.sum((0, 1)), (go * go).sum((0, 1))], 1)


def _gauss_window(dt):
    x = torch.arange(11, dtype=dt) - 5
    g = torch.exp(-0.5 * (x / 1.5) ** 2)
    return g / g.sum()


def ssim(prediction, target):
    """reference/loss.py:10-35 on HWC images (SAME zero padding, clipped mean)."""
    dt = prediction.dtype
    g = _gauss_window(dt)
    kernel = (g[:, None] * g[None, :])[None, None].repeat(3, 1, 1, 1)

    def blur(img):
        return torch.nn.functional.conv2d(img.permute(2, 0, 1)[None], kernel, padding=5, groups=3)[0].permute(1, 2, 0)

    mu_x, mu_y = blur(prediction), blur(target)
    sx = blur(prediction ** 2) - mu_x ** 2
    sy = blur(target ** 2) - mu_y ** 2
    sxy = blur(prediction * target) - mu_x * mu_y
    c1, c2 = 0.01 ** 2, 0.03 ** 2
    num = (2 * mu_x * mu_y + c1) * (2 * sxy + c2)
    den = (mu_x ** 2 + mu_y ** 2 + c1) * (sx + sy + c2)
    return torch.clamp((num / den).mean(), -1.0, 1.0)


def photometric_loss(prediction, target, ssim_weight=0.2):
    """reference/loss.py:38-43."""
    return (1 - ssim_weight) * (prediction - target).abs().mean() + ssim_weight * (1 - ssim(prediction, target))


def finite(x):
    return bool(torch.isfinite(x).all()) and not math.isnan(float(x.sum()))
