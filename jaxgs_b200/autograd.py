"""PyTorch autograd for the render and the loss: the torch counterpart of
the reference's custom_vjp rules (kernels/projector.py:152-224 for the
projection, kernels/sorted_rasterizer.py:165-236 for the fp32 rasterizer,
kernels/fused_loss.py:333-352 for the loss), so that a torch program can
write `loss = fused_loss(render(pool, ...)[0], target); loss.backward()`.

render() runs the forward half of the training step (cluster cull, compact
projection with visible-colour-only SH, binning, the recording fp32 raster
forward) and keeps what the backward needs; its backward runs the raster
backward over the listed clusters and the projection pullback in pool
order, so the gradients of xyz, log_scale, rotation, opacity and sh have
their parameters' shapes (rows of culled clusters and SH coefficients above
the active degree zero).  fused_loss() returns the loss and saves the image
gradient the same kernel computes, scaled by the upstream gradient in the
backward.  Both need CUDA tensors, as every binding of this package does.
"""

from __future__ import annotations

import torch

from . import kernels as K
from .scene import CapacityConfig
from .types import DeviceCamera, GaussianArrays


def _render_forward(pool: GaussianArrays, bounds, camera: DeviceCamera, config: CapacityConfig,
                    active_degree: int):
    """(rgb [H, W, 3], backward state, overflow [1]) of one view."""
    clusters, _ = K.compact_visible_clusters(bounds, camera, config, want_slots=False)
    projected, pullback = K.project_with_compact_pullback(
        pool, camera, config, active_degree, clusters, rgb_only=True, visible_color_only=True)
    table = K.build_sorted_visibility_table_cute(projected, camera, config)
    result, cache = K.rasterize_forward(projected, table, camera, config, want_depth=False,
                                        want_alpha=False)
    return result.rgb, (projected, pullback, table, cache, clusters), table.overflow


def _render_backward(state, grad_rgb: torch.Tensor, camera: DeviceCamera, config: CapacityConfig):
    """Pool-order (xyz, log_scale, rotation, opacity, sh) gradients."""
    projected, pullback, table, cache, clusters = state
    cot = K.rasterize_backward(projected, table, cache, grad_rgb, camera, config,
                               visible_clusters=clusters)
    return pullback(cot, compact=False)


class _Render(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xyz, log_scale, rotation, opacity, sh, alive, bounds, camera, config,
                active_degree):
        pool = GaussianArrays(xyz, log_scale, rotation, opacity, sh, alive)
        rgb, state, overflow = _render_forward(pool, bounds, camera, config, active_degree)
        ctx.state, ctx.camera, ctx.config = state, camera, config
        ctx.mark_non_differentiable(overflow)
        return rgb, overflow

    @staticmethod
    def backward(ctx, grad_rgb, _grad_overflow):
        # Each call allocates its own cotangent buffers, so a retained graph
        # may run the backward again.
        grads = _render_backward(ctx.state, grad_rgb.contiguous(), ctx.camera, ctx.config)
        return (*grads, None, None, None, None, None)


def render(pool: GaussianArrays, bounds, camera: DeviceCamera, config: CapacityConfig,
           active_degree: int | None = None):
    """Differentiable render of one view: (rgb [H, W, 3] float32, overflow
    [1] int32).  Gradients flow to pool.xyz, log_scale, rotation, opacity
    and sh; bounds are the cluster bounds (center, extent, valid) on the
    device.  The image is not clipped (the training loss clips it,
    fused_loss(..., clip_input=True))."""
    degree = config.sh_degree if active_degree is None else int(active_degree)
    return _Render.apply(pool.xyz, pool.log_scale, pool.rotation, pool.opacity, pool.sh,
                         pool.alive, bounds, camera, config, degree)


class _FusedLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, image, target, clip_input):
        loss, grad, _ = K._fused_loss(image, target, False, clip_input=clip_input)
        ctx.save_for_backward(grad)
        return loss.clone()  # a tensor of its own, not a view of the kernel's output

    @staticmethod
    def backward(ctx, grad_loss):
        (grad,) = ctx.saved_tensors
        return grad * grad_loss, None, None


def fused_loss(image: torch.Tensor, target: torch.Tensor, clip_input: bool = False) -> torch.Tensor:
    """Mean 0.8 L1 + 0.2 (1 - SSIM) of an [H, W, 3] float32 image against a
    uint8 or float target (kernels/fused_loss.py:333-352), differentiable in
    the image.  clip_input: the loss of clip(image, 0, 1), its gradient
    through the clip (1/2 at a bound), as rasterize_loss_and_grad (the
    fp32 step path) takes it."""
    return _FusedLoss.apply(image, target, bool(clip_input))
