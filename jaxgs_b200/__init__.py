"""B200 (sm_100a) backend for the jax-gs render-and-loss hot path.

Modules:
  scene    — host-side camera / pool / synthetic scenes (numpy)
  types    — device pytrees (torch) with the reference's layouts
  kernels  — one function per reference binding, calling libgsb200.so
  step     — the training step (cull, project, bin, raster, loss, pullbacks)
  build    — nvcc build of libgsb200.so (sm_100a)
The CUDA library is loaded by `jaxgs_b200.kernels` (via `_lib`); importing it
without the library raises — there is no CPU fallback.
"""

__all__ = ["scene", "types", "kernels", "step", "build"]
