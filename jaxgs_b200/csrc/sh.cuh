// Real spherical-harmonics basis (LiteGS/3DGS order) and the per-view SH
// cotangent expansion, shared by the projection kernels and the sparse Adam
// that reconstructs SH gradients itself, so both produce identical bits.
#pragma once

#include "gsb_common.cuh"

namespace gsb {

constexpr float kC0 = 0.28209479177387814f;
constexpr float kC1 = 0.4886025119029199f;

// SH basis values (reference/sh.py:8-36).
template <int DEGREE>
__device__ __forceinline__ void sh_basis(float dx, float dy, float dz, float b[16])
{
    float xx = dx * dx, yy = dy * dy, zz = dz * dz;
    b[0] = kC0;
    if (DEGREE >= 1) {
        b[1] = -kC1 * dy;
        b[2] = kC1 * dz;
        b[3] = -kC1 * dx;
    }
    if (DEGREE >= 2) {
        b[4] = 1.0925484305920792f * dx * dy;
        b[5] = -1.0925484305920792f * dy * dz;
        b[6] = 0.31539156525252005f * (2.0f * zz - xx - yy);
        b[7] = -1.0925484305920792f * dx * dz;
        b[8] = 0.5462742152960396f * (xx - yy);
    }
    if (DEGREE >= 3) {
        b[9] = -0.5900435899266435f * dy * (3.0f * xx - yy);
        b[10] = 2.890611442640554f * dx * dy * dz;
        b[11] = -0.4570457994644658f * dy * (4.0f * zz - xx - yy);
        b[12] = 0.3731763325901154f * dz * (2.0f * zz - 3.0f * xx - 3.0f * yy);
        b[13] = -0.4570457994644658f * dx * (4.0f * zz - xx - yy);
        b[14] = 1.445305721320277f * dz * (xx - yy);
        b[15] = -0.5900435899266435f * dx * (xx - 3.0f * yy);
    }
}

// SH basis at the unit direction from a camera centre (cv[0..2]) to the
// Gaussian at (wx, wy, wz) (training/sh_pullback.py:19-24).  The direction
// is scaled by the hardware reciprocal square root of its squared length
// (floored at 1e-16 like the reference's norm): a few ulps from the
// reference's divide by sqrt, inside the gradient tolerance, and about
// forty instructions cheaper per view than IEEE sqrt and three divides.
template <int DEGREE>
__device__ __forceinline__ void sh_view_basis(float wx, float wy, float wz, const float* cv,
                                              float bas[16])
{
    const float vx = wx - __ldg(cv), vy = wy - __ldg(cv + 1), vz = wz - __ldg(cv + 2);
    const float inv = rsqrtf(fmaxf(vx * vx + vy * vy + vz * vz, 1e-16f));
    sh_basis<DEGREE>(vx * inv, vy * inv, vz * inv, bas);
}

// training/sh_pullback.py:18-53 summed over views: for each view v with a
// non-zero masked colour cotangent g_v (colors + v * view_stride), the SH
// basis of its direction (centers + v * center_stride) adds Y_k g_v[c] to
// acc[3k + c] for the (DEGREE + 1)^2 active coefficients.  acc is not
// cleared here.
template <int DEGREE>
__device__ __forceinline__ void sh_expand_views(float wx, float wy, float wz, int views,
                                                const float* colors, int64_t view_stride,
                                                const float* centers, int64_t center_stride,
                                                float* acc)
{
    constexpr int NB = (DEGREE + 1) * (DEGREE + 1);
    for (int v = 0; v < views; v++) {
        const float* col = colors + v * view_stride;
        const float c0 = col[0], c1 = col[1], c2 = col[2];
        if (c0 == 0.0f && c1 == 0.0f && c2 == 0.0f) continue;
        float bas[16];
        sh_view_basis<DEGREE>(wx, wy, wz, centers + v * center_stride, bas);
#pragma unroll
        for (int k = 0; k < NB; k++) {
            acc[k * 3] = fmaf(bas[k], c0, acc[k * 3]);
            acc[k * 3 + 1] = fmaf(bas[k], c1, acc[k * 3 + 1]);
            acc[k * 3 + 2] = fmaf(bas[k], c2, acc[k * 3 + 2]);
        }
    }
}

}  // namespace gsb
