/*
 * CPU oracle for the jax-gs render-and-loss hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates the reference algorithms so
 * that the CUDA kernels in jaxgs_b200/csrc can be checked against them.  It is
 * loaded by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline
 * leg; the product path never calls it.
 *
 * Every function cites the reference file:line it restates (paths are inside
 * the imgengineer/jax-gs project, src/jaxgs/...).  Compile with
 * -ffp-contract=off: each C expression then rounds once per operation, and
 * fmaf() is the only fused form, exactly where the reference uses an explicit
 * fma.rn.f32 (kernels/half2.py:296-317).
 *
 * Parity anchors: the binning restatement is bit-exact by construction (IEEE
 * add/mul/div/sqrt/fma in round-to-nearest plus the project-written logarithm
 * gs_logf below, which the GPU kernels evaluate with the same operation
 * sequence).  Projection, compositing and loss are evaluated in float (loss
 * and gradient accumulators in double) and compared within tolerances.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* Project-written natural logarithm.                                         */
/*                                                                           */
/* Method: Cody & Waite style range reduction x = 2^e * m, m in [sqrt(1/2),  */
/* sqrt(2)), then log(m) = 2*atanh(s) with s = (m-1)/(m+1) and the Taylor    */
/* series atanh(s) = s + s^3/3 + s^5/5 + ...  (|s| <= 0.1716, five terms      */
/* leave a truncation error below 2e-9 relative).  ln(2) is split into a     */
/* high part with 14 trailing zero bits and a low remainder so that e*ln2_hi */
/* is exact.  Only IEEE round-to-nearest +,-,*,/ and fma are used, so the     */
/* host and the GPU produce identical bits.  Valid for finite x > 0; returns  */
/* -inf for 0 and NaN for negative or NaN input (not reached by callers).     */
/* ------------------------------------------------------------------------- */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

EXPORT float gs_logf(float x)
{
    if (!(x > 0.0f)) return x == 0.0f ? -INFINITY : NAN;
    if (isinf(x)) return x;
    uint32_t bits = f2u(x);
    int e = 0;
    if (bits < 0x00800000u) {            /* subnormal: scale by 2^23 */
        x = x * 8388608.0f;
        bits = f2u(x);
        e = -23;
    }
    e += (int)(bits >> 23) - 127;
    float m = u2f((bits & 0x007FFFFFu) | 0x3F800000u);   /* [1, 2) */
    if (m > 1.41421356f) { m = m * 0.5f; e += 1; }       /* [sqrt(1/2), sqrt(2)] */
    float f = m - 1.0f;                                   /* exact (Sterbenz) */
    float s = f / (m + 1.0f);
    float z = s * s;
    float p = fmaf(z, 1.0f / 11.0f, 1.0f / 9.0f);
    p = fmaf(z, p, 1.0f / 7.0f);
    p = fmaf(z, p, 1.0f / 5.0f);
    p = fmaf(z, p, 1.0f / 3.0f);
    float sz = s * z;
    float tail = fmaf(sz, p, s);                          /* atanh(s) */
    float lm = tail * 2.0f;                               /* exact */
    float ef = (float)e;
    const float ln2_hi = 0.693145751953125f;              /* 0x3F317200 */
    const float ln2_lo = 1.42860682030941723212e-6f;
    return fmaf(ef, ln2_hi, fmaf(ef, ln2_lo, lm));
}

/* PTX cvt.rzi.s32.f32: truncate toward zero, saturate, NaN -> 0. */
static inline int32_t trunc_i32(float x)
{
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x <= -2147483648.0f) return INT32_MIN;
    return (int32_t)x;
}
static inline int32_t imin(int32_t a, int32_t b) { return a < b ? a : b; }
static inline int32_t imax(int32_t a, int32_t b) { return a > b ? a : b; }

/* ------------------------------------------------------------------------- */
/* Projection forward: kernels/projection.py:47-175 (per-slot body) and the  */
/* compact thread->slot mapping of :42-47.  The JAX restatement of the same  */
/* math is render/projection.py:33-74 and reference/sh.py:8-36.             */
/* ------------------------------------------------------------------------- */
#define SH_C0 0.28209479177387814f
#define SH_C1 0.4886025119029199f

static void sh_color(const float* coef, int degree, float dx, float dy, float dz, float out[3])
{
    float xx = dx * dx, yy = dy * dy, zz = dz * dz;
    for (int ch = 0; ch < 3; ch++) {
        float value = SH_C0 * coef[ch];
        if (degree >= 1)
            value += (-SH_C1 * dy * coef[ch + 3] + SH_C1 * dz * coef[ch + 6]
                      - SH_C1 * dx * coef[ch + 9]);
        if (degree >= 2)
            value += (1.0925484305920792f * dx * dy * coef[ch + 12]
                      - 1.0925484305920792f * dy * dz * coef[ch + 15]
                      + 0.31539156525252005f * (2.0f * zz - xx - yy) * coef[ch + 18]
                      - 1.0925484305920792f * dx * dz * coef[ch + 21]
                      + 0.5462742152960396f * (xx - yy) * coef[ch + 24]);
        if (degree >= 3)
            value += (-0.5900435899266435f * dy * (3.0f * xx - yy) * coef[ch + 27]
                      + 2.890611442640554f * dx * dy * dz * coef[ch + 30]
                      - 0.4570457994644658f * dy * (4.0f * zz - xx - yy) * coef[ch + 33]
                      + 0.3731763325901154f * dz * (2.0f * zz - 3.0f * xx - 3.0f * yy) * coef[ch + 36]
                      - 0.4570457994644658f * dx * (4.0f * zz - xx - yy) * coef[ch + 39]
                      + 1.445305721320277f * dz * (xx - yy) * coef[ch + 42]
                      - 0.5900435899266435f * dx * (xx - 3.0f * yy) * coef[ch + 45]);
        out[ch] = fmaxf(value + 0.5f, 0.0f);
    }
}

/* Slot list of the compact mapping: slot of compact index i, or -1. */
static int64_t compact_slot(int64_t i, int capacity, const int32_t* cluster_ids,
                            int cluster_count, int cluster_size)
{
    if (!cluster_ids) return i < capacity ? i : -1;
    if (i >= (int64_t)cluster_count * cluster_size) return -1;
    int64_t slot = (int64_t)cluster_ids[i / cluster_size] * cluster_size + i % cluster_size;
    return slot < capacity ? slot : -1;
}

EXPORT void orc_project_fwd(
    const float* xyz, const float* log_scale, const float* rotation, const float* opacity,
    const float* sh, const uint8_t* alive, const float* view, const float* intr,
    const float* center, const int32_t* cluster_ids, int cluster_count, int capacity,
    int sh_dim, int degree, int width, int height, float near, float far, int cluster_size,
    int visible_color_only, float* out_mean, float* out_depth, float* out_conic,
    float* out_radius, float* out_color, float* out_alpha, int8_t* out_visible)
{
    /* Slots outside the listed clusters define only visible = 0
       (kernels/projector.py:334-337 via _clear_visible, projection.py:204-210). */
    if (cluster_ids) memset(out_visible, 0, (size_t)capacity);
    int64_t n = cluster_ids ? (int64_t)cluster_count * cluster_size : capacity;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        int64_t g = compact_slot(i, capacity, cluster_ids, cluster_count, cluster_size);
        if (g < 0) continue;
        float wx = xyz[g * 3], wy = xyz[g * 3 + 1], wz = xyz[g * 3 + 2];
        float x = view[0] * wx + view[1] * wy + view[2] * wz + view[3];
        float y = view[4] * wx + view[5] * wy + view[6] * wz + view[7];
        float z = view[8] * wx + view[9] * wy + view[10] * wz + view[11];
        float safe_z = fmaxf(z, near);
        float fx = intr[0], fy = intr[1], cx = intr[2], cy = intr[3];
        float u = fx * x / safe_z + cx;
        float v = fy * y / safe_z + cy;
        out_mean[g * 2] = u;
        out_mean[g * 2 + 1] = v;
        out_depth[g] = z;
        float qw = rotation[g * 4], qx = rotation[g * 4 + 1], qy = rotation[g * 4 + 2],
              qz = rotation[g * 4 + 3];
        float qnorm = 1.0f / sqrtf(fmaxf(qw * qw + qx * qx + qy * qy + qz * qz, 1e-16f));
        qw *= qnorm; qx *= qnorm; qy *= qnorm; qz *= qnorm;
        float r00 = 1.0f - 2.0f * (qy * qy + qz * qz), r01 = 2.0f * (qx * qy - qw * qz),
              r02 = 2.0f * (qx * qz + qw * qy);
        float r10 = 2.0f * (qx * qy + qw * qz), r11 = 1.0f - 2.0f * (qx * qx + qz * qz),
              r12 = 2.0f * (qy * qz - qw * qx);
        float r20 = 2.0f * (qx * qz - qw * qy), r21 = 2.0f * (qy * qz + qw * qx),
              r22 = 1.0f - 2.0f * (qx * qx + qy * qy);
        float s0 = expf(log_scale[g * 3]), s1 = expf(log_scale[g * 3 + 1]),
              s2 = expf(log_scale[g * 3 + 2]);
        float m00 = (view[0] * r00 + view[1] * r10 + view[2] * r20) * s0;
        float m01 = (view[0] * r01 + view[1] * r11 + view[2] * r21) * s1;
        float m02 = (view[0] * r02 + view[1] * r12 + view[2] * r22) * s2;
        float m10 = (view[4] * r00 + view[5] * r10 + view[6] * r20) * s0;
        float m11 = (view[4] * r01 + view[5] * r11 + view[6] * r21) * s1;
        float m12 = (view[4] * r02 + view[5] * r12 + view[6] * r22) * s2;
        float m20 = (view[8] * r00 + view[9] * r10 + view[10] * r20) * s0;
        float m21 = (view[8] * r01 + view[9] * r11 + view[10] * r21) * s1;
        float m22 = (view[8] * r02 + view[9] * r12 + view[10] * r22) * s2;
        float j0 = fx / safe_z, j1 = fy / safe_z;
        float j2 = fx * x / (safe_z * safe_z), j3 = fy * y / (safe_z * safe_z);
        float a0 = j0 * m00 - j2 * m20, a1 = j0 * m01 - j2 * m21, a2 = j0 * m02 - j2 * m22;
        float b0 = j1 * m10 - j3 * m20, b1 = j1 * m11 - j3 * m21, b2 = j1 * m12 - j3 * m22;
        float a = a0 * a0 + a1 * a1 + a2 * a2 + 0.3f;
        float b = a0 * b0 + a1 * b1 + a2 * b2;
        float d = b0 * b0 + b1 * b1 + b2 * b2 + 0.3f;
        float det = fmaxf(a * d - b * b, 1e-8f);
        out_conic[g * 4] = d / det;
        out_conic[g * 4 + 1] = -b / det;
        out_conic[g * 4 + 2] = -b / det;
        out_conic[g * 4 + 3] = a / det;
        out_radius[g] = 3.0f * sqrtf(0.5f * (a + d + sqrtf(fmaxf((a - d) * (a - d) + 4.0f * b * b, 1e-12f))));
        float alpha = 1.0f / (1.0f + expf(-opacity[g]));
        out_alpha[g] = alpha;
        int vis = alive[g] != 0 && z > near && z < far && alpha >= (float)(1.0 / 255)
                  && u >= -0.15f * (float)width && u <= 1.15f * (float)width
                  && v >= -0.15f * (float)height && v <= 1.15f * (float)height;
        out_visible[g] = (int8_t)vis;
        if (!visible_color_only || vis) {
            float dx = wx - center[0], dy = wy - center[1], dz = wz - center[2];
            float dn = 1.0f / sqrtf(fmaxf(dx * dx + dy * dy + dz * dz, 1e-16f));
            float rgb[3];
            sh_color(sh + g * (int64_t)sh_dim * 3, degree, dx * dn, dy * dn, dz * dn, rgb);
            out_color[g * 3] = rgb[0];
            out_color[g * 3 + 1] = rgb[1];
            out_color[g * 3 + 2] = rgb[2];
        } else {
            out_color[g * 3] = out_color[g * 3 + 1] = out_color[g * 3 + 2] = 0.0f;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Projection pullback: kernels/projection_backward.py:42-367.               */
/* Gradients are written at the compact index when compact_gradients, else   */
/* at the pool slot; out_sh holds sh_gradient_dim coefficients per point.    */
/* ------------------------------------------------------------------------- */
EXPORT void orc_project_bwd(
    const float* xyz, const float* log_scale, const float* rotation, const float* opacity,
    const float* sh, const float* view, const float* intr, const float* center,
    const float* color, const int32_t* cluster_ids, int cluster_count, int capacity,
    int sh_dim, int sh_gradient_dim, int degree, float near, int cluster_size,
    int compact_gradients, int rgb_only, int sh_color_only, const float* gmean,
    const float* gdepth, const float* gconic, const float* gradius, const float* gcolor,
    const float* galpha, float* out_xyz, float* out_log_scale, float* out_rotation,
    float* out_opacity, float* out_sh)
{
    int64_t n = cluster_ids ? (int64_t)cluster_count * cluster_size : capacity;
    int shg = sh_gradient_dim * 3;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        int64_t g = compact_slot(i, capacity, cluster_ids, cluster_count, cluster_size);
        if (g < 0) continue;
        int64_t o = compact_gradients ? i : g;
        float* osh = out_sh + o * shg;
        int has = galpha[g] != 0.0f;
        if (!rgb_only) has = has || gdepth[g] != 0.0f || gradius[g] != 0.0f;
        for (int k = 0; k < 2; k++) has = has || gmean[g * 2 + k] != 0.0f;
        for (int k = 0; k < 4; k++) has = has || gconic[g * 4 + k] != 0.0f;
        for (int k = 0; k < 3; k++) has = has || gcolor[g * 3 + k] != 0.0f;
        if (!has) {
            for (int k = 0; k < 3; k++) out_xyz[o * 3 + k] = out_log_scale[o * 3 + k] = 0.0f;
            for (int k = 0; k < 4; k++) out_rotation[o * 4 + k] = 0.0f;
            out_opacity[o] = 0.0f;
            for (int k = 0; k < shg; k++) osh[k] = 0.0f;
            continue;
        }
        float wx = xyz[g * 3], wy = xyz[g * 3 + 1], wz = xyz[g * 3 + 2];
        float x = view[0] * wx + view[1] * wy + view[2] * wz + view[3];
        float y = view[4] * wx + view[5] * wy + view[6] * wz + view[7];
        float z = view[8] * wx + view[9] * wy + view[10] * wz + view[11];
        float safe_z = fmaxf(z, near);
        float fx = intr[0], fy = intr[1];
        float inv_z = 1.0f / safe_z, inv_z2 = inv_z * inv_z;
        float gx = gmean[g * 2] * fx * inv_z;
        float gy = gmean[g * 2 + 1] * fy * inv_z;
        float gz = rgb_only ? 0.0f : gdepth[g];
        float gsafe_z = -gmean[g * 2] * fx * x * inv_z2;
        gsafe_z -= gmean[g * 2 + 1] * fy * y * inv_z2;
        float qw0 = rotation[g * 4], qx0 = rotation[g * 4 + 1], qy0 = rotation[g * 4 + 2],
              qz0 = rotation[g * 4 + 3];
        float qdenom = sqrtf(fmaxf(qw0 * qw0 + qx0 * qx0 + qy0 * qy0 + qz0 * qz0, 1e-16f));
        float qw = qw0 / qdenom, qx = qx0 / qdenom, qy = qy0 / qdenom, qz = qz0 / qdenom;
        float r00 = 1.0f - 2.0f * (qy * qy + qz * qz), r01 = 2.0f * (qx * qy - qw * qz),
              r02 = 2.0f * (qx * qz + qw * qy);
        float r10 = 2.0f * (qx * qy + qw * qz), r11 = 1.0f - 2.0f * (qx * qx + qz * qz),
              r12 = 2.0f * (qy * qz - qw * qx);
        float r20 = 2.0f * (qx * qz - qw * qy), r21 = 2.0f * (qy * qz + qw * qx),
              r22 = 1.0f - 2.0f * (qx * qx + qy * qy);
        float s0 = expf(log_scale[g * 3]), s1 = expf(log_scale[g * 3 + 1]),
              s2 = expf(log_scale[g * 3 + 2]);
        float m00 = (view[0] * r00 + view[1] * r10 + view[2] * r20) * s0;
        float m01 = (view[0] * r01 + view[1] * r11 + view[2] * r21) * s1;
        float m02 = (view[0] * r02 + view[1] * r12 + view[2] * r22) * s2;
        float m10 = (view[4] * r00 + view[5] * r10 + view[6] * r20) * s0;
        float m11 = (view[4] * r01 + view[5] * r11 + view[6] * r21) * s1;
        float m12 = (view[4] * r02 + view[5] * r12 + view[6] * r22) * s2;
        float m20 = (view[8] * r00 + view[9] * r10 + view[10] * r20) * s0;
        float m21 = (view[8] * r01 + view[9] * r11 + view[10] * r21) * s1;
        float m22 = (view[8] * r02 + view[9] * r12 + view[10] * r22) * s2;
        float j0 = fx * inv_z, j1 = fy * inv_z, j2 = fx * x * inv_z2, j3 = fy * y * inv_z2;
        float a0 = j0 * m00 - j2 * m20, a1 = j0 * m01 - j2 * m21, a2 = j0 * m02 - j2 * m22;
        float b0 = j1 * m10 - j3 * m20, b1 = j1 * m11 - j3 * m21, b2 = j1 * m12 - j3 * m22;
        float a = a0 * a0 + a1 * a1 + a2 * a2 + 0.3f;
        float b = a0 * b0 + a1 * b1 + a2 * b2;
        float d = b0 * b0 + b1 * b1 + b2 * b2 + 0.3f;
        float raw_det = a * d - b * b;
        float det = fmaxf(raw_det, 1e-8f);
        float gc00 = gconic[g * 4], gc01 = gconic[g * 4 + 1], gc10 = gconic[g * 4 + 2],
              gc11 = gconic[g * 4 + 3];
        float gdet = 0.0f;
        if (raw_det > 1e-8f) gdet = -(gc00 * d - (gc01 + gc10) * b + gc11 * a) / (det * det);
        float ga = gc11 / det + gdet * d;
        float gb = -(gc01 + gc10) / det - 2.0f * b * gdet;
        float gd = gc00 / det + gdet * a;
        if (!rgb_only) {
            float disc = (a - d) * (a - d) + 4.0f * b * b;
            float disc_root = sqrtf(fmaxf(disc, 1e-12f));
            float eigen = 0.5f * (a + d + disc_root);
            float geigen = gradius[g] * 1.5f / sqrtf(eigen);
            float gdisc = 0.0f;
            if (disc > 1e-12f) gdisc = geigen * 0.25f / disc_root;
            ga += 0.5f * geigen + 2.0f * (a - d) * gdisc;
            gb += 8.0f * b * gdisc;
            gd += 0.5f * geigen - 2.0f * (a - d) * gdisc;
        }
        float ga0 = 2 * a0 * ga + b0 * gb, ga1 = 2 * a1 * ga + b1 * gb, ga2 = 2 * a2 * ga + b2 * gb;
        float gb0 = 2 * b0 * gd + a0 * gb, gb1 = 2 * b1 * gd + a1 * gb, gb2 = 2 * b2 * gd + a2 * gb;
        float gj0 = ga0 * m00 + ga1 * m01 + ga2 * m02;
        float gj1 = gb0 * m10 + gb1 * m11 + gb2 * m12;
        float gj2 = -(ga0 * m20 + ga1 * m21 + ga2 * m22);
        float gj3 = -(gb0 * m20 + gb1 * m21 + gb2 * m22);
        gx += gj2 * fx * inv_z2;
        gy += gj3 * fy * inv_z2;
        gsafe_z -= (gj0 * fx + gj1 * fy) * inv_z2;
        gsafe_z -= 2.0f * (gj2 * fx * x + gj3 * fy * y) * inv_z2 * inv_z;
        if (z > near) gz += gsafe_z;
        float gm00 = j0 * ga0, gm01 = j0 * ga1, gm02 = j0 * ga2;
        float gm10 = j1 * gb0, gm11 = j1 * gb1, gm12 = j1 * gb2;
        float gm20 = -j2 * ga0 - j3 * gb0, gm21 = -j2 * ga1 - j3 * gb1, gm22 = -j2 * ga2 - j3 * gb2;
        out_log_scale[o * 3] = gm00 * m00 + gm10 * m10 + gm20 * m20;
        out_log_scale[o * 3 + 1] = gm01 * m01 + gm11 * m11 + gm21 * m21;
        out_log_scale[o * 3 + 2] = gm02 * m02 + gm12 * m12 + gm22 * m22;
        float gr00 = s0 * (view[0] * gm00 + view[4] * gm10 + view[8] * gm20);
        float gr10 = s0 * (view[1] * gm00 + view[5] * gm10 + view[9] * gm20);
        float gr20 = s0 * (view[2] * gm00 + view[6] * gm10 + view[10] * gm20);
        float gr01 = s1 * (view[0] * gm01 + view[4] * gm11 + view[8] * gm21);
        float gr11 = s1 * (view[1] * gm01 + view[5] * gm11 + view[9] * gm21);
        float gr21 = s1 * (view[2] * gm01 + view[6] * gm11 + view[10] * gm21);
        float gr02 = s2 * (view[0] * gm02 + view[4] * gm12 + view[8] * gm22);
        float gr12 = s2 * (view[1] * gm02 + view[5] * gm12 + view[9] * gm22);
        float gr22 = s2 * (view[2] * gm02 + view[6] * gm12 + view[10] * gm22);
        float gqw = -2 * qz * gr01 + 2 * qy * gr02 + 2 * qz * gr10 - 2 * qx * gr12
                    - 2 * qy * gr20 + 2 * qx * gr21;
        float gqx = 2 * qy * (gr01 + gr10) + 2 * qz * (gr02 + gr20) - 4 * qx * (gr11 + gr22)
                    - 2 * qw * gr12 + 2 * qw * gr21;
        float gqy = -4 * qy * (gr00 + gr22) + 2 * qx * (gr01 + gr10) + 2 * qw * gr02
                    + 2 * qz * (gr12 + gr21) - 2 * qw * gr20;
        float gqz = -4 * qz * (gr00 + gr11) - 2 * qw * gr01 + 2 * qx * (gr02 + gr20)
                    + 2 * qw * gr10 + 2 * qy * (gr12 + gr21);
        float qdot = gqw * qw + gqx * qx + gqy * qy + gqz * qz;
        if (qdenom > 1e-8f) {
            gqw = (gqw - qdot * qw) / qdenom;
            gqx = (gqx - qdot * qx) / qdenom;
            gqy = (gqy - qdot * qy) / qdenom;
            gqz = (gqz - qdot * qz) / qdenom;
        } else {
            gqw /= qdenom; gqx /= qdenom; gqy /= qdenom; gqz /= qdenom;
        }
        out_rotation[o * 4] = gqw;
        out_rotation[o * 4 + 1] = gqx;
        out_rotation[o * 4 + 2] = gqy;
        out_rotation[o * 4 + 3] = gqz;
        float alpha = 1.0f / (1.0f + expf(-opacity[g]));
        out_opacity[o] = galpha[g] * alpha * (1.0f - alpha);

        float vx = wx - center[0], vy = wy - center[1], vz = wz - center[2];
        float dir_denom = sqrtf(fmaxf(vx * vx + vy * vy + vz * vz, 1e-16f));
        float dx = vx / dir_denom, dy = vy / dir_denom, dz = vz / dir_denom;
        float xx = dx * dx, yy = dy * dy, zz = dz * dz;
        float gdx = 0.0f, gdy = 0.0f, gdz = 0.0f;
        const float* c = sh + g * (int64_t)sh_dim * 3;
        int used = (degree + 1) * (degree + 1);
        for (int k = 0; k < shg; k++) osh[k] = 0.0f;
        for (int ch = 0; ch < 3; ch++) {
            float gc = color[g * 3 + ch] > 0.0f ? gcolor[g * 3 + ch] : 0.0f;
            if (sh_color_only) {
                osh[ch] = gc;
            } else {
                osh[ch] = gc * SH_C0;
            }
            if (degree >= 1) {
                if (!sh_color_only) {
                    osh[3 + ch] = -gc * SH_C1 * dy;
                    osh[6 + ch] = gc * SH_C1 * dz;
                    osh[9 + ch] = -gc * SH_C1 * dx;
                }
                gdx -= gc * SH_C1 * c[ch + 9];
                gdy -= gc * SH_C1 * c[ch + 3];
                gdz += gc * SH_C1 * c[ch + 6];
            }
            if (degree >= 2) {
                if (!sh_color_only) {
                    osh[12 + ch] = gc * 1.0925484305920792f * dx * dy;
                    osh[15 + ch] = -gc * 1.0925484305920792f * dy * dz;
                    osh[18 + ch] = gc * 0.31539156525252005f * (2 * zz - xx - yy);
                    osh[21 + ch] = -gc * 1.0925484305920792f * dx * dz;
                    osh[24 + ch] = gc * 0.5462742152960396f * (xx - yy);
                }
                gdx += gc * (1.0925484305920792f * dy * c[ch + 12] - 0.6307831305050401f * dx * c[ch + 18]
                             - 1.0925484305920792f * dz * c[ch + 21] + 1.0925484305920792f * dx * c[ch + 24]);
                gdy += gc * (1.0925484305920792f * dx * c[ch + 12] - 1.0925484305920792f * dz * c[ch + 15]
                             - 0.6307831305050401f * dy * c[ch + 18] - 1.0925484305920792f * dy * c[ch + 24]);
                gdz += gc * (-1.0925484305920792f * dy * c[ch + 15] + 1.2615662610100802f * dz * c[ch + 18]
                             - 1.0925484305920792f * dx * c[ch + 21]);
            }
            if (degree >= 3) {
                if (!sh_color_only) {
                    osh[27 + ch] = -gc * 0.5900435899266435f * dy * (3 * xx - yy);
                    osh[30 + ch] = gc * 2.890611442640554f * dx * dy * dz;
                    osh[33 + ch] = -gc * 0.4570457994644658f * dy * (4 * zz - xx - yy);
                    osh[36 + ch] = gc * 0.3731763325901154f * dz * (2 * zz - 3 * xx - 3 * yy);
                    osh[39 + ch] = -gc * 0.4570457994644658f * dx * (4 * zz - xx - yy);
                    osh[42 + ch] = gc * 1.445305721320277f * dz * (xx - yy);
                    osh[45 + ch] = -gc * 0.5900435899266435f * dx * (xx - 3 * yy);
                }
                gdx += gc * (-3.540261539559861f * dx * dy * c[ch + 27] + 2.890611442640554f * dy * dz * c[ch + 30]
                             + 0.9140915989289316f * dx * dy * c[ch + 33] - 2.2390579955406924f * dx * dz * c[ch + 36]
                             - 0.4570457994644658f * (4 * zz - 3 * xx - yy) * c[ch + 39]
                             + 2.890611442640554f * dx * dz * c[ch + 42] - 1.7701307697799305f * (xx - yy) * c[ch + 45]);
                gdy += gc * (-1.7701307697799305f * (xx - yy) * c[ch + 27] + 2.890611442640554f * dx * dz * c[ch + 30]
                             - 0.4570457994644658f * (4 * zz - xx - 3 * yy) * c[ch + 33]
                             - 2.2390579955406924f * dy * dz * c[ch + 36] + 0.9140915989289316f * dx * dy * c[ch + 39]
                             - 2.890611442640554f * dy * dz * c[ch + 42] + 3.540261539559861f * dx * dy * c[ch + 45]);
                gdz += gc * (2.890611442640554f * dx * dy * c[ch + 30] - 3.6563663957157264f * dy * dz * c[ch + 33]
                             + 0.3731763325901154f * (6 * zz - 3 * xx - 3 * yy) * c[ch + 36]
                             - 3.6563663957157264f * dx * dz * c[ch + 39] + 1.445305721320277f * (xx - yy) * c[ch + 42]);
            }
        }
        (void)used;
        float dir_dot = gdx * dx + gdy * dy + gdz * dz;
        float gxw = gdx / dir_denom, gyw = gdy / dir_denom, gzw = gdz / dir_denom;
        if (dir_denom > 1e-8f) {
            gxw = (gdx - dir_dot * dx) / dir_denom;
            gyw = (gdy - dir_dot * dy) / dir_denom;
            gzw = (gdz - dir_dot * dz) / dir_denom;
        }
        out_xyz[o * 3] = view[0] * gx + view[4] * gy + view[8] * gz + gxw;
        out_xyz[o * 3 + 1] = view[1] * gx + view[5] * gy + view[9] * gz + gyw;
        out_xyz[o * 3 + 2] = view[2] * gx + view[6] * gy + view[10] * gz + gzw;
    }
}

/* ------------------------------------------------------------------------- */
/* AccuTile binning: kernels/sorted_visibility.py:34-224 and _count :307-370.*/
/* ------------------------------------------------------------------------- */
typedef struct {
    float disc, level;
    int is_y;
    float block_u, block_v;
    int32_t u0, u1, v0, v1;
    float bbox_u_min, bbox_u_max, bbox_v_min, bbox_v_max, arg_min, arg_max;
} Ellipse;

/* sorted_visibility.py:34-74 */
static void intersection(float px, float py, float c00, float c01, float c11, float disc,
                         float level, int is_y, float coord, int side, int sliced,
                         float* out_low, float* out_high)
{
    float pu = px, pv = py, coeff = c11;
    if (is_y) { pu = py; pv = px; coeff = c00; }
    float delta = coord - pu;
    float radicand;
    if (sliced) radicand = fmaf(delta, disc * delta, level * coeff);
    else radicand = fmaf(level, coeff, (disc * delta) * delta);
    float root = sqrtf(fmaxf(radicand, 0.0f));
    float low = 0.0f, high = 0.0f;
    if (side == 0) {
        float shared = c01 * -delta;
        low = shared - root;
        high = shared + root;
    } else if (side < 0) {
        low = fmaf(-c01, delta, -root);
    } else {
        high = fmaf(-c01, delta, root);
    }
    *out_low = low / coeff + pv;
    *out_high = high / coeff + pv;
}

/* sorted_visibility.py:77-126 */
static Ellipse ellipse_bounds(float px, float py, float c00, float c01, float c11, float alpha,
                              int tile_w, int tile_h, int tiles_x, int tiles_y)
{
    Ellipse e;
    float c01_sq = c01 * c01;
    float disc = c01_sq - c00 * c11;
    float level = 2.0f * gs_logf(alpha * 255.0f);
    float numerator = c01_sq * -level;
    float x_term = sqrtf(numerator / (c00 * disc));
    float y_term = sqrtf(numerator / (c11 * disc));
    if (c01 >= 0.0f) { x_term = -x_term; y_term = -y_term; }
    float argmin_x = py - y_term, argmin_y = px - x_term;
    float argmax_x = py + y_term, argmax_y = px + x_term;
    float xmin, ymin, xmax, ymax, unused;
    intersection(px, py, c00, c01, c11, disc, level, 1, argmin_x, -1, 0, &xmin, &unused);
    intersection(px, py, c00, c01, c11, disc, level, 0, argmin_y, -1, 0, &ymin, &unused);
    intersection(px, py, c00, c01, c11, disc, level, 1, argmax_x, 1, 0, &unused, &xmax);
    intersection(px, py, c00, c01, c11, disc, level, 0, argmax_y, 1, 0, &unused, &ymax);
    float tw = (float)tile_w, th = (float)tile_h;
    int32_t x0 = imax(0, imin(tiles_x, trunc_i32(xmin / tw)));
    int32_t y0 = imax(0, imin(tiles_y, trunc_i32(ymin / th)));
    int32_t x1 = imax(0, imin(tiles_x, trunc_i32(((xmax + tw) - 1.0f) / tw)));
    int32_t y1 = imax(0, imin(tiles_y, trunc_i32(((ymax + th) - 1.0f) / th)));
    e.disc = disc;
    e.level = level;
    e.is_y = (y1 - y0) < (x1 - x0);
    e.block_u = tw; e.block_v = th;
    e.u0 = x0; e.u1 = x1; e.v0 = y0; e.v1 = y1;
    e.bbox_u_min = xmin; e.bbox_u_max = xmax; e.bbox_v_min = ymin; e.bbox_v_max = ymax;
    e.arg_min = argmin_y; e.arg_max = argmax_y;
    if (e.is_y) {
        e.block_u = th; e.block_v = tw;
        e.u0 = y0; e.u1 = y1; e.v0 = x0; e.v1 = x1;
        e.bbox_u_min = ymin; e.bbox_u_max = ymax; e.bbox_v_min = xmin; e.bbox_v_max = xmax;
        e.arg_min = argmin_x; e.arg_max = argmax_x;
    }
    if ((int64_t)(y1 - y0) * (int64_t)(x1 - x0) <= 0) e.u1 = e.u0;
    return e;
}

/* sorted_visibility.py:129-141 */
static void span(const Ellipse* e, float line, float next_line, float lower_min, float lower_max,
                 float upper_min, float upper_max, int32_t* first, int32_t* end)
{
    float emin = fminf(lower_min, upper_min);
    float emax = fmaxf(lower_max, upper_max);
    if (line <= e->arg_min && e->arg_min < next_line) emin = e->bbox_v_min;
    if (line <= e->arg_max && e->arg_max < next_line) emax = e->bbox_v_max;
    *first = imax(e->v0, imin(e->v1, trunc_i32(emin / e->block_v)));
    *end = imin(e->v1, imax(e->v0, trunc_i32(emax / e->block_v + 1.0f)));
}

/* sorted_visibility.py:170-175 */
static inline int64_t tile_key(int is_y, int32_t u, int32_t v, int tiles_x)
{
    return is_y ? (int64_t)u * tiles_x + v : (int64_t)v * tiles_x + u;
}

/* sorted_visibility.py:178-224.  keys == NULL counts only; otherwise keys
   receives the tile of every pair, in the reference's emission order. */
static int32_t process_tiles(float px, float py, float c00, float c01, float c11, float alpha,
                             int tile_w, int tile_h, int tiles_x, int tiles_y, int64_t* keys)
{
    Ellipse e = ellipse_bounds(px, py, c00, c01, c11, alpha, tile_w, tile_h, tiles_x, tiles_y);
    int32_t count = 0;
    if (e.u1 > e.u0) {
        float upper_min = e.bbox_v_max, upper_max = e.bbox_v_min;
        float lower_min = upper_min, lower_max = upper_max;
        float line = (float)e.u0 * e.block_u;
        if (e.bbox_u_min <= line)
            intersection(px, py, c00, c01, c11, e.disc, e.level, e.is_y, line, 0, 0, &lower_min,
                         &lower_max);
        for (int32_t u = e.u0; u < e.u1; u++) {
            float next_line = line + e.block_u;
            if (next_line <= e.bbox_u_max)
                intersection(px, py, c00, c01, c11, e.disc, e.level, e.is_y, next_line, 0, 1,
                             &upper_min, &upper_max);
            int32_t first, end;
            span(&e, line, next_line, lower_min, lower_max, upper_min, upper_max, &first, &end);
            if (keys)
                for (int32_t v = first; v < end; v++) keys[count + v - first] = tile_key(e.is_y, u, v, tiles_x);
            count += end - first;
            lower_min = upper_min;
            lower_max = upper_max;
            line = next_line;
        }
    }
    return count;
}

static int count_gate(float mx, float my, float c00, float c01, float c11, float a, int width,
                      int height)
{
    /* sorted_visibility.py:333-342 */
    return a >= (float)(1.0 / 255.0) && c00 > 0.0f && c11 > 0.0f && c00 * c11 - c01 * c01 > 0.0f
           && mx >= -0.15f * (float)width && mx <= 1.15f * (float)width
           && my >= -0.15f * (float)height && my <= 1.15f * (float)height;
}

/* Depth sort key: sorted_visibility.py:362-370. */
static inline uint32_t depth_key(float depth, int32_t count)
{
    if (count <= 0) return 0xFFFFFFFFu;
    uint32_t bits = f2u(depth);
    return (bits >> 31) ? ~bits : (bits ^ 0x80000000u);
}

/* _count kernel, sorted_visibility.py:307-370. */
EXPORT void orc_count(const float* mean, const float* conic, const float* alpha,
                      const float* depth, const int8_t* visible, int capacity, int tile_w,
                      int tile_h, int tiles_x, int tiles_y, int width, int height,
                      int32_t* counts, uint32_t* keys)
{
#pragma omp parallel for schedule(dynamic, 256)
    for (int g = 0; g < capacity; g++) {
        int32_t count = 0;
        if (visible[g] != 0) {
            float mx = mean[(int64_t)g * 2], my = mean[(int64_t)g * 2 + 1];
            float c00 = conic[(int64_t)g * 4], c01 = conic[(int64_t)g * 4 + 1],
                  c11 = conic[(int64_t)g * 4 + 3];
            if (count_gate(mx, my, c00, c01, c11, alpha[g], width, height))
                count = process_tiles(mx - 0.5f, my - 0.5f, c00, c01, c11, alpha[g], tile_w, tile_h,
                                      tiles_x, tiles_y, NULL);
        }
        counts[g] = count;
        keys[g] = depth_key(depth[g], count);
    }
}

/* Tiles of one Gaussian in emission order (for tests); returns the count. */
EXPORT int32_t orc_gaussian_tiles(float mx, float my, float c00, float c01, float c11, float a,
                                  int tile_w, int tile_h, int tiles_x, int tiles_y,
                                  int64_t* keys)
{
    return process_tiles(mx - 0.5f, my - 0.5f, c00, c01, c11, a, tile_w, tile_h, tiles_x,
                         tiles_y, keys);
}

typedef struct { uint32_t key; int32_t id; } KeyId;
static int cmp_keyid(const void* a, const void* b)
{
    const KeyId* x = (const KeyId*)a;
    const KeyId* y = (const KeyId*)b;
    if (x->key != y->key) return x->key < y->key ? -1 : 1;
    return (x->id > y->id) - (x->id < y->id);
}

/*
 * Whole binning pipeline, kernels/sorted_binning.py:9-117:
 * count -> stable depth sort of (key, id) (:62-64) -> inclusive scan of the
 * ordered counts (sorted_visibility.py:511-603) -> emission into the arena,
 * truncated at max_pairs (:373-484) -> stable tile sort of the first
 * min(pair_count, max_pairs) pairs (pair_sort.py:1-16) -> tile ranges
 * (sorted_visibility.py:628-659).  Outputs: point_counts[C], gaussian_ids
 * [max_pairs] (entries past the pairs are -1), tile_offsets[T+1],
 * pair_count (unclamped) and overflow (pair_count > max_pairs).
 */
EXPORT int64_t orc_bin(const float* mean, const float* conic, const float* alpha,
                       const float* depth, const int8_t* visible, int capacity, int width,
                       int height, int tile_w, int tile_h, int64_t max_pairs,
                       int32_t* point_counts, int32_t* gaussian_ids, int32_t* tile_offsets,
                       int32_t* overflow)
{
    int tiles_x = (width + tile_w - 1) / tile_w;
    int tiles_y = (height + tile_h - 1) / tile_h;
    int64_t tiles = (int64_t)tiles_x * tiles_y;
    uint32_t* keys = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(capacity > 0 ? capacity : 1));
    orc_count(mean, conic, alpha, depth, visible, capacity, tile_w, tile_h, tiles_x, tiles_y,
              width, height, point_counts, keys);
    KeyId* order = (KeyId*)malloc(sizeof(KeyId) * (size_t)(capacity > 0 ? capacity : 1));
    int64_t nvis = 0;
    for (int g = 0; g < capacity; g++)
        if (point_counts[g] > 0) { order[nvis].key = keys[g]; order[nvis].id = g; nvis++; }
    qsort(order, (size_t)nvis, sizeof(KeyId), cmp_keyid);
    int64_t total = 0;
    for (int64_t r = 0; r < nvis; r++) total += point_counts[order[r].id];
    int64_t used = total < max_pairs ? total : max_pairs;
    int64_t* pair_tile = (int64_t*)malloc(sizeof(int64_t) * (size_t)(used > 0 ? used : 1));
    int32_t* pair_id = (int32_t*)malloc(sizeof(int32_t) * (size_t)(used > 0 ? used : 1));
    int64_t* scratch = NULL;
    int64_t scratch_cap = 0;
    int64_t offset = 0;
    for (int64_t r = 0; r < nvis && offset < used; r++) {
        int32_t g = order[r].id;
        int32_t c = point_counts[g];
        if (c > scratch_cap) {
            scratch_cap = c;
            scratch = (int64_t*)realloc(scratch, sizeof(int64_t) * (size_t)scratch_cap);
        }
        int32_t emitted = process_tiles(mean[(int64_t)g * 2] - 0.5f, mean[(int64_t)g * 2 + 1] - 0.5f,
                                        conic[(int64_t)g * 4], conic[(int64_t)g * 4 + 1],
                                        conic[(int64_t)g * 4 + 3], alpha[g], tile_w, tile_h,
                                        tiles_x, tiles_y, scratch);
        for (int32_t k = 0; k < emitted && offset + k < used; k++) {
            pair_tile[offset + k] = scratch[k];
            pair_id[offset + k] = g;
        }
        offset += c;
    }
    free(scratch);
    /* Stable counting sort by tile, then ranges (== searchsorted left). */
    int64_t* hist = (int64_t*)calloc((size_t)tiles + 1, sizeof(int64_t));
    for (int64_t i = 0; i < used; i++) hist[pair_tile[i] + 1]++;
    for (int64_t t = 0; t < tiles; t++) hist[t + 1] += hist[t];
    for (int64_t t = 0; t <= tiles; t++) tile_offsets[t] = (int32_t)hist[t];
    for (int64_t i = 0; i < max_pairs; i++) gaussian_ids[i] = -1;
    for (int64_t i = 0; i < used; i++) gaussian_ids[hist[pair_tile[i]]++] = pair_id[i];
    *overflow = total > max_pairs;
    free(hist); free(pair_tile); free(pair_id); free(order); free(keys);
    return total;
}

/* ------------------------------------------------------------------------- */
/* fp32 compositing: kernels/sorted_rasterize.py:28-88 with rectangular      */
/* tile_w x tile_h tiles (the pixel arithmetic and the T >= 1/8192 early    */
/* stop are unchanged).  ambiguous[p] (optional) marks pixels where one     */
/* threshold decision lay within a relative 2e-5 of its cut, so an          */
/* implementation whose exp differs by a few ulp may legitimately differ.    */
/* ------------------------------------------------------------------------- */
/* Atomic accumulation for the pixel-parallel backward. */
#define ACC_ADD(slot, val)                 \
    do {                                   \
        double v_ = (val);                 \
        _Pragma("omp atomic") (slot) += v_; \
    } while (0)

/*
 * power = -0.5 * (dx*(c00*dx + c01*dy) + dy*(c10*dx + c11*dy))
 * (sorted_rasterize.py:67-70) in one fixed operation order: the conic is
 * scaled by -1/2 (exact), the dx products are rounded first and the dy terms
 * fused, so an implementation that shares c00*dx and c10*dx between pixels of
 * one column reproduces these bits.
 */
static inline float power_of(const float* c, float dx, float dy)
{
    float c00 = -0.5f * c[0], c01 = -0.5f * c[1], c10 = -0.5f * c[2], c11 = -0.5f * c[3];
    float t1 = fmaf(c01, dy, c00 * dx);
    float t2 = fmaf(c11, dy, c10 * dx);
    return fmaf(dy, t2, dx * t1);
}

static inline int near_cut(float value, float cut, float rel)
{
    return fabsf(value - cut) <= rel * cut;
}

EXPORT void orc_raster_fwd(int width, int height, int tile_w, int tile_h, const float* mean,
                           const float* conic, const float* depth, const float* color,
                           const float* opacity, const int32_t* ids,
                           const int32_t* tile_offsets, const float* background,
                           float* out_rgb, float* out_depth, float* out_alpha,
                           float* out_final_t, int32_t* out_last, uint8_t* ambiguous)
{
    int tiles_x = (width + tile_w - 1) / tile_w;
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t p = 0; p < (int64_t)width * height; p++) {
        int px = (int)(p % width), py = (int)(p / width);
        int tile = (py / tile_h) * tiles_x + px / tile_w;
        float r = 0.0f, gr = 0.0f, bl = 0.0f, wd = 0.0f, T = 1.0f;
        int amb = 0;
        int32_t index = tile_offsets[tile], end = tile_offsets[tile + 1];
        while (index < end && T >= 1.0f / 8192.0f) {
            int64_t g = ids[index];
            float dx = (float)px + 0.5f - mean[g * 2];
            float dy = (float)py + 0.5f - mean[g * 2 + 1];
            float exponent = power_of(conic + g * 4, dx, dy);
            if (exponent <= 0.0f) {
                float raw = opacity[g] * expf(exponent);
                if (near_cut(raw, 1.0f / 256.0f, 2e-5f)) amb = 1;
                if (raw >= 1.0f / 256.0f) {
                    float a = fminf(255.0f / 256.0f, raw);
                    float w = a * T;
                    r += w * color[g * 3];
                    gr += w * color[g * 3 + 1];
                    bl += w * color[g * 3 + 2];
                    wd += w * depth[g];
                    T *= 1.0f - a;
                    if (near_cut(T, 1.0f / 8192.0f, 2e-5f)) amb = 1;
                }
            }
            index += 1;
        }
        out_rgb[p * 3] = r + T * background[0];
        out_rgb[p * 3 + 1] = gr + T * background[1];
        out_rgb[p * 3 + 2] = bl + T * background[2];
        if (out_depth) out_depth[p] = wd;
        if (out_alpha) out_alpha[p] = 1.0f - T;
        if (out_final_t) out_final_t[p] = T;
        if (out_last) out_last[p] = index;
        if (ambiguous) ambiguous[p] = (uint8_t)amb;
    }
}

/*
 * fp32 compositing pullback: kernels/sorted_rasterize.py:91-236, per pixel
 * in reverse from last-1.  Gradients accumulate in double and are written
 * (overwriting) to gmean[C*2], gconic[C*4], gdepth[C], gcolor[C*3],
 * gopacity[C].  ddepth / dalpha may be NULL (zero).
 */
EXPORT void orc_raster_bwd(int width, int height, int tile_w, int tile_h, int capacity,
                           const float* mean, const float* conic, const float* depth,
                           const float* color, const float* opacity, const int32_t* ids,
                           const int32_t* tile_offsets, const float* background,
                           const float* final_t, const int32_t* last, const float* drgb,
                           const float* ddepth, const float* dalpha, float* gmean,
                           float* gconic, float* gdepth, float* gcolor, float* gopacity,
                           float* stats)
{
    /* stats (may be NULL): per Gaussian (fragment count, sum of compositing
     * weights, sum of squared per-pixel opacity gradients), the fragment
     * statistics of kernels/sorted_rasterize.py:155-203. */
    int tiles_x = (width + tile_w - 1) / tile_w;
    double* acc = (double*)calloc((size_t)capacity * 14, sizeof(double));
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t p = 0; p < (int64_t)width * height; p++) {
        int px = (int)(p % width), py = (int)(p / width);
        int tile = (py / tile_h) * tiles_x + px / tile_w;
        int32_t start = tile_offsets[tile];
        float g_r = drgb[p * 3], g_g = drgb[p * 3 + 1], g_b = drgb[p * 3 + 2];
        float g_d = ddepth ? ddepth[p] : 0.0f;
        float gtrans = g_r * background[0] + g_g * background[1] + g_b * background[2]
                       - (dalpha ? dalpha[p] : 0.0f);
        float T_after = final_t[p];
        for (int32_t index = last[p] - 1; index >= start; index--) {
            int64_t g = ids[index];
            float dx = (float)px + 0.5f - mean[g * 2];
            float dy = (float)py + 0.5f - mean[g * 2 + 1];
            float c00 = conic[g * 4], c01 = conic[g * 4 + 1], c10 = conic[g * 4 + 2],
                  c11 = conic[g * 4 + 3];
            float exponent = power_of(conic + g * 4, dx, dy);
            if (!(exponent <= 0.0f)) continue;
            float e = expf(exponent);
            float raw = opacity[g] * e;
            if (!(raw >= 1.0f / 256.0f)) continue;
            float a = fminf(255.0f / 256.0f, raw);
            float T_before = T_after / (1.0f - a);
            float w = T_before * a;
            float gw = g_r * color[g * 3] + g_g * color[g * 3 + 1] + g_b * color[g * 3 + 2]
                       + g_d * depth[g];
            float ga = T_before * (gw - gtrans);
            gtrans = a * gw + (1.0f - a) * gtrans;
            double* acc_g = acc + g * 14;
            ACC_ADD(acc_g[11], 1.0);
            ACC_ADD(acc_g[12], (double)w);
            ACC_ADD(acc_g[6], (double)w * g_d);
            ACC_ADD(acc_g[7], (double)w * g_r);
            ACC_ADD(acc_g[8], (double)w * g_g);
            ACC_ADD(acc_g[9], (double)w * g_b);
            if (raw < 255.0f / 256.0f) {
                float ge = ga * raw;
                ACC_ADD(acc_g[10], (double)ga * e);
                ACC_ADD(acc_g[13], (double)(ga * e) * (double)(ga * e));
                ACC_ADD(acc_g[0], (double)ge * (c00 * dx + 0.5f * (c01 + c10) * dy));
                ACC_ADD(acc_g[1], (double)ge * (c11 * dy + 0.5f * (c01 + c10) * dx));
                ACC_ADD(acc_g[2], -0.5 * ge * dx * dx);
                ACC_ADD(acc_g[3], -0.5 * ge * dx * dy);
                ACC_ADD(acc_g[4], -0.5 * ge * dy * dx);
                ACC_ADD(acc_g[5], -0.5 * ge * dy * dy);
            }
            T_after = T_before;
        }
    }
    for (int64_t g = 0; g < capacity; g++) {
        double* acc_g = acc + g * 14;
        if (stats)
            for (int k = 0; k < 3; k++) stats[g * 3 + k] = (float)acc_g[11 + k];
        gmean[g * 2] = (float)acc_g[0];
        gmean[g * 2 + 1] = (float)acc_g[1];
        for (int k = 0; k < 4; k++) gconic[g * 4 + k] = (float)acc_g[2 + k];
        gdepth[g] = (float)acc_g[6];
        for (int k = 0; k < 3; k++) gcolor[g * 3 + k] = (float)acc_g[7 + k];
        gopacity[g] = (float)acc_g[10];
    }
    free(acc);
}

/* ------------------------------------------------------------------------- */
/* Fused L1 + SSIM: reference/loss.py:6-43 (SAME zero padding, 11x11         */
/* Gaussian window, sigma 1.5) with the per-pixel gradient form of           */
/* kernels/fused_loss.py:229-288.  Evaluated in double.  target is float     */
/* in [0,1] or, when target_u8 != NULL, uint8 divided by 255 (fused_loss.py  */
/* :102-106).  Returns the mean loss; grad may be NULL.                      */
/* ------------------------------------------------------------------------- */
static void gauss_taps(double w[11])
{
    double s = 0.0;
    for (int i = 0; i < 11; i++) { double x = (i - 5) / 1.5; w[i] = exp(-0.5 * x * x); s += w[i]; }
    for (int i = 0; i < 11; i++) w[i] /= s;
}

/* Zero-padded separable blur of an H x W plane (double). */
static void blur(const double* in, double* out, double* tmp, int H, int W, const double w[11])
{
    for (int y = 0; y < H; y++)
        for (int x = 0; x < W; x++) {
            double s = 0.0;
            for (int d = -5; d <= 5; d++) {
                int xx = x + d;
                if (xx >= 0 && xx < W) s += in[(int64_t)y * W + xx] * w[d + 5];
            }
            tmp[(int64_t)y * W + x] = s;
        }
    for (int y = 0; y < H; y++)
        for (int x = 0; x < W; x++) {
            double s = 0.0;
            for (int d = -5; d <= 5; d++) {
                int yy = y + d;
                if (yy >= 0 && yy < H) s += tmp[(int64_t)yy * W + x] * w[d + 5];
            }
            out[(int64_t)y * W + x] = s;
        }
}

EXPORT double orc_loss(int H, int W, const float* image, const float* target_f,
                       const uint8_t* target_u8, float* grad)
{
    double w[11];
    gauss_taps(w);
    int64_t n = (int64_t)H * W;
    double total = 0.0;
    double N = 3.0 * (double)n;
    double* buf = (double*)malloc(sizeof(double) * (size_t)n * 12);
    double *x = buf, *y = buf + n, *mx = buf + 2 * n, *my = buf + 3 * n, *xx = buf + 4 * n,
           *yy = buf + 5 * n, *xy = buf + 6 * n, *tmp = buf + 7 * n, *p0 = buf + 8 * n,
           *p1 = buf + 9 * n, *p2 = buf + 10 * n, *q = buf + 11 * n;
    for (int c = 0; c < 3; c++) {
        for (int64_t i = 0; i < n; i++) {
            x[i] = image[i * 3 + c];
            y[i] = target_u8 ? (double)((float)target_u8[i * 3 + c] * (float)(1.0 / 255))
                             : (double)target_f[i * 3 + c];
        }
        blur(x, mx, tmp, H, W, w);
        blur(y, my, tmp, H, W, w);
        for (int64_t i = 0; i < n; i++) q[i] = x[i] * x[i];
        blur(q, xx, tmp, H, W, w);
        for (int64_t i = 0; i < n; i++) q[i] = y[i] * y[i];
        blur(q, yy, tmp, H, W, w);
        for (int64_t i = 0; i < n; i++) q[i] = x[i] * y[i];
        blur(q, xy, tmp, H, W, w);
        double weight = -0.2 / N;
        for (int64_t i = 0; i < n; i++) {
            double a = mx[i] * mx[i] + my[i] * my[i] + 1e-4;
            double b = (xx[i] - mx[i] * mx[i]) + (yy[i] - my[i] * my[i]) + 9e-4;
            double cc = 2.0 * mx[i] * my[i] + 1e-4;
            double dd = 2.0 * (xy[i] - mx[i] * my[i]) + 9e-4;
            double ssim = cc * dd / (a * b);
            total += 0.2 * (1.0 - ssim) + 0.8 * fabs(x[i] - y[i]);
            p0[i] = (2.0 * my[i] * (dd - cc) / (a * b) + 2.0 * mx[i] * ssim * (1.0 / b - 1.0 / a)) * weight;
            p1[i] = -ssim / b * weight;
            p2[i] = 2.0 * cc / (a * b) * weight;
        }
        if (grad) {
            blur(p0, mx, tmp, H, W, w);
            blur(p1, my, tmp, H, W, w);
            blur(p2, xx, tmp, H, W, w);
            for (int64_t i = 0; i < n; i++) {
                double s = (x[i] > y[i]) ? 1.0 : (x[i] < y[i] ? -1.0 : 0.0);
                grad[i * 3 + c] = (float)(mx[i] + 2.0 * x[i] * my[i] + y[i] * xx[i] + 0.8 * s / N);
            }
        }
    }
    free(buf);
    return total / N;
}

/* ------------------------------------------------------------------------- */
/* Cluster frustum mask and compaction: scene/cluster.py:40-67 and           */
/* kernels/cluster_compact.py:31-44.  planes[24] are the six (a,b,c,d)       */
/* planes computed on the host.  Returns the visible-cluster count; ids      */
/* receives them in ascending order.                                         */
/* ------------------------------------------------------------------------- */
EXPORT int orc_cluster_compact(int num_clusters, const float* center, const float* extent,
                               const uint8_t* valid, const float* planes, int32_t* ids,
                               uint8_t* cluster_visible)
{
    int count = 0;
    for (int c = 0; c < num_clusters; c++) {
        int vis = valid[c] != 0;
        for (int k = 0; k < 6 && vis; k++) {
            const float* pl = planes + k * 4;
            float dist = center[c * 3] * pl[0] + center[c * 3 + 1] * pl[1] + center[c * 3 + 2] * pl[2] + pl[3];
            float rad = extent[c * 3] * fabsf(pl[0]) + extent[c * 3 + 1] * fabsf(pl[1])
                        + extent[c * 3 + 2] * fabsf(pl[2]);
            if (!(dist + rad >= 0.0f)) vis = 0;
        }
        cluster_visible[c] = (uint8_t)vis;
        if (vis) ids[count++] = c;
    }
    return count;
}

EXPORT int orc_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Threads of the parallel loops from here on (n >= 1; ignored without
 * OpenMP).  A launcher may have set OMP_NUM_THREADS=1 for every rank; the
 * one rank that runs the oracle takes the host's threads back with this. */
EXPORT void orc_set_num_threads(int n)
{
#ifdef _OPENMP
    if (n >= 1) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
