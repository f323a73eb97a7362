// Projection forward / pullback and visible-cluster compaction (sm_100a).
//
// One thread per compact index (128 per block).  The compact index i maps to
// pool slot cluster_ids[i / cluster_size] * cluster_size + i % cluster_size
// (kernels/projection.py:42-47), so a 128-slot cluster is one contiguous run
// of 128 Gaussians.  The SH block (the bulk of the 236 B/Gaussian that the
// pass reads) is staged through shared memory with coalesced 16-byte loads
// and read back per thread; all other fields are per-thread loads whose warps
// cover contiguous runs.  HBM-bound: 286 B/Gaussian forward, 524 B/Gaussian
// backward.
#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr int kProjThreads = 128;
constexpr float kC0 = 0.28209479177387814f;
constexpr float kC1 = 0.4886025119029199f;

struct Cam {
    float v[12];
    float fx, fy, cx, cy;
    float c[3];
};

__device__ __forceinline__ void load_cam(Cam& cam, const float* view, const float* intr,
                                         const float* center)
{
#pragma unroll
    for (int k = 0; k < 12; k++) cam.v[k] = __ldg(view + k);
    cam.fx = __ldg(intr);
    cam.fy = __ldg(intr + 1);
    cam.cx = __ldg(intr + 2);
    cam.cy = __ldg(intr + 3);
    cam.c[0] = __ldg(center);
    cam.c[1] = __ldg(center + 1);
    cam.c[2] = __ldg(center + 2);
}

// Slot of compact index i, or -1 (kernels/projection.py:40-47).
__device__ __forceinline__ int64_t slot_of(int64_t i, int capacity, const int32_t* ids,
                                           int count, int cluster_size, bool compacted)
{
    if (!compacted) return i < capacity ? i : -1;
    if (i >= (int64_t)count * cluster_size) return -1;
    int64_t s = (int64_t)__ldg(ids + i / cluster_size) * cluster_size + i % cluster_size;
    return s < capacity ? s : -1;
}

// Stage the SH prefix of the block's Gaussians: floats [0, width) of each
// point's row, width a multiple of 4, into sh_s[point * (width + 4) + k]
// (padding keeps 16-byte alignment and spreads banks).
__device__ __forceinline__ void stage_sh(float* sh_s, const float* sh, int sh_row, int width,
                                         const int64_t* slots)
{
    int vec = width / 4;
    int stride = width + 4;
    for (int k = threadIdx.x; k < kProjThreads * vec; k += kProjThreads) {
        int point = k / vec, part = k % vec;
        int64_t s = slots[point];
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s >= 0) {
            const float* src = sh + s * sh_row + part * 4;
            if ((sh_row & 3) == 0) {
                val = __ldg(reinterpret_cast<const float4*>(src));
            } else {
                int valid = min(4, sh_row - part * 4);
                float t[4] = {0.f, 0.f, 0.f, 0.f};
                for (int q = 0; q < valid; q++) t[q] = __ldg(src + q);
                val = make_float4(t[0], t[1], t[2], t[3]);
            }
        }
        *reinterpret_cast<float4*>(sh_s + point * stride + part * 4) = val;
    }
}

// SH colour, kernels/projection.py:142-171 (reference/sh.py:8-36).
__device__ __forceinline__ float sh_channel(const float* c, int ch, int degree, float dx,
                                            float dy, float dz, float xx, float yy, float zz)
{
    float value = kC0 * c[ch];
    if (degree >= 1)
        value += (-kC1 * dy * c[ch + 3] + kC1 * dz * c[ch + 6] - kC1 * dx * c[ch + 9]);
    if (degree >= 2)
        value += (1.0925484305920792f * dx * dy * c[ch + 12] - 1.0925484305920792f * dy * dz * c[ch + 15]
                  + 0.31539156525252005f * (2.0f * zz - xx - yy) * c[ch + 18]
                  - 1.0925484305920792f * dx * dz * c[ch + 21]
                  + 0.5462742152960396f * (xx - yy) * c[ch + 24]);
    if (degree >= 3)
        value += (-0.5900435899266435f * dy * (3.0f * xx - yy) * c[ch + 27]
                  + 2.890611442640554f * dx * dy * dz * c[ch + 30]
                  - 0.4570457994644658f * dy * (4.0f * zz - xx - yy) * c[ch + 33]
                  + 0.3731763325901154f * dz * (2.0f * zz - 3.0f * xx - 3.0f * yy) * c[ch + 36]
                  - 0.4570457994644658f * dx * (4.0f * zz - xx - yy) * c[ch + 39]
                  + 1.445305721320277f * dz * (xx - yy) * c[ch + 42]
                  - 0.5900435899266435f * dx * (xx - 3.0f * yy) * c[ch + 45]);
    return fmaxf(value + 0.5f, 0.0f);
}

struct Geometry {
    float x, y, z, safe_z;
    float qw, qx, qy, qz, qdenom;
    float s0, s1, s2;
    float m[9];
    float j0, j1, j2, j3;
    float a0, a1, a2, b0, b1, b2;
    float a, b, d;
};

// Shared forward geometry of kernels/projection.py:48-98 (and the same
// recomputation in projection_backward.py:82-139).
__device__ __forceinline__ void geometry(Geometry& g, const Cam& cam, float wx, float wy, float wz,
                                         float4 q, float ls0, float ls1, float ls2, float near)
{
    const float* v = cam.v;
    g.x = v[0] * wx + v[1] * wy + v[2] * wz + v[3];
    g.y = v[4] * wx + v[5] * wy + v[6] * wz + v[7];
    g.z = v[8] * wx + v[9] * wy + v[10] * wz + v[11];
    g.safe_z = fmaxf(g.z, near);
    g.qdenom = sqrtf(fmaxf(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w, 1e-16f));
    float inv = 1.0f / g.qdenom;
    g.qw = q.x * inv;
    g.qx = q.y * inv;
    g.qy = q.z * inv;
    g.qz = q.w * inv;
    float qw = g.qw, qx = g.qx, qy = g.qy, qz = g.qz;
    float r00 = 1.0f - 2.0f * (qy * qy + qz * qz), r01 = 2.0f * (qx * qy - qw * qz),
          r02 = 2.0f * (qx * qz + qw * qy);
    float r10 = 2.0f * (qx * qy + qw * qz), r11 = 1.0f - 2.0f * (qx * qx + qz * qz),
          r12 = 2.0f * (qy * qz - qw * qx);
    float r20 = 2.0f * (qx * qz - qw * qy), r21 = 2.0f * (qy * qz + qw * qx),
          r22 = 1.0f - 2.0f * (qx * qx + qy * qy);
    g.s0 = expf(ls0);
    g.s1 = expf(ls1);
    g.s2 = expf(ls2);
    g.m[0] = (v[0] * r00 + v[1] * r10 + v[2] * r20) * g.s0;
    g.m[1] = (v[0] * r01 + v[1] * r11 + v[2] * r21) * g.s1;
    g.m[2] = (v[0] * r02 + v[1] * r12 + v[2] * r22) * g.s2;
    g.m[3] = (v[4] * r00 + v[5] * r10 + v[6] * r20) * g.s0;
    g.m[4] = (v[4] * r01 + v[5] * r11 + v[6] * r21) * g.s1;
    g.m[5] = (v[4] * r02 + v[5] * r12 + v[6] * r22) * g.s2;
    g.m[6] = (v[8] * r00 + v[9] * r10 + v[10] * r20) * g.s0;
    g.m[7] = (v[8] * r01 + v[9] * r11 + v[10] * r21) * g.s1;
    g.m[8] = (v[8] * r02 + v[9] * r12 + v[10] * r22) * g.s2;
    float inv_z = 1.0f / g.safe_z;
    g.j0 = cam.fx * inv_z;
    g.j1 = cam.fy * inv_z;
    g.j2 = cam.fx * g.x * inv_z * inv_z;
    g.j3 = cam.fy * g.y * inv_z * inv_z;
    g.a0 = g.j0 * g.m[0] - g.j2 * g.m[6];
    g.a1 = g.j0 * g.m[1] - g.j2 * g.m[7];
    g.a2 = g.j0 * g.m[2] - g.j2 * g.m[8];
    g.b0 = g.j1 * g.m[3] - g.j3 * g.m[6];
    g.b1 = g.j1 * g.m[4] - g.j3 * g.m[7];
    g.b2 = g.j1 * g.m[5] - g.j3 * g.m[8];
    g.a = g.a0 * g.a0 + g.a1 * g.a1 + g.a2 * g.a2 + 0.3f;
    g.b = g.a0 * g.b0 + g.a1 * g.b1 + g.a2 * g.b2;
    g.d = g.b0 * g.b0 + g.b1 * g.b1 + g.b2 * g.b2 + 0.3f;
}

__global__ void __launch_bounds__(kProjThreads) project_fwd_kernel(
    gsb_project_params p, const float* __restrict__ xyz, const float* __restrict__ log_scale,
    const float* __restrict__ rotation, const float* __restrict__ opacity,
    const float* __restrict__ sh, const uint8_t* __restrict__ alive, const float* view,
    const float* intr, const float* center, const int32_t* __restrict__ cluster_ids,
    const int32_t* __restrict__ cluster_count, float* __restrict__ out_mean,
    float* __restrict__ out_depth, float* __restrict__ out_conic, float* __restrict__ out_radius,
    float* __restrict__ out_color, float* __restrict__ out_alpha, int8_t* __restrict__ out_visible)
{
    extern __shared__ float4 smem4[];
    float* sh_s = reinterpret_cast<float*>(smem4);
    __shared__ int64_t slots[kProjThreads];
    int count = p.compacted ? __ldg(cluster_count) : 0;
    int64_t first = (int64_t)blockIdx.x * kProjThreads;
    if (p.compacted && first >= (int64_t)count * p.cluster_size) return;  // uniform per block
    int64_t i = first + threadIdx.x;
    int64_t g = slot_of(i, p.capacity, cluster_ids, count, p.cluster_size, p.compacted);
    slots[threadIdx.x] = g;
    __syncthreads();
    int used = (p.degree + 1) * (p.degree + 1) * 3;
    int width = (used + 3) & ~3;
    if (width > p.sh_dim * 3) width = (p.sh_dim * 3 + 3) & ~3;
    stage_sh(sh_s, sh, p.sh_dim * 3, width, slots);
    __syncthreads();
    if (g < 0) return;

    Cam cam;
    load_cam(cam, view, intr, center);
    float wx = xyz[g * 3], wy = xyz[g * 3 + 1], wz = xyz[g * 3 + 2];
    float4 q = *reinterpret_cast<const float4*>(rotation + g * 4);
    Geometry geo;
    geometry(geo, cam, wx, wy, wz, q, log_scale[g * 3], log_scale[g * 3 + 1],
             log_scale[g * 3 + 2], p.near_plane);
    float u = cam.fx * geo.x / geo.safe_z + cam.cx;
    float v = cam.fy * geo.y / geo.safe_z + cam.cy;
    *reinterpret_cast<float2*>(out_mean + g * 2) = make_float2(u, v);
    out_depth[g] = geo.z;
    float a = geo.a, b = geo.b, d = geo.d;
    float det = fmaxf(a * d - b * b, 1e-8f);
    float nb = -b / det;
    *reinterpret_cast<float4*>(out_conic + g * 4) = make_float4(d / det, nb, nb, a / det);
    out_radius[g] = 3.0f * sqrtf(0.5f * (a + d + sqrtf(fmaxf((a - d) * (a - d) + 4.0f * b * b, 1e-12f))));
    float alpha = 1.0f / (1.0f + expf(-opacity[g]));
    out_alpha[g] = alpha;
    float W = (float)p.width, H = (float)p.height;
    bool vis = alive[g] != 0 && geo.z > p.near_plane && geo.z < p.far_plane &&
               alpha >= (float)(1.0 / 255) && u >= -0.15f * W && u <= 1.15f * W &&
               v >= -0.15f * H && v <= 1.15f * H;
    out_visible[g] = vis ? 1 : 0;
    float r = 0.0f, gr = 0.0f, bl = 0.0f;
    if (!p.visible_color_only || vis) {
        float dx = wx - cam.c[0], dy = wy - cam.c[1], dz = wz - cam.c[2];
        float dn = rsqrtf(fmaxf(dx * dx + dy * dy + dz * dz, 1e-16f));
        dx *= dn;
        dy *= dn;
        dz *= dn;
        const float* c = sh_s + threadIdx.x * (width + 4);
        float xx = dx * dx, yy = dy * dy, zz = dz * dz;
        r = sh_channel(c, 0, p.degree, dx, dy, dz, xx, yy, zz);
        gr = sh_channel(c, 1, p.degree, dx, dy, dz, xx, yy, zz);
        bl = sh_channel(c, 2, p.degree, dx, dy, dz, xx, yy, zz);
    }
    out_color[g * 3] = r;
    out_color[g * 3 + 1] = gr;
    out_color[g * 3 + 2] = bl;
}

// kernels/projection.py:178-201 (_clear_projected) / :204-210 (_clear_visible).
__global__ void clear_projected_kernel(int64_t capacity, int clear_all, float* mean, float* depth,
                                       float* conic, float* radius, float* color, float* alpha,
                                       int8_t* visible)
{
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= capacity) return;
    visible[i] = 0;
    if (!clear_all) return;
    *reinterpret_cast<float2*>(mean + i * 2) = make_float2(0.f, 0.f);
    *reinterpret_cast<float4*>(conic + i * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
    color[i * 3] = color[i * 3 + 1] = color[i * 3 + 2] = 0.0f;
    depth[i] = __int_as_float(0x7f800000);
    radius[i] = 0.0f;
    alpha[i] = 0.0f;
}

// ---------------------------------------------------------------------------
// Pullback: kernels/projection_backward.py:42-367.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kProjThreads) project_bwd_kernel(
    gsb_project_bwd_params p, const float* __restrict__ xyz, const float* __restrict__ log_scale,
    const float* __restrict__ rotation, const float* __restrict__ opacity,
    const float* __restrict__ sh, const float* view, const float* intr, const float* center,
    const float* __restrict__ color, const int32_t* __restrict__ cluster_ids,
    const int32_t* __restrict__ cluster_count, const float* __restrict__ gmean,
    const float* __restrict__ gdepth, const float* __restrict__ gconic,
    const float* __restrict__ gradius, const float* __restrict__ gcolor,
    const float* __restrict__ galpha, float* __restrict__ out_xyz,
    float* __restrict__ out_log_scale, float* __restrict__ out_rotation,
    float* __restrict__ out_opacity, float* __restrict__ out_sh)
{
    extern __shared__ float4 smem4[];
    __shared__ int64_t slots[kProjThreads];
    int count = p.compacted ? __ldg(cluster_count) : 0;
    int64_t first = (int64_t)blockIdx.x * kProjThreads;
    if (p.compacted && first >= (int64_t)count * p.cluster_size) return;  // uniform per block
    int64_t i = first + threadIdx.x;
    int64_t g = slot_of(i, p.capacity, cluster_ids, count, p.cluster_size, p.compacted);
    slots[threadIdx.x] = g;
    __syncthreads();
    const int used = (p.degree + 1) * (p.degree + 1) * 3;
    int width = (used + 3) & ~3;
    if (width > p.sh_dim * 3) width = (p.sh_dim * 3 + 3) & ~3;
    const int shg = p.sh_gradient_dim * 3;
    const int gstride = shg + 1;
    float* sh_s = reinterpret_cast<float*>(smem4);                 // staged coefficients
    float* gsh_s = sh_s + kProjThreads * (width + 4);               // transposed gradients
    stage_sh(sh_s, sh, p.sh_dim * 3, width, slots);
    __syncthreads();
    int64_t o = p.compact_gradients ? i : g;
    float* my_gsh = gsh_s + threadIdx.x * gstride;
    for (int k = 0; k < shg; k++) my_gsh[k] = 0.0f;

    bool has = false;
    if (g >= 0) {
        has = galpha[g] != 0.0f;
        if (!p.rgb_only) has = has || gdepth[g] != 0.0f || gradius[g] != 0.0f;
        float2 gm = *reinterpret_cast<const float2*>(gmean + g * 2);
        float4 gc = *reinterpret_cast<const float4*>(gconic + g * 4);
        has = has || gm.x != 0.0f || gm.y != 0.0f || gc.x != 0.0f || gc.y != 0.0f ||
              gc.z != 0.0f || gc.w != 0.0f || gcolor[g * 3] != 0.0f ||
              gcolor[g * 3 + 1] != 0.0f || gcolor[g * 3 + 2] != 0.0f;
        if (!has) {
            for (int k = 0; k < 3; k++) out_xyz[o * 3 + k] = out_log_scale[o * 3 + k] = 0.0f;
            *reinterpret_cast<float4*>(out_rotation + o * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
            out_opacity[o] = 0.0f;
        }
    }
    if (has) {
        Cam cam;
        load_cam(cam, view, intr, center);
        float wx = xyz[g * 3], wy = xyz[g * 3 + 1], wz = xyz[g * 3 + 2];
        float4 q = *reinterpret_cast<const float4*>(rotation + g * 4);
        Geometry geo;
        geometry(geo, cam, wx, wy, wz, q, log_scale[g * 3], log_scale[g * 3 + 1],
                 log_scale[g * 3 + 2], p.near_plane);
        const float* v = cam.v;
        float fx = cam.fx, fy = cam.fy;
        float inv_z = 1.0f / geo.safe_z, inv_z2 = inv_z * inv_z;
        float x = geo.x, y = geo.y;
        float gmx = gmean[g * 2], gmy = gmean[g * 2 + 1];
        float gx = gmx * fx * inv_z;
        float gy = gmy * fy * inv_z;
        float gz = p.rgb_only ? 0.0f : gdepth[g];
        float gsafe_z = -gmx * fx * x * inv_z2;
        gsafe_z -= gmy * fy * y * inv_z2;
        float a = geo.a, b = geo.b, d = geo.d;
        float raw_det = a * d - b * b;
        float det = fmaxf(raw_det, 1e-8f);
        float4 gcn = *reinterpret_cast<const float4*>(gconic + g * 4);
        float gdet = 0.0f;
        if (raw_det > 1e-8f) gdet = -(gcn.x * d - (gcn.y + gcn.z) * b + gcn.w * a) / (det * det);
        float ga = gcn.w / det + gdet * d;
        float gb = -(gcn.y + gcn.z) / det - 2.0f * b * gdet;
        float gd = gcn.x / det + gdet * a;
        if (!p.rgb_only) {
            float disc = (a - d) * (a - d) + 4.0f * b * b;
            float disc_root = sqrtf(fmaxf(disc, 1e-12f));
            float eigen = 0.5f * (a + d + disc_root);
            float geigen = gradius[g] * 1.5f / sqrtf(eigen);
            float gdisc = disc > 1e-12f ? geigen * 0.25f / disc_root : 0.0f;
            ga += 0.5f * geigen + 2.0f * (a - d) * gdisc;
            gb += 8.0f * b * gdisc;
            gd += 0.5f * geigen - 2.0f * (a - d) * gdisc;
        }
        const float* m = geo.m;
        float ga0 = 2 * geo.a0 * ga + geo.b0 * gb, ga1 = 2 * geo.a1 * ga + geo.b1 * gb,
              ga2 = 2 * geo.a2 * ga + geo.b2 * gb;
        float gb0 = 2 * geo.b0 * gd + geo.a0 * gb, gb1 = 2 * geo.b1 * gd + geo.a1 * gb,
              gb2 = 2 * geo.b2 * gd + geo.a2 * gb;
        float gj0 = ga0 * m[0] + ga1 * m[1] + ga2 * m[2];
        float gj1 = gb0 * m[3] + gb1 * m[4] + gb2 * m[5];
        float gj2 = -(ga0 * m[6] + ga1 * m[7] + ga2 * m[8]);
        float gj3 = -(gb0 * m[6] + gb1 * m[7] + gb2 * m[8]);
        gx += gj2 * fx * inv_z2;
        gy += gj3 * fy * inv_z2;
        gsafe_z -= (gj0 * fx + gj1 * fy) * inv_z2;
        gsafe_z -= 2.0f * (gj2 * fx * x + gj3 * fy * y) * inv_z2 * inv_z;
        if (geo.z > p.near_plane) gz += gsafe_z;
        float j0 = geo.j0, j1 = geo.j1, j2 = geo.j2, j3 = geo.j3;
        float gm00 = j0 * ga0, gm01 = j0 * ga1, gm02 = j0 * ga2;
        float gm10 = j1 * gb0, gm11 = j1 * gb1, gm12 = j1 * gb2;
        float gm20 = -j2 * ga0 - j3 * gb0, gm21 = -j2 * ga1 - j3 * gb1, gm22 = -j2 * ga2 - j3 * gb2;
        out_log_scale[o * 3] = gm00 * m[0] + gm10 * m[3] + gm20 * m[6];
        out_log_scale[o * 3 + 1] = gm01 * m[1] + gm11 * m[4] + gm21 * m[7];
        out_log_scale[o * 3 + 2] = gm02 * m[2] + gm12 * m[5] + gm22 * m[8];
        float s0 = geo.s0, s1 = geo.s1, s2 = geo.s2;
        float gr00 = s0 * (v[0] * gm00 + v[4] * gm10 + v[8] * gm20);
        float gr10 = s0 * (v[1] * gm00 + v[5] * gm10 + v[9] * gm20);
        float gr20 = s0 * (v[2] * gm00 + v[6] * gm10 + v[10] * gm20);
        float gr01 = s1 * (v[0] * gm01 + v[4] * gm11 + v[8] * gm21);
        float gr11 = s1 * (v[1] * gm01 + v[5] * gm11 + v[9] * gm21);
        float gr21 = s1 * (v[2] * gm01 + v[6] * gm11 + v[10] * gm21);
        float gr02 = s2 * (v[0] * gm02 + v[4] * gm12 + v[8] * gm22);
        float gr12 = s2 * (v[1] * gm02 + v[5] * gm12 + v[9] * gm22);
        float gr22 = s2 * (v[2] * gm02 + v[6] * gm12 + v[10] * gm22);
        float qw = geo.qw, qx = geo.qx, qy = geo.qy, qz = geo.qz;
        float gqw = -2 * qz * gr01 + 2 * qy * gr02 + 2 * qz * gr10 - 2 * qx * gr12 - 2 * qy * gr20 + 2 * qx * gr21;
        float gqx = 2 * qy * (gr01 + gr10) + 2 * qz * (gr02 + gr20) - 4 * qx * (gr11 + gr22) - 2 * qw * gr12 + 2 * qw * gr21;
        float gqy = -4 * qy * (gr00 + gr22) + 2 * qx * (gr01 + gr10) + 2 * qw * gr02 + 2 * qz * (gr12 + gr21) - 2 * qw * gr20;
        float gqz = -4 * qz * (gr00 + gr11) - 2 * qw * gr01 + 2 * qx * (gr02 + gr20) + 2 * qw * gr10 + 2 * qy * (gr12 + gr21);
        float qdenom = geo.qdenom;
        float qdot = gqw * qw + gqx * qx + gqy * qy + gqz * qz;
        if (qdenom > 1e-8f) {
            gqw = (gqw - qdot * qw) / qdenom;
            gqx = (gqx - qdot * qx) / qdenom;
            gqy = (gqy - qdot * qy) / qdenom;
            gqz = (gqz - qdot * qz) / qdenom;
        } else {
            gqw /= qdenom;
            gqx /= qdenom;
            gqy /= qdenom;
            gqz /= qdenom;
        }
        *reinterpret_cast<float4*>(out_rotation + o * 4) = make_float4(gqw, gqx, gqy, gqz);
        float alpha = 1.0f / (1.0f + expf(-opacity[g]));
        out_opacity[o] = galpha[g] * alpha * (1.0f - alpha);

        float vx = wx - cam.c[0], vy = wy - cam.c[1], vz = wz - cam.c[2];
        float dir_denom = sqrtf(fmaxf(vx * vx + vy * vy + vz * vz, 1e-16f));
        float dx = vx / dir_denom, dy = vy / dir_denom, dz = vz / dir_denom;
        float xx = dx * dx, yy = dy * dy, zz = dz * dz;
        float gdx = 0.0f, gdy = 0.0f, gdz = 0.0f;
        const float* c = sh_s + threadIdx.x * (width + 4);
        const int degree = p.degree;
        for (int ch = 0; ch < 3; ch++) {
            float gc = color[g * 3 + ch] > 0.0f ? gcolor[g * 3 + ch] : 0.0f;
            if (p.sh_color_only) {
                my_gsh[ch] = gc;
            } else {
                my_gsh[ch] = gc * kC0;
            }
            if (degree >= 1) {
                if (!p.sh_color_only) {
                    my_gsh[3 + ch] = -gc * kC1 * dy;
                    my_gsh[6 + ch] = gc * kC1 * dz;
                    my_gsh[9 + ch] = -gc * kC1 * dx;
                }
                gdx -= gc * kC1 * c[ch + 9];
                gdy -= gc * kC1 * c[ch + 3];
                gdz += gc * kC1 * c[ch + 6];
            }
            if (degree >= 2) {
                if (!p.sh_color_only) {
                    my_gsh[12 + ch] = gc * 1.0925484305920792f * dx * dy;
                    my_gsh[15 + ch] = -gc * 1.0925484305920792f * dy * dz;
                    my_gsh[18 + ch] = gc * 0.31539156525252005f * (2 * zz - xx - yy);
                    my_gsh[21 + ch] = -gc * 1.0925484305920792f * dx * dz;
                    my_gsh[24 + ch] = gc * 0.5462742152960396f * (xx - yy);
                }
                gdx += gc * (1.0925484305920792f * dy * c[ch + 12] - 0.6307831305050401f * dx * c[ch + 18] -
                             1.0925484305920792f * dz * c[ch + 21] + 1.0925484305920792f * dx * c[ch + 24]);
                gdy += gc * (1.0925484305920792f * dx * c[ch + 12] - 1.0925484305920792f * dz * c[ch + 15] -
                             0.6307831305050401f * dy * c[ch + 18] - 1.0925484305920792f * dy * c[ch + 24]);
                gdz += gc * (-1.0925484305920792f * dy * c[ch + 15] + 1.2615662610100802f * dz * c[ch + 18] -
                             1.0925484305920792f * dx * c[ch + 21]);
            }
            if (degree >= 3) {
                if (!p.sh_color_only) {
                    my_gsh[27 + ch] = -gc * 0.5900435899266435f * dy * (3 * xx - yy);
                    my_gsh[30 + ch] = gc * 2.890611442640554f * dx * dy * dz;
                    my_gsh[33 + ch] = -gc * 0.4570457994644658f * dy * (4 * zz - xx - yy);
                    my_gsh[36 + ch] = gc * 0.3731763325901154f * dz * (2 * zz - 3 * xx - 3 * yy);
                    my_gsh[39 + ch] = -gc * 0.4570457994644658f * dx * (4 * zz - xx - yy);
                    my_gsh[42 + ch] = gc * 1.445305721320277f * dz * (xx - yy);
                    my_gsh[45 + ch] = -gc * 0.5900435899266435f * dx * (xx - 3 * yy);
                }
                gdx += gc * (-3.540261539559861f * dx * dy * c[ch + 27] + 2.890611442640554f * dy * dz * c[ch + 30] +
                             0.9140915989289316f * dx * dy * c[ch + 33] - 2.2390579955406924f * dx * dz * c[ch + 36] -
                             0.4570457994644658f * (4 * zz - 3 * xx - yy) * c[ch + 39] +
                             2.890611442640554f * dx * dz * c[ch + 42] - 1.7701307697799305f * (xx - yy) * c[ch + 45]);
                gdy += gc * (-1.7701307697799305f * (xx - yy) * c[ch + 27] + 2.890611442640554f * dx * dz * c[ch + 30] -
                             0.4570457994644658f * (4 * zz - xx - 3 * yy) * c[ch + 33] -
                             2.2390579955406924f * dy * dz * c[ch + 36] + 0.9140915989289316f * dx * dy * c[ch + 39] -
                             2.890611442640554f * dy * dz * c[ch + 42] + 3.540261539559861f * dx * dy * c[ch + 45]);
                gdz += gc * (2.890611442640554f * dx * dy * c[ch + 30] - 3.6563663957157264f * dy * dz * c[ch + 33] +
                             0.3731763325901154f * (6 * zz - 3 * xx - 3 * yy) * c[ch + 36] -
                             3.6563663957157264f * dx * dz * c[ch + 39] + 1.445305721320277f * (xx - yy) * c[ch + 42]);
            }
        }
        float dir_dot = gdx * dx + gdy * dy + gdz * dz;
        float gxw = gdx / dir_denom, gyw = gdy / dir_denom, gzw = gdz / dir_denom;
        if (dir_denom > 1e-8f) {
            gxw = (gdx - dir_dot * dx) / dir_denom;
            gyw = (gdy - dir_dot * dy) / dir_denom;
            gzw = (gdz - dir_dot * dz) / dir_denom;
        }
        out_xyz[o * 3] = v[0] * gx + v[4] * gy + v[8] * gz + gxw;
        out_xyz[o * 3 + 1] = v[1] * gx + v[5] * gy + v[9] * gz + gyw;
        out_xyz[o * 3 + 2] = v[2] * gx + v[6] * gy + v[10] * gz + gzw;
    }
    // Coalesced write of the transposed SH gradients (projection_backward.py:342-367).
    __syncthreads();
    for (int k = threadIdx.x; k < kProjThreads * shg; k += kProjThreads) {
        int point = k / shg, coef = k % shg;
        int64_t slot = slots[point];
        if (slot < 0) continue;
        int64_t out_point = p.compact_gradients ? first + point : slot;
        out_sh[out_point * shg + coef] = gsh_s[point * gstride + coef];
    }
}

// kernels/projection_backward.py:370-390 (_clear_parameter_grads).
__global__ void clear_grads_kernel(int64_t capacity, int shg, float* gxyz, float* gscale,
                                   float* grot, float* gop, float* gsh)
{
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < capacity * shg) gsh[i] = 0.0f;
    if (i < capacity * 4) grot[i] = 0.0f;
    if (i < capacity * 3) gxyz[i] = gscale[i] = 0.0f;
    if (i < capacity) gop[i] = 0.0f;
}

// ---------------------------------------------------------------------------
// Cluster frustum test + stable compaction (scene/cluster.py:40-67,
// kernels/cluster_compact.py:31-44).  One block of 1024 threads handles up to
// 1024 clusters per chunk with a block scan, so the ids come out in ascending
// order without atomics.
// ---------------------------------------------------------------------------
constexpr int kClusterThreads = 1024;

__global__ void __launch_bounds__(kClusterThreads) cluster_compact_kernel(
    int num_clusters, const float* __restrict__ center, const float* __restrict__ extent,
    const uint8_t* __restrict__ valid, const float* __restrict__ planes, int32_t* ids,
    int32_t* count_out, uint8_t* cluster_vis)
{
    __shared__ float pl[24];
    __shared__ int warp_totals[32];
    __shared__ int running;
    if (threadIdx.x < 24) pl[threadIdx.x] = planes[threadIdx.x];
    if (threadIdx.x == 0) running = 0;
    __syncthreads();
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int base = 0; base < num_clusters; base += kClusterThreads) {
        int c = base + threadIdx.x;
        int vis = 0;
        if (c < num_clusters) {
            vis = valid[c] != 0;
            float cx = center[c * 3], cy = center[c * 3 + 1], cz = center[c * 3 + 2];
            float ex = extent[c * 3], ey = extent[c * 3 + 1], ez = extent[c * 3 + 2];
            for (int k = 0; k < 6 && vis; k++) {
                const float* q = pl + k * 4;
                float dist = cx * q[0] + cy * q[1] + cz * q[2] + q[3];
                float rad = ex * fabsf(q[0]) + ey * fabsf(q[1]) + ez * fabsf(q[2]);
                if (!(dist + rad >= 0.0f)) vis = 0;
            }
            cluster_vis[c] = (uint8_t)vis;
        }
        unsigned ballot = __ballot_sync(GSB_FULL_MASK, vis);
        if (lane == 0) warp_totals[warp] = __popc(ballot);
        __syncthreads();
        if (warp == 0) {
            int t = warp_totals[lane];
            int inc = warp_inclusive_scan(t, lane);
            warp_totals[lane] = inc - t;
        }
        __syncthreads();
        int pos = running + warp_totals[warp] + __popc(ballot & lanemask_lt());
        if (vis) ids[pos] = c;
        __syncthreads();
        if (threadIdx.x == kClusterThreads - 1) running = pos + vis;
        __syncthreads();
    }
    if (threadIdx.x == 0) *count_out = running;
}

__global__ void expand_slots_kernel(int64_t capacity, int cluster_size, const uint8_t* cluster_vis,
                                    uint8_t* slots)
{
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < capacity) slots[i] = cluster_vis[i / cluster_size];
}

size_t project_smem(int width_floats, int shg)
{
    return (size_t)kProjThreads * (width_floats + 4) * sizeof(float) +
           (size_t)kProjThreads * (shg + 1) * sizeof(float);
}

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gsb_project_fwd(gsb_stream_t stream, const gsb_project_params* p, const float* xyz,
                               const float* log_scale, const float* rotation, const float* opacity,
                               const float* sh, const uint8_t* alive, const float* view,
                               const float* intrinsics, const float* center,
                               const int32_t* cluster_ids, const int32_t* cluster_count,
                               float* mean, float* depth, float* conic, float* radius,
                               float* color, float* alpha, int8_t* visible)
{
    if (!p) return GSB_ERR_NULL;
    if (p->capacity < 0 || p->sh_dim < 1 || p->degree < 0 || p->degree > 3 ||
        (p->degree + 1) * (p->degree + 1) > p->sh_dim || p->cluster_size <= 0)
        return GSB_ERR_INVALID;
    if (p->capacity == 0) return GSB_OK;
    if (!xyz || !log_scale || !rotation || !opacity || !sh || !alive || !view || !intrinsics ||
        !center || !mean || !depth || !conic || !radius || !color || !alpha || !visible)
        return GSB_ERR_NULL;
    if (p->compacted && (!cluster_ids || !cluster_count)) return GSB_ERR_NULL;
    if ((reinterpret_cast<uintptr_t>(rotation) | reinterpret_cast<uintptr_t>(conic)) & 15)
        return GSB_ERR_INVALID;
    cudaStream_t s = as_stream(stream);
    if (p->compacted) {
        clear_projected_kernel<<<ceil_div(p->capacity, 256), 256, 0, s>>>(
            p->capacity, p->clear_invisible, mean, depth, conic, radius, color, alpha, visible);
        if (int e = check_launch()) return e;
    }
    int used = (p->degree + 1) * (p->degree + 1) * 3;
    int width = (used + 3) & ~3;
    if (width > p->sh_dim * 3) width = (p->sh_dim * 3 + 3) & ~3;
    size_t smem = (size_t)kProjThreads * (width + 4) * sizeof(float);
    int blocks = ceil_div(p->capacity, kProjThreads);
    project_fwd_kernel<<<blocks, kProjThreads, smem, s>>>(
        *p, xyz, log_scale, rotation, opacity, sh, alive, view, intrinsics, center, cluster_ids,
        cluster_count, mean, depth, conic, radius, color, alpha, visible);
    return check_launch();
}

extern "C" int gsb_project_bwd(gsb_stream_t stream, const gsb_project_bwd_params* p,
                               const float* xyz, const float* log_scale, const float* rotation,
                               const float* opacity, const float* sh, const float* view,
                               const float* intrinsics, const float* center, const float* color,
                               const int32_t* cluster_ids, const int32_t* cluster_count,
                               const float* gmean, const float* gdepth, const float* gconic,
                               const float* gradius, const float* gcolor, const float* galpha,
                               float* gxyz, float* glog_scale, float* grotation, float* gopacity,
                               float* gsh)
{
    if (!p) return GSB_ERR_NULL;
    if (p->capacity < 0 || p->sh_dim < 1 || p->degree < 0 || p->degree > 3 ||
        (p->degree + 1) * (p->degree + 1) > p->sh_dim || p->cluster_size <= 0 ||
        p->sh_gradient_dim < 1 || p->sh_gradient_dim > p->sh_dim)
        return GSB_ERR_INVALID;
    if (p->sh_color_only ? p->sh_gradient_dim != 1
                         : p->sh_gradient_dim < (p->degree + 1) * (p->degree + 1))
        return GSB_ERR_INVALID;
    if (p->capacity == 0) return GSB_OK;
    if (!xyz || !log_scale || !rotation || !opacity || !sh || !view || !intrinsics || !center ||
        !color || !gmean || !gconic || !gcolor || !galpha || !gxyz || !glog_scale ||
        !grotation || !gopacity || !gsh)
        return GSB_ERR_NULL;
    if (!p->rgb_only && (!gdepth || !gradius)) return GSB_ERR_NULL;
    if (p->compacted && (!cluster_ids || !cluster_count)) return GSB_ERR_NULL;
    if ((reinterpret_cast<uintptr_t>(rotation) | reinterpret_cast<uintptr_t>(gconic) |
         reinterpret_cast<uintptr_t>(grotation) | reinterpret_cast<uintptr_t>(gmean)) & 15)
        return GSB_ERR_INVALID;
    cudaStream_t s = as_stream(stream);
    int shg = p->sh_gradient_dim * 3;
    if (p->compacted && !p->compact_gradients) {
        int64_t n = (int64_t)p->capacity * (shg > 4 ? shg : 4);
        clear_grads_kernel<<<ceil_div(n, 256), 256, 0, s>>>(p->capacity, shg, gxyz, glog_scale,
                                                            grotation, gopacity, gsh);
        if (int e = check_launch()) return e;
    }
    int used = (p->degree + 1) * (p->degree + 1) * 3;
    int width = (used + 3) & ~3;
    if (width > p->sh_dim * 3) width = (p->sh_dim * 3 + 3) & ~3;
    size_t smem = project_smem(width, shg);
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(project_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             96 * 1024);
        configured = true;
    }
    project_bwd_kernel<<<ceil_div(p->capacity, kProjThreads), kProjThreads, smem, s>>>(
        *p, xyz, log_scale, rotation, opacity, sh, view, intrinsics, center, color, cluster_ids,
        cluster_count, gmean, gdepth, gconic, gradius, gcolor, galpha, gxyz, glog_scale,
        grotation, gopacity, gsh);
    return check_launch();
}

extern "C" size_t gsb_cluster_compact_workspace_size(const gsb_cluster_params* p)
{
    return p ? (((size_t)(p->num_clusters > 0 ? p->num_clusters : 1) + 255) & ~size_t(255)) : 0;
}

extern "C" int gsb_cluster_compact(gsb_stream_t stream, const gsb_cluster_params* p,
                                   void* workspace, size_t workspace_bytes, const float* center,
                                   const float* extent, const uint8_t* valid, const float* planes,
                                   int32_t* ids, int32_t* count, uint8_t* visible_slots)
{
    if (!p) return GSB_ERR_NULL;
    if (p->num_clusters < 0 || p->cluster_size <= 0 || p->capacity < 0 ||
        (int64_t)p->num_clusters * p->cluster_size < p->capacity)
        return GSB_ERR_INVALID;
    if (workspace_bytes < gsb_cluster_compact_workspace_size(p) || !workspace)
        return GSB_ERR_WORKSPACE;
    if (!count || (p->num_clusters > 0 && (!center || !extent || !valid || !planes || !ids)))
        return GSB_ERR_NULL;
    cudaStream_t s = as_stream(stream);
    uint8_t* cluster_vis = static_cast<uint8_t*>(workspace);
    cluster_compact_kernel<<<1, kClusterThreads, 0, s>>>(p->num_clusters, center, extent, valid,
                                                         planes, ids, count, cluster_vis);
    if (int e = check_launch()) return e;
    if (visible_slots && p->capacity > 0) {
        expand_slots_kernel<<<ceil_div(p->capacity, 256), 256, 0, s>>>(
            p->capacity, p->cluster_size, cluster_vis, visible_slots);
        return check_launch();
    }
    return GSB_OK;
}
