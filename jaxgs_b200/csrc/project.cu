// Projection forward / pullback and visible-cluster compaction (sm_100a).
//
// One thread per compact index (128 per block).  The compact index i maps to
// pool slot cluster_ids[i / cluster_size] * cluster_size + i % cluster_size
// (kernels/projection.py:42-47), so a 128-slot cluster is one contiguous run
// of 128 Gaussians and every warp reads and writes contiguous runs.  The SH
// rows (the bulk of the 236 B/Gaussian) move as 16-byte vectors per thread;
// the SH degree is a template parameter so the basis and its derivatives are
// straight-line code.  HBM-bound: 286 B/Gaussian forward, 524 B/Gaussian
// backward (236 B with colour-only SH gradients).
#include "gsb_common.cuh"
#include "sh.cuh"

namespace gsb {
namespace {

constexpr int kProjThreads = 128;

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

// Is cluster c among the ascending visible-cluster ids[0:count]?
__device__ __forceinline__ bool cluster_listed(const int32_t* ids, int count, int64_t c)
{
    int lo = 0, hi = count;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(ids + mid) < c) lo = mid + 1;
        else hi = mid;
    }
    return lo < count && __ldg(ids + lo) == c;
}

// cluster_listed for a whole warp: when all lanes ask about the same
// cluster, the warp narrows the search 32-way per round (3 rounds of loads
// for 8k clusters instead of 13 dependent ones); otherwise each lane
// searches alone.  Every lane of the warp must call it.
__device__ __forceinline__ bool cluster_listed_warp(const int32_t* ids, int count, int64_t c)
{
    const int lane = threadIdx.x & 31;
    const int64_t c0 = __shfl_sync(GSB_FULL_MASK, c, 0);
    if (!__all_sync(GSB_FULL_MASK, c == c0)) return cluster_listed(ids, count, c);
    int lo = 0, hi = count;  // lower bound of c0 lies in [lo, hi]
    while (hi - lo > 32) {
        const int step = (hi - lo + 31) / 32;
        const int pos = lo + lane * step;
        const bool below = pos < hi && __ldg(ids + pos) < c0;
        const int k = __popc(__ballot_sync(GSB_FULL_MASK, below));  // lanes 0..k-1 below
        const int new_lo = k > 0 ? lo + (k - 1) * step + 1 : lo;
        const int new_hi = k < 32 && lo + k * step < hi ? lo + k * step : hi;
        lo = new_lo;
        hi = new_hi;
    }
    const int pos = lo + lane;
    const bool below = pos < hi && __ldg(ids + pos) < c0;
    const int first = lo + __popc(__ballot_sync(GSB_FULL_MASK, below));
    return first < count && __ldg(ids + first) == c0;
}

// Loads floats [0, N) of one Gaussian's SH row (row stride `row` floats):
// 16-byte vector loads when the row and the base are 16-byte aligned.
template <int N>
__device__ __forceinline__ void load_sh(const float* __restrict__ sh, int64_t g, int row, bool vec,
                                        float c[N])
{
    const float* src = sh + g * row;
    if (vec) {
#pragma unroll
        for (int k = 0; k < N / 4; k++) {
            float4 v = __ldg(reinterpret_cast<const float4*>(src) + k);
            c[4 * k] = v.x;
            c[4 * k + 1] = v.y;
            c[4 * k + 2] = v.z;
            c[4 * k + 3] = v.w;
        }
#pragma unroll
        for (int k = (N / 4) * 4; k < N; k++) c[k] = __ldg(src + k);
    } else {
#pragma unroll
        for (int k = 0; k < N; k++) c[k] = __ldg(src + k);
    }
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

template <int DEGREE>
__global__ void __launch_bounds__(kProjThreads) project_fwd_kernel(
    gsb_project_params p, const float* __restrict__ xyz, const float* __restrict__ log_scale,
    const float* __restrict__ rotation, const float* __restrict__ opacity,
    const float* __restrict__ sh, const uint8_t* __restrict__ alive, const float* view,
    const float* intr, const float* center, const int32_t* __restrict__ cluster_ids,
    const int32_t* __restrict__ cluster_count, float* __restrict__ out_mean,
    float* __restrict__ out_depth, float* __restrict__ out_conic, float* __restrict__ out_radius,
    float* __restrict__ out_color, float* __restrict__ out_alpha, int8_t* __restrict__ out_visible)
{
    pdl_begin();
    constexpr int NC = (DEGREE + 1) * (DEGREE + 1) * 3;
    int count = p.compacted ? __ldg(cluster_count) : 0;
    // One thread per pool slot.  With a cluster list, slots of unlisted
    // clusters are cleared here (kernels/projection.py:178-210: visible = 0,
    // and with clear_invisible every field), so no separate clear pass runs.
    const int64_t g = (int64_t)blockIdx.x * kProjThreads + threadIdx.x;
    const bool listed = !p.compacted ||
        cluster_listed_warp(cluster_ids, count, (g < p.capacity ? g : p.capacity - 1) / p.cluster_size);
    if (g >= p.capacity) return;
    if (!listed) {
        out_visible[g] = 0;
        if (p.clear_invisible) {
            *reinterpret_cast<float2*>(out_mean + g * 2) = make_float2(0.f, 0.f);
            *reinterpret_cast<float4*>(out_conic + g * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
            out_color[g * 3] = out_color[g * 3 + 1] = out_color[g * 3 + 2] = 0.0f;
            out_depth[g] = __int_as_float(0x7f800000);
            out_radius[g] = 0.0f;
            out_alpha[g] = 0.0f;
        }
        return;
    }
    const int row = p.sh_dim * 3;
    const bool vec = (row & 3) == 0 && (reinterpret_cast<uintptr_t>(sh) & 15) == 0;
    Cam cam;
    load_cam(cam, view, intr, center);
    float wx = xyz[g * 3], wy = xyz[g * 3 + 1], wz = xyz[g * 3 + 2];
    float4 q = __ldg(reinterpret_cast<const float4*>(rotation + g * 4));
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
    float rgb[3] = {0.0f, 0.0f, 0.0f};
    if (!p.visible_color_only || vis) {
        float dx = wx - cam.c[0], dy = wy - cam.c[1], dz = wz - cam.c[2];
        float dn = rsqrtf(fmaxf(dx * dx + dy * dy + dz * dz, 1e-16f));
        float c[NC];
        load_sh<NC>(sh, g, row, vec, c);
        float bas[16];
        sh_basis<DEGREE>(dx * dn, dy * dn, dz * dn, bas);
#pragma unroll
        for (int ch = 0; ch < 3; ch++) {
            // kernels/projection.py:142-171 adds the bands in this grouping.
            float value = bas[0] * c[ch];
            if (DEGREE >= 1) value += (bas[1] * c[ch + 3] + bas[2] * c[ch + 6] + bas[3] * c[ch + 9]);
            if (DEGREE >= 2)
                value += (bas[4] * c[ch + 12] + bas[5] * c[ch + 15] + bas[6] * c[ch + 18] +
                          bas[7] * c[ch + 21] + bas[8] * c[ch + 24]);
            if (DEGREE >= 3)
                value += (bas[9] * c[ch + 27] + bas[10] * c[ch + 30] + bas[11] * c[ch + 33] +
                          bas[12] * c[ch + 36] + bas[13] * c[ch + 39] + bas[14] * c[ch + 42] +
                          bas[15] * c[ch + 45]);
            rgb[ch] = fmaxf(value + 0.5f, 0.0f);
        }
    }
    out_color[g * 3] = rgb[0];
    out_color[g * 3 + 1] = rgb[1];
    out_color[g * 3 + 2] = rgb[2];
}

// ---------------------------------------------------------------------------
// Pullback: kernels/projection_backward.py:42-367.
// SH_MODE: 0 = all sh_gradient_dim coefficients (bands above DEGREE zero),
//          1 = colour cotangents only (sh_color_only, 3 floats per point).
// ---------------------------------------------------------------------------
// sh_stage (all-coefficient mode): write the thread's SH gradient row to sh_stage[threadIdx.x *
// sh_stage_stride] (16-byte aligned, shg a multiple of 4) for the block to
// store coalesced.  Returns whether the thread's output row was produced.
template <int DEGREE, int SH_MODE>
__device__ __forceinline__ bool project_bwd_body(
    const gsb_project_bwd_params& p, const float* __restrict__ xyz,
    const float* __restrict__ log_scale, const float* __restrict__ rotation,
    const float* __restrict__ opacity, const float* __restrict__ sh, const float* view,
    const float* intr, const float* center, const float* __restrict__ color,
    const int32_t* __restrict__ cluster_ids, const int32_t* __restrict__ cluster_count,
    const float* __restrict__ gmean, const float* __restrict__ gdepth,
    const float* __restrict__ gconic, const float* __restrict__ gradius,
    const float* __restrict__ gcolor, const float* __restrict__ galpha,
    float* __restrict__ out_xyz, float* __restrict__ out_log_scale,
    float* __restrict__ out_rotation, float* __restrict__ out_opacity, float* __restrict__ out_sh,
    float* sh_stage = nullptr, int sh_stage_stride = 0)
{
    constexpr int NB = (DEGREE + 1) * (DEGREE + 1);
    int count = p.compacted ? __ldg(cluster_count) : 0;
    int64_t i = (int64_t)blockIdx.x * kProjThreads + threadIdx.x;
    // Pool-order output of a compacted pullback covers every slot: the rows of
    // unlisted clusters are written as zeros (their cotangents are not read).
    const bool pool_order = p.compacted && !p.compact_gradients;
    int64_t g;
    bool listed = true;
    if (pool_order) {
        listed = cluster_listed_warp(cluster_ids, count,
                                     (i < p.capacity ? i : p.capacity - 1) / p.cluster_size);
        if (i >= p.capacity) return false;
        g = i;
    } else {
        g = slot_of(i, p.capacity, cluster_ids, count, p.cluster_size, p.compacted);
        if (g < 0) return false;
    }
    const int64_t o = p.compact_gradients ? i : g;
    const int shg = SH_MODE == 1 ? 3 : p.sh_gradient_dim * 3;
    float* osh = (SH_MODE == 0 && sh_stage) ? sh_stage + threadIdx.x * sh_stage_stride
                                            : out_sh + o * shg;
    const bool vec_out = (SH_MODE == 0 && sh_stage) ||
                         ((shg & 3) == 0 && (reinterpret_cast<uintptr_t>(out_sh) & 15) == 0);

    float2 gm = make_float2(0.f, 0.f);
    float4 gcn = make_float4(0.f, 0.f, 0.f, 0.f);
    float gc0 = 0.f, gc1 = 0.f, gc2 = 0.f, gal = 0.f;
    // The parameters and the colour are loaded with the cotangents, in one
    // round trip, before it is known whether they are needed: a dependent
    // chain of loads, not bandwidth, bounds this kernel.
    float wx = 0.f, wy = 0.f, wz = 0.f, ls0 = 0.f, ls1 = 0.f, ls2 = 0.f, op = 0.f;
    float col0 = 0.f, col1 = 0.f, col2 = 0.f;
    float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
    bool has = false;
    if (listed) {
        gm = __ldg(reinterpret_cast<const float2*>(gmean + g * 2));
        gcn = __ldg(reinterpret_cast<const float4*>(gconic + g * 4));
        gc0 = gcolor[g * 3];
        gc1 = gcolor[g * 3 + 1];
        gc2 = gcolor[g * 3 + 2];
        gal = galpha[g];
        wx = __ldg(xyz + g * 3);
        wy = __ldg(xyz + g * 3 + 1);
        wz = __ldg(xyz + g * 3 + 2);
        q = __ldg(reinterpret_cast<const float4*>(rotation + g * 4));
        ls0 = __ldg(log_scale + g * 3);
        ls1 = __ldg(log_scale + g * 3 + 1);
        ls2 = __ldg(log_scale + g * 3 + 2);
        op = __ldg(opacity + g);
        col0 = __ldg(color + g * 3);
        col1 = __ldg(color + g * 3 + 1);
        col2 = __ldg(color + g * 3 + 2);
        has = gal != 0.0f || gm.x != 0.0f || gm.y != 0.0f || gcn.x != 0.0f || gcn.y != 0.0f ||
              gcn.z != 0.0f || gcn.w != 0.0f || gc0 != 0.0f || gc1 != 0.0f || gc2 != 0.0f;
        if (!p.rgb_only) has = has || gdepth[g] != 0.0f || gradius[g] != 0.0f;
    }
    if (!has) {
        // Occluded or culled splats: zero gradients (projection_backward.py:61-80).
        out_xyz[o * 3] = out_xyz[o * 3 + 1] = out_xyz[o * 3 + 2] = 0.0f;
        out_log_scale[o * 3] = out_log_scale[o * 3 + 1] = out_log_scale[o * 3 + 2] = 0.0f;
        *reinterpret_cast<float4*>(out_rotation + o * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
        out_opacity[o] = 0.0f;
        if (vec_out) {
            for (int k = 0; k < shg / 4; k++)
                reinterpret_cast<float4*>(osh)[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            for (int k = 0; k < shg; k++) osh[k] = 0.0f;
        }
        return true;
    }
    // With a staged SH output row, the SH input coefficients the direction
    // gradient needs are copied into that row asynchronously now (16-byte
    // cp.async, the thread's own row, so no barrier), overlapping the
    // geometry; they are read back before the row is overwritten.
    constexpr int kInChunks = (NB * 3) / 4;
    const bool sh_async = SH_MODE == 0 && DEGREE >= 1 && sh_stage != nullptr &&
                          (NB * 3) % 4 == 0 && ((p.sh_dim * 3) & 3) == 0 &&
                          (reinterpret_cast<uintptr_t>(sh) & 15) == 0 &&
                          kInChunks * 4 <= sh_stage_stride;
    if (sh_async) {
        const float4* src = reinterpret_cast<const float4*>(sh + g * (p.sh_dim * 3));
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(osh);
#pragma unroll
        for (int k = 0; k < kInChunks; k++)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst + 16 * k),
                         "l"(src + k)
                         : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    Cam cam;
    load_cam(cam, view, intr, center);
    Geometry geo;
    geometry(geo, cam, wx, wy, wz, q, ls0, ls1, ls2, p.near_plane);
    const float* v = cam.v;
    const float fx = cam.fx, fy = cam.fy;
    const float inv_z = 1.0f / geo.safe_z, inv_z2 = inv_z * inv_z;
    const float x = geo.x, y = geo.y;
    float gx = gm.x * fx * inv_z;
    float gy = gm.y * fy * inv_z;
    float gz = p.rgb_only ? 0.0f : gdepth[g];
    float gsafe_z = -gm.x * fx * x * inv_z2;
    gsafe_z -= gm.y * fy * y * inv_z2;
    const float a = geo.a, b = geo.b, d = geo.d;
    const float raw_det = a * d - b * b;
    const float det = fmaxf(raw_det, 1e-8f);
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
    const float j0 = geo.j0, j1 = geo.j1, j2 = geo.j2, j3 = geo.j3;
    float gm00 = j0 * ga0, gm01 = j0 * ga1, gm02 = j0 * ga2;
    float gm10 = j1 * gb0, gm11 = j1 * gb1, gm12 = j1 * gb2;
    float gm20 = -j2 * ga0 - j3 * gb0, gm21 = -j2 * ga1 - j3 * gb1, gm22 = -j2 * ga2 - j3 * gb2;
    out_log_scale[o * 3] = gm00 * m[0] + gm10 * m[3] + gm20 * m[6];
    out_log_scale[o * 3 + 1] = gm01 * m[1] + gm11 * m[4] + gm21 * m[7];
    out_log_scale[o * 3 + 2] = gm02 * m[2] + gm12 * m[5] + gm22 * m[8];
    const float s0 = geo.s0, s1 = geo.s1, s2 = geo.s2;
    float gr00 = s0 * (v[0] * gm00 + v[4] * gm10 + v[8] * gm20);
    float gr10 = s0 * (v[1] * gm00 + v[5] * gm10 + v[9] * gm20);
    float gr20 = s0 * (v[2] * gm00 + v[6] * gm10 + v[10] * gm20);
    float gr01 = s1 * (v[0] * gm01 + v[4] * gm11 + v[8] * gm21);
    float gr11 = s1 * (v[1] * gm01 + v[5] * gm11 + v[9] * gm21);
    float gr21 = s1 * (v[2] * gm01 + v[6] * gm11 + v[10] * gm21);
    float gr02 = s2 * (v[0] * gm02 + v[4] * gm12 + v[8] * gm22);
    float gr12 = s2 * (v[1] * gm02 + v[5] * gm12 + v[9] * gm22);
    float gr22 = s2 * (v[2] * gm02 + v[6] * gm12 + v[10] * gm22);
    const float qw = geo.qw, qx = geo.qx, qy = geo.qy, qz = geo.qz;
    float gqw = -2 * qz * gr01 + 2 * qy * gr02 + 2 * qz * gr10 - 2 * qx * gr12 - 2 * qy * gr20 + 2 * qx * gr21;
    float gqx = 2 * qy * (gr01 + gr10) + 2 * qz * (gr02 + gr20) - 4 * qx * (gr11 + gr22) - 2 * qw * gr12 + 2 * qw * gr21;
    float gqy = -4 * qy * (gr00 + gr22) + 2 * qx * (gr01 + gr10) + 2 * qw * gr02 + 2 * qz * (gr12 + gr21) - 2 * qw * gr20;
    float gqz = -4 * qz * (gr00 + gr11) - 2 * qw * gr01 + 2 * qx * (gr02 + gr20) + 2 * qw * gr10 + 2 * qy * (gr12 + gr21);
    const float qdenom = geo.qdenom;
    const float qdot = gqw * qw + gqx * qx + gqy * qy + gqz * qz;
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
    const float alpha = 1.0f / (1.0f + expf(-op));
    out_opacity[o] = gal * alpha * (1.0f - alpha);

    // SH: colour cotangents pass only where the colour was not clamped.
    const float vx = wx - cam.c[0], vy = wy - cam.c[1], vz = wz - cam.c[2];
    const float dir_denom = sqrtf(fmaxf(vx * vx + vy * vy + vz * vz, 1e-16f));
    const float dx = vx / dir_denom, dy = vy / dir_denom, dz = vz / dir_denom;
    float gcc[3];
    gcc[0] = col0 > 0.0f ? gc0 : 0.0f;
    gcc[1] = col1 > 0.0f ? gc1 : 0.0f;
    gcc[2] = col2 > 0.0f ? gc2 : 0.0f;
    // dot_k = sum_ch gc_ch * coef[k][ch] for the direction gradient, formed
    // before the SH gradient row (which may reuse the staged coefficients'
    // storage) is written.
    float dot[16];
    if (DEGREE >= 1) {
        float cf[NB * 3];
        if (sh_async) {
            asm volatile("cp.async.wait_all;" ::: "memory");
#pragma unroll
            for (int k = 0; k < kInChunks; k++) {
                const float4 v4 = reinterpret_cast<const float4*>(osh)[k];
                cf[4 * k] = v4.x;
                cf[4 * k + 1] = v4.y;
                cf[4 * k + 2] = v4.z;
                cf[4 * k + 3] = v4.w;
            }
        } else {
            load_sh<NB * 3>(sh, g, p.sh_dim * 3,
                            ((p.sh_dim * 3) & 3) == 0 && (reinterpret_cast<uintptr_t>(sh) & 15) == 0,
                            cf);
        }
#pragma unroll
        for (int k = 0; k < NB; k++) dot[k] = gcc[0] * cf[3 * k] + gcc[1] * cf[3 * k + 1] + gcc[2] * cf[3 * k + 2];
    }
    if (SH_MODE == 1) {
        osh[0] = gcc[0];
        osh[1] = gcc[1];
        osh[2] = gcc[2];
    } else {
        float bas[16];
        sh_basis<DEGREE>(dx, dy, dz, bas);
        const int nval = NB * 3;
        if (vec_out) {
            constexpr int kChunks = (NB * 3 + 3) / 4;
#pragma unroll
            for (int k = 0; k < kChunks; k++) {
                float e[4];
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const int c = 4 * k + t;
                    e[t] = c < NB * 3 ? gcc[c % 3] * bas[c / 3] : 0.0f;
                }
                reinterpret_cast<float4*>(osh)[k] = make_float4(e[0], e[1], e[2], e[3]);
            }
            for (int k = kChunks; k < shg / 4; k++)
                reinterpret_cast<float4*>(osh)[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
#pragma unroll
            for (int c = 0; c < nval; c++) osh[c] = gcc[c % 3] * bas[c / 3];
            for (int c = nval; c < shg; c++) osh[c] = 0.0f;
        }
    }
    // Direction gradient: dot_k = sum_ch gc_ch * coef[k][ch], then the basis
    // derivatives of projection_backward.py:259-330.
    float gdx = 0.0f, gdy = 0.0f, gdz = 0.0f;
    if (DEGREE >= 1) {
        const float xx = dx * dx, yy = dy * dy, zz = dz * dz;
        gdx -= kC1 * dot[3];
        gdy -= kC1 * dot[1];
        gdz += kC1 * dot[2];
        if (DEGREE >= 2) {
            gdx += 1.0925484305920792f * dy * dot[4] - 0.6307831305050401f * dx * dot[6] -
                   1.0925484305920792f * dz * dot[7] + 1.0925484305920792f * dx * dot[8];
            gdy += 1.0925484305920792f * dx * dot[4] - 1.0925484305920792f * dz * dot[5] -
                   0.6307831305050401f * dy * dot[6] - 1.0925484305920792f * dy * dot[8];
            gdz += -1.0925484305920792f * dy * dot[5] + 1.2615662610100802f * dz * dot[6] -
                   1.0925484305920792f * dx * dot[7];
        }
        if (DEGREE >= 3) {
            gdx += -3.540261539559861f * dx * dy * dot[9] + 2.890611442640554f * dy * dz * dot[10] +
                   0.9140915989289316f * dx * dy * dot[11] - 2.2390579955406924f * dx * dz * dot[12] -
                   0.4570457994644658f * (4 * zz - 3 * xx - yy) * dot[13] +
                   2.890611442640554f * dx * dz * dot[14] - 1.7701307697799305f * (xx - yy) * dot[15];
            gdy += -1.7701307697799305f * (xx - yy) * dot[9] + 2.890611442640554f * dx * dz * dot[10] -
                   0.4570457994644658f * (4 * zz - xx - 3 * yy) * dot[11] -
                   2.2390579955406924f * dy * dz * dot[12] + 0.9140915989289316f * dx * dy * dot[13] -
                   2.890611442640554f * dy * dz * dot[14] + 3.540261539559861f * dx * dy * dot[15];
            gdz += 2.890611442640554f * dx * dy * dot[10] - 3.6563663957157264f * dy * dz * dot[11] +
                   0.3731763325901154f * (6 * zz - 3 * xx - 3 * yy) * dot[12] -
                   3.6563663957157264f * dx * dz * dot[13] + 1.445305721320277f * (xx - yy) * dot[14];
        }
    }
    const float dir_dot = gdx * dx + gdy * dy + gdz * dz;
    float gxw = gdx / dir_denom, gyw = gdy / dir_denom, gzw = gdz / dir_denom;
    if (dir_denom > 1e-8f) {
        gxw = (gdx - dir_dot * dx) / dir_denom;
        gyw = (gdy - dir_dot * dy) / dir_denom;
        gzw = (gdz - dir_dot * dz) / dir_denom;
    }
    out_xyz[o * 3] = v[0] * gx + v[4] * gy + v[8] * gz + gxw;
    out_xyz[o * 3 + 1] = v[1] * gx + v[5] * gy + v[9] * gz + gyw;
    out_xyz[o * 3 + 2] = v[2] * gx + v[6] * gy + v[10] * gz + gzw;
    return true;
}

// Rows of SH gradients are 4 * chunks floats (chunks <= kStageChunks); a
// block's rows are staged in shared memory with an odd float4 stride (no
// bank conflicts for the per-thread float4 writes) and leave as consecutive
// float4 stores of the whole block.
constexpr int kStageChunks = 12;
constexpr int kStageStride4 = kStageChunks + 1;

// Six blocks per SM (80 registers, a few bytes spilled) measured faster than
// the five that 94 registers allow: the kernel waits on loads, so more
// resident warps overlap more of them (config 2: 90 -> 84 us).
template <int DEGREE, int SH_MODE>
__global__ void __launch_bounds__(kProjThreads, 6) project_bwd_kernel(
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
    pdl_begin();
    const int shg = p.sh_gradient_dim * 3;
    const int chunks = shg >> 2;
    const bool staged = SH_MODE == 0 && (shg & 3) == 0 && chunks <= kStageChunks &&
                        (reinterpret_cast<uintptr_t>(out_sh) & 15) == 0;
    if (!staged) {
        project_bwd_body<DEGREE, SH_MODE>(p, xyz, log_scale, rotation, opacity, sh, view, intr,
                                          center, color, cluster_ids, cluster_count, gmean, gdepth,
                                          gconic, gradius, gcolor, galpha, out_xyz, out_log_scale,
                                          out_rotation, out_opacity, out_sh);
        return;
    }
    __shared__ __align__(16) float4 stage[kProjThreads * kStageStride4];
    __shared__ int row_count;
    const bool wrote = project_bwd_body<DEGREE, SH_MODE>(
        p, xyz, log_scale, rotation, opacity, sh, view, intr, center, color, cluster_ids,
        cluster_count, gmean, gdepth, gconic, gradius, gcolor, galpha, out_xyz, out_log_scale,
        out_rotation, out_opacity, nullptr, reinterpret_cast<float*>(stage),
        kStageStride4 * 4);
    // The rows produced form a prefix of the block's slots (validity only
    // ends at the last listed slot or the capacity).
    if (threadIdx.x == 0) row_count = 0;
    __syncthreads();
    const unsigned ballot = __ballot_sync(GSB_FULL_MASK, wrote);
    if ((threadIdx.x & 31) == 0 && ballot) atomicAdd(&row_count, __popc(ballot));
    __syncthreads();
    const int rows = row_count;
    // Row r of the block is output row blockIdx.x * kProjThreads + r (the
    // compact index, or the pool slot in pool order).
    float4* out4 = reinterpret_cast<float4*>(out_sh) +
                   (int64_t)blockIdx.x * kProjThreads * chunks;
    const uint32_t magic = ((1u << 20) + chunks - 1) / chunks;  // exact for idx < 2^16
    for (int idx = threadIdx.x; idx < rows * chunks; idx += kProjThreads) {
        const int r = (int)(((uint32_t)idx * magic) >> 20);
        const int k = idx - r * chunks;
        out4[idx] = stage[r * kStageStride4 + k];
    }
}

// training/sh_pullback.py:18-53 summed over views: the SH coefficient
// cotangents of colour cotangents that were masked where the colour clamped
// (the sh_color_only pullback output),
//   gsh[g][k][c] = sum_v B_k(dir_gv) colors[v][g][c],
// with dir_gv normalised exactly as the pullback does; bands above DEGREE and
// coefficients past (DEGREE+1)^2 are zero.  A view whose three cotangents
// are zero (the Gaussian was culled or occluded there) adds nothing.
template <int DEGREE>
__global__ void __launch_bounds__(kProjThreads) sh_from_colors_kernel(
    int64_t capacity, int sh_dim, int views, int64_t view_stride, int64_t center_stride,
    const float* __restrict__ xyz, const float* __restrict__ centers,
    const float* __restrict__ colors, float* __restrict__ gsh)
{
    pdl_begin();
    constexpr int NB = (DEGREE + 1) * (DEGREE + 1);
    const int64_t g = (int64_t)blockIdx.x * kProjThreads + threadIdx.x;
    const bool active = g < capacity;
    float acc[NB * 3];
#pragma unroll
    for (int c = 0; c < NB * 3; c++) acc[c] = 0.0f;
    if (active) {
        sh_expand_views<DEGREE>(xyz[g * 3], xyz[g * 3 + 1], xyz[g * 3 + 2], views,
                                colors + g * 3, view_stride, centers, center_stride, acc);
    }
    const int n = sh_dim * 3;
    const int chunks = n >> 2;
    constexpr int kChunks = (NB * 3 + 3) / 4;
    // Uniform over the block: rows staged in shared memory and stored as
    // whole-block coalesced float4 runs when they are float4 rows.
    if ((n & 3) != 0 || chunks > kStageChunks || (reinterpret_cast<uintptr_t>(gsh) & 15) != 0) {
        if (!active) return;
        float* out = gsh + g * (int64_t)n;
#pragma unroll
        for (int c = 0; c < NB * 3; c++) out[c] = acc[c];
        for (int c = NB * 3; c < n; c++) out[c] = 0.0f;
        return;
    }
    __shared__ __align__(16) float4 stage[kProjThreads * kStageStride4];
    float4* row = stage + threadIdx.x * kStageStride4;
#pragma unroll
    for (int k = 0; k < kChunks; k++) {
        float e[4];
#pragma unroll
        for (int t = 0; t < 4; t++) e[t] = 4 * k + t < NB * 3 ? acc[4 * k + t] : 0.0f;
        row[k] = make_float4(e[0], e[1], e[2], e[3]);
    }
    for (int k = kChunks; k < chunks; k++) row[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    const int64_t first = (int64_t)blockIdx.x * kProjThreads;
    const int rows = (int)(capacity - first < kProjThreads ? capacity - first : kProjThreads);
    float4* out4 = reinterpret_cast<float4*>(gsh) + first * chunks;
    const uint32_t magic = ((1u << 20) + chunks - 1) / chunks;  // exact for idx < 2^16
    for (int idx = threadIdx.x; idx < rows * chunks; idx += kProjThreads) {
        const int r = (int)(((uint32_t)idx * magic) >> 20);
        out4[idx] = stage[r * kStageStride4 + (idx - r * chunks)];
    }
}

// ---------------------------------------------------------------------------
// Cluster frustum test + stable compaction (scene/cluster.py:40-67,
// kernels/cluster_compact.py:31-44).  One block of 1024 threads per round of
// 8192 clusters: the tests read the bounds coalesced (cluster j*1024 + t) and
// leave one visibility byte per cluster in shared memory; then thread t
// takes clusters 8t..8t+7, and one block scan of the per-thread counts
// writes the ids in ascending order without atomics.
// ---------------------------------------------------------------------------
constexpr int kClusterThreads = 1024;
constexpr int kClustersPerThread = 8;
constexpr int kClusterRound = kClusterThreads * kClustersPerThread;

__global__ void __launch_bounds__(kClusterThreads) cluster_compact_kernel(
    int num_clusters, const float* __restrict__ center, const float* __restrict__ extent,
    const uint8_t* __restrict__ valid, const float* __restrict__ planes, int32_t* ids,
    int32_t* count_out, uint8_t* cluster_vis)
{
    pdl_begin();
    __shared__ float pl[24];
    __shared__ int warp_totals[32];
    __shared__ int running;
    __shared__ __align__(8) uint8_t vis_s[kClusterRound];
    if (threadIdx.x < 24) pl[threadIdx.x] = planes[threadIdx.x];
    if (threadIdx.x == 0) running = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int base = 0; base < num_clusters; base += kClusterRound) {
        // All eight clusters' bounds are loaded before any test, so their
        // memory latencies overlap.
        float b[kClustersPerThread][6];
        int ok[kClustersPerThread];
#pragma unroll
        for (int j = 0; j < kClustersPerThread; j++) {
            const int c = base + j * kClusterThreads + threadIdx.x;
            ok[j] = c < num_clusters ? valid[c] != 0 : 0;
#pragma unroll
            for (int k = 0; k < 3; k++) {
                b[j][k] = c < num_clusters ? center[c * 3 + k] : 0.0f;
                b[j][3 + k] = c < num_clusters ? extent[c * 3 + k] : 0.0f;
            }
        }
#pragma unroll
        for (int j = 0; j < kClustersPerThread; j++) {
            const int local = j * kClusterThreads + threadIdx.x;
            const int c = base + local;
            int vis = ok[j];
#pragma unroll
            for (int k = 0; k < 6; k++) {
                const float* q = pl + k * 4;
                const float dist = b[j][0] * q[0] + b[j][1] * q[1] + b[j][2] * q[2] + q[3];
                const float rad = b[j][3] * fabsf(q[0]) + b[j][4] * fabsf(q[1]) + b[j][5] * fabsf(q[2]);
                if (!(dist + rad >= 0.0f)) vis = 0;
            }
            if (c < num_clusters) cluster_vis[c] = (uint8_t)vis;
            vis_s[local] = (uint8_t)vis;
        }
        __syncthreads();
        const uint2 packed = reinterpret_cast<const uint2*>(vis_s)[threadIdx.x];
        unsigned bits = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            bits |= ((packed.x >> (8 * j)) & 1u) << j;
            bits |= ((packed.y >> (8 * j)) & 1u) << (j + 4);
        }
        const int first = base + threadIdx.x * kClustersPerThread;
        const int cnt = __popc(bits);
        const int inc = warp_inclusive_scan(cnt, lane);
        if (lane == 31) warp_totals[warp] = inc;
        __syncthreads();
        if (warp == 0) {
            const int t = warp_totals[lane];
            warp_totals[lane] = warp_inclusive_scan(t, lane) - t;
        }
        __syncthreads();
        int pos = running + warp_totals[warp] + inc - cnt;
        for (int j = 0; j < kClustersPerThread; j++)
            if ((bits >> j) & 1u) ids[pos++] = first + j;
        __syncthreads();
        if (threadIdx.x == kClusterThreads - 1) running = pos;
        __syncthreads();
    }
    if (threadIdx.x == 0) *count_out = running;
}

__global__ void expand_slots_kernel(int64_t capacity, int cluster_size, const uint8_t* cluster_vis,
                                    uint8_t* slots)
{
    pdl_begin();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < capacity) slots[i] = cluster_vis[i / cluster_size];
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
    int blocks = ceil_div(p->capacity, kProjThreads);
#define GSB_PROJ_FWD(D)                                                                          \
    gsb::launch(project_fwd_kernel<D>, blocks, kProjThreads, 0, s,                                        \
        *p, xyz, log_scale, rotation, opacity, sh, alive, view, intrinsics, center, cluster_ids, \
        cluster_count, mean, depth, conic, radius, color, alpha, visible)
    switch (p->degree) {
        case 0: GSB_PROJ_FWD(0); break;
        case 1: GSB_PROJ_FWD(1); break;
        case 2: GSB_PROJ_FWD(2); break;
        default: GSB_PROJ_FWD(3); break;
    }
#undef GSB_PROJ_FWD
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
    int blocks = ceil_div(p->capacity, kProjThreads);
#define GSB_PROJ_BWD(D, M)                                                                        \
    gsb::launch(project_bwd_kernel<D, M>, blocks, kProjThreads, 0, s,                                      \
        *p, xyz, log_scale, rotation, opacity, sh, view, intrinsics, center, color, cluster_ids,  \
        cluster_count, gmean, gdepth, gconic, gradius, gcolor, galpha, gxyz, glog_scale,          \
        grotation, gopacity, gsh)
    if (p->sh_color_only) {
        switch (p->degree) {
            case 0: GSB_PROJ_BWD(0, 1); break;
            case 1: GSB_PROJ_BWD(1, 1); break;
            case 2: GSB_PROJ_BWD(2, 1); break;
            default: GSB_PROJ_BWD(3, 1); break;
        }
    } else {
        switch (p->degree) {
            case 0: GSB_PROJ_BWD(0, 0); break;
            case 1: GSB_PROJ_BWD(1, 0); break;
            case 2: GSB_PROJ_BWD(2, 0); break;
            default: GSB_PROJ_BWD(3, 0); break;
        }
    }
#undef GSB_PROJ_BWD
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
    gsb::launch(cluster_compact_kernel, 1, kClusterThreads, 0, s, p->num_clusters, center, extent, valid,
                                                         planes, ids, count, cluster_vis);
    if (int e = check_launch()) return e;
    if (visible_slots && p->capacity > 0) {
        gsb::launch(expand_slots_kernel, ceil_div(p->capacity, 256), 256, 0, s, 
            p->capacity, p->cluster_size, cluster_vis, visible_slots);
        return check_launch();
    }
    return GSB_OK;
}

extern "C" int gsb_sh_from_colors(gsb_stream_t stream, const gsb_sh_params* p, const float* xyz,
                                  const float* centers, const float* colors, float* gsh)
{
    if (!p) return GSB_ERR_NULL;
    const int64_t view_stride = p->view_stride ? p->view_stride : (int64_t)p->capacity * 3;
    const int64_t center_stride = p->center_stride ? p->center_stride : 3;
    if (p->capacity < 0 || p->sh_dim < 1 || p->degree < 0 || p->degree > 3 ||
        (p->degree + 1) * (p->degree + 1) > p->sh_dim || p->views < 0 ||
        view_stride < (int64_t)p->capacity * 3 || center_stride < 3)
        return GSB_ERR_INVALID;
    if (p->capacity == 0) return GSB_OK;
    if (!xyz || !gsh || (p->views > 0 && (!centers || !colors))) return GSB_ERR_NULL;
    cudaStream_t s = as_stream(stream);
    const int blocks = ceil_div(p->capacity, kProjThreads);
#define GSB_SH_FROM_COLORS(D)                                                               \
    gsb::launch(sh_from_colors_kernel<D>, blocks, kProjThreads, 0, s,                                \
        p->capacity, p->sh_dim, p->views, view_stride, center_stride, xyz, centers, colors, \
        gsh)
    switch (p->degree) {
        case 0: GSB_SH_FROM_COLORS(0); break;
        case 1: GSB_SH_FROM_COLORS(1); break;
        case 2: GSB_SH_FROM_COLORS(2); break;
        default: GSB_SH_FROM_COLORS(3); break;
    }
#undef GSB_SH_FROM_COLORS
    return check_launch();
}
