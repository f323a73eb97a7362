// Visible-cluster sparse Adam (sm_100a): the LiteGS update without bias
// correction (kernels/sparse_adam.py:16-54, training/optimizer.py:276-341):
// for every element of the listed clusters' alive slots
//     m = 0.9 m + 0.1 g;  v = 0.999 v + 0.001 g^2;  x -= lr m / (sqrt(v) + 1e-15)
// with lr = rate[0] (times 10 for the first three channels of an SH row).
// Slots outside the listed clusters, and dead slots, are left untouched.
//
// A listed cluster's elements of one field are a contiguous run of
// cluster_size * channels floats in pool order (and in compact gradient
// order), so the kernel walks them four at a time with 16-byte loads and
// stores of the value, both moments and the gradient: 28 bytes of traffic
// per element, the whole cost of the update.  Vectors that would reach past
// the pool's end, or that are not 16-byte aligned, fall back to scalars.
//
// The SH field can also be updated from the step's colour cotangents
// (sparse_adam_sh_kernel): a lane per slot computes the SH basis of the
// slot's view direction into shared memory, then the warp updates its slots'
// rows with 16-byte vectors as above, forming each element's gradient from
// the basis and the colour cotangent, so no gradient row is written or read:
// 24 bytes of traffic per SH element instead of 28, plus 24 per slot.
#include "gsb_common.cuh"
#include "sh.cuh"

namespace gsb {
namespace {

constexpr int kAdamThreads = 256;
constexpr int kAdamVec = 4;

__device__ __forceinline__ void adam_element(float& x, float& m, float& v, float g, float lr)
{
    m = __fadd_rn(__fmul_rn(0.9f, m), __fmul_rn(0.1f, g));
    v = __fadd_rn(__fmul_rn(0.999f, v), __fmul_rn(__fmul_rn(0.001f, g), g));
    x = __fsub_rn(x, __fdiv_rn(__fmul_rn(lr, m), __fadd_rn(__fsqrt_rn(v), 1e-15f)));
}

// grid.x: listed-cluster index (blocks past the count exit); grid.y: parts
// of the cluster's run of cluster_size * channels elements.
__global__ void __launch_bounds__(kAdamThreads) sparse_adam_kernel(
    gsb_adam_params p, float* __restrict__ value, float* __restrict__ mean,
    float* __restrict__ variance, const float* __restrict__ gradient,
    const int8_t* __restrict__ alive, const int32_t* __restrict__ cluster_ids,
    const int32_t* __restrict__ cluster_count, const float* __restrict__ rate)
{
    pdl_begin();
    const int cluster = blockIdx.x;
    if (cluster >= __ldg(cluster_count)) return;
    const int64_t run = (int64_t)p.cluster_size * p.channels;
    const int64_t local = ((int64_t)blockIdx.y * kAdamThreads + threadIdx.x) * kAdamVec;
    if (local >= run) return;
    const int64_t first_slot = (int64_t)__ldg(cluster_ids + cluster) * p.cluster_size;
    const int64_t base = first_slot * p.channels;                 // pool-order element
    const int64_t gbase = p.compact_gradients ? (int64_t)cluster * run : base;
    const int64_t limit = (int64_t)p.capacity * p.channels;        // pool elements
    const float lr0 = __ldg(rate);
    const int n = (int)(run - local < kAdamVec ? run - local : kAdamVec);
    const bool aligned = ((reinterpret_cast<uintptr_t>(value) | reinterpret_cast<uintptr_t>(mean) |
                           reinterpret_cast<uintptr_t>(variance) |
                           reinterpret_cast<uintptr_t>(gradient)) & 15) == 0;
    const bool vec = aligned && n == kAdamVec && base + local + kAdamVec <= limit &&
                     (((base + local) | (gbase + local)) & 3) == 0;
    float x[kAdamVec], m[kAdamVec], v[kAdamVec], g[kAdamVec];
    if (vec) {
        const float4 xv = *reinterpret_cast<const float4*>(value + base + local);
        const float4 mv = *reinterpret_cast<const float4*>(mean + base + local);
        const float4 vv = *reinterpret_cast<const float4*>(variance + base + local);
        const float4 gv = __ldg(reinterpret_cast<const float4*>(gradient + gbase + local));
        x[0] = xv.x; x[1] = xv.y; x[2] = xv.z; x[3] = xv.w;
        m[0] = mv.x; m[1] = mv.y; m[2] = mv.z; m[3] = mv.w;
        v[0] = vv.x; v[1] = vv.y; v[2] = vv.z; v[3] = vv.w;
        g[0] = gv.x; g[1] = gv.y; g[2] = gv.z; g[3] = gv.w;
    }
    bool any = false;
    // Slot and channel of the first element with one 32-bit division (a run
    // holds fewer than 2^26 elements); the next three follow by carrying.
    int rel = (int)local / p.channels;
    int chan = (int)local - rel * p.channels;
#pragma unroll
    for (int k = 0; k < kAdamVec; k++) {
        if (k > 0 && ++chan == p.channels) {
            chan = 0;
            rel++;
        }
        if (k >= n) break;
        const int64_t e = local + k;
        const int64_t slot = first_slot + rel;
        if (slot >= p.capacity || __ldg(alive + slot) == 0) continue;
        if (!vec) {
            x[k] = value[base + e];
            m[k] = mean[base + e];
            v[k] = variance[base + e];
            g[k] = __ldg(gradient + gbase + e);
        }
        const float lr = p.is_sh && chan < 3 ? lr0 * 10.0f : lr0;
        adam_element(x[k], m[k], v[k], g[k], lr);
        any = true;
        if (!vec) {
            value[base + e] = x[k];
            mean[base + e] = m[k];
            variance[base + e] = v[k];
        }
    }
    // Dead slots inside a vector are stored back unchanged.
    if (vec && any) {
        *reinterpret_cast<float4*>(value + base + local) = make_float4(x[0], x[1], x[2], x[3]);
        *reinterpret_cast<float4*>(mean + base + local) = make_float4(m[0], m[1], m[2], m[3]);
        *reinterpret_cast<float4*>(variance + base + local) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// Each warp of sparse_adam_sh_kernel owns 32 consecutive slots of a listed
// cluster.  Phase 1, lane l: slot l's gradient ingredients into the warp's
// shared rows -- with one view the SH basis of its direction (16 floats) and
// its colour cotangent (3 floats); with several views the summed gradient
// row itself (sh_expand_views).  Phase 2: the lanes walk the warp's rows of
// value and moments as consecutive 16-byte vectors and update them.  With
// one view the gradient of element (coefficient q, channel c) is
// fmaf(Y_q, colour[c], 0), the first step of sh_expand_views, so the bits
// equal the expanded gradient's (an all-zero colour gives +0 either way).
constexpr int kShWarpSlots = 32;
constexpr int kShWarps = 4;
constexpr int kShOneView = 20;  // 16 basis values, 3 colour channels, a pad
constexpr int kShStride = 16 * 3 + 1;  // a whole gradient row, odd stride

template <int DEGREE, bool ONE_VIEW>
__global__ void __launch_bounds__(kShWarps * 32) sparse_adam_sh_kernel(
    gsb_adam_sh_params p, int64_t view_stride, int64_t center_stride, float* __restrict__ sh,
    float* __restrict__ mean, float* __restrict__ variance, const float* __restrict__ xyz,
    const float* __restrict__ centers, const float* __restrict__ colors,
    const int8_t* __restrict__ alive, const int32_t* __restrict__ cluster_ids,
    const int32_t* __restrict__ cluster_count, const float* __restrict__ rate)
{
    pdl_begin();
    constexpr int NB = (DEGREE + 1) * (DEGREE + 1);
    constexpr int kRow = ONE_VIEW ? kShOneView : kShStride;
    __shared__ float stage[kShWarps][kShWarpSlots * kRow];
    __shared__ int8_t live[kShWarps][kShWarpSlots];
    const int cluster = blockIdx.x;
    if (cluster >= __ldg(cluster_count)) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rel0 = (blockIdx.y * kShWarps + warp) * kShWarpSlots;
    if (rel0 >= p.cluster_size) return;
    const int64_t slot0 = (int64_t)__ldg(cluster_ids + cluster) * p.cluster_size + rel0;
    if (slot0 >= p.capacity) return;
    int64_t rows64 = p.cluster_size - rel0 < kShWarpSlots ? p.cluster_size - rel0 : kShWarpSlots;
    if (p.capacity - slot0 < rows64) rows64 = p.capacity - slot0;
    const int rows = (int)rows64;
    const int n = p.sh_dim * 3;
    float* st = stage[warp];
    if (lane < rows) {
        const int64_t slot = slot0 + lane;
        const bool ok = __ldg(alive + slot) != 0;
        live[warp][lane] = ok;
        const int64_t row = p.compact_colors ? (int64_t)cluster * p.cluster_size + rel0 + lane
                                             : slot;
        const float wx = __ldg(xyz + slot * 3), wy = __ldg(xyz + slot * 3 + 1),
                    wz = __ldg(xyz + slot * 3 + 2);
        float* dst = st + lane * kRow;
        if (ONE_VIEW) {
            float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f;
            float bas[16];
#pragma unroll
            for (int q = 0; q < 16; q++) bas[q] = 0.0f;
            if (ok) {
                c0 = __ldg(colors + row * 3);
                c1 = __ldg(colors + row * 3 + 1);
                c2 = __ldg(colors + row * 3 + 2);
                if (c0 != 0.0f || c1 != 0.0f || c2 != 0.0f)
                    sh_view_basis<DEGREE>(wx, wy, wz, centers, bas);
            }
#pragma unroll
            for (int q = 0; q < NB; q++) dst[q] = bas[q];
            dst[16] = c0;
            dst[17] = c1;
            dst[18] = c2;
        } else {
            float acc[NB * 3];
#pragma unroll
            for (int c = 0; c < NB * 3; c++) acc[c] = 0.0f;
            if (ok)
                sh_expand_views<DEGREE>(wx, wy, wz, p.views, colors + row * 3, view_stride,
                                        centers, center_stride, acc);
#pragma unroll
            for (int c = 0; c < NB * 3; c++) dst[c] = acc[c];
            for (int c = NB * 3; c < n; c++) dst[c] = 0.0f;
        }
    }
    __syncwarp();
    const float lr0 = __ldg(rate);
    const int total4 = rows * n / 4;  // n % 4 == 0 for this kernel
    float4* xs = reinterpret_cast<float4*>(sh + slot0 * n);
    float4* ms = reinterpret_cast<float4*>(mean + slot0 * n);
    float4* vs = reinterpret_cast<float4*>(variance + slot0 * n);
#pragma unroll 2
    for (int i = lane; i < total4; i += 32) {
        const int e = 4 * i;
        const int r = e / n;  // the vector's four elements share a row
        if (!live[warp][r]) continue;
        const int chan = e - r * n;
        const float* src = st + r * kRow;
        const float4 xv = xs[i], mv = ms[i], vv = vs[i];
        float x[4] = {xv.x, xv.y, xv.z, xv.w}, m[4] = {mv.x, mv.y, mv.z, mv.w},
              v[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
        for (int k = 0; k < kAdamVec; k++) {
            const int ch = chan + k;
            float g;
            if (ONE_VIEW) {
                const int q = ch / 3, c = ch - 3 * q;
                g = q < NB ? fmaf(src[q], src[16 + c], 0.0f) : 0.0f;
            } else {
                g = src[ch];
            }
            adam_element(x[k], m[k], v[k], g, ch < 3 ? lr0 * 10.0f : lr0);
        }
        xs[i] = make_float4(x[0], x[1], x[2], x[3]);
        ms[i] = make_float4(m[0], m[1], m[2], m[3]);
        vs[i] = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// Any row length and alignment: one thread per element, the row's gradient
// rebuilt whole (sh_expand_views) and the element's entry taken.
template <int DEGREE>
__global__ void __launch_bounds__(kAdamThreads) sparse_adam_sh_scalar_kernel(
    gsb_adam_sh_params p, int64_t view_stride, int64_t center_stride, float* __restrict__ sh,
    float* __restrict__ mean, float* __restrict__ variance, const float* __restrict__ xyz,
    const float* __restrict__ centers, const float* __restrict__ colors,
    const int8_t* __restrict__ alive, const int32_t* __restrict__ cluster_ids,
    const int32_t* __restrict__ cluster_count, const float* __restrict__ rate)
{
    pdl_begin();
    constexpr int NB = (DEGREE + 1) * (DEGREE + 1);
    const int cluster = blockIdx.x;
    if (cluster >= __ldg(cluster_count)) return;
    const int n = p.sh_dim * 3;
    const int64_t e = (int64_t)blockIdx.y * kAdamThreads + threadIdx.x;
    if (e >= (int64_t)p.cluster_size * n) return;
    const int rel = (int)(e / n), chan = (int)(e - (int64_t)rel * n);
    const int64_t slot = (int64_t)__ldg(cluster_ids + cluster) * p.cluster_size + rel;
    if (slot >= p.capacity || __ldg(alive + slot) == 0) return;
    const int64_t row = p.compact_colors ? (int64_t)cluster * p.cluster_size + rel : slot;
    float acc[48];
#pragma unroll
    for (int c = 0; c < 48; c++) acc[c] = 0.0f;
    sh_expand_views<DEGREE>(__ldg(xyz + slot * 3), __ldg(xyz + slot * 3 + 1),
                            __ldg(xyz + slot * 3 + 2), p.views, colors + row * 3, view_stride,
                            centers, center_stride, acc);
    const float g = chan < NB * 3 ? acc[chan] : 0.0f;
    const int64_t at = slot * n + chan;
    float x = sh[at], m = mean[at], v = variance[at];
    adam_element(x, m, v, g, chan < 3 ? __ldg(rate) * 10.0f : __ldg(rate));
    sh[at] = x;
    mean[at] = m;
    variance[at] = v;
}

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gsb_sparse_adam(gsb_stream_t stream, const gsb_adam_params* p, float* value,
                               float* mean, float* variance, const float* gradient,
                               const int8_t* alive, const int32_t* cluster_ids,
                               const int32_t* cluster_count, const float* rate)
{
    if (!p) return GSB_ERR_NULL;
    if (p->capacity < 0 || p->channels < 1 || p->cluster_size < 1 ||
        (int64_t)p->cluster_size * p->channels > (int64_t)65535 * kAdamThreads * kAdamVec)
        return GSB_ERR_INVALID;
    if (p->capacity == 0) return GSB_OK;
    if (!value || !mean || !variance || !gradient || !alive || !cluster_ids || !cluster_count ||
        !rate)
        return GSB_ERR_NULL;
    const int64_t run = (int64_t)p->cluster_size * p->channels;
    const int clusters = ceil_div(p->capacity, p->cluster_size);
    const int parts = ceil_div(run, (int64_t)kAdamThreads * kAdamVec);
    gsb::launch(sparse_adam_kernel, dim3(clusters, parts), kAdamThreads, 0, as_stream(stream), *p,
                value, mean, variance, gradient, alive, cluster_ids, cluster_count, rate);
    return check_launch();
}

extern "C" int gsb_sparse_adam_sh(gsb_stream_t stream, const gsb_adam_sh_params* p, float* sh,
                                  float* mean, float* variance, const float* xyz,
                                  const float* centers, const float* colors, const int8_t* alive,
                                  const int32_t* cluster_ids, const int32_t* cluster_count,
                                  const float* rate)
{
    if (!p) return GSB_ERR_NULL;
    if (p->capacity < 0 || p->sh_dim < 1 || p->sh_dim > 16 || p->degree < 0 || p->degree > 3 ||
        (p->degree + 1) * (p->degree + 1) > p->sh_dim || p->cluster_size < 1 || p->views < 0)
        return GSB_ERR_INVALID;
    const int64_t view_stride = p->view_stride ? p->view_stride : (int64_t)p->capacity * 3;
    const int64_t center_stride = p->center_stride ? p->center_stride : 3;
    if (center_stride < 3 || view_stride < 0) return GSB_ERR_INVALID;
    if (p->capacity == 0) return GSB_OK;
    if (!sh || !mean || !variance || !xyz || !alive || !cluster_ids || !cluster_count || !rate ||
        (p->views > 0 && (!centers || !colors)))
        return GSB_ERR_NULL;
    const int clusters = ceil_div(p->capacity, p->cluster_size);
    const int n = p->sh_dim * 3;
    const bool vec = (n & 3) == 0 &&
                     ((reinterpret_cast<uintptr_t>(sh) | reinterpret_cast<uintptr_t>(mean) |
                       reinterpret_cast<uintptr_t>(variance)) & 15) == 0;
    const int64_t run = (int64_t)p->cluster_size * n;
    const int64_t groups64 = ceil_div((int64_t)p->cluster_size, (int64_t)kShWarps * kShWarpSlots);
    if (groups64 > 65535 || ceil_div(run, (int64_t)kAdamThreads) > 65535) return GSB_ERR_INVALID;
    const int groups = (int)groups64;
    cudaStream_t s = as_stream(stream);
#define GSB_ADAM_SH(D)                                                                        \
    if (vec && p->views == 1)                                                                 \
        gsb::launch(sparse_adam_sh_kernel<D, true>, dim3(clusters, groups), kShWarps * 32, 0, \
                    s, *p, view_stride, center_stride, sh, mean, variance, xyz, centers,      \
                    colors, alive, cluster_ids, cluster_count, rate);                         \
    else if (vec)                                                                             \
        gsb::launch(sparse_adam_sh_kernel<D, false>, dim3(clusters, groups), kShWarps * 32,   \
                    0, s, *p, view_stride, center_stride, sh, mean, variance, xyz, centers,   \
                    colors, alive, cluster_ids, cluster_count, rate);                         \
    else                                                                                      \
        gsb::launch(sparse_adam_sh_scalar_kernel<D>,                                          \
                    dim3(clusters, (int)ceil_div(run, (int64_t)kAdamThreads)), kAdamThreads,  \
                    0, s, *p, view_stride, center_stride, sh, mean, variance, xyz, centers,   \
                    colors, alive, cluster_ids, cluster_count, rate)
    switch (p->degree) {
        case 0: GSB_ADAM_SH(0); break;
        case 1: GSB_ADAM_SH(1); break;
        case 2: GSB_ADAM_SH(2); break;
        default: GSB_ADAM_SH(3); break;
    }
#undef GSB_ADAM_SH
    return check_launch();
}
