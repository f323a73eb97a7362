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
#include "gsb_common.cuh"

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
