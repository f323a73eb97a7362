// Consumers of the fragment statistics and the opacity reset of LiteGS
// density control (training/densify.py:20-35, :158-165), elementwise over
// the pool (sm_100a).
//  * densify_scores_kernel: per slot, from (count n, weight w, sum s, squared
//    sum q) of the fragment statistics, the opacity-weighted gradient
//    variance score max(q/(n+1) - (s/(n+1))^2, 0) * n * sigmoid(o)^2 (0 for
//    dead slots and non-finite values) and the prune flag alive & w == 0.
//  * decay_opacity_kernel: alive slots' opacity logits become
//    logit(max(sigmoid(o) / 2, 1/128)).
#include "gsb_common.cuh"

namespace gsb {
namespace {

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

__global__ void densify_scores_kernel(int64_t capacity, const float4* __restrict__ stats,
                                      const float* __restrict__ opacity,
                                      const int8_t* __restrict__ alive, float* __restrict__ scores,
                                      int8_t* __restrict__ prune)
{
    pdl_begin();
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= capacity) return;
    const float4 st = stats[g];
    const bool live = alive[g] != 0;
    const float n1 = st.x + 1.0f;
    const float mean = st.z / n1;
    const float variance = fmaxf(st.w / n1 - mean * mean, 0.0f);
    const float a = sigmoid(opacity[g]);
    float score = variance * st.x * (a * a);
    if (!isfinite(score)) score = 0.0f;
    scores[g] = live ? score : 0.0f;
    prune[g] = live && st.y == 0.0f ? 1 : 0;
}

__global__ void decay_opacity_kernel(int64_t capacity, float* __restrict__ opacity,
                                     const int8_t* __restrict__ alive)
{
    pdl_begin();
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= capacity || alive[g] == 0) return;
    const float a = fmaxf(sigmoid(opacity[g]) * 0.5f, 1.0f / 128.0f);
    opacity[g] = logf(a / (1.0f - a));
}

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gsb_densify_scores(gsb_stream_t stream, int64_t capacity, const float* stats,
                                  const float* opacity, const int8_t* alive, float* scores,
                                  int8_t* prune)
{
    if (capacity < 0) return GSB_ERR_INVALID;
    if (capacity == 0) return GSB_OK;
    if (!stats || !opacity || !alive || !scores || !prune) return GSB_ERR_NULL;
    if (reinterpret_cast<uintptr_t>(stats) & 15) return GSB_ERR_INVALID;
    gsb::launch(densify_scores_kernel, ceil_div(capacity, 256), 256, 0, as_stream(stream),
                capacity, reinterpret_cast<const float4*>(stats), opacity, alive, scores, prune);
    return check_launch();
}

extern "C" int gsb_decay_opacity(gsb_stream_t stream, int64_t capacity, float* opacity,
                                 const int8_t* alive)
{
    if (capacity < 0) return GSB_ERR_INVALID;
    if (capacity == 0) return GSB_OK;
    if (!opacity || !alive) return GSB_ERR_NULL;
    gsb::launch(decay_opacity_kernel, ceil_div(capacity, 256), 256, 0, as_stream(stream), capacity,
                opacity, alive);
    return check_launch();
}
