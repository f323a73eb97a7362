// fp32 tile rasterization forward / backward for sm_100a.
//
// Semantics: kernels/sorted_rasterize.py:28-236 (per-pixel front-to-back
// compositing, alpha = min(o*exp(power), 255/256) when >= 1/256 and
// power <= 0, early stop once T < 1/8192, backward from the pixel's last
// composited pair), on rectangular tile_w x tile_h tiles.
//
// Work decomposition (B200-first, not the reference's): one CTA per tile,
// one warp per 8x4 block of the tile, one pixel per lane.  Warps walk the
// tile's pair list in 32-pair batches; each lane stages one 48-byte splat
// record and tests the splat's conservative 1/256-level bounding box against
// its warp's 8x4 block, so a warp skips (with one ballot) every splat that
// cannot give any of its pixels alpha >= 1/256 — the result is identical to
// visiting them.  Warps stop independently once all their pixels are
// saturated.  The backward reduces each splat's nine gradients with a
// transposed butterfly (8 values in 9 shuffles + 1 in 5) and issues one
// float atomic per value per warp.
//
// The power is computed with the exact operation sequence of the host
// oracle (pre-scaled conic, fmaf form), so only exp differs between them.
#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr float kMinAlpha = 1.0f / 256.0f;
constexpr float kMaxAlpha = 255.0f / 256.0f;
constexpr float kMinT = 1.0f / 8192.0f;

// Record layout (3 x float4 per Gaussian):
//   r0 = (mean_x, mean_y, ext_x, ext_y)   ext: bbox half extents at 1/256
//   r1 = (-c00/2, -c01/2, -c10/2, -c11/2)
//   r2 = (red, green, blue, opacity)
// ext_x = -inf marks a splat that can never reach alpha 1/256; +inf one whose
// conic is not positive definite (never skipped).
__global__ void pack_kernel(int64_t capacity, const float* __restrict__ mean,
                            const float* __restrict__ conic, const float* __restrict__ color,
                            const float* __restrict__ alpha, const int8_t* __restrict__ visible,
                            float4* __restrict__ splats)
{
    int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= capacity || visible[g] == 0) return;
    float2 m = *reinterpret_cast<const float2*>(mean + g * 2);
    float4 c = *reinterpret_cast<const float4*>(conic + g * 4);
    float o = alpha[g];
    float ex, ey;
    float b = 0.5f * (c.y + c.z);
    float det = c.x * c.w - b * b;
    if (!(o * 256.0f >= 0.99999f)) {
        ex = ey = -__int_as_float(0x7f800000);
    } else if (!(c.x > 0.0f && c.w > 0.0f && det > 0.0f)) {
        ex = ey = __int_as_float(0x7f800000);
    } else {
        // q = d^T C d <= level  <=>  o * exp(-q/2) >= 1/256; 0.1% + margin.
        float level = 2.0f * logf(fmaxf(o * 256.0f, 1.0f)) * 1.001f + 1e-3f;
        ex = sqrtf(level * c.w / det) * 1.0005f + 1e-3f;
        ey = sqrtf(level * c.x / det) * 1.0005f + 1e-3f;
    }
    float4* r = splats + g * 3;
    r[0] = make_float4(m.x, m.y, ex, ey);
    r[1] = make_float4(-0.5f * c.x, -0.5f * c.y, -0.5f * c.z, -0.5f * c.w);
    r[2] = make_float4(color[g * 3], color[g * 3 + 1], color[g * 3 + 2], o);
}

// Heaviest-first tile permutation: counting sort into 256 buckets, eight per
// octave of (work + 1) (kernels/packed_rasterize.py:38-89 describes the same
// bucketing); order inside a bucket is unspecified.
constexpr int kOrderThreads = 1024;
constexpr int kOrderBuckets = 256;

__device__ __forceinline__ int work_bucket(int64_t work)
{
    float f = (float)(work < 0 ? 1 : work + 1);
    int b = (int)(__float_as_uint(f) >> 20) - (127 << 3);
    b = max(0, min(kOrderBuckets - 1, b));
    return kOrderBuckets - 1 - b;
}

__global__ void __launch_bounds__(kOrderThreads) order_tiles_kernel(const int32_t* __restrict__ work,
                                                                    int tiles, int from_offsets,
                                                                    int32_t* __restrict__ order)
{
    __shared__ int starts[kOrderBuckets];
    int tid = threadIdx.x;
    if (tid < kOrderBuckets) starts[tid] = 0;
    __syncthreads();
    for (int t = tid; t < tiles; t += kOrderThreads) {
        int64_t w = from_offsets ? (int64_t)work[t + 1] - work[t] : work[t];
        atomicAdd(&starts[work_bucket(w)], 1);
    }
    __syncthreads();
    if (tid < 32) {
        int per = kOrderBuckets / 32;
        int total = 0;
        for (int i = 0; i < per; i++) total += starts[tid * per + i];
        int inc = warp_inclusive_scan(total, tid);
        int running = inc - total;
        for (int i = 0; i < per; i++) {
            int c = starts[tid * per + i];
            starts[tid * per + i] = running;
            running += c;
        }
    }
    __syncthreads();
    for (int t = tid; t < tiles; t += kOrderThreads) {
        int64_t w = from_offsets ? (int64_t)work[t + 1] - work[t] : work[t];
        int pos = atomicAdd(&starts[work_bucket(w)], 1);
        order[pos] = t;
    }
}

struct TileGeom {
    int tile, tx0, ty0;     // tile id and pixel origin
    int bx0, by0;           // this warp's 8x4 block origin (pixels)
    int px, py;             // this lane's pixel
    bool in_image;
};

__device__ __forceinline__ TileGeom tile_geom(const gsb_raster_params& p, int tile, int warp,
                                              int lane)
{
    TileGeom t;
    int tiles_x = (p.width + p.tile_w - 1) / p.tile_w;
    t.tile = tile;
    t.tx0 = (tile % tiles_x) * p.tile_w;
    t.ty0 = (tile / tiles_x) * p.tile_h;
    int blocks_x = p.tile_w / 8;
    t.bx0 = t.tx0 + (warp % blocks_x) * 8;
    t.by0 = t.ty0 + (warp / blocks_x) * 4;
    t.px = t.bx0 + (lane & 7);
    t.py = t.by0 + (lane >> 3);
    t.in_image = t.px < p.width && t.py < p.height;
    return t;
}

// Can the splat reach alpha >= 1/256 at any pixel centre of the 8x4 block?
__device__ __forceinline__ bool block_hit(float4 r0, float bx0, float by0)
{
    return r0.x - r0.z <= bx0 + 7.5f && r0.x + r0.z >= bx0 + 0.5f && r0.y - r0.w <= by0 + 3.5f &&
           r0.y + r0.w >= by0 + 0.5f;
}

// Power (= -q/2) with the oracle's operation sequence.
__device__ __forceinline__ float power_of(float4 r1, float dx, float dy)
{
    float t1 = __fmaf_rn(r1.x, dx, __fmul_rn(r1.y, dy));
    float t2 = __fmaf_rn(r1.z, dx, __fmul_rn(r1.w, dy));
    return __fmaf_rn(dx, t1, __fmul_rn(dy, t2));
}

struct Stash {
    float4 r0[32], r1[32], r2[32];
    float depth[32];
};

template <bool WANT_DEPTH>
__global__ void __launch_bounds__(256) raster_fwd_kernel(
    gsb_raster_params p, const float4* __restrict__ splats, const float* __restrict__ depth,
    const int32_t* __restrict__ ids, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ order, const float* __restrict__ background,
    float* __restrict__ rgb, float* __restrict__ out_depth, float* __restrict__ out_alpha,
    float* __restrict__ final_t, int32_t* __restrict__ last_out,
    int32_t* __restrict__ backward_work)
{
    extern __shared__ Stash stash_all[];
    __shared__ int tile_work;
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Stash& st = stash_all[warp];
    int tile = order[blockIdx.x];
    TileGeom tg = tile_geom(p, tile, warp, lane);
    if (threadIdx.x == 0) tile_work = 0;
    int32_t start = offsets[tile], end = offsets[tile + 1];
    float pcx = (float)tg.px + 0.5f, pcy = (float)tg.py + 0.5f;
    float bx0 = (float)tg.bx0, by0 = (float)tg.by0;
    float T = 1.0f, cr = 0.0f, cg = 0.0f, cb = 0.0f, cd = 0.0f;
    int32_t last = end;
    bool done = !tg.in_image;
    for (int32_t base = start; base < end; base += 32) {
        if (__all_sync(GSB_FULL_MASK, done)) break;
        int32_t i = base + lane;
        bool hit = false;
        if (i < end) {
            int32_t g = __ldg(ids + i);
            const float4* rec = splats + (int64_t)g * 3;
            float4 r0 = __ldg(rec);
            hit = block_hit(r0, bx0, by0);
            if (hit) {
                st.r0[lane] = r0;
                st.r1[lane] = __ldg(rec + 1);
                st.r2[lane] = __ldg(rec + 2);
                if (WANT_DEPTH) st.depth[lane] = __ldg(depth + g);
            }
        }
        unsigned mask = __ballot_sync(GSB_FULL_MASK, hit);
        __syncwarp();
        while (mask) {
            int k = __ffs(mask) - 1;
            mask &= mask - 1;
            float4 r0 = st.r0[k], r1 = st.r1[k], r2 = st.r2[k];
            float dx = pcx - r0.x, dy = pcy - r0.y;
            float power = power_of(r1, dx, dy);
            float raw = r2.w * __expf(power);
            if (!done && power <= 0.0f && raw >= kMinAlpha) {
                float a = fminf(kMaxAlpha, raw);
                float w = a * T;
                cr = __fmaf_rn(w, r2.x, cr);
                cg = __fmaf_rn(w, r2.y, cg);
                cb = __fmaf_rn(w, r2.z, cb);
                if (WANT_DEPTH) cd = __fmaf_rn(w, st.depth[k], cd);
                T = T * (1.0f - a);
                if (T < kMinT) {
                    done = true;
                    last = base + k + 1;
                }
            }
            if (__all_sync(GSB_FULL_MASK, done)) break;
        }
        __syncwarp();
    }
    if (tg.in_image) {
        int64_t pix = (int64_t)tg.py * p.width + tg.px;
        rgb[pix * 3] = cr + T * __ldg(background);
        rgb[pix * 3 + 1] = cg + T * __ldg(background + 1);
        rgb[pix * 3 + 2] = cb + T * __ldg(background + 2);
        if (out_depth) out_depth[pix] = cd;
        if (out_alpha) out_alpha[pix] = 1.0f - T;
        final_t[pix] = T;
        last_out[pix] = last;
    }
    int work = tg.in_image ? last - start : 0;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) work = max(work, __shfl_xor_sync(GSB_FULL_MASK, work, d));
    __syncthreads();
    if (lane == 0) atomicMax(&tile_work, work);
    __syncthreads();
    if (threadIdx.x == 0) backward_work[tile] = tile_work;
}

// Transposed butterfly over 8 values: afterwards lane l holds the warp sum
// of value (l >> 2).  9 shuffles instead of 8 x 5.
__device__ __forceinline__ float warp_sum8(float v[8], int lane)
{
    bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        float keep = b4 ? v[j + 4] : v[j];
        float send = b4 ? v[j] : v[j + 4];
        v[j] = keep + __shfl_xor_sync(GSB_FULL_MASK, send, 16);
    }
#pragma unroll
    for (int j = 0; j < 2; j++) {
        float keep = b3 ? v[j + 2] : v[j];
        float send = b3 ? v[j] : v[j + 2];
        v[j] = keep + __shfl_xor_sync(GSB_FULL_MASK, send, 8);
    }
    {
        float keep = b2 ? v[1] : v[0];
        float send = b2 ? v[0] : v[1];
        v[0] = keep + __shfl_xor_sync(GSB_FULL_MASK, send, 4);
    }
    float s = v[0];
    s += __shfl_xor_sync(GSB_FULL_MASK, s, 2);
    s += __shfl_xor_sync(GSB_FULL_MASK, s, 1);
    return s;
}

template <bool WANT_DEPTH>
__global__ void __launch_bounds__(256) raster_bwd_kernel(
    gsb_raster_bwd_params p, const float4* __restrict__ splats, const float* __restrict__ depth,
    const int32_t* __restrict__ ids, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ order, const float* __restrict__ background,
    const float* __restrict__ final_t, const int32_t* __restrict__ last_in,
    const float* __restrict__ drgb, const float* __restrict__ ddepth,
    const float* __restrict__ dalpha, float* __restrict__ gmean, float* __restrict__ gconic,
    float* __restrict__ gdepth, float* __restrict__ gcolor, float* __restrict__ galpha)
{
    extern __shared__ Stash stash_all[];
    __shared__ int32_t stash_id[8][32];
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Stash& st = stash_all[warp];
    int tile = order[blockIdx.x];
    gsb_raster_params rp{p.capacity, p.width, p.height, p.tile_w, p.tile_h};
    TileGeom tg = tile_geom(rp, tile, warp, lane);
    int32_t start = offsets[tile];
    float pcx = (float)tg.px + 0.5f, pcy = (float)tg.py + 0.5f;
    float bx0 = (float)tg.bx0, by0 = (float)tg.by0;
    float gR = 0.0f, gG = 0.0f, gB = 0.0f, gD = 0.0f, gtrans = 0.0f, T_after = 1.0f;
    int32_t last = start;
    if (tg.in_image) {
        int64_t pix = (int64_t)tg.py * p.width + tg.px;
        last = last_in[pix];
        gR = drgb[pix * 3];
        gG = drgb[pix * 3 + 1];
        gB = drgb[pix * 3 + 2];
        if (WANT_DEPTH) gD = ddepth ? ddepth[pix] : 0.0f;
        gtrans = gR * __ldg(background) + gG * __ldg(background + 1) + gB * __ldg(background + 2) -
                 (dalpha ? dalpha[pix] : 0.0f);
        T_after = final_t[pix];
    }
    int32_t top = last;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) top = max(top, __shfl_xor_sync(GSB_FULL_MASK, top, d));
    // Walk batches [base, chunk_end) from the end back to the tile start.
    for (int32_t chunk_end = top; chunk_end > start; chunk_end -= 32) {
        int32_t base = max(start, chunk_end - 32);
        int32_t i = base + lane;
        bool hit = false;
        if (i < chunk_end) {
            int32_t g = __ldg(ids + i);
            const float4* rec = splats + (int64_t)g * 3;
            float4 r0 = __ldg(rec);
            hit = block_hit(r0, bx0, by0);
            if (hit) {
                st.r0[lane] = r0;
                st.r1[lane] = __ldg(rec + 1);
                st.r2[lane] = __ldg(rec + 2);
                stash_id[warp][lane] = g;
                if (WANT_DEPTH) st.depth[lane] = __ldg(depth + g);
            }
        }
        unsigned mask = __ballot_sync(GSB_FULL_MASK, hit);
        __syncwarp();
        while (mask) {
            int k = 31 - __clz(mask);
            mask &= ~(1u << k);
            int32_t idx = base + k;
            float4 r0 = st.r0[k], r1 = st.r1[k], r2 = st.r2[k];
            float dx = pcx - r0.x, dy = pcy - r0.y;
            float power = power_of(r1, dx, dy);
            float e = __expf(power);
            float raw = r2.w * e;
            bool contrib = idx < last && power <= 0.0f && raw >= kMinAlpha;
            float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            float go = 0.0f, gz = 0.0f;
            if (contrib) {
                float a = fminf(kMaxAlpha, raw);
                float one_minus = 1.0f - a;
                float T_before = __fdividef(T_after, one_minus);
                float w = T_before * a;
                float gw = gR * r2.x + gG * r2.y + gB * r2.z;
                if (WANT_DEPTH) gw += gD * st.depth[k];
                float ga = T_before * (gw - gtrans);
                gtrans = a * gw + one_minus * gtrans;
                v[5] = w * gR;
                v[6] = w * gG;
                v[7] = w * gB;
                if (WANT_DEPTH) gz = w * gD;
                if (raw < kMaxAlpha) {
                    float ge = ga * raw;
                    go = ga * e;
                    // r1 holds -c/2: c00*dx + cbar*dy = -2 (r1.x dx + rbar dy).
                    float rbar = 0.5f * (r1.y + r1.z);
                    float m0 = __fmaf_rn(r1.x, dx, rbar * dy);
                    float m1 = __fmaf_rn(r1.w, dy, rbar * dx);
                    v[0] = -2.0f * ge * m0;
                    v[1] = -2.0f * ge * m1;
                    float h = -0.5f * ge;
                    v[2] = h * dx * dx;
                    v[3] = h * dx * dy;
                    v[4] = h * dy * dy;
                }
                T_after = T_before;
            }
            if (__any_sync(GSB_FULL_MASK, contrib)) {
                int64_t g = stash_id[warp][k];
                float s = warp_sum8(v, lane);
                go = warp_sum(go);
                if (WANT_DEPTH) gz = warp_sum(gz);
                int which = lane >> 2, role = lane & 3;
                if (role == 0) {
                    float* dst = which < 2 ? gmean + g * 2 + which
                                 : which < 5 ? gconic + g * 4 + (which == 2 ? 0 : which == 3 ? 1 : 3)
                                             : gcolor + g * 3 + (which - 5);
                    atomicAdd(dst, s);
                } else if (role == 1 && which == 3) {
                    atomicAdd(gconic + g * 4 + 2, s);
                } else if (lane == 1) {
                    atomicAdd(galpha + g, go);
                } else if (WANT_DEPTH && lane == 2) {
                    atomicAdd(gdepth + g, gz);
                }
            }
        }
        __syncwarp();
    }
}

__global__ void zero_cotangents_kernel(int64_t capacity, float* gmean, float* gconic, float* gdepth,
                                       float* gcolor, float* galpha)
{
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= capacity) return;
    *reinterpret_cast<float2*>(gmean + i * 2) = make_float2(0.f, 0.f);
    *reinterpret_cast<float4*>(gconic + i * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
    gcolor[i * 3] = gcolor[i * 3 + 1] = gcolor[i * 3 + 2] = 0.0f;
    galpha[i] = 0.0f;
    if (gdepth) gdepth[i] = 0.0f;
}

// kernels/packed_rasterize.py:619-645: zero only the listed clusters' slots.
__global__ void zero_cluster_cotangents_kernel(int64_t capacity, int cluster_size,
                                               const int32_t* __restrict__ ids,
                                               const int32_t* __restrict__ count, float* gmean,
                                               float* gconic, float* gcolor, float* galpha)
{
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)(*count) * cluster_size) return;
    int64_t g = (int64_t)ids[i / cluster_size] * cluster_size + i % cluster_size;
    if (g >= capacity) return;
    *reinterpret_cast<float2*>(gmean + g * 2) = make_float2(0.f, 0.f);
    *reinterpret_cast<float4*>(gconic + g * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
    gcolor[g * 3] = gcolor[g * 3 + 1] = gcolor[g * 3 + 2] = 0.0f;
    galpha[g] = 0.0f;
}

bool tiles_ok(int tile_w, int tile_h)
{
    return tile_w > 0 && tile_h > 0 && tile_w % 8 == 0 && tile_h % 4 == 0 &&
           (tile_w / 8) * (tile_h / 4) <= 8;
}

size_t raster_ws(const gsb_raster_params& p)
{
    int64_t tiles = (int64_t)ceil_div(p.width, p.tile_w) * ceil_div(p.height, p.tile_h);
    return ((size_t)tiles * sizeof(int32_t) + 255) & ~size_t(255);
}

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" size_t gsb_raster_workspace_size(const gsb_raster_params* p)
{
    return p ? raster_ws(*p) : 0;
}

extern "C" int gsb_raster_fwd(gsb_stream_t stream, const gsb_raster_params* p, void* workspace,
                              size_t workspace_bytes, const float* mean, const float* conic,
                              const float* depth, const float* color, const float* alpha,
                              const int8_t* visible, const int32_t* gaussian_ids,
                              const int32_t* tile_offsets, const float* background, float* rgb,
                              float* out_depth, float* out_alpha, float* final_t, int32_t* last,
                              int32_t* backward_work, float* splats)
{
    if (!p) return GSB_ERR_NULL;
    if (p->capacity < 0 || p->width <= 0 || p->height <= 0 || !tiles_ok(p->tile_w, p->tile_h))
        return GSB_ERR_INVALID;
    if (!workspace || workspace_bytes < raster_ws(*p)) return GSB_ERR_WORKSPACE;
    if (!gaussian_ids || !tile_offsets || !background || !rgb || !final_t || !last ||
        !backward_work || !splats ||
        (p->capacity > 0 && (!mean || !conic || !color || !alpha || !visible)) ||
        (out_depth && !depth))
        return GSB_ERR_NULL;
    if ((reinterpret_cast<uintptr_t>(splats) | reinterpret_cast<uintptr_t>(conic)) & 15)
        return GSB_ERR_INVALID;
    cudaStream_t s = as_stream(stream);
    int tiles = ceil_div(p->width, p->tile_w) * ceil_div(p->height, p->tile_h);
    int32_t* order = static_cast<int32_t*>(workspace);
    if (p->capacity > 0) {
        pack_kernel<<<ceil_div(p->capacity, 256), 256, 0, s>>>(p->capacity, mean, conic, color,
                                                               alpha, visible,
                                                               reinterpret_cast<float4*>(splats));
        if (int e = check_launch()) return e;
    }
    order_tiles_kernel<<<1, kOrderThreads, 0, s>>>(tile_offsets, tiles, 1, order);
    if (int e = check_launch()) return e;
    int warps = (p->tile_w / 8) * (p->tile_h / 4);
    size_t smem = (size_t)warps * sizeof(Stash);
    if (out_depth)
        raster_fwd_kernel<true><<<tiles, warps * 32, smem, s>>>(
            *p, reinterpret_cast<const float4*>(splats), depth, gaussian_ids, tile_offsets, order,
            background, rgb, out_depth, out_alpha, final_t, last, backward_work);
    else
        raster_fwd_kernel<false><<<tiles, warps * 32, smem, s>>>(
            *p, reinterpret_cast<const float4*>(splats), depth, gaussian_ids, tile_offsets, order,
            background, rgb, out_depth, out_alpha, final_t, last, backward_work);
    return check_launch();
}

extern "C" int gsb_raster_bwd(gsb_stream_t stream, const gsb_raster_bwd_params* p,
                              void* workspace, size_t workspace_bytes, const float* splats,
                              const float* depth, const int32_t* gaussian_ids,
                              const int32_t* tile_offsets, const float* background,
                              const float* final_t, const int32_t* last,
                              const int32_t* backward_work, const float* drgb,
                              const float* ddepth, const float* dalpha,
                              const int32_t* cluster_ids, const int32_t* cluster_count,
                              float* gmean, float* gconic, float* gdepth, float* gcolor,
                              float* galpha)
{
    if (!p) return GSB_ERR_NULL;
    gsb_raster_params rp{p->capacity, p->width, p->height, p->tile_w, p->tile_h};
    if (p->capacity < 0 || p->width <= 0 || p->height <= 0 || !tiles_ok(p->tile_w, p->tile_h))
        return GSB_ERR_INVALID;
    if (!workspace || workspace_bytes < raster_ws(rp)) return GSB_ERR_WORKSPACE;
    if (!splats || !gaussian_ids || !tile_offsets || !background || !final_t || !last ||
        !backward_work || !drgb || !gmean || !gconic || !gcolor || !galpha)
        return GSB_ERR_NULL;
    bool want_depth = ddepth != nullptr;
    if (want_depth && (!depth || !gdepth)) return GSB_ERR_NULL;
    if (cluster_ids && (!cluster_count || p->cluster_size <= 0)) return GSB_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(splats) | reinterpret_cast<uintptr_t>(gconic)) & 15)
        return GSB_ERR_INVALID;
    cudaStream_t s = as_stream(stream);
    int tiles = ceil_div(p->width, p->tile_w) * ceil_div(p->height, p->tile_h);
    int32_t* order = static_cast<int32_t*>(workspace);
    if (p->capacity > 0) {
        if (cluster_ids) {
            zero_cluster_cotangents_kernel<<<ceil_div(p->capacity, 256), 256, 0, s>>>(
                p->capacity, p->cluster_size, cluster_ids, cluster_count, gmean, gconic, gcolor,
                galpha);
        } else {
            zero_cotangents_kernel<<<ceil_div(p->capacity, 256), 256, 0, s>>>(
                p->capacity, gmean, gconic, gdepth, gcolor, galpha);
        }
        if (int e = check_launch()) return e;
    }
    order_tiles_kernel<<<1, kOrderThreads, 0, s>>>(backward_work, tiles, 0, order);
    if (int e = check_launch()) return e;
    int warps = (p->tile_w / 8) * (p->tile_h / 4);
    size_t smem = (size_t)warps * sizeof(Stash);
    const float4* sp = reinterpret_cast<const float4*>(splats);
    if (want_depth)
        raster_bwd_kernel<true><<<tiles, warps * 32, smem, s>>>(
            *p, sp, depth, gaussian_ids, tile_offsets, order, background, final_t, last, drgb,
            ddepth, dalpha, gmean, gconic, gdepth, gcolor, galpha);
    else
        raster_bwd_kernel<false><<<tiles, warps * 32, smem, s>>>(
            *p, sp, depth, gaussian_ids, tile_offsets, order, background, final_t, last, drgb,
            ddepth, dalpha, gmean, gconic, gdepth, gcolor, galpha);
    return check_launch();
}
