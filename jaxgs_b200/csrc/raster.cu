// fp32 tile rasterization forward / backward for sm_100a.
//
// Semantics: kernels/sorted_rasterize.py:28-236 (per-pixel front-to-back
// compositing, alpha = min(o*exp(power), 255/256) when >= 1/256 and
// power <= 0, early stop once T < 1/8192, backward from the pixel's last
// composited pair), on rectangular tile_w x tile_h tiles.
//
// Work decomposition (B200-first, not the reference's): one CTA per tile, one
// warp per 8 x (4*ROWS) pixel block, ROWS vertically adjacent pixels per lane
// (ROWS = 2 when tile_h is a multiple of 8, else 1).
//  * Forward: a warp walks the tile's pairs in 32-pair batches; each lane
//    stages one 48-byte splat record and tests the splat's conservative
//    1/256-level bounding box, then the ellipse itself (ellipse_hit), against
//    the warp's block, so one ballot skips every splat that cannot reach the
//    block.  Warps stop independently once
//    all their pixels are saturated, and record per batch a 32-bit word of
//    the pairs that composited at least one fragment of the block.
//  * Backward: a warp reads those words from its top pair down and visits
//    only the set bits (exact pruning), recomputing each fragment in reverse.
//    Per splat every lane accumulates moments of its pixels' power gradients
//    (sum ge, ge*dy, ge*dy^2; the lane's column fixes dx) and colour
//    gradients; the moments of two contributing splats are reduced together
//    by one 16-value transposed butterfly, and one predicated RED per warp
//    adds both splats' cotangents.
//
// The power is evaluated with the host oracle's operation order (the conic
// scaled by -1/2, shared c00*dx / c10*dx, fused dy terms), so it is
// bit-identical; only exp differs (__expf here, libm there).
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
__host__ __device__ __forceinline__ void pack_record(float2 m, float4 c, float o, float red,
                                                    float green, float blue, float4 r[3])
{
    float ex, ey;
    float b = 0.5f * (c.y + c.z);
    float det = c.x * c.w - b * b;
    if (!(o * 256.0f >= 0.99999f)) {
        ex = ey = -INFINITY;
    } else if (!(c.x > 0.0f && c.w > 0.0f && det > 0.0f)) {
        ex = ey = INFINITY;
    } else {
        // q = d^T C d <= level  <=>  o * exp(-q/2) >= 1/256; 0.1% + margin.
        float level = 2.0f * logf(fmaxf(o * 256.0f, 1.0f)) * 1.001f + 1e-3f;
        ex = sqrtf(level * c.w / det) * 1.0005f + 1e-3f;
        ey = sqrtf(level * c.x / det) * 1.0005f + 1e-3f;
    }
    r[0] = make_float4(m.x, m.y, ex, ey);
    r[1] = make_float4(-0.5f * c.x, -0.5f * c.y, -0.5f * c.z, -0.5f * c.w);
    r[2] = make_float4(red, green, blue, o);
}

__global__ void pack_kernel(int64_t capacity, const float* __restrict__ mean,
                            const float* __restrict__ conic, const float* __restrict__ color,
                            const float* __restrict__ alpha, const int8_t* __restrict__ visible,
                            float4* __restrict__ splats)
{
    pdl_begin();
    int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= capacity || visible[g] == 0) return;
    float4 r[3];
    pack_record(*reinterpret_cast<const float2*>(mean + g * 2),
                *reinterpret_cast<const float4*>(conic + g * 4), alpha[g], color[g * 3],
                color[g * 3 + 1], color[g * 3 + 2], r);
    float4* out = splats + g * 3;
    out[0] = r[0];
    out[1] = r[1];
    out[2] = r[2];
}

// Heaviest-first tile permutation: counting sort into 256 buckets, eight per
// octave of (work + 1) (the bucketing of kernels/packed_rasterize.py:38-89);
// order inside a bucket is unspecified.
constexpr int kOrderThreads = 1024;
constexpr int kOrderBuckets = 256;

__device__ __forceinline__ int work_bucket(int64_t work)
{
    float f = (float)(work < 0 ? 1 : work + 1);
    int b = (int)(__float_as_uint(f) >> 20) - (127 << 3);
    b = max(0, min(kOrderBuckets - 1, b));
    return kOrderBuckets - 1 - b;
}

// Tiles are taken 8 per thread per round (round r, thread t: tiles
// r*8192 + j*1024 + t); a round's loads are issued before its atomics so
// their latencies overlap, and one round's buckets stay in registers for the
// scatter (larger images reload theirs).
constexpr int kOrderPerThread = 8;

__device__ __forceinline__ void order_round_buckets(const int32_t* __restrict__ work, int tiles,
                                                    int from_offsets, int round, int bucket[])
{
    int64_t w[kOrderPerThread];
#pragma unroll
    for (int j = 0; j < kOrderPerThread; j++) {
        const int t = round * kOrderThreads * kOrderPerThread + j * kOrderThreads + threadIdx.x;
        w[j] = t < tiles ? (from_offsets ? (int64_t)work[t + 1] - work[t] : (int64_t)work[t]) : 0;
    }
#pragma unroll
    for (int j = 0; j < kOrderPerThread; j++) {
        const int t = round * kOrderThreads * kOrderPerThread + j * kOrderThreads + threadIdx.x;
        bucket[j] = t < tiles ? work_bucket(w[j]) : -1;
    }
}

__global__ void __launch_bounds__(kOrderThreads) order_tiles_kernel(const int32_t* __restrict__ work,
                                                                    int tiles, int from_offsets,
                                                                    int32_t* __restrict__ order)
{
    pdl_begin();
    __shared__ int starts[kOrderBuckets];
    const int tid = threadIdx.x;
    const int rounds = (tiles + kOrderThreads * kOrderPerThread - 1) / (kOrderThreads * kOrderPerThread);
    if (tid < kOrderBuckets) starts[tid] = 0;
    __syncthreads();
    int bucket[kOrderPerThread];
    for (int r = 0; r < rounds; r++) {
        order_round_buckets(work, tiles, from_offsets, r, bucket);
#pragma unroll
        for (int j = 0; j < kOrderPerThread; j++)
            if (bucket[j] >= 0) atomicAdd(&starts[bucket[j]], 1);
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
    for (int r = 0; r < rounds; r++) {
        if (rounds > 1) order_round_buckets(work, tiles, from_offsets, r, bucket);
#pragma unroll
        for (int j = 0; j < kOrderPerThread; j++) {
            if (bucket[j] < 0) continue;
            const int t = r * kOrderThreads * kOrderPerThread + j * kOrderThreads + tid;
            order[atomicAdd(&starts[bucket[j]], 1)] = t;
        }
    }
}

template <int ROWS>
struct Geom {
    int tile;
    int bx0, by0;  // block origin (pixels)
    int px;        // lane column
    int py0;       // lane's first row
};

template <int ROWS>
__device__ __forceinline__ Geom<ROWS> geom(int width, int tile_w, int tile_h, int tile, int warp,
                                           int lane)
{
    Geom<ROWS> t;
    int tiles_x = (width + tile_w - 1) / tile_w;
    int blocks_x = tile_w / 8;
    t.tile = tile;
    t.bx0 = (tile % tiles_x) * tile_w + (warp % blocks_x) * 8;
    t.by0 = (tile / tiles_x) * tile_h + (warp / blocks_x) * 4 * ROWS;
    t.px = t.bx0 + (lane & 7);
    t.py0 = t.by0 + (lane >> 3) * ROWS;
    return t;
}

// Can the splat reach alpha >= 1/256 at any pixel centre of the block?
template <int ROWS>
__host__ __device__ __forceinline__ bool block_hit(float4 r0, float bx0, float by0)
{
    return r0.x - r0.z <= bx0 + 7.5f && r0.x + r0.z >= bx0 + 0.5f &&
           r0.y - r0.w <= by0 + (4 * ROWS - 0.5f) && r0.y + r0.w >= by0 + 0.5f;
}

// Can the splat reach alpha >= 1/256 at any pixel centre of the block?  The
// exact form of block_hit: the largest power over the rectangle of the
// block's pixel centres (a concave quadratic, so its maximum is the mean when
// the rectangle holds it, else on an edge at the clamped vertex) against
// ln(1 / (256 o)), less a margin far above the rounding of both this
// evaluation and the fragment's (1e-4 plus 1e-5 of the quadratic's term
// sizes), so it never rejects a splat a pixel would composite.  Splats with
// a non-positive-definite conic (ext = +inf) always pass.
__host__ __device__ __forceinline__ float fast_recip(float x)
{
#ifdef __CUDA_ARCH__
    return __fdividef(1.0f, x);
#else
    return 1.0f / x;
#endif
}

__host__ __device__ __forceinline__ float fast_log(float x)
{
#ifdef __CUDA_ARCH__
    return __logf(x);
#else
    return logf(x);
#endif
}

template <int ROWS>
__host__ __device__ __forceinline__ bool ellipse_hit(float4 r0, float4 r1, float o, float bx0,
                                                     float by0)
{
    if (!(r0.z < INFINITY)) return true;
    const float x0 = bx0 + 0.5f - r0.x, x1 = bx0 + 7.5f - r0.x;
    const float y0 = by0 + 0.5f - r0.y, y1 = by0 + (4 * ROWS - 0.5f) - r0.y;
    if (x0 <= 0.0f && x1 >= 0.0f && y0 <= 0.0f && y1 >= 0.0f) return true;
    // power(dx, dy) = a dx^2 + b dx dy + c dy^2, a = -c00/2 < 0, c = -c11/2 < 0.
    const float a = r1.x, b = r1.y + r1.z, c = r1.w;
    const float ky = -0.5f * b * fast_recip(c), kx = -0.5f * b * fast_recip(a);
    float best = -INFINITY;
    const float xs[2] = {x0, x1}, ys[2] = {y0, y1};
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const float x = xs[i];
        const float y = fminf(fmaxf(ky * x, y0), y1);
        best = fmaxf(best, fmaf(x, fmaf(a, x, b * y), c * y * y));
        const float yy = ys[i];
        const float xx = fminf(fmaxf(kx * yy, x0), x1);
        best = fmaxf(best, fmaf(xx, fmaf(a, xx, b * yy), c * yy * yy));
    }
    const float mx = fmaxf(fabsf(x0), fabsf(x1)), my = fmaxf(fabsf(y0), fabsf(y1));
    const float size = fabsf(a) * mx * mx + fabsf(b) * mx * my + fabsf(c) * my * my;
    const float thr = -fast_log(256.0f * o);
    return best >= thr - (1e-4f + 1e-5f * size);
}

__device__ __forceinline__ uint32_t bit_word(int32_t start, int tile, int batch, int warps, int warp)
{
    return (uint32_t)(((start >> 5) + tile + batch) * warps + warp);
}

// Lane arithmetic over the lane's ROWS pixels: with two rows every add, mul
// and fma is one packed f32x2 instruction (sm_100), rounded exactly like its
// scalar form, so one- and two-row kernels produce identical fragments.
template <int ROWS>
struct Vec;

template <>
struct Vec<2> {
    using T = float2;
    static __device__ __forceinline__ T add(T a, T b) { return __fadd2_rn(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) { return __fmul2_rn(a, b); }
    static __device__ __forceinline__ T fma(T a, T b, T c) { return __ffma2_rn(a, b, c); }
    static __device__ __forceinline__ T lo(float4 v) { return make_float2(v.x, v.y); }
    static __device__ __forceinline__ T hi(float4 v) { return make_float2(v.z, v.w); }
    static __device__ __forceinline__ T splat(float x) { return make_float2(x, x); }
    static __device__ __forceinline__ float get(T v, int r) { return r ? v.y : v.x; }
    static __device__ __forceinline__ void set(T& v, int r, float x)
    {
        if (r) v.y = x;
        else v.x = x;
    }
};

template <>
struct Vec<1> {
    using T = float;
    static __device__ __forceinline__ T add(T a, T b) { return __fadd_rn(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) { return __fmul_rn(a, b); }
    static __device__ __forceinline__ T fma(T a, T b, T c) { return __fmaf_rn(a, b, c); }
    static __device__ __forceinline__ T lo(float4 v) { return v.x; }
    static __device__ __forceinline__ T hi(float4 v) { return v.z; }
    static __device__ __forceinline__ T splat(float x) { return x; }
    static __device__ __forceinline__ float get(T v, int) { return v; }
    static __device__ __forceinline__ void set(T& v, int, float x) { v = x; }
};

template <int ROWS>
__device__ __forceinline__ float row_sum(typename Vec<ROWS>::T v)
{
    float s = Vec<ROWS>::get(v, 0);
#pragma unroll
    for (int r = 1; r < ROWS; r++) s += Vec<ROWS>::get(v, r);
    return s;
}

// Per-warp stash of up to 32 staged splats, every scalar duplicated so that
// one broadcast shared load yields the (value, value) operand of a packed
// instruction.
struct Stash {
    float4 q0[32];     // (-mean_x, -mean_x, -mean_y, -mean_y)
    float4 q1[32];     // (c00', c00', c10', c10')   c' = -c / 2
    float4 q2[32];     // (c01', c01', c11', c11')
    float4 q3[32];     // (opacity, opacity, red, red)
    float4 q4[32];     // (green, green, blue, blue)
    float2 depth[32];  // (depth, depth)
    int32_t id[32];
};

__device__ __forceinline__ void stash_splat(Stash& st, int lane, float4 r0, float4 r1, float4 r2)
{
    st.q0[lane] = make_float4(-r0.x, -r0.x, -r0.y, -r0.y);
    st.q1[lane] = make_float4(r1.x, r1.x, r1.z, r1.z);
    st.q2[lane] = make_float4(r1.y, r1.y, r1.w, r1.w);
    st.q3[lane] = make_float4(r2.w, r2.w, r2.x, r2.x);
    st.q4[lane] = make_float4(r2.y, r2.y, r2.z, r2.z);
}

// Offsets and power of splat k at the lane's pixels, in the oracle's order:
// power = dy * (c11' dy + c10' dx) + dx * (c01' dy + c00' dx), fused.
template <int ROWS>
struct Fragment {
    typename Vec<ROWS>::T dx, dy, power;
};

template <int ROWS>
__device__ __forceinline__ Fragment<ROWS> fragment(const Stash& st, int k,
                                                   typename Vec<ROWS>::T pcx,
                                                   typename Vec<ROWS>::T pcy)
{
    using V = Vec<ROWS>;
    const float4 q0 = st.q0[k], q1 = st.q1[k], q2 = st.q2[k];
    Fragment<ROWS> f;
    f.dx = V::add(pcx, V::lo(q0));
    f.dy = V::add(pcy, V::hi(q0));
    const auto t1 = V::fma(V::lo(q2), f.dy, V::mul(V::lo(q1), f.dx));
    const auto t2 = V::fma(V::hi(q2), f.dy, V::mul(V::hi(q1), f.dx));
    f.power = V::fma(f.dy, t2, V::mul(f.dx, t1));
    return f;
}

// RECORD = false is the RGB-only forward of inference (the reference's
// record_contributions = False, packed_rasterizer.py:219-232): the same
// compositing, without final T, last index, backward work or contribution
// bits.  STATS also gathers the forward's fragment statistics per Gaussian
// (packed_rasterize.py:363-377): the number of composited fragments and the
// sum of their compositing weights T * alpha, as interleaved pairs.
template <int ROWS, bool WANT_DEPTH, bool RECORD, bool STATS>
// At most 48 registers (five 256-thread blocks' worth per SM): with the
// exact block test the compiler would take 58, and 48 keeps 19 two-warp CTAs
// per SM (2 % faster on config 2; the depth-writing instances spill 8-16 B).
__global__ void __launch_bounds__(256, 5) raster_fwd_kernel(
    gsb_raster_params p, const float4* __restrict__ splats, const float* __restrict__ depth,
    const int32_t* __restrict__ ids, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ order, const float* __restrict__ background,
    float* __restrict__ rgb, float* __restrict__ out_depth, float* __restrict__ out_alpha,
    float* __restrict__ final_t, int32_t* __restrict__ last_out,
    int32_t* __restrict__ backward_work, uint32_t* __restrict__ bits,
    float* __restrict__ stats)
{
    pdl_begin();
    using V = Vec<ROWS>;
    using T = typename V::T;
    extern __shared__ Stash stash_all[];
    __shared__ int tile_work;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    Stash& st = stash_all[warp];
    const int tile = order[blockIdx.x];
    const Geom<ROWS> tg = geom<ROWS>(p.width, p.tile_w, p.tile_h, tile, warp, lane);
    if (RECORD && threadIdx.x == 0) tile_work = 0;
    const int32_t start = offsets[tile], end = offsets[tile + 1];
    const T pcx = V::splat((float)tg.px + 0.5f);
    const float bx0 = (float)tg.bx0, by0 = (float)tg.by0;
    T pcy, trans = V::splat(1.0f), cr = V::splat(0.0f), cg = cr, cb = cr, cd = cr;
    int32_t last[ROWS];
    bool active[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; r++) {
        V::set(pcy, r, (float)(tg.py0 + r) + 0.5f);
        last[r] = end;
        active[r] = tg.px < p.width && tg.py0 + r < p.height;
    }
    bool any_active = false;
#pragma unroll
    for (int r = 0; r < ROWS; r++) any_active |= active[r];
    for (int32_t base = start, batch = 0; base < end; base += 32, batch++) {
        if (!__any_sync(GSB_FULL_MASK, any_active)) break;
        int32_t i = base + lane;
        bool hit = false;
        if (i < end) {
            int32_t g = __ldg(ids + i);
            const float4* rec = splats + (int64_t)g * 3;
            float4 r0 = __ldg(rec);
            hit = block_hit<ROWS>(r0, bx0, by0);
            float4 r1, r2;
            if (hit) {
                r1 = __ldg(rec + 1);
                r2 = __ldg(rec + 2);
                hit = ellipse_hit<ROWS>(r0, r1, r2.w, bx0, by0);
            }
            if (hit) {
                stash_splat(st, lane, r0, r1, r2);
                if (STATS) st.id[lane] = g;
                if (WANT_DEPTH) {
                    const float d = __ldg(depth + g);
                    st.depth[lane] = make_float2(d, d);
                }
            }
        }
        unsigned mask = __ballot_sync(GSB_FULL_MASK, hit);
        // Bit k: this lane composited splat k of the batch (OR-reduced over
        // the warp once per batch).
        unsigned mine = 0;
        __syncwarp();
        while (mask) {
            const int k = __ffs(mask) - 1;
            mask &= mask - 1;
            const Fragment<ROWS> f = fragment<ROWS>(st, k, pcx, pcy);
            const float4 q3 = st.q3[k], q4 = st.q4[k];
            T e;
#pragma unroll
            for (int r = 0; r < ROWS; r++) V::set(e, r, __expf(V::get(f.power, r)));
            const T raw = V::mul(V::lo(q3), e);
            T a;
            bool valid_any = false;
            bool valid[ROWS];
#pragma unroll
            for (int r = 0; r < ROWS; r++) {
                const float rr = V::get(raw, r);
                valid[r] = active[r] && V::get(f.power, r) <= 0.0f && rr >= kMinAlpha;
                // Branch-free: with a = 0 every update below is an exact no-op.
                V::set(a, r, valid[r] ? fminf(kMaxAlpha, rr) : 0.0f);
                valid_any |= valid[r];
            }
            const T w = V::mul(a, trans);
            cr = V::fma(w, V::hi(q3), cr);
            cg = V::fma(w, V::lo(q4), cg);
            cb = V::fma(w, V::hi(q4), cb);
            if (WANT_DEPTH) {
                const float2 d = st.depth[k];
                cd = V::fma(w, V::lo(make_float4(d.x, d.y, d.x, d.y)), cd);
            }
            // T (1 - a), with 1 - a formed as fma(a, -1, 1) (exact same rounding).
            trans = V::mul(trans, V::fma(a, V::splat(-1.0f), V::splat(1.0f)));
            const int32_t next = base + k + 1;
#pragma unroll
            for (int r = 0; r < ROWS; r++) {
                const bool stop = valid[r] && V::get(trans, r) < kMinT;
                last[r] = stop ? next : last[r];
                active[r] = active[r] && !stop;
            }
            if (RECORD && valid_any) mine |= 1u << k;
            if (STATS) {
                // w is exactly zero where the fragment is not composited.
                float count = 0.0f;
#pragma unroll
                for (int r = 0; r < ROWS; r++) count += valid[r] ? 1.0f : 0.0f;
                count = warp_sum(count);
                const float weight = warp_sum(row_sum<ROWS>(w));
                if (lane == 0 && count != 0.0f) {
                    float* sg = stats + (int64_t)st.id[k] * 2;
                    atomicAdd(sg, count);
                    atomicAdd(sg + 1, weight);
                }
            }
        }
        // Saturated lanes composite nothing more, so the warp's exit is
        // tested once per batch.
        any_active = false;
#pragma unroll
        for (int r = 0; r < ROWS; r++) any_active |= active[r];
        if (RECORD) {
            const unsigned contributed = __reduce_or_sync(GSB_FULL_MASK, mine);
            if (lane == 0) bits[bit_word(start, tile, batch, warps, warp)] = contributed;
        }
        __syncwarp();
    }
    int work = 0;
#pragma unroll
    for (int r = 0; r < ROWS; r++) {
        const int y = tg.py0 + r;
        if (tg.px < p.width && y < p.height) {
            const int64_t pix = (int64_t)y * p.width + tg.px;
            const float t = V::get(trans, r);
            float out_r = V::get(cr, r) + t * __ldg(background);
            float out_g = V::get(cg, r) + t * __ldg(background + 1);
            float out_b = V::get(cb, r) + t * __ldg(background + 2);
            if (p.flags & GSB_RASTER_CLAMP_RGB) {
                // The packed rasterizer's output, min(colour, 1)
                // (packed_rasterize.py:396).
                out_r = fminf(out_r, 1.0f);
                out_g = fminf(out_g, 1.0f);
                out_b = fminf(out_b, 1.0f);
            }
            rgb[pix * 3] = out_r;
            rgb[pix * 3 + 1] = out_g;
            rgb[pix * 3 + 2] = out_b;
            if (out_depth) out_depth[pix] = V::get(cd, r);
            if (out_alpha) out_alpha[pix] = 1.0f - t;
            if (RECORD) {
                final_t[pix] = t;
                last_out[pix] = last[r];
                work = max(work, last[r] - start);
            }
        }
    }
    if constexpr (RECORD) {
#pragma unroll
        for (int d = 16; d > 0; d >>= 1)
            work = max(work, __shfl_xor_sync(GSB_FULL_MASK, work, d));
        __syncthreads();
        if (lane == 0) atomicMax(&tile_work, work);
        __syncthreads();
        if (threadIdx.x == 0) backward_work[tile] = tile_work;
    }
}

// Transposed butterfly over 16 values: afterwards lane l holds the warp sum
// of value ((l >> 1) & 15).  16 shuffles for 16 sums.
__device__ __forceinline__ float warp_sum16(float v[16], int lane)
{
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        float keep = b4 ? v[j + 8] : v[j];
        float send = b4 ? v[j] : v[j + 8];
        v[j] = keep + __shfl_xor_sync(GSB_FULL_MASK, send, 16);
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
        float keep = b3 ? v[j + 4] : v[j];
        float send = b3 ? v[j] : v[j + 4];
        v[j] = keep + __shfl_xor_sync(GSB_FULL_MASK, send, 8);
    }
#pragma unroll
    for (int j = 0; j < 2; j++) {
        float keep = b2 ? v[j + 2] : v[j];
        float send = b2 ? v[j] : v[j + 2];
        v[j] = keep + __shfl_xor_sync(GSB_FULL_MASK, send, 4);
    }
    float keep = b1 ? v[1] : v[0];
    float send = b1 ? v[0] : v[1];
    float s = keep + __shfl_xor_sync(GSB_FULL_MASK, send, 2);
    s += __shfl_xor_sync(GSB_FULL_MASK, s, 1);
    return s;
}

// Warp sums of two values: lanes 0-15 get the first's, 16-31 the second's.
__device__ __forceinline__ float warp_sum_pair(float a, float b, int lane)
{
    const bool hi = lane & 16;
    float t = (hi ? b : a) + __shfl_xor_sync(GSB_FULL_MASK, hi ? a : b, 16);
    t += __shfl_xor_sync(GSB_FULL_MASK, t, 8);
    t += __shfl_xor_sync(GSB_FULL_MASK, t, 4);
    t += __shfl_xor_sync(GSB_FULL_MASK, t, 2);
    t += __shfl_xor_sync(GSB_FULL_MASK, t, 1);
    return t;
}

template <int ROWS, bool WANT_DEPTH, bool STATS>
__global__ void __launch_bounds__(256) raster_bwd_kernel(
    gsb_raster_bwd_params p, const float4* __restrict__ splats, const float* __restrict__ depth,
    const int32_t* __restrict__ ids, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ order, const uint32_t* __restrict__ bits,
    const float* __restrict__ background, const float* __restrict__ final_t,
    const int32_t* __restrict__ last_in, const float* __restrict__ drgb,
    const float* __restrict__ ddepth, const float* __restrict__ dalpha, float* __restrict__ gmean,
    float* __restrict__ gconic, float* __restrict__ gdepth, float* __restrict__ gcolor,
    float* __restrict__ galpha, float* __restrict__ stats)
{
    pdl_begin();
    using V = Vec<ROWS>;
    using T = typename V::T;
    extern __shared__ Stash stash_all[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    Stash& st = stash_all[warp];
    const int tile = order[blockIdx.x];
    const Geom<ROWS> tg = geom<ROWS>(p.width, p.tile_w, p.tile_h, tile, warp, lane);
    const int32_t start = offsets[tile];
    const T pcx = V::splat((float)tg.px + 0.5f);
    T pcy, gR = V::splat(0.0f), gG = gR, gB = gR, gD = gR, gtrans = gR, T_after = V::splat(1.0f);
    int32_t last[ROWS];
    int32_t top = start;
#pragma unroll
    for (int r = 0; r < ROWS; r++) {
        const int y = tg.py0 + r;
        V::set(pcy, r, (float)y + 0.5f);
        last[r] = start;
        if (tg.px < p.width && y < p.height) {
            const int64_t pix = (int64_t)y * p.width + tg.px;
            last[r] = last_in[pix];
            const float r_ = drgb[pix * 3], g_ = drgb[pix * 3 + 1], b_ = drgb[pix * 3 + 2];
            V::set(gR, r, r_);
            V::set(gG, r, g_);
            V::set(gB, r, b_);
            if (WANT_DEPTH) V::set(gD, r, ddepth[pix]);
            V::set(gtrans, r, r_ * __ldg(background) + g_ * __ldg(background + 1) +
                                  b_ * __ldg(background + 2) - (dalpha ? dalpha[pix] : 0.0f));
            V::set(T_after, r, final_t[pix]);
            top = max(top, last[r]);
        }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) top = max(top, __shfl_xor_sync(GSB_FULL_MASK, top, d));
    // Two contributing splats per pass of the reduction: after warp_sum16
    // lanes 2j, 2j+1 hold moment j (Sx, Sy, Sxx, Sxy, Syy, R, G, B) of the
    // first splat and lanes 16 + 2j, 16 + 2j + 1 that of the second.  Even
    // lanes add their moment; odd lane 1 the opacity gradient sum(ge) / o,
    // odd lane 3 the depth one, odd lane 7 repeats Sxy for conic[2] (unless
    // the symmetric convention folds it into conic[1]); the same +16.
    const int role_lane = lane & 15, j = role_lane >> 1;
    float* target = nullptr;
    int stride = 0;
    if ((role_lane & 1) == 0) {
        if (j < 2) { target = gmean + j; stride = 2; }
        else if (j < 5) { target = gconic + (j == 2 ? 0 : j == 3 ? 1 : 3); stride = 4; }
        else { target = gcolor + (j - 5); stride = 3; }
    } else if (role_lane == 7 && !(p.flags & GSB_RASTER_BWD_SYMMETRIC_CONIC)) {
        target = gconic + 2; stride = 4;
    } else if (role_lane == 1) {
        target = galpha; stride = 1;
    } else if (WANT_DEPTH && role_lane == 3) {
        target = gdepth; stride = 1;
    }
    // Constant coefficient of the lane's moment (2-4: -1/2, 5-7: 1).
    // Symmetric convention (packed_rasterize.py:130-175): conic[0][1] takes
    // both off-diagonal contributions and conic[1][0] stays zero.
    const float kA = j < 5 ? ((j == 3 && (p.flags & GSB_RASTER_BWD_SYMMETRIC_CONIC)) ? -1.0f
                                                                                      : -0.5f)
                           : 1.0f;
    const bool second = lane & 16;
    if (top <= start) return;
    // One splat's pass over the lane's pixels, in reverse compositing
    // order: updates T_after and gtrans, returns the lane's moments.
    auto visit = [&](int k, int32_t idx, float (&v)[8], float& S0, float& Z) {
        const Fragment<ROWS> f = fragment<ROWS>(st, k, pcx, pcy);
        const float4 q3 = st.q3[k], q4 = st.q4[k];
        T e;
#pragma unroll
        for (int r = 0; r < ROWS; r++) V::set(e, r, __expf(V::get(f.power, r)));
        const T raw = V::mul(V::lo(q3), e);
        T a, inv;
        bool valid[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; r++) {
            const float rr = V::get(raw, r);
            valid[r] = idx < last[r] && V::get(f.power, r) <= 0.0f && rr >= kMinAlpha;
            // Branch-free: with a = 0 the transmittance, the colour
            // behind and every accumulated term stay exactly unchanged.
            V::set(a, r, valid[r] ? fminf(kMaxAlpha, rr) : 0.0f);
        }
        const T one_minus = V::fma(a, V::splat(-1.0f), V::splat(1.0f));
#pragma unroll
        for (int r = 0; r < ROWS; r++) V::set(inv, r, __fdividef(1.0f, V::get(one_minus, r)));
        const T T_before = V::mul(T_after, inv);
        const T w = V::mul(T_before, a);
        T gw = V::fma(gB, V::hi(q4), V::fma(gG, V::lo(q4), V::mul(gR, V::hi(q3))));
        if (WANT_DEPTH) {
            const float2 d = st.depth[k];
            gw = V::fma(gD, V::lo(make_float4(d.x, d.y, d.x, d.y)), gw);
        }
        // ga = T_before (gw - gtrans); gtrans' = a gw + (1 - a) gtrans
        // (an exact no-op when a = 0).
        const T ga = V::mul(T_before, V::fma(gtrans, V::splat(-1.0f), gw));
        gtrans = V::fma(a, gw, V::mul(one_minus, gtrans));
        const float R = row_sum<ROWS>(V::mul(w, gR));
        const float G = row_sum<ROWS>(V::mul(w, gG));
        const float B = row_sum<ROWS>(V::mul(w, gB));
        Z = 0.0f;
        if (WANT_DEPTH) Z = row_sum<ROWS>(V::mul(w, gD));
        T ge = V::mul(ga, raw);
        float count = 0.0f, square = 0.0f;
#pragma unroll
        for (int r = 0; r < ROWS; r++) {
            const bool live = valid[r] && V::get(raw, r) < kMaxAlpha;
            V::set(ge, r, live ? V::get(ge, r) : 0.0f);
            V::set(T_after, r, valid[r] ? V::get(T_before, r) : V::get(T_after, r));
            if (STATS) {
                // Fragment statistics (sorted_rasterize.py:155-203): one
                // count per composited fragment, and the squared opacity
                // cotangent ga * e of each unsaturated one.
                const float go = live ? V::get(ga, r) * V::get(e, r) : 0.0f;
                count += valid[r] ? 1.0f : 0.0f;
                square = fmaf(go, go, square);
            }
        }
        if (STATS) {
            // w is exactly zero where the fragment is not composited.
            const float weight = warp_sum(row_sum<ROWS>(w));
            count = warp_sum(count);
            square = warp_sum(square);
            if (lane == 0 && count != 0.0f) {
                float* st_g = stats + (int64_t)st.id[k] * 3;
                atomicAdd(st_g, count);
                atomicAdd(st_g + 1, weight);
                atomicAdd(st_g + 2, square);
            }
        }
        const T gedy = V::mul(ge, f.dy);
        S0 = row_sum<ROWS>(ge);
        const float Sy = row_sum<ROWS>(gedy);
        const float Syy = row_sum<ROWS>(V::mul(gedy, f.dy));
        const float dx = V::get(f.dx, 0);
        const float Sx = dx * S0;
        v[0] = Sx; v[1] = Sy; v[2] = dx * Sx; v[3] = dx * Sy;
        v[4] = Syy; v[5] = R; v[6] = G; v[7] = B;
    };
    const int32_t top_batch = (top - 1 - start) >> 5;
    for (int32_t batch = top_batch; batch >= 0; batch--) {
        uint32_t word = __ldg(bits + bit_word(start, tile, batch, warps, warp));
        if (batch == top_batch) {
            const int k_max = (top - 1 - start) & 31;
            word &= k_max == 31 ? 0xffffffffu : ((2u << k_max) - 1u);
        }
        if (word == 0) continue;
        const int32_t base = start + batch * 32;
        if (word & (1u << lane)) {
            const int32_t g = __ldg(ids + base + lane);
            const float4* rec = splats + (int64_t)g * 3;
            stash_splat(st, lane, __ldg(rec), __ldg(rec + 1), __ldg(rec + 2));
            st.id[lane] = g;
            if (WANT_DEPTH) {
                const float d = __ldg(depth + g);
                st.depth[lane] = make_float2(d, d);
            }
        }
        __syncwarp();
        while (word) {
            const int k1 = 31 - __clz(word);
            word &= ~(1u << k1);
            float v[16], S0a, Za;
            float (&va)[8] = *reinterpret_cast<float(*)[8]>(&v[0]);
            float (&vb)[8] = *reinterpret_cast<float(*)[8]>(&v[8]);
            visit(k1, base + k1, va, S0a, Za);
            const bool has2 = word != 0;  // uniform over the warp
            int k2 = k1;
            float S0b = 0.0f, Zb = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++) vb[i] = 0.0f;
            if (has2) {
                k2 = 31 - __clz(word);
                word &= ~(1u << k2);
                visit(k2, base + k2, vb, S0b, Zb);
            }
            const float s = warp_sum16(v, lane);
            const float S0 = warp_sum_pair(S0a, S0b, lane);
            float Z = 0.0f;
            if (WANT_DEPTH) Z = warp_sum_pair(Za, Zb, lane);
            // gmean.x = c00 Sx + cbar Sy, gmean.y = c11 Sy + cbar Sx with c = -2 c';
            // gconic = -Sxx/2, -Sxy/2 (twice), -Syy/2; gcolor = R, G, B;
            // galpha = sum(ge) / o.
            const int k = second ? k2 : k1;
            const float4 q1 = st.q1[k], q2 = st.q2[k];
            const float other = __shfl_xor_sync(GSB_FULL_MASK, s, 2);
            const float coef_a = j == 0 ? -2.0f * q1.x : (j == 1 ? -2.0f * q2.z : kA);
            const float coef_b = j < 2 ? -(q2.x + q1.z) : 0.0f;
            float value = coef_a * s + coef_b * other;
            if (role_lane == 1) value = __fdividef(S0, st.q3[k].x);
            if (WANT_DEPTH && role_lane == 3) value = Z;
            if (target && (has2 || !second)) atomicAdd(target + (int64_t)st.id[k] * stride, value);
        }
        __syncwarp();
    }
}

__global__ void zero_cotangents_kernel(int64_t capacity, float* gmean, float* gconic, float* gdepth,
                                       float* gcolor, float* galpha)
{
    pdl_begin();
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
    pdl_begin();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)(*count) * cluster_size) return;
    int64_t g = (int64_t)ids[i / cluster_size] * cluster_size + i % cluster_size;
    if (g >= capacity) return;
    *reinterpret_cast<float2*>(gmean + g * 2) = make_float2(0.f, 0.f);
    *reinterpret_cast<float4*>(gconic + g * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
    gcolor[g * 3] = gcolor[g * 3 + 1] = gcolor[g * 3 + 2] = 0.0f;
    galpha[g] = 0.0f;
}

// Fragment statistics start from zero over the whole pool, and so does the
// opacity cotangent, their fourth column (kernels/packed_rasterize.py:759-766).
__global__ void zero_stats_kernel(int64_t capacity, float* stats, float* galpha)
{
    pdl_begin();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= capacity * 3) return;
    stats[i] = 0.0f;
    if (i < capacity) galpha[i] = 0.0f;
}

bool tiles_ok(int tile_w, int tile_h)
{
    return tile_w > 0 && tile_h > 0 && tile_w % 8 == 0 && tile_h % 4 == 0 && tile_w <= 16 &&
           tile_h <= 16;
}

int rows_per_lane(int tile_h) { return tile_h % 8 == 0 ? 2 : 1; }

int warps_per_tile(int tile_w, int tile_h)
{
    return (tile_w / 8) * (tile_h / (4 * rows_per_lane(tile_h)));
}

int64_t num_tiles(const gsb_raster_params& p)
{
    return (int64_t)ceil_div(p.width, p.tile_w) * ceil_div(p.height, p.tile_h);
}

size_t raster_ws(const gsb_raster_params& p)
{
    return ((size_t)num_tiles(p) * sizeof(int32_t) + 255) & ~size_t(255);
}

size_t bit_words(const gsb_raster_params& p)
{
    int64_t pairs = p.max_pairs > 0 ? p.max_pairs : 0;
    return (size_t)(pairs / 32 + num_tiles(p) + 1) * warps_per_tile(p.tile_w, p.tile_h);
}

template <int ROWS>
void launch_fwd(cudaStream_t s, int tiles, int warps, bool want_depth, bool record,
                const gsb_raster_params& p, const float4* sp, const float* depth,
                const int32_t* ids, const int32_t* offsets, const int32_t* order, const float* bg,
                float* rgb, float* od, float* oa, float* final_t, int32_t* last, int32_t* work,
                uint32_t* bits, float* stats)
{
    size_t smem = (size_t)warps * sizeof(Stash);
    auto go = [&](auto kernel) {
        gsb::launch(kernel, tiles, warps * 32, smem, s, p, sp, depth, ids, offsets, order, bg, rgb,
                    od, oa, final_t, last, work, bits, stats);
    };
    if (stats) {
        if (want_depth) go(raster_fwd_kernel<ROWS, true, true, true>);
        else go(raster_fwd_kernel<ROWS, false, true, true>);
    } else if (record) {
        if (want_depth) go(raster_fwd_kernel<ROWS, true, true, false>);
        else go(raster_fwd_kernel<ROWS, false, true, false>);
    } else {
        if (want_depth) go(raster_fwd_kernel<ROWS, true, false, false>);
        else go(raster_fwd_kernel<ROWS, false, false, false>);
    }
}

__global__ void zero_f32_kernel(float* p, int64_t n)
{
    pdl_begin();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        p[i] = 0.0f;
}

template <int ROWS>
void launch_bwd(cudaStream_t s, int tiles, int warps, bool want_depth,
                const gsb_raster_bwd_params& p, const float4* sp, const float* depth,
                const int32_t* ids, const int32_t* offsets, const int32_t* order,
                const uint32_t* bits, const float* bg, const float* final_t, const int32_t* last,
                const float* drgb, const float* ddepth, const float* dalpha, float* gmean,
                float* gconic, float* gdepth, float* gcolor, float* galpha, float* stats)
{
    size_t smem = (size_t)warps * sizeof(Stash);
    auto go = [&](auto kernel) {
        gsb::launch(kernel, tiles, warps * 32, smem, s, p, sp, depth, ids, offsets, order, bits,
                    bg, final_t, last, drgb, ddepth, dalpha, gmean, gconic, gdepth, gcolor,
                    galpha, stats);
    };
    if (stats) {
        if (want_depth) go(raster_bwd_kernel<ROWS, true, true>);
        else go(raster_bwd_kernel<ROWS, false, true>);
    } else {
        if (want_depth) go(raster_bwd_kernel<ROWS, true, false>);
        else go(raster_bwd_kernel<ROWS, false, false>);
    }
}

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" size_t gsb_raster_workspace_size(const gsb_raster_params* p)
{
    return p ? raster_ws(*p) : 0;
}

extern "C" size_t gsb_raster_bit_words(const gsb_raster_params* p)
{
    if (!p || !tiles_ok(p->tile_w, p->tile_h) || p->width <= 0 || p->height <= 0) return 0;
    return bit_words(*p);
}

namespace gsb {
namespace {

int launch_pack(cudaStream_t s, const gsb_raster_params& p, const float* mean, const float* conic,
                const float* color, const float* alpha, const int8_t* visible, float* splats)
{
    if (p.capacity == 0) return GSB_OK;
    gsb::launch(pack_kernel, ceil_div(p.capacity, 256), 256, 0, s, p.capacity, mean, conic, color, alpha,
                                                          visible,
                                                          reinterpret_cast<float4*>(splats));
    return check_launch();
}

// Zero the cotangents and order the tiles by backward work (into workspace).
int launch_bwd_prepare(cudaStream_t s, const gsb_raster_bwd_params& p, int tiles,
                       const int32_t* backward_work, const int32_t* cluster_ids,
                       const int32_t* cluster_count, int32_t* order, float* gmean, float* gconic,
                       float* gdepth, float* gcolor, float* galpha, float* stats)
{
    if (p.capacity > 0 && stats) {
        gsb::launch(zero_stats_kernel, ceil_div((int64_t)p.capacity * 3, 256), 256, 0, s,
                    (int64_t)p.capacity, stats, galpha);
        if (int e = check_launch()) return e;
    }
    if (p.capacity > 0) {
        if (cluster_ids) {
            gsb::launch(zero_cluster_cotangents_kernel, ceil_div(p.capacity, 256), 256, 0, s, 
                p.capacity, p.cluster_size, cluster_ids, cluster_count, gmean, gconic, gcolor,
                galpha);
        } else {
            gsb::launch(zero_cotangents_kernel, ceil_div(p.capacity, 256), 256, 0, s, 
                p.capacity, gmean, gconic, gdepth, gcolor, galpha);
        }
        if (int e = check_launch()) return e;
    }
    gsb::launch(order_tiles_kernel, 1, kOrderThreads, 0, s, backward_work, tiles, 0, order);
    return check_launch();
}

bool raster_shape_ok(const gsb_raster_params& p)
{
    return p.capacity >= 0 && p.width > 0 && p.height > 0 && tiles_ok(p.tile_w, p.tile_h) &&
           p.max_pairs >= 0 && p.max_pairs < (int64_t(1) << 31) &&
           (p.flags & ~(GSB_RASTER_SPLATS_READY | GSB_RASTER_RGB_ONLY | GSB_RASTER_CLAMP_RGB)) == 0;
}

bool raster_bwd_shape_ok(const gsb_raster_bwd_params& p)
{
    return p.capacity >= 0 && p.width > 0 && p.height > 0 && tiles_ok(p.tile_w, p.tile_h) &&
           (p.flags & ~(GSB_RASTER_BWD_PREPARED | GSB_RASTER_BWD_SYMMETRIC_CONIC)) == 0;
}

bool misaligned16(const void* a, const void* b)
{
    return ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) != 0;
}

}  // namespace
}  // namespace gsb

extern "C" int gsb_raster_pack(gsb_stream_t stream, const gsb_raster_params* p, const float* mean,
                               const float* conic, const float* color, const float* alpha,
                               const int8_t* visible, float* splats)
{
    if (!p) return GSB_ERR_NULL;
    if (!raster_shape_ok(*p)) return GSB_ERR_INVALID;
    if (!splats || (p->capacity > 0 && (!mean || !conic || !color || !alpha || !visible)))
        return GSB_ERR_NULL;
    if (misaligned16(splats, conic)) return GSB_ERR_INVALID;
    return launch_pack(as_stream(stream), *p, mean, conic, color, alpha, visible, splats);
}

extern "C" int gsb_raster_fwd(gsb_stream_t stream, const gsb_raster_params* p, void* workspace,
                              size_t workspace_bytes, const float* mean, const float* conic,
                              const float* depth, const float* color, const float* alpha,
                              const int8_t* visible, const int32_t* gaussian_ids,
                              const int32_t* tile_offsets, const float* background, float* rgb,
                              float* out_depth, float* out_alpha, float* final_t, int32_t* last,
                              int32_t* backward_work, float* splats, uint32_t* contribution_bits,
                              float* fragment_stats)
{
    if (!p) return GSB_ERR_NULL;
    if (!raster_shape_ok(*p)) return GSB_ERR_INVALID;
    if (fragment_stats && (p->flags & GSB_RASTER_RGB_ONLY)) return GSB_ERR_INVALID;
    if (!workspace || workspace_bytes < raster_ws(*p)) return GSB_ERR_WORKSPACE;
    const bool packed = (p->flags & GSB_RASTER_SPLATS_READY) != 0;
    const bool record = (p->flags & GSB_RASTER_RGB_ONLY) == 0;
    if (!gaussian_ids || !tile_offsets || !background || !rgb || !splats ||
        (record && (!final_t || !last || !backward_work || !contribution_bits)) ||
        (p->capacity > 0 && !packed && (!mean || !conic || !color || !alpha || !visible)) ||
        (out_depth && !depth))
        return GSB_ERR_NULL;
    if (misaligned16(splats, packed ? nullptr : conic)) return GSB_ERR_INVALID;
    cudaStream_t s = as_stream(stream);
    int tiles = (int)num_tiles(*p);
    int32_t* order = static_cast<int32_t*>(workspace);
    if (!packed) {
        if (int e = launch_pack(s, *p, mean, conic, color, alpha, visible, splats)) return e;
    }
    if (fragment_stats && p->capacity > 0) {
        gsb::launch(zero_f32_kernel, 296, 256, 0, s, fragment_stats, (int64_t)p->capacity * 2);
        if (int e = check_launch()) return e;
    }
    gsb::launch(order_tiles_kernel, 1, kOrderThreads, 0, s, tile_offsets, tiles, 1, order);
    if (int e = check_launch()) return e;
    int warps = warps_per_tile(p->tile_w, p->tile_h);
    const float4* sp = reinterpret_cast<const float4*>(splats);
    if (rows_per_lane(p->tile_h) == 2)
        launch_fwd<2>(s, tiles, warps, out_depth != nullptr, record, *p, sp, depth, gaussian_ids,
                      tile_offsets, order, background, rgb, out_depth, out_alpha, final_t, last,
                      backward_work, contribution_bits, fragment_stats);
    else
        launch_fwd<1>(s, tiles, warps, out_depth != nullptr, record, *p, sp, depth, gaussian_ids,
                      tile_offsets, order, background, rgb, out_depth, out_alpha, final_t, last,
                      backward_work, contribution_bits, fragment_stats);
    return check_launch();
}

extern "C" int gsb_raster_bwd_prepare(gsb_stream_t stream, const gsb_raster_bwd_params* p,
                                      void* workspace, size_t workspace_bytes,
                                      const int32_t* backward_work, const int32_t* cluster_ids,
                                      const int32_t* cluster_count, float* gmean, float* gconic,
                                      float* gdepth, float* gcolor, float* galpha,
                                      float* fragment_stats)
{
    if (!p) return GSB_ERR_NULL;
    gsb_raster_params rp{p->capacity, p->width, p->height, p->tile_w, p->tile_h, p->max_pairs, 0};
    if (!raster_bwd_shape_ok(*p)) return GSB_ERR_INVALID;
    if (!workspace || workspace_bytes < raster_ws(rp)) return GSB_ERR_WORKSPACE;
    if (!backward_work || !gmean || !gconic || !gcolor || !galpha) return GSB_ERR_NULL;
    if (cluster_ids && (!cluster_count || p->cluster_size <= 0)) return GSB_ERR_INVALID;
    if (!cluster_ids && !gdepth) return GSB_ERR_NULL;
    if (misaligned16(gconic, nullptr)) return GSB_ERR_INVALID;
    return launch_bwd_prepare(as_stream(stream), *p, (int)num_tiles(rp), backward_work,
                              cluster_ids, cluster_count, static_cast<int32_t*>(workspace), gmean,
                              gconic, gdepth, gcolor, galpha, fragment_stats);
}

extern "C" int gsb_raster_bwd(gsb_stream_t stream, const gsb_raster_bwd_params* p,
                              void* workspace, size_t workspace_bytes, const float* splats,
                              const float* depth, const int32_t* gaussian_ids,
                              const int32_t* tile_offsets, const float* background,
                              const float* final_t, const int32_t* last,
                              const int32_t* backward_work, const uint32_t* contribution_bits,
                              const float* drgb, const float* ddepth, const float* dalpha,
                              const int32_t* cluster_ids, const int32_t* cluster_count,
                              float* gmean, float* gconic, float* gdepth, float* gcolor,
                              float* galpha, float* fragment_stats)
{
    if (!p) return GSB_ERR_NULL;
    gsb_raster_params rp{p->capacity, p->width, p->height, p->tile_w, p->tile_h, p->max_pairs, 0};
    if (!raster_bwd_shape_ok(*p)) return GSB_ERR_INVALID;
    if (!workspace || workspace_bytes < raster_ws(rp)) return GSB_ERR_WORKSPACE;
    if (!splats || !gaussian_ids || !tile_offsets || !background || !final_t || !last ||
        !backward_work || !contribution_bits || !drgb || !gmean || !gconic || !gcolor || !galpha)
        return GSB_ERR_NULL;
    bool want_depth = ddepth != nullptr;
    if (want_depth && (!depth || !gdepth)) return GSB_ERR_NULL;
    if (cluster_ids && (!cluster_count || p->cluster_size <= 0)) return GSB_ERR_INVALID;
    if (!cluster_ids && !gdepth) return GSB_ERR_NULL;
    if (misaligned16(splats, gconic)) return GSB_ERR_INVALID;
    cudaStream_t s = as_stream(stream);
    int tiles = (int)num_tiles(rp);
    int32_t* order = static_cast<int32_t*>(workspace);
    if (!(p->flags & GSB_RASTER_BWD_PREPARED)) {
        if (int e = launch_bwd_prepare(s, *p, tiles, backward_work, cluster_ids, cluster_count,
                                       order, gmean, gconic, gdepth, gcolor, galpha,
                                       fragment_stats))
            return e;
    }
    int warps = warps_per_tile(p->tile_w, p->tile_h);
    const float4* sp = reinterpret_cast<const float4*>(splats);
    if (rows_per_lane(p->tile_h) == 2)
        launch_bwd<2>(s, tiles, warps, want_depth, *p, sp, depth, gaussian_ids, tile_offsets,
                      order, contribution_bits, background, final_t, last, drgb, ddepth, dalpha,
                      gmean, gconic, gdepth, gcolor, galpha, fragment_stats);
    else
        launch_bwd<1>(s, tiles, warps, want_depth, *p, sp, depth, gaussian_ids, tile_offsets,
                      order, contribution_bits, background, final_t, last, drgb, ddepth, dalpha,
                      gmean, gconic, gdepth, gcolor, galpha, fragment_stats);
    return check_launch();
}
