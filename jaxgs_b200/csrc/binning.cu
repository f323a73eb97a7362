// Tile binning for sm_100a: AccuTile count + depth keys, stable depth sort,
// depth-ordered scan, pair emission, stable LSD tile sort and tile ranges.
//
// Result contract (kernels/sorted_binning.py:9-117): the valid prefix of
// gaussian_ids lists, tile by tile, every Gaussian whose AccuTile ellipse
// covers the tile, ordered by (depth key, Gaussian id).  Internally:
//   1. count_kernel      — per Gaussian pair count and 32-bit depth key.
//   2. depth sort        — 4 stable 8-bit LSD passes; the first pass drops the
//                          0xFFFFFFFF keys of Gaussians without pairs, so the
//                          remaining passes sort only binned Gaussians.
//   3. scan              — inclusive scan of the counts in depth order.
//   4. emission          — each Gaussian writes its pairs to its segment; one
//                          thread per small Gaussian, one warp per large one.
//   5. tile sort         — stable LSD passes over the tile key (digit plan of
//                          kernels/pair_sort.py:33-37) of the emitted pairs.
//   6. tile ranges       — offsets[t] = first pair with tile >= t.
// Every stage is a plain kernel launch on one stream: no inter-block waits,
// no host synchronisation; counts that only the device knows (binned
// Gaussians, pairs) are read by the kernels, whose grids are sized for the
// capacity and whose surplus blocks exit at once.
#include "gsb_common.cuh"

namespace gsb {
namespace {

// ---------------------------------------------------------------------------
// AccuTile geometry (kernels/sorted_visibility.py:34-224), explicitly rounded
// so that the host oracle (oracle/gs_oracle.c) gives identical bits.
// ---------------------------------------------------------------------------
struct Ellipse {
    float disc, level;
    int is_y;
    float block_u, block_v;
    int32_t u0, u1, v0, v1;
    float bbox_u_min, bbox_u_max, bbox_v_min, bbox_v_max, arg_min, arg_max;
};

// sorted_visibility.py:34-74
__device__ __forceinline__ void intersection(float px, float py, float c00, float c01, float c11,
                                             float disc, float level, int is_y, float coord,
                                             int side, bool sliced, float& out_low, float& out_high)
{
    float pu = is_y ? py : px;
    float pv = is_y ? px : py;
    float coeff = is_y ? c00 : c11;
    float delta = fsub(coord, pu);
    float radicand = sliced ? ffma(delta, fmul(disc, delta), fmul(level, coeff))
                            : ffma(level, coeff, fmul(fmul(disc, delta), delta));
    float root = fsqrt(fmaxf(radicand, 0.0f));
    float low = 0.0f, high = 0.0f;
    if (side == 0) {
        float shared = fmul(c01, -delta);
        low = fsub(shared, root);
        high = fadd(shared, root);
    } else if (side < 0) {
        low = ffma(-c01, delta, -root);
    } else {
        high = ffma(-c01, delta, root);
    }
    out_low = fadd(fdiv(low, coeff), pv);
    out_high = fadd(fdiv(high, coeff), pv);
}

// sorted_visibility.py:77-126
__device__ __forceinline__ Ellipse ellipse_bounds(float px, float py, float c00, float c01,
                                                  float c11, float alpha, int tile_w, int tile_h,
                                                  int tiles_x, int tiles_y)
{
    Ellipse e;
    float c01_sq = fmul(c01, c01);
    float disc = fsub(c01_sq, fmul(c00, c11));
    float level = fmul(2.0f, gs_logf(fmul(alpha, 255.0f)));
    float numerator = fmul(c01_sq, -level);
    float x_term = fsqrt(fdiv(numerator, fmul(c00, disc)));
    float y_term = fsqrt(fdiv(numerator, fmul(c11, disc)));
    if (c01 >= 0.0f) {
        x_term = -x_term;
        y_term = -y_term;
    }
    float argmin_x = fsub(py, y_term), argmin_y = fsub(px, x_term);
    float argmax_x = fadd(py, y_term), argmax_y = fadd(px, x_term);
    float xmin, ymin, xmax, ymax, unused;
    intersection(px, py, c00, c01, c11, disc, level, 1, argmin_x, -1, false, xmin, unused);
    intersection(px, py, c00, c01, c11, disc, level, 0, argmin_y, -1, false, ymin, unused);
    intersection(px, py, c00, c01, c11, disc, level, 1, argmax_x, 1, false, unused, xmax);
    intersection(px, py, c00, c01, c11, disc, level, 0, argmax_y, 1, false, unused, ymax);
    float tw = (float)tile_w, th = (float)tile_h;
    int32_t x0 = max(0, min(tiles_x, trunc_i32(fdiv(xmin, tw))));
    int32_t y0 = max(0, min(tiles_y, trunc_i32(fdiv(ymin, th))));
    int32_t x1 = max(0, min(tiles_x, trunc_i32(fdiv(fsub(fadd(xmax, tw), 1.0f), tw))));
    int32_t y1 = max(0, min(tiles_y, trunc_i32(fdiv(fsub(fadd(ymax, th), 1.0f), th))));
    e.disc = disc;
    e.level = level;
    e.is_y = (y1 - y0) < (x1 - x0);
    if (e.is_y) {
        e.block_u = th; e.block_v = tw;
        e.u0 = y0; e.u1 = y1; e.v0 = x0; e.v1 = x1;
        e.bbox_u_min = ymin; e.bbox_u_max = ymax; e.bbox_v_min = xmin; e.bbox_v_max = xmax;
        e.arg_min = argmin_x; e.arg_max = argmax_x;
    } else {
        e.block_u = tw; e.block_v = th;
        e.u0 = x0; e.u1 = x1; e.v0 = y0; e.v1 = y1;
        e.bbox_u_min = xmin; e.bbox_u_max = xmax; e.bbox_v_min = ymin; e.bbox_v_max = ymax;
        e.arg_min = argmin_y; e.arg_max = argmax_y;
    }
    if ((int64_t)(y1 - y0) * (int64_t)(x1 - x0) <= 0) e.u1 = e.u0;
    return e;
}

// sorted_visibility.py:129-141
__device__ __forceinline__ void span(const Ellipse& e, float line, float next_line, float lower_min,
                                     float lower_max, float upper_min, float upper_max,
                                     int32_t& first, int32_t& end)
{
    float emin = fminf(lower_min, upper_min);
    float emax = fmaxf(lower_max, upper_max);
    if (line <= e.arg_min && e.arg_min < next_line) emin = e.bbox_v_min;
    if (line <= e.arg_max && e.arg_max < next_line) emax = e.bbox_v_max;
    first = max(e.v0, min(e.v1, trunc_i32(fdiv(emin, e.block_v))));
    end = min(e.v1, max(e.v0, trunc_i32(fadd(fdiv(emax, e.block_v), 1.0f))));
}

__device__ __forceinline__ uint32_t tile_key(int is_y, int32_t u, int32_t v, int tiles_x)
{
    return is_y ? (uint32_t)(u * tiles_x + v) : (uint32_t)(v * tiles_x + u);
}

struct Splat {
    float px, py, c00, c01, c11, alpha;
};

// sorted_visibility.py:333-342
__device__ __forceinline__ bool count_gate(float mx, float my, float c00, float c01, float c11,
                                           float a, int width, int height)
{
    float W = (float)width, H = (float)height;
    return a >= (float)(1.0 / 255.0) && c00 > 0.0f && c11 > 0.0f &&
           fsub(fmul(c00, c11), fmul(c01, c01)) > 0.0f && mx >= fmul(-0.15f, W) &&
           mx <= fmul(1.15f, W) && my >= fmul(-0.15f, H) && my <= fmul(1.15f, H);
}

__device__ __forceinline__ Splat load_splat(const float* mean, const float* conic,
                                            const float* alpha, int64_t g)
{
    Splat s;
    float2 m = *reinterpret_cast<const float2*>(mean + g * 2);
    float4 c = *reinterpret_cast<const float4*>(conic + g * 4);
    s.px = fsub(m.x, 0.5f);
    s.py = fsub(m.y, 0.5f);
    s.c00 = c.x;
    s.c01 = c.y;
    s.c11 = c.w;
    s.alpha = alpha[g];
    return s;
}

// sorted_visibility.py:178-224: sequential row walk; EMIT writes the pairs.
template <bool EMIT, typename K>
__device__ int32_t process_tiles(const Splat& s, int tile_w, int tile_h, int tiles_x, int tiles_y,
                                 int32_t gid, int64_t offset, int64_t max_pairs, K* keys,
                                 int32_t* values)
{
    Ellipse e = ellipse_bounds(s.px, s.py, s.c00, s.c01, s.c11, s.alpha, tile_w, tile_h, tiles_x,
                               tiles_y);
    int32_t count = 0;
    if (e.u1 > e.u0) {
        float upper_min = e.bbox_v_max, upper_max = e.bbox_v_min;
        float lower_min = upper_min, lower_max = upper_max;
        float line = fmul((float)e.u0, e.block_u);
        if (e.bbox_u_min <= line)
            intersection(s.px, s.py, s.c00, s.c01, s.c11, e.disc, e.level, e.is_y, line, 0, false,
                         lower_min, lower_max);
        for (int32_t u = e.u0; u < e.u1; u++) {
            float next_line = fadd(line, e.block_u);
            if (next_line <= e.bbox_u_max)
                intersection(s.px, s.py, s.c00, s.c01, s.c11, e.disc, e.level, e.is_y, next_line,
                             0, true, upper_min, upper_max);
            int32_t first, end;
            span(e, line, next_line, lower_min, lower_max, upper_min, upper_max, first, end);
            if (EMIT) {
                for (int32_t v = first; v < end; v++) {
                    int64_t slot = offset + count + v - first;
                    if (slot < max_pairs) {
                        keys[slot] = (K)tile_key(e.is_y, u, v, tiles_x);
                        values[slot] = gid;
                    }
                }
            }
            count += end - first;
            lower_min = upper_min;
            lower_max = upper_max;
            line = next_line;
        }
    }
    return count;
}

// Row u's span computed independently but equal to process_tiles's: the
// sequential walk's upper bound after row k is the slice at line m*, the
// largest m <= k+1 with m*block_u <= bbox_u_max (the slice is recomputed only
// while next_line <= bbox_u_max), or the empty interval when m* <= u0.
__device__ __forceinline__ void row_span(const Splat& s, const Ellipse& e, int32_t m_max, int32_t u,
                                         int32_t& first, int32_t& end)
{
    float line = fmul((float)u, e.block_u);
    float next_line = fadd(line, e.block_u);
    float lower_min = e.bbox_v_max, lower_max = e.bbox_v_min;
    if (u == e.u0) {
        if (e.bbox_u_min <= line)
            intersection(s.px, s.py, s.c00, s.c01, s.c11, e.disc, e.level, e.is_y, line, 0, false,
                         lower_min, lower_max);
    } else {
        int32_t m = min(u, m_max);
        if (m >= e.u0 + 1)
            intersection(s.px, s.py, s.c00, s.c01, s.c11, e.disc, e.level, e.is_y,
                         fmul((float)m, e.block_u), 0, true, lower_min, lower_max);
    }
    float upper_min = e.bbox_v_max, upper_max = e.bbox_v_min;
    int32_t m = min(u + 1, m_max);
    if (m >= e.u0 + 1)
        intersection(s.px, s.py, s.c00, s.c01, s.c11, e.disc, e.level, e.is_y,
                     fmul((float)m, e.block_u), 0, true, upper_min, upper_max);
    span(e, line, next_line, lower_min, lower_max, upper_min, upper_max, first, end);
}

// Largest integer m with m * block_u <= bbox_u_max (exact comparison).
__device__ __forceinline__ int32_t last_line(const Ellipse& e)
{
    float q = floorf(e.bbox_u_max / e.block_u);
    int32_t m;
    if (!(q > -1.0f)) return -1;
    m = q > 1.0e7f ? 10000000 : (int32_t)q;
    for (int it = 0; it < 3 && fmul((float)(m + 1), e.block_u) <= e.bbox_u_max; it++) m++;
    for (int it = 0; it < 3 && m >= 0 && fmul((float)m, e.block_u) > e.bbox_u_max; it++) m--;
    return m;
}

// Radix-sortable depth bits (sorted_visibility.py:362-370).
__device__ __forceinline__ uint32_t depth_key(float depth, int32_t count)
{
    if (count <= 0) return 0xFFFFFFFFu;
    uint32_t bits = __float_as_uint(depth);
    return (bits >> 31) ? ~bits : (bits ^ 0x80000000u);
}

// _count, sorted_visibility.py:307-370.
__global__ void __launch_bounds__(256) count_kernel(int capacity, const float* __restrict__ mean,
                                                    const float* __restrict__ conic,
                                                    const float* __restrict__ alpha,
                                                    const float* __restrict__ depth,
                                                    const int8_t* __restrict__ visible,
                                                    gsb_bin_params p, int tiles_x, int tiles_y,
                                                    int32_t* __restrict__ counts,
                                                    uint32_t* __restrict__ keys)
{
    int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= capacity) return;
    int32_t count = 0;
    if (visible[g] != 0) {
        float2 m = *reinterpret_cast<const float2*>(mean + g * 2);
        float4 c = *reinterpret_cast<const float4*>(conic + g * 4);
        float a = alpha[g];
        if (count_gate(m.x, m.y, c.x, c.y, c.w, a, p.width, p.height)) {
            Splat s{fsub(m.x, 0.5f), fsub(m.y, 0.5f), c.x, c.y, c.w, a};
            count = process_tiles<false, uint32_t>(s, p.tile_w, p.tile_h, tiles_x, tiles_y, 0, 0,
                                                   0, nullptr, nullptr);
        }
    }
    counts[g] = count;
    keys[g] = depth_key(depth[g], count);
}

// ---------------------------------------------------------------------------
// Stable LSD radix sort pass (reduce-then-scan, no inter-block waits).
// Block tile: 256 threads x 16 items; warp w owns 512 consecutive items,
// ranked round by round with match.any so equal digits keep their order.
// ---------------------------------------------------------------------------
constexpr int kSortThreads = 256;
constexpr int kSortItems = 16;
constexpr int kSortTile = kSortThreads * kSortItems;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kMaxRadix = 256;

__device__ __forceinline__ int64_t read_count(const int32_t* ptr, int64_t cap)
{
    if (!ptr) return cap;
    int64_t v = *ptr;
    return v < 0 ? 0 : (v < cap ? v : cap);
}

template <typename K>
__global__ void __launch_bounds__(kSortThreads) radix_hist_kernel(
    const K* __restrict__ keys, const int32_t* n_ptr, int64_t n_cap, int shift, int bits,
    int max_blocks, bool drop_sentinel, uint32_t* __restrict__ hist)
{
    __shared__ uint32_t counters[kMaxRadix];
    int64_t n = read_count(n_ptr, n_cap);
    int64_t base = (int64_t)blockIdx.x * kSortTile;
    if (base >= n) return;
    int radix = 1 << bits;
    for (int d = threadIdx.x; d < radix; d += kSortThreads) counters[d] = 0;
    __syncthreads();
    for (int k = 0; k < kSortItems; k++) {
        int64_t i = base + (int64_t)k * kSortThreads + threadIdx.x;
        if (i < n) {
            uint32_t key = (uint32_t)keys[i];
            if (!(drop_sentinel && key == 0xFFFFFFFFu))
                atomicAdd(&counters[(key >> shift) & (radix - 1)], 1u);
        }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < radix; d += kSortThreads)
        hist[(int64_t)d * max_blocks + blockIdx.x] = counters[d];
}

// One block per digit: exclusive scan over the active blocks, digit total.
__global__ void __launch_bounds__(kSortThreads) radix_scan_kernel(
    const int32_t* n_ptr, int64_t n_cap, int max_blocks, uint32_t* __restrict__ hist,
    uint32_t* __restrict__ digit_totals)
{
    __shared__ uint32_t warp_sums[kSortWarps];
    int64_t n = read_count(n_ptr, n_cap);
    int blocks = (int)((n + kSortTile - 1) / kSortTile);
    uint32_t* row = hist + (int64_t)blockIdx.x * max_blocks;
    int per = (blocks + kSortThreads - 1) / kSortThreads;
    int lo = threadIdx.x * per, hi = min(blocks, lo + per);
    uint32_t local = 0;
    for (int b = lo; b < hi; b++) local += row[b];
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t inc = warp_inclusive_scan(local, lane);
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    uint32_t warp_base = 0;
    for (int w = 0; w < warp; w++) warp_base += warp_sums[w];
    uint32_t running = warp_base + inc - local;
    for (int b = lo; b < hi; b++) {
        uint32_t c = row[b];
        row[b] = running;
        running += c;
    }
    if (threadIdx.x == kSortThreads - 1) digit_totals[blockIdx.x] = warp_base + inc;
}

template <typename K>
__global__ void __launch_bounds__(kSortThreads) radix_scatter_kernel(
    const K* __restrict__ keys_in, const int32_t* __restrict__ vals_in, K* __restrict__ keys_out,
    int32_t* __restrict__ vals_out, const int32_t* n_ptr, int64_t n_cap, int shift, int bits,
    int max_blocks, bool drop_sentinel, const uint32_t* __restrict__ hist,
    const uint32_t* __restrict__ digit_totals, int32_t* n_out)
{
    __shared__ uint32_t warp_hist[kSortWarps][kMaxRadix + 1];
    __shared__ uint32_t digit_off[kMaxRadix];
    __shared__ uint32_t scan_tmp[kSortWarps];
    int64_t n = read_count(n_ptr, n_cap);
    int64_t base = (int64_t)blockIdx.x * kSortTile;
    int radix = 1 << bits;
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (base >= n) {
        // Block 0 still reports the surviving count when n == 0.
        if (blockIdx.x == 0 && threadIdx.x == 0 && n_out) *n_out = 0;
        return;
    }
    // Exclusive scan of the digit totals -> digit base offsets.
    {
        uint32_t t = threadIdx.x < radix ? digit_totals[threadIdx.x] : 0u;
        uint32_t inc = warp_inclusive_scan(t, lane);
        if (lane == 31) scan_tmp[warp] = inc;
        __syncthreads();
        uint32_t wb = 0;
        for (int w = 0; w < warp; w++) wb += scan_tmp[w];
        if (threadIdx.x < radix) digit_off[threadIdx.x] = wb + inc - t + hist[(int64_t)threadIdx.x * max_blocks + blockIdx.x];
        if (blockIdx.x == 0 && threadIdx.x == kSortThreads - 1 && n_out) *n_out = (int32_t)(wb + inc);
    }
    for (int d = lane; d <= radix; d += 32) warp_hist[warp][d] = 0;
    __syncwarp();
    K key[kSortItems];
    int32_t val[kSortItems];
    uint32_t rank[kSortItems];
    int digit[kSortItems];
    int64_t wbase = base + (int64_t)warp * 32 * kSortItems;
    unsigned lt = lanemask_lt();
#pragma unroll
    for (int r = 0; r < kSortItems; r++) {
        int64_t i = wbase + r * 32 + lane;
        bool valid = i < n;
        key[r] = valid ? keys_in[i] : (K)0;
        val[r] = valid ? (vals_in ? vals_in[i] : (int32_t)i) : 0;
        if (valid && drop_sentinel && (uint32_t)key[r] == 0xFFFFFFFFu) valid = false;
        int d = valid ? (int)(((uint32_t)key[r] >> shift) & (radix - 1)) : radix;
        digit[r] = d;
        unsigned peers = __match_any_sync(GSB_FULL_MASK, d);
        uint32_t before = warp_hist[warp][d];
        __syncwarp();
        rank[r] = before + __popc(peers & lt);
        if ((peers & lt) == 0) warp_hist[warp][d] = before + __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    for (int d = threadIdx.x; d < radix; d += kSortThreads) {
        uint32_t running = 0;
        for (int w = 0; w < kSortWarps; w++) {
            uint32_t c = warp_hist[w][d];
            warp_hist[w][d] = running;
            running += c;
        }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kSortItems; r++) {
        int d = digit[r];
        if (d < radix) {
            uint32_t dest = digit_off[d] + warp_hist[warp][d] + rank[r];
            keys_out[dest] = key[r];
            vals_out[dest] = val[r];
        }
    }
}

template <typename K>
int radix_pass(cudaStream_t s, const K* keys_in, const int32_t* vals_in, K* keys_out,
               int32_t* vals_out, const int32_t* n_ptr, int64_t n_cap, int shift, int bits,
               bool drop_sentinel, uint32_t* hist, uint32_t* totals, int32_t* n_out)
{
    int max_blocks = ceil_div(n_cap > 0 ? n_cap : 1, kSortTile);
    radix_hist_kernel<K><<<max_blocks, kSortThreads, 0, s>>>(keys_in, n_ptr, n_cap, shift, bits,
                                                             max_blocks, drop_sentinel, hist);
    radix_scan_kernel<<<1 << bits, kSortThreads, 0, s>>>(n_ptr, n_cap, max_blocks, hist, totals);
    radix_scatter_kernel<K><<<max_blocks, kSortThreads, 0, s>>>(
        keys_in, vals_in, keys_out, vals_out, n_ptr, n_cap, shift, bits, max_blocks,
        drop_sentinel, hist, totals, n_out);
    return check_launch();
}

// ---------------------------------------------------------------------------
// Depth-ordered scan (sorted_visibility.py:511-603): ends[r] = sum of the
// counts of ranks <= r; pair_count = ends[n-1]; overflow = pair_count > cap.
// ---------------------------------------------------------------------------
constexpr int kScanThreads = 256;
constexpr int kScanItems = 4;
constexpr int kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ int64_t block_reduce_i64(int64_t v, int64_t* shared)
{
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) shared[warp] = v;
    __syncthreads();
    int64_t total = 0;
    for (int w = 0; w < kScanThreads / 32; w++) total += shared[w];
    __syncthreads();
    return total;
}

__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(
    const int32_t* __restrict__ order, const int32_t* __restrict__ counts, const int32_t* n_ptr,
    int64_t n_cap, int64_t* __restrict__ block_sums)
{
    __shared__ int64_t shared[kScanThreads / 32];
    int64_t n = read_count(n_ptr, n_cap);
    int64_t base = (int64_t)blockIdx.x * kScanTile;
    if (base >= n) return;
    int64_t sum = 0;
    for (int k = 0; k < kScanItems; k++) {
        int64_t i = base + threadIdx.x * kScanItems + k;
        if (i < n) sum += counts[order[i]];
    }
    sum = block_reduce_i64(sum, shared);
    if (threadIdx.x == 0) block_sums[blockIdx.x] = sum;
}

__global__ void __launch_bounds__(kScanThreads) scan_kernel(
    const int32_t* __restrict__ order, const int32_t* __restrict__ counts, const int32_t* n_ptr,
    int64_t n_cap, const int64_t* __restrict__ block_sums, int64_t* __restrict__ ends,
    int64_t max_pairs, int32_t* pair_count, int32_t* overflow, int32_t* n_pairs_clamped)
{
    __shared__ int64_t shared[kScanThreads / 32];
    __shared__ int64_t warp_inc[kScanThreads / 32];
    int64_t n = read_count(n_ptr, n_cap);
    int64_t base = (int64_t)blockIdx.x * kScanTile;
    if (n == 0) {
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            *pair_count = 0;
            *overflow = 0;
            *n_pairs_clamped = 0;
        }
        return;
    }
    if (base >= n) return;
    int64_t earlier = 0;
    for (int64_t b = threadIdx.x; b < blockIdx.x; b += kScanThreads) earlier += block_sums[b];
    earlier = block_reduce_i64(earlier, shared);
    int64_t v[kScanItems];
    int64_t running = 0;
    for (int k = 0; k < kScanItems; k++) {
        int64_t i = base + threadIdx.x * kScanItems + k;
        v[k] = i < n ? counts[order[i]] : 0;
        running += v[k];
        v[k] = running;
    }
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int64_t inc = warp_inclusive_scan(running, lane);
    if (lane == 31) warp_inc[warp] = inc;
    __syncthreads();
    int64_t wb = 0;
    for (int w = 0; w < warp; w++) wb += warp_inc[w];
    int64_t before = earlier + wb + inc - running;
    for (int k = 0; k < kScanItems; k++) {
        int64_t i = base + threadIdx.x * kScanItems + k;
        if (i < n) {
            int64_t end = before + v[k];
            ends[i] = end;
            if (i == n - 1) {
                *pair_count = (int32_t)(end < 0x7fffffff ? end : 0x7fffffff);
                *overflow = end > max_pairs ? 1 : 0;
                *n_pairs_clamped = (int32_t)(end < max_pairs ? end : max_pairs);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Emission (sorted_visibility.py:373-484).
// ---------------------------------------------------------------------------
constexpr int kLanePairs = 16;

template <typename K>
__global__ void __launch_bounds__(256) emit_kernel(
    const int32_t* __restrict__ order, const int32_t* __restrict__ counts,
    const int64_t* __restrict__ ends, const int32_t* n_ptr, int64_t n_cap,
    const float* __restrict__ mean, const float* __restrict__ conic,
    const float* __restrict__ alpha, gsb_bin_params p, int tiles_x, int tiles_y,
    K* __restrict__ keys, int32_t* __restrict__ values, int32_t* __restrict__ queue,
    int32_t* __restrict__ queue_count)
{
    int64_t n = read_count(n_ptr, n_cap);
    int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int32_t count = 0, gid = 0;
    int64_t offset = 0;
    if (r < n) {
        gid = order[r];
        count = counts[gid];
        offset = ends[r] - count;
    }
    if (count > 0 && count <= kLanePairs && offset < p.max_pairs) {
        Splat s = load_splat(mean, conic, alpha, gid);
        process_tiles<true, K>(s, p.tile_w, p.tile_h, tiles_x, tiles_y, gid, offset, p.max_pairs,
                               keys, values);
    }
    bool large = count > kLanePairs && offset < p.max_pairs;
    unsigned queued = __ballot_sync(GSB_FULL_MASK, large);
    if (queued) {
        int lane = threadIdx.x & 31;
        int leader = __ffs(queued) - 1;
        int first = 0;
        if (lane == leader) first = atomicAdd(queue_count, __popc(queued));
        first = __shfl_sync(GSB_FULL_MASK, first, leader);
        if (large) queue[first + __popc(queued & lanemask_lt())] = (int32_t)r;
    }
}

// One warp per queued Gaussian: lanes take 32 rows at a time, then write the
// pairs of those rows as consecutive 32-pair chunks (each lane finds its row
// by binary search over the rows' exclusive offsets).
template <typename K>
__global__ void __launch_bounds__(256) emit_large_kernel(
    const int32_t* __restrict__ queue, const int32_t* __restrict__ queue_count,
    const int32_t* __restrict__ order, const int32_t* __restrict__ counts,
    const int64_t* __restrict__ ends, const float* __restrict__ mean,
    const float* __restrict__ conic, const float* __restrict__ alpha, gsb_bin_params p,
    int tiles_x, int tiles_y, K* __restrict__ keys, int32_t* __restrict__ values)
{
    int lane = threadIdx.x & 31;
    int warps = gridDim.x * (blockDim.x / 32);
    int total = *queue_count;
    for (int item = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); item < total; item += warps) {
        int64_t r = queue[item];
        int32_t gid = order[r];
        int64_t offset = ends[r] - counts[gid];
        Splat s = load_splat(mean, conic, alpha, gid);
        Ellipse e = ellipse_bounds(s.px, s.py, s.c00, s.c01, s.c11, s.alpha, p.tile_w, p.tile_h,
                                   tiles_x, tiles_y);
        int32_t m_max = last_line(e);
        for (int32_t base = e.u0; base < e.u1; base += 32) {
            int32_t u = base + lane;
            int32_t first = 0, cnt = 0;
            if (u < e.u1) {
                int32_t end;
                row_span(s, e, m_max, u, first, end);
                cnt = end - first;
            }
            int32_t inc = warp_inclusive_scan(cnt, lane);
            int32_t before = inc - cnt;
            int32_t rows_total = __shfl_sync(GSB_FULL_MASK, inc, 31);
            for (int32_t chunk = 0; chunk < rows_total; chunk += 32) {
                int32_t pair = chunk + lane;
                int row = 0;
#pragma unroll
                for (int step = 16; step > 0; step >>= 1) {
                    int32_t b = __shfl_sync(GSB_FULL_MASK, before, row + step);
                    if (b <= pair) row += step;
                }
                int32_t row_first = __shfl_sync(GSB_FULL_MASK, first, row);
                int32_t row_before = __shfl_sync(GSB_FULL_MASK, before, row);
                int64_t slot = offset + pair;
                if (pair < rows_total && slot < p.max_pairs) {
                    keys[slot] = (K)tile_key(e.is_y, base + row, row_first + pair - row_before,
                                             tiles_x);
                    values[slot] = gid;
                }
            }
            offset += rows_total;
        }
    }
}

// ---------------------------------------------------------------------------
// Tile ranges (sorted_visibility.py:628-659): offsets[t] = first index with
// key >= t over the first n sorted keys; empty tiles get contiguous offsets.
// ---------------------------------------------------------------------------
template <typename K>
__global__ void ranges_kernel(const K* __restrict__ keys, const int32_t* n_ptr, int64_t n_cap,
                              int num_tiles, int32_t* __restrict__ offsets)
{
    int64_t n = read_count(n_ptr, n_cap);
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (n == 0) {
        for (; i <= num_tiles; i += stride) offsets[i] = 0;
        return;
    }
    for (; i <= n; i += stride) {
        int64_t previous = i > 0 ? (int64_t)(uint32_t)keys[i - 1] : -1;
        int64_t current = i < n ? (int64_t)(uint32_t)keys[i] : num_tiles;
        if (current > num_tiles) current = num_tiles;
        for (int64_t t = previous + 1; t <= current; t++) offsets[t] = (int32_t)i;
    }
}

__global__ void zero_i32_kernel(int32_t* p, int n)
{
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = 0;
}

// digit_plan, kernels/pair_sort.py:33-37.
void digit_plan(int64_t num_tiles, int& passes, int& bits)
{
    int b = 1;
    while ((int64_t(1) << b) < num_tiles) b++;
    if (num_tiles <= 1) b = 1;
    passes = (b + 7) / 8;
    bits = (b + passes - 1) / passes;
}

struct BinLayout {
    uint32_t *depth_keys, *keys_a, *keys_b;
    int32_t *order_a, *order_b;
    int64_t* ends;
    int64_t* block_sums;
    int32_t *queue, *scalars;  // scalars: [0] binned count, [1] queue count, [2] clamped pairs
    void *pair_keys_a, *pair_keys_b;
    int32_t *pair_ids_a, *pair_ids_b;
    uint32_t *hist, *totals;
};

BinLayout carve_bin(char* base, const gsb_bin_params& p, size_t& used)
{
    Carver c{base, 0, 0};
    BinLayout L;
    int64_t C = p.capacity > 0 ? p.capacity : 1;
    int64_t P = p.max_pairs > 0 ? p.max_pairs : 1;
    int64_t tiles = (int64_t)ceil_div(p.width, p.tile_w) * ceil_div(p.height, p.tile_h);
    size_t key_bytes = tiles <= 65535 ? 2 : 4;
    L.depth_keys = c.take<uint32_t>(C);
    L.keys_a = c.take<uint32_t>(C);
    L.keys_b = c.take<uint32_t>(C);
    L.order_a = c.take<int32_t>(C);
    L.order_b = c.take<int32_t>(C);
    L.ends = c.take<int64_t>(C);
    L.block_sums = c.take<int64_t>(ceil_div(C, kScanTile));
    L.queue = c.take<int32_t>(C);
    L.scalars = c.take<int32_t>(8);
    L.pair_keys_a = c.take<char>(P * key_bytes);
    L.pair_keys_b = c.take<char>(P * key_bytes);
    L.pair_ids_a = c.take<int32_t>(P);
    L.pair_ids_b = c.take<int32_t>(P);
    int64_t max_items = C > P ? C : P;
    L.hist = c.take<uint32_t>((int64_t)kMaxRadix * ceil_div(max_items, kSortTile));
    L.totals = c.take<uint32_t>(kMaxRadix);
    used = c.used;
    return L;
}

template <typename K>
int tile_stage(cudaStream_t s, const gsb_bin_params& p, const BinLayout& L, int tiles_x,
               int tiles_y, int64_t num_tiles, const float* mean, const float* conic,
               const float* alpha, const int32_t* point_counts, int32_t* gaussian_ids,
               int32_t* tile_offsets)
{
    K* keys_a = static_cast<K*>(L.pair_keys_a);
    K* keys_b = static_cast<K*>(L.pair_keys_b);
    const int32_t* order = L.order_b;  // depth order after 4 passes
    const int32_t* n_binned = L.scalars + 0;
    int64_t C = p.capacity;
    emit_kernel<K><<<ceil_div(C, 256), 256, 0, s>>>(order, point_counts, L.ends, n_binned, C, mean,
                                                    conic, alpha, p, tiles_x, tiles_y, keys_a,
                                                    L.pair_ids_a, L.queue, L.scalars + 1);
    if (int e = check_launch()) return e;
    emit_large_kernel<K><<<148 * 8, 256, 0, s>>>(L.queue, L.scalars + 1, order, point_counts,
                                                 L.ends, mean, conic, alpha, p, tiles_x, tiles_y,
                                                 keys_a, L.pair_ids_a);
    if (int e = check_launch()) return e;
    int passes, bits;
    digit_plan(num_tiles, passes, bits);
    const int32_t* n_pairs = L.scalars + 2;
    const K* src_k = keys_a;
    const int32_t* src_v = L.pair_ids_a;
    // Ping-pong so that the last pass writes the ids into gaussian_ids.
    for (int pass = 0; pass < passes; pass++) {
        bool last = pass == passes - 1;
        K* dst_k = (src_k == keys_a) ? keys_b : keys_a;
        int32_t* dst_v = last ? gaussian_ids
                              : (src_v == L.pair_ids_a ? L.pair_ids_b : L.pair_ids_a);
        if (int e = radix_pass<K>(s, src_k, src_v, dst_k, dst_v, n_pairs, p.max_pairs,
                                  pass * bits, bits, false, L.hist, L.totals, nullptr))
            return e;
        src_k = dst_k;
        src_v = dst_v;
    }
    ranges_kernel<K><<<1024, 256, 0, s>>>(src_k, n_pairs, p.max_pairs, (int)num_tiles, tile_offsets);
    return check_launch();
}

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gsb_tile_sort_plan(int64_t num_tiles, int* passes, int* bits)
{
    if (!passes || !bits) return GSB_ERR_NULL;
    if (num_tiles <= 0) return GSB_ERR_INVALID;
    digit_plan(num_tiles, *passes, *bits);
    return GSB_OK;
}

extern "C" size_t gsb_bin_workspace_size(const gsb_bin_params* p)
{
    if (!p) return 0;
    size_t used = 0;
    carve_bin(nullptr, *p, used);
    return used;
}

extern "C" int gsb_bin(gsb_stream_t stream, const gsb_bin_params* p, void* workspace,
                       size_t workspace_bytes, const float* mean, const float* conic,
                       const float* alpha, const float* depth, const int8_t* visible,
                       int32_t* point_counts, int32_t* gaussian_ids, int32_t* tile_offsets,
                       int32_t* pair_count, int32_t* overflow)
{
    if (!p) return GSB_ERR_NULL;
    if (p->capacity < 0 || p->width <= 0 || p->height <= 0 || p->tile_w <= 0 || p->tile_h <= 0 ||
        p->max_pairs <= 0 || p->max_pairs >= (int64_t(1) << 31))
        return GSB_ERR_INVALID;
    int tiles_x = ceil_div(p->width, p->tile_w), tiles_y = ceil_div(p->height, p->tile_h);
    int64_t num_tiles = (int64_t)tiles_x * tiles_y;
    if (num_tiles >= (int64_t(1) << 31)) return GSB_ERR_INVALID;
    if (!workspace || workspace_bytes < gsb_bin_workspace_size(p) ||
        (reinterpret_cast<uintptr_t>(workspace) & 255))
        return GSB_ERR_WORKSPACE;
    if (!gaussian_ids || !tile_offsets || !pair_count || !overflow ||
        (p->capacity > 0 && (!mean || !conic || !alpha || !depth || !visible || !point_counts)))
        return GSB_ERR_NULL;
    if ((reinterpret_cast<uintptr_t>(conic) & 15) || (reinterpret_cast<uintptr_t>(mean) & 7))
        return GSB_ERR_INVALID;
    cudaStream_t s = as_stream(stream);
    size_t used = 0;
    BinLayout L = carve_bin(static_cast<char*>(workspace), *p, used);
    zero_i32_kernel<<<1, 32, 0, s>>>(L.scalars, 8);
    if (int e = check_launch()) return e;
    int64_t C = p->capacity;
    if (C > 0) {
        count_kernel<<<ceil_div(C, 256), 256, 0, s>>>((int)C, mean, conic, alpha, depth, visible,
                                                      *p, tiles_x, tiles_y, point_counts,
                                                      L.depth_keys);
        if (int e = check_launch()) return e;
        // Depth sort: pass 0 drops the Gaussians without pairs.
        if (int e = radix_pass<uint32_t>(s, L.depth_keys, nullptr, L.keys_a, L.order_a, nullptr, C,
                                         0, 8, true, L.hist, L.totals, L.scalars + 0))
            return e;
        const int32_t* nb = L.scalars + 0;
        if (int e = radix_pass<uint32_t>(s, L.keys_a, L.order_a, L.keys_b, L.order_b, nb, C, 8, 8,
                                         false, L.hist, L.totals, nullptr))
            return e;
        if (int e = radix_pass<uint32_t>(s, L.keys_b, L.order_b, L.keys_a, L.order_a, nb, C, 16, 8,
                                         false, L.hist, L.totals, nullptr))
            return e;
        if (int e = radix_pass<uint32_t>(s, L.keys_a, L.order_a, L.keys_b, L.order_b, nb, C, 24, 8,
                                         false, L.hist, L.totals, nullptr))
            return e;
    }
    scan_reduce_kernel<<<ceil_div(C > 0 ? C : 1, kScanTile), kScanThreads, 0, s>>>(
        L.order_b, point_counts, L.scalars + 0, C, L.block_sums);
    if (int e = check_launch()) return e;
    scan_kernel<<<ceil_div(C > 0 ? C : 1, kScanTile), kScanThreads, 0, s>>>(
        L.order_b, point_counts, L.scalars + 0, C, L.block_sums, L.ends, p->max_pairs, pair_count,
        overflow, L.scalars + 2);
    if (int e = check_launch()) return e;
    if (num_tiles <= 65535)
        return tile_stage<uint16_t>(s, *p, L, tiles_x, tiles_y, num_tiles, mean, conic, alpha,
                                    point_counts, gaussian_ids, tile_offsets);
    return tile_stage<uint32_t>(s, *p, L, tiles_x, tiles_y, num_tiles, mean, conic, alpha,
                                point_counts, gaussian_ids, tile_offsets);
}
