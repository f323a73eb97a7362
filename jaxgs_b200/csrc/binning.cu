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
// Per-block digit histograms of the emitted tile keys (the tile sort's
// per-pass histograms), accumulated in shared memory during emission.
struct KeyHist {
    uint32_t* local;  // [passes][256] in shared memory, or nullptr
    int passes, bits;
    __device__ __forceinline__ void add(uint32_t key) const
    {
        for (int pass = 0; pass < passes; pass++)
            atomicAdd(local + pass * 256 + ((key >> (pass * bits)) & ((1u << bits) - 1)), 1u);
    }
};

template <bool EMIT, typename K>
__device__ int32_t process_tiles(const Splat& s, int tile_w, int tile_h, int tiles_x, int tiles_y,
                                 int32_t gid, int64_t offset, int64_t max_pairs, K* keys,
                                 int32_t* values, KeyHist hist = KeyHist{nullptr, 0, 0})
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
                        const uint32_t key = tile_key(e.is_y, u, v, tiles_x);
                        keys[slot] = (K)key;
                        values[slot] = gid;
                        if (hist.local) hist.add(key);
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

// _count, sorted_visibility.py:307-370.  Also accumulates the four 8-bit
// digit histograms of the keys of Gaussians with pairs (the depth sort's
// per-pass histograms), one shared-memory update per distinct digit per warp.
__global__ void __launch_bounds__(256) count_kernel(int capacity, const float* __restrict__ mean,
                                                    const float* __restrict__ conic,
                                                    const float* __restrict__ alpha,
                                                    const float* __restrict__ depth,
                                                    const int8_t* __restrict__ visible,
                                                    gsb_bin_params p, int tiles_x, int tiles_y,
                                                    int32_t* __restrict__ counts,
                                                    uint32_t* __restrict__ keys,
                                                    uint32_t* __restrict__ depth_hist)
{
    pdl_begin();
    __shared__ uint32_t hist[4][256];
    for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) (&hist[0][0])[i] = 0;
    __syncthreads();
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int32_t count = 0;
    if (g < capacity && visible[g] != 0) {
        float2 m = *reinterpret_cast<const float2*>(mean + g * 2);
        float4 c = *reinterpret_cast<const float4*>(conic + g * 4);
        float a = alpha[g];
        if (count_gate(m.x, m.y, c.x, c.y, c.w, a, p.width, p.height)) {
            Splat s{fsub(m.x, 0.5f), fsub(m.y, 0.5f), c.x, c.y, c.w, a};
            count = process_tiles<false, uint32_t>(s, p.tile_w, p.tile_h, tiles_x, tiles_y, 0, 0,
                                                   0, nullptr, nullptr);
        }
    }
    if (g < capacity) {
        const uint32_t key = depth_key(depth[g], count);
        counts[g] = count;
        keys[g] = key;
    }
    const uint32_t key = g < capacity ? depth_key(depth[g], count) : 0xFFFFFFFFu;
    const unsigned lt = lanemask_lt();
#pragma unroll
    for (int pass = 0; pass < 4; pass++) {
        const int d = count > 0 ? (int)((key >> (8 * pass)) & 255u) : 256;
        const unsigned peers = __match_any_sync(GSB_FULL_MASK, d);
        if ((peers & lt) == 0 && d < 256) atomicAdd(&hist[pass][d], (uint32_t)__popc(peers));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) {
        const uint32_t v = (&hist[0][0])[i];
        if (v) atomicAdd(depth_hist + i, v);
    }
}

// ---------------------------------------------------------------------------
// Stable LSD radix sort, onesweep style.
//  * onesweep_hist_kernel reads the keys once and accumulates the digit
//    histograms of every pass (a key's digits do not change between passes).
//  * Each pass is one kernel.  A block takes the next partition index from an
//    atomic counter, so every lower partition was taken by a block that is
//    already running; it ranks its 2048 items with bit-ballot multisplit
//    (stable within the tile), publishes its per-digit counts, then looks
//    back over the predecessors' published counts until one carries an
//    inclusive prefix (decoupled look-back), publishes its own inclusive
//    prefix and scatters.  Items are staged in shared memory in digit order,
//    so each digit's run leaves the block as consecutive addresses.
//  * Every look-back spin is bounded; on expiry the block records an error
//    word (reported as GSB_ERR_LAUNCH by the host on the next call) and uses
//    what it has, so a fault can never turn into a hang.
// The first depth-sort pass drops the 0xFFFFFFFF keys of Gaussians without
// pairs; later passes sort only the survivors.
// ---------------------------------------------------------------------------
constexpr int kSortThreads = 256;
constexpr int kSortItems = 8;
constexpr int kSortTile = kSortThreads * kSortItems;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kMaxRadix = 256;
constexpr uint32_t kFlagAggregate = 1u << 30;
constexpr uint32_t kFlagPrefix = 2u << 30;
constexpr uint32_t kValueMask = (1u << 30) - 1;
constexpr int kSpinLimit = 1 << 22;

__device__ __forceinline__ int64_t read_count(const int32_t* ptr, int64_t cap)
{
    if (!ptr) return cap;
    int64_t v = *ptr;
    return v < 0 ? 0 : (v < cap ? v : cap);
}

template <typename K>
__device__ __forceinline__ int item_digit(K key, bool valid, bool drop_sentinel, int shift, int radix)
{
    if (!valid || (drop_sentinel && (uint32_t)key == 0xFFFFFFFFu)) return radix;
    return (int)(((uint32_t)key >> shift) & (radix - 1));
}

// Lanes of the warp holding the same digit (bit-ballot multisplit); digit
// `radix` (invalid items) gets its own class through the extra bit.
__device__ __forceinline__ unsigned same_digit_mask(int d, int bits)
{
    unsigned m = GSB_FULL_MASK;
    for (int k = 0; k <= bits; k++) {
        const bool b = (d >> k) & 1;
        const unsigned bal = __ballot_sync(GSB_FULL_MASK, b);
        m &= b ? bal : ~bal;
    }
    return m;
}

// Digit histograms of all passes: hist[pass * 256 + digit] (global atomics,
// one per digit per block).  passes <= 4.
template <typename K>
__global__ void __launch_bounds__(kSortThreads) onesweep_hist_kernel(
    const K* __restrict__ keys, const int32_t* n_ptr, int64_t n_cap, int passes, int bits,
    bool drop_sentinel, uint32_t* __restrict__ hist)
{
    pdl_begin();
    __shared__ uint32_t local[4][kMaxRadix];
    const int64_t n = read_count(n_ptr, n_cap);
    const int radix = 1 << bits;
    for (int i = threadIdx.x; i < 4 * kMaxRadix; i += kSortThreads) (&local[0][0])[i] = 0;
    __syncthreads();
    const unsigned lt = lanemask_lt();
    const int64_t stride = (int64_t)gridDim.x * kSortThreads;
    for (int64_t base = (int64_t)blockIdx.x * kSortThreads; base < n; base += stride) {
        const int64_t i = base + threadIdx.x;
        const bool valid = i < n;
        const K key = valid ? keys[i] : (K)0;
        for (int pass = 0; pass < passes; pass++) {
            const int d = item_digit(key, valid, drop_sentinel, pass * bits, radix);
            const unsigned m = same_digit_mask(d, bits);
            if ((m & lt) == 0 && d < radix) atomicAdd(&local[pass][d], (uint32_t)__popc(m));
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < passes * radix; i += kSortThreads) {
        const uint32_t c = local[i / radix][i % radix];
        if (c) atomicAdd(hist + (i / radix) * kMaxRadix + (i % radix), c);
    }
}

// Exclusive scan of 256 values held one per thread (all threads participate).
__device__ __forceinline__ uint32_t block_exclusive_scan256(uint32_t v, uint32_t* scratch)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t inc = warp_inclusive_scan(v, lane);
    if (lane == 31) scratch[warp] = inc;
    __syncthreads();
    uint32_t wb = 0;
    for (int w = 0; w < warp; w++) wb += scratch[w];
    __syncthreads();
    return wb + inc - v;
}

template <typename K>
__global__ void __launch_bounds__(kSortThreads) onesweep_pass_kernel(
    const K* __restrict__ keys_in, const int32_t* __restrict__ vals_in, K* __restrict__ keys_out,
    int32_t* __restrict__ vals_out, const int32_t* n_ptr, int64_t n_cap, int shift, int bits,
    bool drop_sentinel, const uint32_t* __restrict__ pass_hist, uint32_t* status,
    int32_t* part_counter, int32_t* n_out, int32_t* error)
{
    pdl_begin();
    __shared__ uint32_t warp_hist[kSortWarps][kMaxRadix + 1];
    __shared__ uint32_t global_off[kMaxRadix];
    __shared__ uint32_t block_start[kMaxRadix];
    __shared__ uint32_t scratch[kSortWarps];
    __shared__ K s_keys[kSortTile];
    __shared__ int32_t s_vals[kSortTile];
    __shared__ int s_part;
    __shared__ uint32_t s_valid;
    const int radix = 1 << bits;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t n = read_count(n_ptr, n_cap);
    if (threadIdx.x == 0) s_part = atomicAdd(part_counter, 1);
    for (int d = lane; d <= radix; d += 32) warp_hist[warp][d] = 0;
    __syncthreads();
    const int part = s_part;
    const int64_t base = (int64_t)part * kSortTile;
    if (part == 0 && threadIdx.x == 0 && n_out) {
        uint32_t total = 0;
        for (int d = 0; d < radix; d++) total += pass_hist[d];
        *n_out = (int32_t)total;
    }
    if (base >= n) return;  // uniform: no later partition waits on this one
    K key[kSortItems];
    int32_t val[kSortItems];
    int digit[kSortItems];
    uint32_t rank[kSortItems];
    const int64_t wbase = base + (int64_t)warp * 32 * kSortItems;
#pragma unroll
    for (int r = 0; r < kSortItems; r++) {
        const int64_t i = wbase + r * 32 + lane;
        const bool valid = i < n;
        key[r] = valid ? keys_in[i] : (K)0;
        val[r] = valid ? (vals_in ? vals_in[i] : (int32_t)i) : 0;
        digit[r] = item_digit(key[r], valid, drop_sentinel, shift, radix);
    }
    const unsigned lt = lanemask_lt();
#pragma unroll
    for (int r = 0; r < kSortItems; r++) {
        const int d = digit[r];
        const unsigned m = same_digit_mask(d, bits);
        const uint32_t before = warp_hist[warp][d];
        __syncwarp();
        rank[r] = before + __popc(m & lt);
        if ((m & lt) == 0) warp_hist[warp][d] = before + __popc(m);
        __syncwarp();
    }
    __syncthreads();
    const int d = threadIdx.x;  // kSortThreads == kMaxRadix
    uint32_t count = 0;
    if (d < radix) {
#pragma unroll
        for (int w = 0; w < kSortWarps; w++) {
            const uint32_t c = warp_hist[w][d];
            warp_hist[w][d] = count;
            count += c;
        }
        // Publish this partition's count, then look back for the prefix.
        volatile uint32_t* st = status;
        if (part == 0) {
            st[d] = kFlagPrefix | count;
        } else {
            st[(int64_t)part * kMaxRadix + d] = kFlagAggregate | count;
        }
    }
    uint32_t excl = 0;
    if (d < radix && part > 0) {
        // Windowed look-back: the status words of up to kWindow predecessors
        // are loaded together, so the walk costs one latency per window.
        constexpr int kWindow = 8;
        volatile uint32_t* st = status;
        int j = part - 1;
        int spins = 0;
        bool done = false;
        while (!done && j >= 0) {
            uint32_t v[kWindow];
#pragma unroll
            for (int k = 0; k < kWindow; k++) v[k] = (j - k >= 0) ? (uint32_t)st[(int64_t)(j - k) * kMaxRadix + d] : (uint32_t)(2u << 30);
            int k = 0;
            uint32_t acc = 0;
            for (; k < kWindow; k++) {
                const uint32_t flag = v[k] & ~kValueMask;
                if (flag == 0) break;  // not published yet: wait here
                acc += v[k] & kValueMask;
                if (flag == kFlagPrefix) {
                    done = true;
                    break;
                }
            }
            if (done) {
                excl += acc;
            } else if (k == kWindow) {
                excl += acc;
                j -= kWindow;
            } else {
                excl += acc;  // consume the published run, retry the first gap
                j -= k;
                if (++spins > kSpinLimit) {
                    atomicExch(error, 1);
                    done = true;
                }
            }
        }
        st[(int64_t)part * kMaxRadix + d] = kFlagPrefix | ((excl + count) & kValueMask);
    }
    const uint32_t start = block_exclusive_scan256(count, scratch);
    const uint32_t digit_base = block_exclusive_scan256(d < radix ? pass_hist[d] : 0u, scratch);
    if (d < radix) {
        block_start[d] = start;
        global_off[d] = digit_base + excl;
    }
    if (d == radix - 1) s_valid = start + count;
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kSortItems; r++) {
        const int dd = digit[r];
        if (dd < radix) {
            const uint32_t pos = block_start[dd] + warp_hist[warp][dd] + rank[r];
            s_keys[pos] = key[r];
            s_vals[pos] = val[r];
        }
    }
    __syncthreads();
    const uint32_t valid_count = s_valid;
    for (uint32_t j = threadIdx.x; j < valid_count; j += kSortThreads) {
        const K k = s_keys[j];
        const int dd = (int)(((uint32_t)k >> shift) & (radix - 1));
        const uint32_t dst = global_off[dd] + (j - block_start[dd]);
        keys_out[dst] = k;
        vals_out[dst] = s_vals[j];
    }
}

__global__ void zero_u32_kernel(uint32_t* p, int64_t n)
{
    pdl_begin();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        p[i] = 0;
}

// Zeroes up to three word ranges in one launch.
__global__ void zero_ranges_kernel(uint32_t* a, int64_t na, uint32_t* b, int64_t nb, uint32_t* c,
                                   int64_t nc)
{
    pdl_begin();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < na + nb + nc; i += stride) {
        if (i < na) a[i] = 0;
        else if (i < na + nb) b[i - na] = 0;
        else c[i - na - nb] = 0;
    }
}

// Sort scratch: histograms [4][256], status [4][partitions][256], counters.
struct SortScratch {
    uint32_t* hist;
    uint32_t* status;
    int32_t* counters;
    int partitions;
};

// Histograms, look-back status words and partition counters are one
// contiguous region, zeroed by one launch.
int64_t sort_scratch_words(const SortScratch& w)
{
    return 4 * kMaxRadix + 4 * (int64_t)w.partitions * kMaxRadix + 8;
}

int zero_sort_scratch(cudaStream_t s, const SortScratch& w)
{
    gsb::launch(zero_u32_kernel, 256, 256, 0, s, w.hist, sort_scratch_words(w));
    return check_launch();
}

// With hist_ready the caller has zeroed the scratch and accumulated the
// per-pass digit histograms into w.hist (the producer kernels do it).
template <typename K>
int onesweep_sort(cudaStream_t s, const K* keys_in, const int32_t* vals_in, K* key_a, K* key_b,
                  int32_t* val_a, int32_t* val_b, int32_t* val_out, const K** sorted_keys,
                  const int32_t** sorted_vals, const int32_t* n_ptr, int64_t n_cap, int passes,
                  int bits, bool drop_sentinel, const SortScratch& w, int32_t* n_out,
                  int32_t* error, bool hist_ready)
{
    if (!hist_ready) {
        if (int e = zero_sort_scratch(s, w)) return e;
        gsb::launch(onesweep_hist_kernel<K>, 148 * 4, kSortThreads, 0, s, keys_in, n_ptr, n_cap, passes,
                                                                 bits, drop_sentinel, w.hist);
        if (int e = check_launch()) return e;
    }
    const K* src_k = keys_in;
    const int32_t* src_v = vals_in;
    const int32_t* pass_n = n_ptr;
    for (int pass = 0; pass < passes; pass++) {
        const bool last = pass == passes - 1;
        K* dst_k = (src_k == key_a) ? key_b : key_a;
        int32_t* dst_v = (last && val_out) ? val_out : ((src_v == val_a) ? val_b : val_a);
        gsb::launch(onesweep_pass_kernel<K>, w.partitions, kSortThreads, 0, s, 
            src_k, src_v, dst_k, dst_v, pass_n, n_cap, pass * bits, bits, drop_sentinel && pass == 0,
            w.hist + pass * kMaxRadix, w.status + (int64_t)pass * w.partitions * kMaxRadix,
            w.counters + pass, (pass == 0 && drop_sentinel) ? n_out : nullptr, error);
        if (int e = check_launch()) return e;
        if (pass == 0 && drop_sentinel) pass_n = n_out;
        src_k = dst_k;
        src_v = dst_v;
    }
    *sorted_keys = src_k;
    *sorted_vals = src_v;
    return GSB_OK;
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
    pdl_begin();
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
    pdl_begin();
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

// Adds the block's digit counts to the tile sort's global histograms
// (hist[pass * 256 + digit], the layout onesweep_sort reads).
__device__ __forceinline__ void flush_key_hist(const uint32_t* local, int passes,
                                               uint32_t* key_hist)
{
    __syncthreads();
    for (int i = threadIdx.x; i < passes * 256; i += blockDim.x) {
        const uint32_t c = local[i];
        if (c) atomicAdd(key_hist + i, c);
    }
}

template <typename K>
__global__ void __launch_bounds__(256) emit_kernel(
    const int32_t* __restrict__ order, const int32_t* __restrict__ counts,
    const int64_t* __restrict__ ends, const int32_t* n_ptr, int64_t n_cap,
    const float* __restrict__ mean, const float* __restrict__ conic,
    const float* __restrict__ alpha, gsb_bin_params p, int tiles_x, int tiles_y,
    K* __restrict__ keys, int32_t* __restrict__ values, int32_t* __restrict__ queue,
    int32_t* __restrict__ queue_count, int passes, int bits, uint32_t* __restrict__ key_hist)
{
    pdl_begin();
    __shared__ uint32_t local[4 * 256];
    for (int i = threadIdx.x; i < passes * 256; i += blockDim.x) local[i] = 0;
    __syncthreads();
    const KeyHist hist{local, passes, bits};
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
                               keys, values, hist);
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
    flush_key_hist(local, passes, key_hist);
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
    int tiles_x, int tiles_y, K* __restrict__ keys, int32_t* __restrict__ values, int passes,
    int bits, uint32_t* __restrict__ key_hist)
{
    pdl_begin();
    __shared__ uint32_t local[4 * 256];
    for (int i = threadIdx.x; i < passes * 256; i += blockDim.x) local[i] = 0;
    __syncthreads();
    const KeyHist hist{local, passes, bits};
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
                    const uint32_t key =
                        tile_key(e.is_y, base + row, row_first + pair - row_before, tiles_x);
                    keys[slot] = (K)key;
                    values[slot] = gid;
                    hist.add(key);
                }
            }
            offset += rows_total;
        }
    }
    flush_key_hist(local, passes, key_hist);
}

// ---------------------------------------------------------------------------
// Tile ranges (sorted_visibility.py:628-659): offsets[t] = first index with
// key >= t over the first n sorted keys; empty tiles get contiguous offsets.
// Also reports an internal sort time-out as bit 1 of overflow.
// ---------------------------------------------------------------------------
template <typename K>
__global__ void ranges_kernel(const K* __restrict__ keys, const int32_t* n_ptr, int64_t n_cap,
                              int num_tiles, int32_t* __restrict__ offsets,
                              const int32_t* __restrict__ sort_error, int32_t* overflow)
{
    pdl_begin();
    if (blockIdx.x == 0 && threadIdx.x == 0 && *sort_error) atomicOr(overflow, 2);
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
    int32_t *queue, *scalars;  // [0] binned, [1] queue count, [2] clamped pairs, [3] sort error
    void *emit_keys, *pair_keys_a, *pair_keys_b;
    int32_t *emit_ids, *pair_ids_a, *pair_ids_b;
    SortScratch depth_sort, pair_sort;
};

SortScratch carve_sort(Carver& c, int64_t items)
{
    SortScratch w;
    w.partitions = ceil_div(items > 0 ? items : 1, kSortTile);
    uint32_t* base = c.take<uint32_t>(4 * kMaxRadix + 4 * (int64_t)w.partitions * kMaxRadix + 8);
    w.hist = base;
    w.status = base ? base + 4 * kMaxRadix : nullptr;
    w.counters = base ? reinterpret_cast<int32_t*>(w.status + 4 * (int64_t)w.partitions * kMaxRadix) : nullptr;
    return w;
}

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
    L.emit_keys = c.take<char>(P * key_bytes);
    L.pair_keys_a = c.take<char>(P * key_bytes);
    L.pair_keys_b = c.take<char>(P * key_bytes);
    L.emit_ids = c.take<int32_t>(P);
    L.pair_ids_a = c.take<int32_t>(P);
    L.pair_ids_b = c.take<int32_t>(P);
    L.depth_sort = carve_sort(c, C);
    L.pair_sort = carve_sort(c, P);
    used = c.used;
    return L;
}

template <typename K>
int tile_stage(cudaStream_t s, const gsb_bin_params& p, const BinLayout& L, int tiles_x,
               int tiles_y, int64_t num_tiles, const float* mean, const float* conic,
               const float* alpha, const int32_t* point_counts, const int32_t* order,
               int32_t* gaussian_ids, int32_t* tile_offsets, int32_t* overflow)
{
    K* emit_keys = static_cast<K*>(L.emit_keys);
    const int32_t* n_binned = L.scalars + 0;
    int64_t C = p.capacity;
    int passes, bits;
    digit_plan(num_tiles, passes, bits);
    // The emission kernels also accumulate the tile sort's digit histograms
    // (its scratch was zeroed at the start of gsb_bin).
    gsb::launch(emit_kernel<K>, ceil_div(C > 0 ? C : 1, 256), 256, 0, s, 
        order, point_counts, L.ends, n_binned, C, mean, conic, alpha, p, tiles_x, tiles_y,
        emit_keys, L.emit_ids, L.queue, L.scalars + 1, passes, bits, L.pair_sort.hist);
    if (int e = check_launch()) return e;
    gsb::launch(emit_large_kernel<K>, 148 * 8, 256, 0, s, L.queue, L.scalars + 1, order, point_counts,
                                                 L.ends, mean, conic, alpha, p, tiles_x, tiles_y,
                                                 emit_keys, L.emit_ids, passes, bits,
                                                 L.pair_sort.hist);
    if (int e = check_launch()) return e;
    const K* sorted_keys = nullptr;
    const int32_t* sorted_ids = nullptr;
    if (int e = onesweep_sort<K>(s, emit_keys, L.emit_ids, static_cast<K*>(L.pair_keys_a),
                                 static_cast<K*>(L.pair_keys_b), L.pair_ids_a, L.pair_ids_b,
                                 gaussian_ids, &sorted_keys, &sorted_ids, L.scalars + 2,
                                 p.max_pairs, passes, bits, false, L.pair_sort, nullptr,
                                 L.scalars + 3, true))
        return e;
    gsb::launch(ranges_kernel<K>, 1024, 256, 0, s, sorted_keys, L.scalars + 2, p.max_pairs, (int)num_tiles,
                                          tile_offsets, L.scalars + 3, overflow);
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
        p->max_pairs <= 0 || p->max_pairs >= (int64_t(1) << 30))
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
    // Scalars, the depth sort's and the tile sort's scratch: one launch.
    gsb::launch(zero_ranges_kernel, 296, 256, 0, s, reinterpret_cast<uint32_t*>(L.scalars), 8,
                                           L.depth_sort.hist, sort_scratch_words(L.depth_sort),
                                           L.pair_sort.hist, sort_scratch_words(L.pair_sort));
    if (int e = check_launch()) return e;
    int64_t C = p->capacity;
    const uint32_t* sorted_depth_keys = nullptr;
    const int32_t* depth_order = L.order_a;
    if (C > 0) {
        gsb::launch(count_kernel, ceil_div(C, 256), 256, 0, s, (int)C, mean, conic, alpha, depth, visible,
                                                      *p, tiles_x, tiles_y, point_counts,
                                                      L.depth_keys, L.depth_sort.hist);
        if (int e = check_launch()) return e;
        // Depth sort: pass 0 drops the Gaussians without pairs.
        if (int e = onesweep_sort<uint32_t>(s, L.depth_keys, nullptr, L.keys_a, L.keys_b, L.order_a,
                                            L.order_b, nullptr, &sorted_depth_keys, &depth_order,
                                            nullptr, C, 4, 8, true, L.depth_sort, L.scalars + 0,
                                            L.scalars + 3, true))
            return e;
    }
    gsb::launch(scan_reduce_kernel, ceil_div(C > 0 ? C : 1, kScanTile), kScanThreads, 0, s, 
        depth_order, point_counts, L.scalars + 0, C, L.block_sums);
    if (int e = check_launch()) return e;
    gsb::launch(scan_kernel, ceil_div(C > 0 ? C : 1, kScanTile), kScanThreads, 0, s, 
        depth_order, point_counts, L.scalars + 0, C, L.block_sums, L.ends, p->max_pairs, pair_count,
        overflow, L.scalars + 2);
    if (int e = check_launch()) return e;
    if (num_tiles <= 65535)
        return tile_stage<uint16_t>(s, *p, L, tiles_x, tiles_y, num_tiles, mean, conic, alpha,
                                    point_counts, depth_order, gaussian_ids, tile_offsets, overflow);
    return tile_stage<uint32_t>(s, *p, L, tiles_x, tiles_y, num_tiles, mean, conic, alpha,
                                point_counts, depth_order, gaussian_ids, tile_offsets, overflow);
}
