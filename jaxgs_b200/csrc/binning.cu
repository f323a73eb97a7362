// Tile binning for sm_100a: AccuTile count + depth keys, stable depth sort,
// depth-ordered scan, pair emission, stable LSD tile sort and tile ranges.
//
// Result contract (kernels/sorted_binning.py:9-117): the valid prefix of
// gaussian_ids lists, tile by tile, every Gaussian whose AccuTile ellipse
// covers the tile, ordered by (depth key, Gaussian id).  Internally:
//   1. count_kernel      — per Gaussian pair count and 32-bit depth key.
//   2. depth sort        — 4 stable 8-bit LSD passes; the first pass drops the
//                          0xFFFFFFFF keys of Gaussians without pairs, so the
//                          remaining passes sort only binned Gaussians.  The
//                          last pass also writes the counts in depth order and
//                          sums them per block of 256 depth ranks.
//   3. emission          — each block adds up the earlier blocks' sums and
//                          scans its own counts (the inclusive scan of counts
//                          in depth order), then each Gaussian writes its pairs
//                          to its segment; one thread per small Gaussian, one
//                          warp per large one.
//   4. tile sort         — stable LSD passes over the tile key (digit plan of
//                          kernels/pair_sort.py:33-37) of the emitted pairs.
//   5. tile ranges       — offsets[t] = first pair with tile >= t.
// Every stage is a plain kernel launch on one stream, with no host
// synchronisation; the only inter-block waits are the sort passes' bounded
// look-backs.  Counts that only the device knows (binned Gaussians, pairs)
// are read by the kernels, whose grids are sized for the capacity and whose
// surplus blocks exit at once.
#include <atomic>

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
    float block_u, block_v, inv_block_v;
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

// x / d for a tile dimension d.  When d is a power of two (inv = 1/d, else
// inv = 0), x * inv is the same correctly rounded quotient -- the product
// x * 2^-k is exact before its one rounding, as the quotient is -- so the
// IEEE division becomes one multiply without changing a bit.
__device__ __forceinline__ float div_dim(float x, float d, float inv)
{
    return inv != 0.0f ? fmul(x, inv) : fdiv(x, d);
}

__host__ __device__ inline float pow2_reciprocal(int d)
{
    return (d > 0 && (d & (d - 1)) == 0) ? 1.0f / (float)d : 0.0f;
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
    const float inv_tw = pow2_reciprocal(tile_w), inv_th = pow2_reciprocal(tile_h);
    int32_t x0 = max(0, min(tiles_x, trunc_i32(div_dim(xmin, tw, inv_tw))));
    int32_t y0 = max(0, min(tiles_y, trunc_i32(div_dim(ymin, th, inv_th))));
    int32_t x1 = max(0, min(tiles_x, trunc_i32(div_dim(fsub(fadd(xmax, tw), 1.0f), tw, inv_tw))));
    int32_t y1 = max(0, min(tiles_y, trunc_i32(div_dim(fsub(fadd(ymax, th), 1.0f), th, inv_th))));
    e.disc = disc;
    e.level = level;
    e.is_y = (y1 - y0) < (x1 - x0);
    if (e.is_y) {
        e.block_u = th; e.block_v = tw; e.inv_block_v = inv_tw;
        e.u0 = y0; e.u1 = y1; e.v0 = x0; e.v1 = x1;
        e.bbox_u_min = ymin; e.bbox_u_max = ymax; e.bbox_v_min = xmin; e.bbox_v_max = xmax;
        e.arg_min = argmin_x; e.arg_max = argmax_x;
    } else {
        e.block_u = tw; e.block_v = th; e.inv_block_v = inv_th;
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
    first = max(e.v0, min(e.v1, trunc_i32(div_dim(emin, e.block_v, e.inv_block_v))));
    end = min(e.v1, max(e.v0, trunc_i32(fadd(div_dim(emax, e.block_v, e.inv_block_v), 1.0f))));
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

// _count, sorted_visibility.py:307-370.  A block covers kCountSlots slots.
// The cheap gate (visible, alpha, conic, screen bounds) runs first; the slots
// that pass it are queued in shared memory and walked with full warps (the
// AccuTile ellipse and row walk are the costly part, and about a third of the
// slots pass).  The kernel also accumulates the four 8-bit digit histograms
// of the keys of Gaussians with pairs (the depth sort's per-pass
// histograms) in shared memory, and
// zeroes this call's sort look-back words and per-block pair sums (`bulk`),
// which only later kernels of the call read.
constexpr int kCountThreads = 256;
constexpr int kCountPerThread = 4;
constexpr int kCountSlots = kCountThreads * kCountPerThread;

__global__ void __launch_bounds__(kCountThreads) count_kernel(
    int capacity, const float* __restrict__ mean, const float* __restrict__ conic,
    const float* __restrict__ alpha, const float* __restrict__ depth,
    const int8_t* __restrict__ visible, gsb_bin_params p, int tiles_x, int tiles_y,
    int32_t* __restrict__ counts, uint32_t* __restrict__ keys, uint32_t* __restrict__ depth_hist,
    uint4* __restrict__ bulk, int64_t bulk_vec4)
{
    pdl_begin();
    __shared__ uint32_t hist[4][256];
    __shared__ int32_t queue[kCountSlots];
    __shared__ int queued;
    for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) (&hist[0][0])[i] = 0;
    if (threadIdx.x == 0) queued = 0;
    {
        const int64_t stride = (int64_t)gridDim.x * blockDim.x;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < bulk_vec4; i += stride)
            bulk[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const unsigned lt = lanemask_lt();
    const int64_t first = (int64_t)blockIdx.x * kCountSlots;
#pragma unroll
    for (int k = 0; k < kCountPerThread; k++) {
        const int64_t g = first + k * kCountThreads + threadIdx.x;
        bool gated = false;
        if (g < capacity && visible[g] != 0) {
            const float2 m = *reinterpret_cast<const float2*>(mean + g * 2);
            const float4 c = *reinterpret_cast<const float4*>(conic + g * 4);
            gated = count_gate(m.x, m.y, c.x, c.y, c.w, alpha[g], p.width, p.height);
        }
        if (g < capacity && !gated) {
            counts[g] = 0;
            keys[g] = 0xFFFFFFFFu;
        }
        const unsigned mask = __ballot_sync(GSB_FULL_MASK, gated);
        int at = 0;
        if (lane == 0 && mask) at = atomicAdd(&queued, __popc(mask));
        at = __shfl_sync(GSB_FULL_MASK, at, 0);
        if (gated) queue[at + __popc(mask & lt)] = (int32_t)(g - first);
    }
    __syncthreads();
    const int total = queued;
    for (int base = 0; base < total; base += kCountThreads) {
        const int q = base + threadIdx.x;
        int32_t count = 0;
        uint32_t key = 0xFFFFFFFFu;
        if (q < total) {
            const int64_t g = first + queue[q];
            const Splat sp = load_splat(mean, conic, alpha, g);
            count = process_tiles<false, uint32_t>(sp, p.tile_w, p.tile_h, tiles_x, tiles_y, 0, 0,
                                                   0, nullptr, nullptr);
            key = depth_key(depth[g], count);
            counts[g] = count;
            keys[g] = key;
        }
        if (count > 0) {
#pragma unroll
            for (int pass = 0; pass < 4; pass++) atomicAdd(&hist[pass][(key >> (8 * pass)) & 255u], 1u);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) {
        const uint32_t v = (&hist[0][0])[i];
        if (v) atomicAdd(depth_hist + i, v);
    }
}

// ---------------------------------------------------------------------------
// Stable LSD radix sort, onesweep style: one kernel per digit pass.
//  * The digit histograms of every pass come from the kernels that produce
//    the keys (count_kernel for the depth keys, the emission kernels for the
//    tile keys; a key's digits do not change between passes), so no pass
//    reads its input twice.
//  * Partitions are large (512 threads x 8 items), so the binning's small
//    sorts (a few hundred thousand to a few million items) have few of them
//    and the look-back chain stays short.
//  * Only the blocks a partition needs take one (blocks past the
//    device-side item count exit at once); each takes the next partition
//    index from an atomic counter, so every lower partition belongs to a
//    block that is already running.  It ranks its items stably (bit-ballot
//    multisplit: bits + 1 ballots per item, which measured faster here than
//    __match_any_sync, whose throughput falls with many distinct digits;
//    items are ordered by index, lane-major inside a warp's 256-item run,
//    warps in order), publishes its per-digit counts at once, stages the
//    items in shared memory in digit order and only then looks back over its
//    predecessors' published counts until one carries an inclusive prefix
//    (decoupled look-back), 32 predecessors per round trip.
//  * Each digit's run leaves the block as consecutive addresses.
//  * Every look-back wait is bounded; on expiry the block records an error
//    word (reported as overflow bit 1) and uses what it has, so a fault can
//    never turn into a hang.
// The first depth pass drops the 0xFFFFFFFF keys of Gaussians without pairs;
// later passes sort only the survivors.  The last depth pass also writes the
// pair counts in depth order and adds them up per emission block, which is
// the depth-ordered scan of sorted_visibility.py:511-603 minus its last step
// (the emission kernel finishes it).
// ---------------------------------------------------------------------------
constexpr int kSortThreads = 512;
constexpr int kSortItems = 8;
constexpr int kSortTile = kSortThreads * kSortItems;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kMaxRadix = 256;
constexpr uint32_t kFlagAggregate = 1u << 30;
constexpr uint32_t kFlagPrefix = 2u << 30;
constexpr uint32_t kValueMask = (1u << 30) - 1;
constexpr int kSpinLimit = 1 << 22;
constexpr int kLookBack = 32;
// Emission: depth ranks per block.
constexpr int kEmitThreads = 256;

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

// Exclusive scan of one value per thread over a block of n_warps warps (all
// threads participate); scratch holds n_warps words.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* scratch)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    const uint32_t inc = warp_inclusive_scan(v, lane);
    if (lane == 31) scratch[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const uint32_t t = lane < warps ? scratch[lane] : 0u;
        const uint32_t ti = warp_inclusive_scan(t, lane);
        __syncwarp();
        if (lane < warps) scratch[lane] = ti - t;
    }
    __syncthreads();
    const uint32_t out = scratch[warp] + inc - v;
    __syncthreads();
    return out;
}

// The last depth pass's extra outputs: pair counts in depth order and their
// sums per emission block.
struct DepthTail {
    const int32_t* counts;           // per Gaussian id
    int32_t* sorted_counts;          // per depth rank
    unsigned long long* block_sums;  // per kEmitThreads ranks
};

// Sum of the published counts of partitions part-1, part-2, ... down to the
// first one that carries an inclusive prefix (that prefix included).  Words
// are read 32 predecessors at a time; at a predecessor that has not
// published yet, only that one word is polled (with a growing sleep).
__device__ __forceinline__ uint32_t look_back(const uint32_t* status, int part, int radix, int d,
                                              int32_t* error)
{
    volatile const uint32_t* st = status;
    uint32_t excl = 0;
    int j = part - 1;
    int spins = 0;
    while (true) {
        uint32_t v[kLookBack];
#pragma unroll
        for (int k = 0; k < kLookBack; k++)
            v[k] = (j - k >= 0) ? st[(int64_t)(j - k) * radix + d] : kFlagPrefix;
        int k = 0;
#pragma unroll
        for (; k < kLookBack; k++) {
            const uint32_t flag = v[k] & ~kValueMask;
            if (flag == 0) break;  // not published yet
            excl += v[k] & kValueMask;
            if (flag == kFlagPrefix) return excl;
        }
        j -= k;
        if (k == kLookBack) continue;
        unsigned sleep_ns = 32;
        while ((st[(int64_t)j * radix + d] & ~kValueMask) == 0) {
            if (++spins > kSpinLimit) {
                atomicExch(error, 1);
                return excl;
            }
            __nanosleep(sleep_ns);
            sleep_ns = sleep_ns < 256 ? sleep_ns * 2 : 256;
        }
    }
}

// Shared memory of one pass block (dynamic: above the 48 KB static limit).
template <typename K>
struct SortSmem {
    uint16_t warp_hist[kSortWarps][kMaxRadix + 2];  // per-warp counts, then offsets
    uint32_t global_off[kMaxRadix];
    uint32_t block_start[kMaxRadix];
    uint32_t scratch[kSortWarps];
    K keys[kSortTile];
    int32_t vals[kSortTile];
    int part;
    uint32_t valid;
};

template <typename K, bool TAIL>
__global__ void __launch_bounds__(kSortThreads) onesweep_pass_kernel(
    const K* __restrict__ keys_in, const int32_t* __restrict__ vals_in, K* __restrict__ keys_out,
    int32_t* __restrict__ vals_out, const int32_t* n_ptr, int64_t n_cap, int shift, int bits,
    bool drop_sentinel, const uint32_t* __restrict__ pass_hist, uint32_t* status,
    int32_t* part_counter, int32_t* n_out, int32_t* error, DepthTail tail)
{
    pdl_begin();
    extern __shared__ __align__(16) unsigned char sort_smem_raw[];
    SortSmem<K>& sm = *reinterpret_cast<SortSmem<K>*>(sort_smem_raw);
    const int radix = 1 << bits;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t n = read_count(n_ptr, n_cap);
    if (blockIdx.x == 0 && threadIdx.x == 0 && n_out) {
        uint32_t total = 0;
        for (int d = 0; d < radix; d++) total += pass_hist[d];
        *n_out = (int32_t)total;
    }
    // Exactly ceil(n / kSortTile) blocks take a partition index.
    if ((int64_t)blockIdx.x * kSortTile >= n) return;
    if (threadIdx.x == 0) sm.part = atomicAdd(part_counter, 1);
    for (int d = lane; d <= radix; d += 32) sm.warp_hist[warp][d] = 0;
    __syncthreads();
    const int part = sm.part;
    const int64_t base = (int64_t)part * kSortTile;
    uint32_t* my_status = status + (int64_t)part * radix;
    const int d = threadIdx.x;
    const unsigned lt = lanemask_lt();
    {
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
#pragma unroll
        for (int r = 0; r < kSortItems; r++) {
            const int dr = digit[r];
            const unsigned peers = same_digit_mask(dr, bits);
            const uint32_t before = sm.warp_hist[warp][dr];
            __syncwarp();
            rank[r] = before + __popc(peers & lt);
            if ((peers & lt) == 0) sm.warp_hist[warp][dr] = (uint16_t)(before + __popc(peers));
            __syncwarp();
        }
        __syncthreads();
        uint32_t count = 0;
        if (d < radix) {
            for (int w = 0; w < kSortWarps; w++) {
                const uint32_t c = sm.warp_hist[w][d];
                sm.warp_hist[w][d] = (uint16_t)count;
                count += c;
            }
            // Publish this partition's count before anything else, so that
            // successors looking back find it early.
            volatile uint32_t* st = my_status;
            st[d] = (part == 0 ? kFlagPrefix : kFlagAggregate) | count;
        }
        const uint32_t start = block_exclusive_scan(d < radix ? count : 0u, sm.scratch);
        if (d < radix) sm.block_start[d] = start;
        if (d == radix - 1) sm.valid = start + count;
        __syncthreads();
        // Stage the items in digit order (registers are free afterwards).
#pragma unroll
        for (int r = 0; r < kSortItems; r++) {
            const int dd = digit[r];
            if (dd < radix) {
                const uint32_t pos = sm.block_start[dd] + sm.warp_hist[warp][dd] + rank[r];
                sm.keys[pos] = key[r];
                sm.vals[pos] = val[r];
            }
        }
    }
    const uint32_t digit_base = block_exclusive_scan(d < radix ? pass_hist[d] : 0u, sm.scratch);
    if (d < radix) {
        uint32_t excl = 0;
        if (part > 0) {
            const uint32_t count =
                (d == radix - 1 ? sm.valid : sm.block_start[d + 1]) - sm.block_start[d];
            excl = look_back(status, part, radix, d, error);
            volatile uint32_t* st = my_status;
            st[d] = kFlagPrefix | ((excl + count) & kValueMask);
        }
        sm.global_off[d] = digit_base + excl;
    }
    __syncthreads();
    const uint32_t valid_count = sm.valid;
    if constexpr (!TAIL) {
        for (uint32_t j = threadIdx.x; j < valid_count; j += kSortThreads) {
            const K k = sm.keys[j];
            const int dd = (int)(((uint32_t)k >> shift) & (radix - 1));
            const uint32_t dst = sm.global_off[dd] + (j - sm.block_start[dd]);
            keys_out[dst] = k;
            vals_out[dst] = sm.vals[j];
        }
    } else {
        // Whole warps iterate so that each warp can add up the counts of the
        // ranks it wrote per emission block before one atomic per block.
        for (uint32_t j0 = (uint32_t)warp * 32; j0 < valid_count; j0 += kSortThreads) {
            const uint32_t j = j0 + lane;
            uint32_t blk = 0xFFFFFFFFu, cnt = 0;
            if (j < valid_count) {
                const K k = sm.keys[j];
                const int dd = (int)(((uint32_t)k >> shift) & (radix - 1));
                const uint32_t dst = sm.global_off[dd] + (j - sm.block_start[dd]);
                const int32_t v = sm.vals[j];
                keys_out[dst] = k;
                vals_out[dst] = v;
                cnt = (uint32_t)tail.counts[v];
                tail.sorted_counts[dst] = (int32_t)cnt;
                blk = dst / kEmitThreads;
            }
            const unsigned peers = __match_any_sync(GSB_FULL_MASK, blk);
            const uint32_t lo = __reduce_add_sync(peers, cnt & 0xFFFFu);
            const uint32_t hi = __reduce_add_sync(peers, cnt >> 16);
            if (blk != 0xFFFFFFFFu && (peers & lt) == 0)
                atomicAdd(tail.block_sums + blk, ((unsigned long long)hi << 16) + lo);
        }
    }
}

__global__ void zero_u32_kernel(uint32_t* p, int64_t n)
{
    pdl_begin();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        p[i] = 0;
}

// The pass kernels' shared memory is above the static limit: raise each
// instance's dynamic limit once per device.
std::atomic<uint64_t> g_sort_configured{0};

int configure_sort_kernels()
{
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) {
        set_error(err);
        return GSB_ERR_LAUNCH;
    }
    const uint64_t bit = dev >= 0 && dev < 64 ? (uint64_t)1 << dev : 0;
    if (bit && (g_sort_configured.load(std::memory_order_acquire) & bit)) return GSB_OK;
    const struct {
        const void* fn;
        int smem;
    } kernels[] = {
        {(const void*)onesweep_pass_kernel<uint32_t, false>, (int)sizeof(SortSmem<uint32_t>)},
        {(const void*)onesweep_pass_kernel<uint32_t, true>, (int)sizeof(SortSmem<uint32_t>)},
        {(const void*)onesweep_pass_kernel<uint16_t, false>, (int)sizeof(SortSmem<uint16_t>)},
    };
    for (const auto& k : kernels) {
        err = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
        if (err != cudaSuccess) {
            set_error(err);
            return GSB_ERR_LAUNCH;
        }
    }
    g_sort_configured.fetch_or(bit, std::memory_order_acq_rel);
    return GSB_OK;
}

// Sort scratch.  hist ([4][256] digit totals per pass) and counters (one
// partition counter per pass) sit in the call's head region, zeroed first;
// status ([passes][partitions][radix] look-back words) in the bulk region,
// zeroed by count_kernel.
struct SortScratch {
    uint32_t* hist;
    uint32_t* status;
    int32_t* counters;
    int partitions;
    int radix;
};

template <typename K>
int onesweep_sort(cudaStream_t s, const K* keys_in, const int32_t* vals_in, K* key_a, K* key_b,
                  int32_t* val_a, int32_t* val_b, int32_t* val_out, const K** sorted_keys,
                  const int32_t** sorted_vals, const int32_t* n_ptr, int64_t n_cap, int passes,
                  int bits, bool drop_sentinel, const SortScratch& w, int32_t* n_out,
                  int32_t* error, const DepthTail* tail)
{
    const K* src_k = keys_in;
    const int32_t* src_v = vals_in;
    const int32_t* pass_n = n_ptr;
    const int radix = 1 << bits;
    const size_t smem = sizeof(SortSmem<K>);
    for (int pass = 0; pass < passes; pass++) {
        const bool last = pass == passes - 1;
        K* dst_k = (src_k == key_a) ? key_b : key_a;
        int32_t* dst_v = (last && val_out) ? val_out : ((src_v == val_a) ? val_b : val_a);
        uint32_t* status = w.status + (int64_t)pass * w.partitions * radix;
        const bool drop = drop_sentinel && pass == 0;
        int32_t* count_out = drop ? n_out : nullptr;
        if (last && tail) {
            gsb::launch(onesweep_pass_kernel<K, true>, w.partitions, kSortThreads, smem, s, src_k,
                        src_v, dst_k, dst_v, pass_n, n_cap, pass * bits, bits, drop,
                        w.hist + pass * kMaxRadix, status, w.counters + pass, count_out, error,
                        *tail);
        } else {
            gsb::launch(onesweep_pass_kernel<K, false>, w.partitions, kSortThreads, smem, s,
                        src_k, src_v, dst_k, dst_v, pass_n, n_cap, pass * bits, bits, drop,
                        w.hist + pass * kMaxRadix, status, w.counters + pass, count_out, error,
                        DepthTail{});
        }
        if (int e = check_launch()) return e;
        if (drop) pass_n = n_out;
        src_k = dst_k;
        src_v = dst_v;
    }
    *sorted_keys = src_k;
    *sorted_vals = src_v;
    return GSB_OK;
}

// ---------------------------------------------------------------------------
// Emission (sorted_visibility.py:373-484), with the last step of the
// depth-ordered scan (sorted_visibility.py:511-603): a block's first pair
// offset is the sum of the pair counts of the earlier blocks (the block's
// threads add the block sums written by the last depth pass; they are
// L2-resident), and its threads' offsets follow from a block scan.
// A Gaussian with at most kLanePairs pairs is walked by its own thread;
// larger ones are queued for a warp each (emit_large_kernel).  32 measured
// fastest on config 2 (8: +10 %, 16: +2.7 %, 64: +3 % of the binning).
// ---------------------------------------------------------------------------
constexpr int kLanePairs = 32;

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

struct EmitScan {
    const int32_t* sorted_counts;
    const unsigned long long* block_sums;
    int32_t* pair_count;
    int32_t* overflow;
    int32_t* n_pairs_clamped;
};

template <typename K>
__global__ void __launch_bounds__(kEmitThreads) emit_kernel(
    const int32_t* __restrict__ order, EmitScan scan, const int32_t* n_ptr, int64_t n_cap,
    const float* __restrict__ mean, const float* __restrict__ conic,
    const float* __restrict__ alpha, gsb_bin_params p, int tiles_x, int tiles_y,
    K* __restrict__ keys, int32_t* __restrict__ values, int32_t* __restrict__ queue_gid,
    int32_t* __restrict__ queue_off, int32_t* __restrict__ queue_count, int passes, int bits,
    uint32_t* __restrict__ key_hist)
{
    pdl_begin();
    __shared__ uint32_t local[4 * 256];
    __shared__ long long warp_total[kEmitThreads / 32];
    __shared__ unsigned long long prefix_part[kEmitThreads / 32];
    const int64_t n = read_count(n_ptr, n_cap);
    const int b = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (n == 0) {
        if (b == 0 && threadIdx.x == 0) {
            *scan.pair_count = 0;
            *scan.overflow = 0;
            *scan.n_pairs_clamped = 0;
        }
        return;
    }
    if ((int64_t)b * kEmitThreads >= n) return;  // uniform per block
    for (int i = threadIdx.x; i < passes * 256; i += blockDim.x) local[i] = 0;
    {
        // Every thread adds a strided share of the earlier blocks' sums, so
        // the loads are in flight together instead of one warp's chain.
        unsigned long long acc = 0;
#pragma unroll 4
        for (int i = threadIdx.x; i < b; i += kEmitThreads) acc += scan.block_sums[i];
        acc = warp_sum(acc);
        if (lane == 0) prefix_part[warp] = acc;
    }
    const int64_t r = (int64_t)b * kEmitThreads + threadIdx.x;
    int32_t count = 0, gid = 0;
    if (r < n) {
        gid = order[r];
        count = scan.sorted_counts[r];
    }
    const long long inc = warp_inclusive_scan((long long)count, lane);
    if (lane == 31) warp_total[warp] = inc;
    __syncthreads();
    long long before = 0;
#pragma unroll
    for (int w = 0; w < kEmitThreads / 32; w++) before += (long long)prefix_part[w];
    for (int w = 0; w < warp; w++) before += warp_total[w];
    const int64_t offset = before + inc - count;
    if (r == n - 1) {
        const int64_t end = offset + count;
        *scan.pair_count = (int32_t)(end < 0x7fffffff ? end : 0x7fffffff);
        *scan.overflow = end > p.max_pairs ? 1 : 0;
        *scan.n_pairs_clamped = (int32_t)(end < p.max_pairs ? end : p.max_pairs);
    }
    const KeyHist hist{local, passes, bits};
    if (count > 0 && count <= kLanePairs && offset < p.max_pairs) {
        Splat s = load_splat(mean, conic, alpha, gid);
        process_tiles<true, K>(s, p.tile_w, p.tile_h, tiles_x, tiles_y, gid, offset, p.max_pairs,
                               keys, values, hist);
    }
    const bool large = count > kLanePairs && offset < p.max_pairs;
    const unsigned queued = __ballot_sync(GSB_FULL_MASK, large);
    if (queued) {
        const int leader = __ffs(queued) - 1;
        int first = 0;
        if (lane == leader) first = atomicAdd(queue_count, __popc(queued));
        first = __shfl_sync(GSB_FULL_MASK, first, leader);
        if (large) {
            const int slot = first + __popc(queued & lanemask_lt());
            queue_gid[slot] = gid;
            queue_off[slot] = (int32_t)offset;
        }
    }
    flush_key_hist(local, passes, key_hist);
}

// One warp per queued Gaussian: lanes take 32 rows at a time, then write the
// pairs of those rows as consecutive 32-pair chunks (each lane finds its row
// by binary search over the rows' exclusive offsets).
template <typename K>
__global__ void __launch_bounds__(256) emit_large_kernel(
    const int32_t* __restrict__ queue_gid, const int32_t* __restrict__ queue_off,
    const int32_t* __restrict__ queue_count, const float* __restrict__ mean,
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
        const int32_t gid = queue_gid[item];
        int64_t offset = queue_off[item];
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

// Workspace of one gsb_bin call.
//  head (zeroed by the call's first kernel): scalars[8] ([0] binned
//    Gaussians, [1] large-emission queue length, [2] pairs kept, [3] sort
//    time-out), the depth and tile sorts' digit totals [4][256] each and
//    their partition counters [4] each.
//  bulk (zeroed by count_kernel): the per-block pair sums of the emission,
//    then the two sorts' look-back words.
struct BinLayout {
    uint32_t *depth_keys, *keys_a, *keys_b;
    int32_t *order_a, *order_b, *sorted_counts;
    int32_t *queue_gid, *queue_off;
    uint32_t* head;
    int64_t head_words;
    uint32_t* bulk;
    int64_t bulk_words;
    int32_t* scalars;
    unsigned long long* block_sums;
    void *emit_keys, *pair_keys_a, *pair_keys_b;
    int32_t *emit_ids, *pair_ids_a, *pair_ids_b;
    SortScratch depth_sort, pair_sort;
    int tile_passes, tile_bits;
};

constexpr int64_t kHeadWords = 8 + 2 * 4 * kMaxRadix + 2 * 4;

BinLayout carve_bin(char* base, const gsb_bin_params& p, size_t& used)
{
    Carver c{base, 0, 0};
    BinLayout L;
    int64_t C = p.capacity > 0 ? p.capacity : 1;
    int64_t P = p.max_pairs > 0 ? p.max_pairs : 1;
    int64_t tiles = (int64_t)ceil_div(p.width, p.tile_w) * ceil_div(p.height, p.tile_h);
    digit_plan(tiles > 0 ? tiles : 1, L.tile_passes, L.tile_bits);
    size_t key_bytes = tiles <= 65535 ? 2 : 4;
    L.depth_keys = c.take<uint32_t>(C);
    L.keys_a = c.take<uint32_t>(C);
    L.keys_b = c.take<uint32_t>(C);
    L.order_a = c.take<int32_t>(C);
    L.order_b = c.take<int32_t>(C);
    L.sorted_counts = c.take<int32_t>(C);
    L.queue_gid = c.take<int32_t>(C);
    L.queue_off = c.take<int32_t>(C);
    L.emit_keys = c.take<char>(P * key_bytes);
    L.pair_keys_a = c.take<char>(P * key_bytes);
    L.pair_keys_b = c.take<char>(P * key_bytes);
    L.emit_ids = c.take<int32_t>(P);
    L.pair_ids_a = c.take<int32_t>(P);
    L.pair_ids_b = c.take<int32_t>(P);
    L.head_words = kHeadWords;
    L.head = c.take<uint32_t>(kHeadWords);
    L.scalars = reinterpret_cast<int32_t*>(L.head);
    L.depth_sort.partitions = ceil_div(C, kSortTile);
    L.depth_sort.radix = 256;
    L.pair_sort.partitions = ceil_div(P, kSortTile);
    L.pair_sort.radix = 1 << L.tile_bits;
    const int64_t blocks = ceil_div(C, kEmitThreads);
    const int64_t depth_status = 4 * (int64_t)L.depth_sort.partitions * L.depth_sort.radix;
    const int64_t pair_status =
        (int64_t)L.tile_passes * L.pair_sort.partitions * L.pair_sort.radix;
    L.bulk_words = ((2 * blocks + depth_status + pair_status) + 3) & ~int64_t(3);
    L.bulk = c.take<uint32_t>(L.bulk_words);
    if (base) {
        L.depth_sort.hist = L.head + 8;
        L.pair_sort.hist = L.head + 8 + 4 * kMaxRadix;
        L.depth_sort.counters = reinterpret_cast<int32_t*>(L.head + 8 + 8 * kMaxRadix);
        L.pair_sort.counters = L.depth_sort.counters + 4;
        L.block_sums = reinterpret_cast<unsigned long long*>(L.bulk);
        L.depth_sort.status = L.bulk + 2 * blocks;
        L.pair_sort.status = L.depth_sort.status + depth_status;
    }
    used = c.used;
    return L;
}

template <typename K>
int tile_stage(cudaStream_t s, const gsb_bin_params& p, const BinLayout& L, int tiles_x,
               int tiles_y, int64_t num_tiles, const float* mean, const float* conic,
               const float* alpha, const int32_t* order, int32_t* gaussian_ids,
               int32_t* tile_offsets, int32_t* pair_count, int32_t* overflow)
{
    K* emit_keys = static_cast<K*>(L.emit_keys);
    const int32_t* n_binned = L.scalars + 0;
    int64_t C = p.capacity;
    const int passes = L.tile_passes, bits = L.tile_bits;
    // The emission kernels also accumulate the tile sort's digit histograms.
    EmitScan scan{L.sorted_counts, L.block_sums, pair_count, overflow, L.scalars + 2};
    gsb::launch(emit_kernel<K>, ceil_div(C > 0 ? C : 1, kEmitThreads), kEmitThreads, 0, s, order,
                scan, n_binned, C, mean, conic, alpha, p, tiles_x, tiles_y, emit_keys, L.emit_ids,
                L.queue_gid, L.queue_off, L.scalars + 1, passes, bits, L.pair_sort.hist);
    if (int e = check_launch()) return e;
    gsb::launch(emit_large_kernel<K>, 148 * 8, 256, 0, s, L.queue_gid, L.queue_off, L.scalars + 1,
                mean, conic, alpha, p, tiles_x, tiles_y, emit_keys, L.emit_ids, passes, bits,
                L.pair_sort.hist);
    if (int e = check_launch()) return e;
    const K* sorted_keys = nullptr;
    const int32_t* sorted_ids = nullptr;
    if (int e = onesweep_sort<K>(s, emit_keys, L.emit_ids, static_cast<K*>(L.pair_keys_a),
                                 static_cast<K*>(L.pair_keys_b), L.pair_ids_a, L.pair_ids_b,
                                 gaussian_ids, &sorted_keys, &sorted_ids, L.scalars + 2,
                                 p.max_pairs, passes, bits, false, L.pair_sort, nullptr,
                                 L.scalars + 3, nullptr))
        return e;
    gsb::launch(ranges_kernel<K>, 1024, 256, 0, s, sorted_keys, L.scalars + 2, p.max_pairs,
                (int)num_tiles, tile_offsets, L.scalars + 3, overflow);
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
    if (int e = configure_sort_kernels()) return e;
    cudaStream_t s = as_stream(stream);
    size_t used = 0;
    BinLayout L = carve_bin(static_cast<char*>(workspace), *p, used);
    gsb::launch(zero_u32_kernel, 8, 256, 0, s, L.head, L.head_words);
    if (int e = check_launch()) return e;
    int64_t C = p->capacity;
    const uint32_t* sorted_depth_keys = nullptr;
    const int32_t* depth_order = L.order_a;
    // count_kernel always runs: it also zeroes the bulk region.
    const int count_blocks =
        ceil_div(C > 0 ? C : 1, kCountSlots) > 296 ? ceil_div(C, kCountSlots) : 296;
    gsb::launch(count_kernel, count_blocks, kCountThreads, 0, s, (int)C, mean, conic, alpha, depth,
                visible, *p, tiles_x, tiles_y, point_counts, L.depth_keys, L.depth_sort.hist,
                reinterpret_cast<uint4*>(L.bulk), L.bulk_words / 4);
    if (int e = check_launch()) return e;
    if (C > 0) {
        // Depth sort: pass 0 drops the Gaussians without pairs; the last pass
        // writes the counts in depth order and their per-block sums.
        const DepthTail tail{point_counts, L.sorted_counts, L.block_sums};
        if (int e = onesweep_sort<uint32_t>(s, L.depth_keys, nullptr, L.keys_a, L.keys_b,
                                            L.order_a, L.order_b, nullptr, &sorted_depth_keys,
                                            &depth_order, nullptr, C, 4, 8, true, L.depth_sort,
                                            L.scalars + 0, L.scalars + 3, &tail))
            return e;
    }
    if (num_tiles <= 65535)
        return tile_stage<uint16_t>(s, *p, L, tiles_x, tiles_y, num_tiles, mean, conic, alpha,
                                    depth_order, gaussian_ids, tile_offsets, pair_count, overflow);
    return tile_stage<uint32_t>(s, *p, L, tiles_x, tiles_y, num_tiles, mean, conic, alpha,
                                depth_order, gaussian_ids, tile_offsets, pair_count, overflow);
}
