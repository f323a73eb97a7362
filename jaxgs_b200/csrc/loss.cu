// Fused L1(0.8) + SSIM(0.2) loss, image gradient and gradient scale (sm_100a).
//
// Semantics: reference/loss.py:6-43 (11x11 Gaussian window, sigma 1.5, SAME
// zero padding, C1 = 0.01^2, C2 = 0.03^2) with the per-pixel gradient of
// kernels/fused_loss.py:229-288: for every pixel the SSIM partials
// dS/dmu_x, dS/dE[x^2], dS/dE[xy] are formed from the window statistics and
// blurred once more, grad = blur(p0) + 2x blur(p1) + y blur(p2)
// + 0.8 sign(x - y) / (3HW).
//
// The SSIM map needs only four blurred statistics per channel: mu_x, mu_y,
// E[x^2 + y^2] (sigma_x^2 and sigma_y^2 enter only as their sum) and E[xy].
// They are carried as two float2 pairs, (mu_x, mu_y) and (E[x^2+y^2], E[xy]),
// so every tap of every separable pass is two packed f32x2 FMAs (sm_100).
//
// Row streaming.  One CTA per (32-column strip, segment of rows, channel)
// walks down its segment 16 rows at a time.  The two vertical windows (the
// statistics' and the partials') live in 32-row ring buffers in shared
// memory, so a row is staged and its partials are formed once per strip
// rather than once per tile: only the 10-column (statistics) and 5-column
// (partials) horizontal halos are computed twice.  Per 16-row chunk k, with
// statistics rows S_k = ys - 11 + 16k .. +15 and output rows S_k - 5 .. +10:
//   stage   16 new (x, y) rows (52 columns) into the patch ring
//   pass 1  vertical window sums of the statistics      (16 x 52)
//   pass 2  horizontal sums -> SSIM partials, SSIM loss (16 x 42) -> ring
//   pass 3  vertical blur of the partials               (16 x 42)
//   pass 4  horizontal blur -> image gradient, L1 loss  (16 x 32)
// Chunk 0 only fills the rings (its outputs precede the segment).  Each
// thread of a pass owns a run of consecutive outputs and accumulates them in
// registers while it streams the inputs once (scatter form).  Row strides
// are padded to odd multiples so that lanes walking down a column hit
// distinct banks.  About 43 KB of shared memory per CTA, four CTAs (32
// warps) per SM.  Per-CTA loss sums and |grad| maxima are reduced by a
// single-block kernel in a fixed order, so the scalar results are
// deterministic.
//
// The stage and pass bodies are __host__ __device__ functions of (thread
// index, shared state): the kernel runs them between barriers, and a host
// build can run the same bodies thread by thread with checked indexing.
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr int kTW = 32, kR = 5, kTaps = 2 * kR + 1;
constexpr int kCH = 16;    // rows per chunk
constexpr int kRing = 32;  // rows held by each ring buffer (a power of two)
constexpr int kThreads = 256;
constexpr int kSW = kTW + 2 * kR;  // 42 statistics / partials columns
constexpr int kPW = kTW + 4 * kR;  // 52 staged columns
constexpr int kPStride = kPW + 1, kQStride = kSW + 1;
constexpr int kRun1 = 4, kRuns1 = kCH / kRun1;  // pass 1: 16 rows as 4 runs of 4, x 52 columns
constexpr int kRun2 = 3, kRuns2 = kSW / kRun2;  // pass 2: 42 columns as 14 runs of 3, x 16 rows
constexpr int kRun3 = 4, kRuns3 = kCH / kRun3;  // pass 3: 16 rows as 4 runs of 4, x 42 columns
constexpr int kRun4 = 4, kRuns4 = kTW / kRun4;  // pass 4: 32 columns as 8 runs of 4, x 16 rows
static_assert(kRuns1 * kRun1 == kCH && kRuns2 * kRun2 == kSW, "run cover");
static_assert(kRuns3 * kRun3 == kCH && kRuns4 * kRun4 == kTW, "run cover");
static_assert(kRuns1 * kPW <= kThreads && kRuns2 * kCH <= kThreads, "pass items");
static_assert(kRuns3 * kSW <= kThreads && kRuns4 * kCH <= kThreads, "pass items");
static_assert(kPW <= 64 && kThreads % 64 == 0 && kCH % (kThreads / 64) == 0, "staging lanes");
// Each ring holds two chunks of rows: the 26-row windows a chunk reads
// (5 rows above its first row to 5 below its last, twice over for the
// patch) stay inside the chunk and its neighbour when 2 kR <= kCH.
static_assert(2 * kR <= kCH && kRing == 2 * kCH, "ring rows");
// Statistics rows run kCH - kR rows ahead of the output rows, and the patch
// rows another kCH - kR ahead of those (so chunk 1's outputs start at ys).
constexpr int kPartLead = kCH - kR, kPatchLead = 2 * (kCH - kR);

// exp(-(d/1.5)^2 / 2) normalised, correctly rounded to float32; d = t - 5.
__host__ __device__ constexpr float tap(int t)
{
    return t == 0 || t == 10 ? 0.001028380123898387f
         : t == 1 || t == 9  ? 0.0075987582094967365f
         : t == 2 || t == 8  ? 0.036000773310661316f
         : t == 3 || t == 7  ? 0.10936068743467331f
         : t == 4 || t == 6  ? 0.21300554275512695f
                             : 0.26601171493530273f;
}

// Packed f32x2 arithmetic on the device (each lane rounded like its scalar
// form), the same lane by lane on the host.
__host__ __device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c)
{
#ifdef __CUDA_ARCH__
    return __ffma2_rn(a, b, c);
#else
    return make_float2(std::fmaf(a.x, b.x, c.x), std::fmaf(a.y, b.y, c.y));
#endif
}

__host__ __device__ __forceinline__ float2 mul2(float2 a, float2 b)
{
#ifdef __CUDA_ARCH__
    return __fmul2_rn(a, b);
#else
    return make_float2(a.x * b.x, a.y * b.y);
#endif
}

__host__ __device__ __forceinline__ float2 tap2(int t) { return make_float2(tap(t), tap(t)); }

// 1/x for the SSIM denominators (both >= 1e-4): the fast reciprocal on the
// device, an IEEE divide on the host.
__host__ __device__ __forceinline__ float recip(float x)
{
#ifdef __CUDA_ARCH__
    return __fdividef(1.0f, x);
#else
    return 1.0f / x;
#endif
}

template <typename T>
__host__ __device__ __forceinline__ T load_ro(const T* p)
{
#ifdef __CUDA_ARCH__
    return __ldg(p);
#else
    return *p;
#endif
}

__host__ __device__ __forceinline__ float clip01(float v) { return fminf(fmaxf(v, 0.0f), 1.0f); }

// d clip(v, 0, 1) / dv with jnp.maximum/minimum tie semantics (1/2 at a bound).
__host__ __device__ __forceinline__ float clip_grad(float v)
{
    if (v > 0.0f && v < 1.0f) return 1.0f;
    if (v == 0.0f || v == 1.0f) return 0.5f;
    return 0.0f;
}

struct LossSmem {
    float2 patch[kRing][kPStride];  // (x, y) rows of the channel, ring; x clipped when requested
    union {
        float4 v[kCH][kPStride];  // pass 1 -> 2: (mu_x, mu_y, E[x^2+y^2], E[xy]) column sums
        struct {
            float2 q01[kCH][kQStride];  // pass 3 -> 4: vertically blurred partials (p0, p1)
            float q2[kCH][kQStride];    //              and p2
        } r;
    } u;
    float2 p01[kRing][kQStride];  // SSIM partials (p0, p1), ring
    float p2[kRing][kQStride];    //               and p2
};

// One CTA's strip: output columns [x0, x0 + 32), output rows [ys, ye) of
// channel c.  Patch row y sits in ring row (y - ys + 22) & 31, partials row
// y in (y - ys + 11) & 31 (both offsets are >= 0 for every row touched).
struct Strip {
    int width, height, x0, ys, ye, c;
    float inv_n;
};

__host__ __device__ __forceinline__ int patch_ring(const Strip& g, int y) { return (y - g.ys + kPatchLead) & (kRing - 1); }
__host__ __device__ __forceinline__ int part_ring(const Strip& g, int y) { return (y - g.ys + kPartLead) & (kRing - 1); }
__host__ __device__ __forceinline__ int stats_row0(const Strip& g, int k) { return g.ys - kPartLead + kCH * k; }

// Stage block j: image rows [ys - 22 + 16 j, +16) of the 52 columns from
// x0 - 10, zero outside the image.  Every load of the thread is issued
// before the first store so their latencies overlap.
template <bool U8, bool CLIP>
__host__ __device__ __forceinline__ void stage_rows(int tid, LossSmem& S, const Strip& g, int j,
                                                    const float* image, const void* target_raw)
{
    constexpr int kSweeps = kCH / (kThreads / 64);
    const int col = tid & 63, row0 = tid >> 6;
    const int gx = g.x0 - 2 * kR + col;
    const bool col_in = col < kPW && gx >= 0 && gx < g.width;
    const uint8_t* t8 = static_cast<const uint8_t*>(target_raw);
    const float* tf = static_cast<const float*>(target_raw);
    float xv[kSweeps], yv[kSweeps];
#pragma unroll
    for (int k = 0; k < kSweeps; k++) {
        const int gy = g.ys - kPatchLead + kCH * j + row0 + k * (kThreads / 64);
        xv[k] = 0.0f;
        yv[k] = 0.0f;
        if (col_in && gy >= 0 && gy < g.height) {
            const int64_t idx = ((int64_t)gy * g.width + gx) * 3 + g.c;
            xv[k] = load_ro(image + idx);
            yv[k] = U8 ? (float)load_ro(t8 + idx) : load_ro(tf + idx);
        }
    }
    if (col < kPW) {
#pragma unroll
        for (int k = 0; k < kSweeps; k++) {
            const int gy = g.ys - kPatchLead + kCH * j + row0 + k * (kThreads / 64);
            const float x = CLIP ? clip01(xv[k]) : xv[k];
            const float y = U8 ? yv[k] * (float)(1.0 / 255.0) : yv[k];
            S.patch[patch_ring(g, gy)][col] = make_float2(x, y);
        }
    }
}

// Pass 1: vertical window sums of (x, y) and (x^2 + y^2, xy) for the
// chunk's 16 statistics rows, all 52 staged columns.
__host__ __device__ __forceinline__ void pass1(int tid, LossSmem& S, const Strip& g, int k)
{
    if (tid >= kRuns1 * kPW) return;
    const int q = tid % kPW, r0 = (tid / kPW) * kRun1;
    const int y0 = stats_row0(g, k) + r0 - kR;  // first patch row of the run's windows
    float2 m[kRun1], s[kRun1];
#pragma unroll
    for (int o = 0; o < kRun1; o++) m[o] = s[o] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < kRun1 + 2 * kR; j++) {
        const float2 v = S.patch[patch_ring(g, y0 + j)][q];
        const float2 sq = mul2(v, v);
        const float2 u = make_float2(sq.x + sq.y, v.x * v.y);
#pragma unroll
        for (int o = 0; o < kRun1; o++) {
            const int t = j - o;
            if (t >= 0 && t < kTaps) {
                m[o] = fma2(tap2(t), v, m[o]);
                s[o] = fma2(tap2(t), u, s[o]);
            }
        }
    }
#pragma unroll
    for (int o = 0; o < kRun1; o++) S.u.v[r0 + o][q] = make_float4(m[o].x, m[o].y, s[o].x, s[o].y);
}

// Pass 2: horizontal sums -> statistics -> SSIM partials (zero outside the
// image) into the partials ring, and the SSIM part of the loss on the
// strip's own pixels.
__host__ __device__ __forceinline__ void pass2(int tid, LossSmem& S, const Strip& g, int k, float& loss)
{
    if (tid >= kRuns2 * kCH) return;
    const int r = tid % kCH, c0 = (tid / kCH) * kRun2;
    const float weight = -0.2f * g.inv_n;
    float2 m[kRun2], s[kRun2];
#pragma unroll
    for (int o = 0; o < kRun2; o++) m[o] = s[o] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < kRun2 + 2 * kR; j++) {
        const float4 v = S.u.v[r][c0 + j];
        const float2 a = make_float2(v.x, v.y), b = make_float2(v.z, v.w);
#pragma unroll
        for (int o = 0; o < kRun2; o++) {
            const int t = j - o;
            if (t >= 0 && t < kTaps) {
                m[o] = fma2(tap2(t), a, m[o]);
                s[o] = fma2(tap2(t), b, s[o]);
            }
        }
    }
    const int gy = stats_row0(g, k) + r;
    const bool row_in = gy >= 0 && gy < g.height;
    const bool row_own = gy >= g.ys && gy < g.ye;
    const int ring = part_ring(g, gy);
#pragma unroll
    for (int o = 0; o < kRun2; o++) {
        const int cc = c0 + o;
        const int gx = g.x0 - kR + cc;
        float p0 = 0.0f, p1 = 0.0f, p2 = 0.0f;
        if (row_in && gx >= 0 && gx < g.width) {
            const float mx = m[o].x, my = m[o].y;
            const float mxy = mx * my;
            const float mm = fmaf(mx, mx, my * my);
            const float A = mm + 1e-4f;
            const float B = (s[o].x - mm) + 9e-4f;
            const float Cc = fmaf(2.0f, mxy, 1e-4f);
            const float D = fmaf(2.0f, s[o].y - mxy, 9e-4f);
            const float inv_a = recip(A), inv_b = recip(B);
            const float inv_ab = inv_a * inv_b;
            const float ssim = Cc * D * inv_ab;
            p0 = (my * (D - Cc) * inv_ab + mx * ssim * (inv_b - inv_a)) * (2.0f * weight);
            p1 = -ssim * inv_b * weight;
            p2 = 2.0f * Cc * inv_ab * weight;
            if (row_own && cc >= kR && cc < kR + kTW) loss += 0.2f * (1.0f - ssim);
        }
        S.p01[ring][cc] = make_float2(p0, p1);
        S.p2[ring][cc] = p2;
    }
}

// Pass 3: vertical blur of the partials onto the chunk's 16 output rows.
__host__ __device__ __forceinline__ void pass3(int tid, LossSmem& S, const Strip& g, int k)
{
    if (tid >= kRuns3 * kSW) return;
    const int cc = tid % kSW, r0 = (tid / kSW) * kRun3;
    const int y0 = stats_row0(g, k) - 2 * kR + r0;  // first partials row of the run's windows
    float2 a[kRun3];
    float b[kRun3];
#pragma unroll
    for (int o = 0; o < kRun3; o++) {
        a[o] = make_float2(0.0f, 0.0f);
        b[o] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < kRun3 + 2 * kR; j++) {
        const int ring = part_ring(g, y0 + j);
        const float2 u = S.p01[ring][cc];
        const float v = S.p2[ring][cc];
#pragma unroll
        for (int o = 0; o < kRun3; o++) {
            const int t = j - o;
            if (t >= 0 && t < kTaps) {
                a[o] = fma2(tap2(t), u, a[o]);
                b[o] = fmaf(tap(t), v, b[o]);
            }
        }
    }
#pragma unroll
    for (int o = 0; o < kRun3; o++) {
        S.u.r.q01[r0 + o][cc] = a[o];
        S.u.r.q2[r0 + o][cc] = b[o];
    }
}

// Pass 4: horizontal blur -> image gradient of the chunk's output rows
// (written straight to global memory), the L1 part of the loss, |grad| max.
template <bool CLIP>
__host__ __device__ __forceinline__ void pass4(int tid, LossSmem& S, const Strip& g, int k,
                                               const float* image, float* grad, float& loss,
                                               uint32_t& scale_bits)
{
    if (tid >= kRuns4 * kCH) return;
    const int r = tid % kCH, c0 = (tid / kCH) * kRun4;
    float2 a[kRun4];
    float b[kRun4];
#pragma unroll
    for (int o = 0; o < kRun4; o++) {
        a[o] = make_float2(0.0f, 0.0f);
        b[o] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < kRun4 + 2 * kR; j++) {
        const float2 u = S.u.r.q01[r][c0 + j];
        const float v = S.u.r.q2[r][c0 + j];
#pragma unroll
        for (int o = 0; o < kRun4; o++) {
            const int t = j - o;
            if (t >= 0 && t < kTaps) {
                a[o] = fma2(tap2(t), u, a[o]);
                b[o] = fmaf(tap(t), v, b[o]);
            }
        }
    }
    const int gy = stats_row0(g, k) - kR + r;
    if (gy < g.ys || gy >= g.ye) return;
    const int ring = patch_ring(g, gy);
#pragma unroll
    for (int o = 0; o < kRun4; o++) {
        const int col = c0 + o;
        const int gx = g.x0 + col;
        if (gx < g.width) {
            const float2 xy = S.patch[ring][col + 2 * kR];
            const float sign = xy.x > xy.y ? 1.0f : (xy.x < xy.y ? -1.0f : 0.0f);
            float value = a[o].x + 2.0f * xy.x * a[o].y + xy.y * b[o] + 0.8f * sign * g.inv_n;
            const int64_t idx = ((int64_t)gy * g.width + gx) * 3 + g.c;
            if (CLIP) value *= clip_grad(load_ro(image + idx));
            grad[idx] = value;
            uint32_t bits;
            memcpy(&bits, &value, sizeof(bits));
            scale_bits = scale_bits > (bits & 0x7fffffffu) ? scale_bits : (bits & 0x7fffffffu);
            loss += 0.8f * fabsf(xy.x - xy.y);
        }
    }
}

// Rows of the segment a CTA covers and the strip geometry of block (bx, by, c).
__host__ __device__ __forceinline__ Strip strip_of(int width, int height, int seg_rows, int bx, int by,
                                                   int c)
{
    Strip g;
    g.width = width;
    g.height = height;
    g.x0 = bx * kTW;
    g.ys = by * seg_rows;
    g.ye = g.ys + seg_rows < height ? g.ys + seg_rows : height;
    g.c = c;
    g.inv_n = 1.0f / (3.0f * (float)width * (float)height);
    return g;
}

// Chunks a CTA runs: one to fill the rings, then one per 16 output rows.
__host__ __device__ __forceinline__ int strip_chunks(const Strip& g)
{
    return 1 + (g.ye - g.ys + kCH - 1) / kCH;
}

template <bool U8, bool CLIP>
__global__ void __launch_bounds__(kThreads, 4) loss_kernel(int width, int height, int seg_rows,
                                                           const float* __restrict__ image,
                                                           const void* __restrict__ target_raw,
                                                           float* __restrict__ grad,
                                                           float* __restrict__ block_loss,
                                                           uint32_t* __restrict__ block_scale)
{
    pdl_begin();
    extern __shared__ float4 smem_raw[];
    LossSmem& S = *reinterpret_cast<LossSmem*>(smem_raw);
    __shared__ float warp_loss[kThreads / 32];
    __shared__ uint32_t warp_scale[kThreads / 32];
    const int tid = threadIdx.x;
    const Strip g = strip_of(width, height, seg_rows, blockIdx.x, blockIdx.y, blockIdx.z);
    const int chunks = strip_chunks(g);
    float loss = 0.0f;
    uint32_t scale_bits = 0;
    for (int k = 0; k < chunks; k++) {
        if (k == 0) stage_rows<U8, CLIP>(tid, S, g, 0, image, target_raw);
        stage_rows<U8, CLIP>(tid, S, g, k + 1, image, target_raw);
        __syncthreads();
        pass1(tid, S, g, k);
        __syncthreads();
        pass2(tid, S, g, k, loss);
        __syncthreads();
        if (k > 0) {
            pass3(tid, S, g, k);
            __syncthreads();
            pass4<CLIP>(tid, S, g, k, image, grad, loss, scale_bits);
            __syncthreads();
        }
    }
    loss = warp_sum(loss);
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) scale_bits = max(scale_bits, __shfl_xor_sync(GSB_FULL_MASK, scale_bits, d));
    if ((tid & 31) == 0) {
        warp_loss[tid >> 5] = loss;
        warp_scale[tid >> 5] = scale_bits;
    }
    __syncthreads();
    if (tid == 0) {
        float total = 0.0f;
        uint32_t sb = 0;
        for (int w = 0; w < kThreads / 32; w++) {
            total += warp_loss[w];
            sb = max(sb, warp_scale[w]);
        }
        const int b = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        block_loss[b] = total;
        block_scale[b] = sb;
    }
}

// Fixed-order reduction of the per-CTA partials (deterministic).
__global__ void __launch_bounds__(1024) loss_finish_kernel(int blocks, float inv_n,
                                                           const float* __restrict__ block_loss,
                                                           const uint32_t* __restrict__ block_scale,
                                                           float* loss, float* scale)
{
    pdl_begin();
    __shared__ double partial[32];
    __shared__ uint32_t pscale[32];
    double s = 0.0;
    uint32_t m = 0;
    // Eight loads per thread in flight before they are summed (fixed order).
    constexpr int kBatch = 8;
    for (int base = threadIdx.x; base < blocks; base += blockDim.x * kBatch) {
        float lv[kBatch];
        uint32_t sv[kBatch];
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            const int b = base + k * (int)blockDim.x;
            lv[k] = b < blocks ? block_loss[b] : 0.0f;
            sv[k] = b < blocks ? block_scale[b] : 0u;
        }
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            s += (double)lv[k];
            m = max(m, sv[k]);
        }
    }
    s = warp_sum(s);
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) m = max(m, __shfl_xor_sync(GSB_FULL_MASK, m, d));
    if ((threadIdx.x & 31) == 0) {
        partial[threadIdx.x >> 5] = s;
        pscale[threadIdx.x >> 5] = m;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        uint32_t mm = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) {
            t += partial[w];
            mm = max(mm, pscale[w]);
        }
        *loss = (float)(t * (double)inv_n);
        if (scale) {
            float v = __uint_as_float(mm);
            *scale = (v != v) ? v : fmaxf(v, 1e-12f);
        }
    }
}


// Per-CTA slots: at most one per 32x16 block of pixels and channel (the
// strips' segments are whole multiples of 16 rows).
constexpr int kSlotRows = 16;

int64_t loss_tiles(const gsb_loss_params& p)
{
    return (int64_t)ceil_div(p.width, kTW) * ceil_div(p.height, kSlotRows);
}

bool loss_shape_ok(const gsb_loss_params& p)
{
    return p.width > 0 && p.height > 0 && ceil_div(p.height, kSlotRows) <= 65535 &&
           loss_tiles(p) <= (int64_t)1 << 28;
}

// Rows per segment: enough segments that the strips x segments x channels
// CTAs fill about four per SM of a 148-SM B200 in one wave, each a whole
// number of 16-row chunks.
int loss_segment_rows(const gsb_loss_params& p)
{
    constexpr double kTargetCtas = 4.0 * 148.0;
    const int strips = ceil_div(p.width, kTW);
    const int chunks = ceil_div(p.height, kCH);
    int segments = (int)std::lround(kTargetCtas / (3.0 * strips));
    segments = segments < 1 ? 1 : (segments > chunks ? chunks : segments);
    return ceil_div(ceil_div(p.height, segments), kCH) * kCH;
}

// The kernels need more than 48 KB of dynamic shared memory on some builds:
// opt in once per device (a host-side function attribute; it never enters a
// graph capture).
std::atomic<uint64_t> g_loss_configured{0};

int configure_loss_kernels()
{
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) {
        set_error(err);
        return GSB_ERR_LAUNCH;
    }
    const uint64_t bit = dev >= 0 && dev < 64 ? (uint64_t)1 << dev : 0;
    if (bit && (g_loss_configured.load(std::memory_order_acquire) & bit)) return GSB_OK;
    const int smem = (int)sizeof(LossSmem);
    const void* kernels[4] = {(const void*)loss_kernel<true, true>,
                              (const void*)loss_kernel<true, false>,
                              (const void*)loss_kernel<false, true>,
                              (const void*)loss_kernel<false, false>};
    for (const void* k : kernels) {
        err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (err != cudaSuccess) {
            set_error(err);
            return GSB_ERR_LAUNCH;
        }
    }
    g_loss_configured.fetch_or(bit, std::memory_order_acq_rel);
    return GSB_OK;
}

// Loss kernel + fixed-order finish.  block_loss / block_scale hold one slot
// per CTA (strip, segment, channel).
int launch_loss(cudaStream_t s, const gsb_loss_params& p, const float* image, const void* target,
                float* loss, float* grad, float* scale, float* block_loss, uint32_t* block_scale)
{
    const int seg_rows = loss_segment_rows(p);
    dim3 grid(ceil_div(p.width, kTW), ceil_div(p.height, seg_rows), 3);
    const size_t smem = sizeof(LossSmem);
    auto launch = [&](auto kernel) {
        gsb::launch(kernel, grid, kThreads, smem, s, p.width, p.height, seg_rows, image, target, grad,
                    block_loss, block_scale);
    };
    if (p.target_u8) {
        if (p.clip_input) launch(loss_kernel<true, true>);
        else launch(loss_kernel<true, false>);
    } else {
        if (p.clip_input) launch(loss_kernel<false, true>);
        else launch(loss_kernel<false, false>);
    }
    if (int e = check_launch()) return e;
    const float inv_n = 1.0f / (3.0f * (float)p.width * (float)p.height);
    const int blocks = (int)(grid.x * grid.y * grid.z);
    gsb::launch(loss_finish_kernel, 1, 1024, 0, s, blocks, inv_n, block_loss, block_scale, loss, scale);
    return check_launch();
}

size_t slot_bytes(const gsb_loss_params& p) { return ((size_t)(3 * loss_tiles(p)) * 4 + 255) & ~size_t(255); }

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" size_t gsb_loss_workspace_size(const gsb_loss_params* p)
{
    if (!p || !loss_shape_ok(*p)) return 0;
    return 2 * slot_bytes(*p);
}

extern "C" int gsb_loss(gsb_stream_t stream, const gsb_loss_params* p, void* workspace,
                        size_t workspace_bytes, const float* image, const void* target, float* loss,
                        float* grad, float* scale)
{
    if (!p) return GSB_ERR_NULL;
    if (!loss_shape_ok(*p)) return GSB_ERR_INVALID;
    if (!workspace || workspace_bytes < gsb_loss_workspace_size(p)) return GSB_ERR_WORKSPACE;
    if (!image || !target || !loss || !grad) return GSB_ERR_NULL;
    if (int e = configure_loss_kernels()) return e;
    float* block_loss = static_cast<float*>(workspace);
    uint32_t* block_scale =
        reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) + slot_bytes(*p));
    return launch_loss(as_stream(stream), *p, image, target, loss, grad, scale, block_loss,
                       block_scale);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of gsb_loss.
//
// Who needs it: callers that may not allocate device memory at the moment
// they compute the loss.  A JAX/XLA host preallocates most of the GPU for its
// own allocator and hands a custom call only the buffers it planned, so a
// cudaMalloc inside the call competes with that pool (and can fail with
// memory nominally free); a serving process with a fixed memory plan forbids
// allocation on its request path; cudaMalloc and cudaFree can synchronise the
// device, stalling every stream a latency-bound caller keeps busy; and a
// plugin boundary that passes only input and output pointers gives the
// callee nowhere to put a workspace.  gsb_loss needs at most 2 x 4 bytes
// per 32x16 block of pixels and channel of temporaries (one loss sum and
// one |grad| maximum per CTA).  Here they
// live in the fixed array below, part of this library's device image.
//
// Limits and sharing:
//  * GSB_LOSS_NOALLOC_MAX_TILES tiles of 32x16 pixels (4096 x 2048 pixels,
//    or any image with ceil(W/32) * ceil(H/16) <= 16384); larger images are
//    rejected with GSB_ERR_INVALID and a message in gsb_last_error().
//  * The array takes 384 KiB on every GPU on which this library's device
//    code is loaded, until the process exits.
//  * Every call on a device shares the one array.  Nothing in it needs to
//    start at zero: each CTA overwrites its own slots before the finishing
//    kernel reads them, so the contents left by the previous call are never
//    read.  Calls whose kernels overlap on the GPU (different streams with
//    no ordering between them) race on the array and give wrong results;
//    order them on one stream or with events.
//  * The first call on a device, with that device current, looks up the
//    array's device address (cudaGetSymbolAddress) and sets the kernels'
//    shared-memory limit on that device; make that first call before any
//    stream capture begins.  Later calls only read the cached address.
// ---------------------------------------------------------------------------
namespace gsb {
namespace {

constexpr int kNoallocMaxTiles = GSB_LOSS_NOALLOC_MAX_TILES;
constexpr int kNoallocSlots = 3 * kNoallocMaxTiles;  // one per 32x16 block and channel
constexpr int kNoallocMaxDevices = 64;

// [0, slots) loss sums (float bits), [slots, 2 slots) |grad| maxima.
static __device__ __align__(256) uint32_t g_loss_scratch[2 * kNoallocSlots];

std::mutex g_noalloc_mutex;
std::atomic<void*> g_noalloc_scratch[kNoallocMaxDevices];

// Device address of g_loss_scratch on the current device (set up on first
// use).  The name g_loss_scratch in host code is only a handle for the
// runtime; the address must come from cudaGetSymbolAddress.
int noalloc_scratch(void** out)
{
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) {
        set_error(err);
        return GSB_ERR_LAUNCH;
    }
    if (dev < 0 || dev >= kNoallocMaxDevices) {
        set_error_text("gsb_loss_noalloc: device ordinal above 63 is not supported");
        return GSB_ERR_INVALID;
    }
    void* ptr = g_noalloc_scratch[dev].load(std::memory_order_acquire);
    if (!ptr) {
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        ptr = g_noalloc_scratch[dev].load(std::memory_order_acquire);
        if (!ptr) {
            err = cudaGetSymbolAddress(&ptr, g_loss_scratch);
            if (err != cudaSuccess || !ptr) {
                set_error(err != cudaSuccess ? err : cudaErrorInvalidSymbol);
                return GSB_ERR_LAUNCH;
            }
            g_noalloc_scratch[dev].store(ptr, std::memory_order_release);
        }
    }
    *out = ptr;
    return GSB_OK;
}

}  // namespace
}  // namespace gsb

extern "C" int gsb_loss_noalloc(gsb_stream_t stream, const gsb_loss_params* p, const float* image,
                                const void* target, float* loss, float* grad, float* scale)
{
    if (!p) return GSB_ERR_NULL;
    if (p->width <= 0 || p->height <= 0) return GSB_ERR_INVALID;
    const int64_t tiles = loss_tiles(*p);
    if (tiles > kNoallocMaxTiles) {
        char msg[200];
        std::snprintf(msg, sizeof(msg),
                      "gsb_loss_noalloc: a %dx%d image has %lld tiles of 32x16, above the "
                      "limit of %d (e.g. 4096x2048); use gsb_loss with a workspace",
                      p->width, p->height, (long long)tiles, kNoallocMaxTiles);
        set_error_text(msg);
        return GSB_ERR_INVALID;
    }
    if (!image || !target || !loss || !grad) return GSB_ERR_NULL;
    void* scratch = nullptr;
    if (int e = noalloc_scratch(&scratch)) return e;
    if (int e = configure_loss_kernels()) return e;
    float* block_loss = static_cast<float*>(scratch);
    uint32_t* block_scale = static_cast<uint32_t*>(scratch) + kNoallocSlots;
    return launch_loss(as_stream(stream), *p, image, target, loss, grad, scale, block_loss,
                       block_scale);
}
