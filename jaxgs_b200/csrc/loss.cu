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
// One CTA per (32x16 output tile, channel).  The CTA stages the 52x36
// zero-padded (x, y) patch of its channel (10-pixel halo), then runs four
// separable 11-tap passes in shared memory.  Each thread owns a run of
// consecutive outputs and accumulates them in registers while it streams
// the inputs once (scatter form), so only the run's accumulators are live:
//   1. vertical sums of the statistics      (26 rows x 52 columns)
//   2. horizontal sums -> SSIM partials, loss (26 x 42)
//   3. vertical blur of the partials          (16 x 42)
//   4. horizontal blur -> image gradient      (16 x 32)
// Row strides are padded to odd multiples so that lanes walking down a
// column hit distinct banks.  About 54 KB of shared memory per CTA, so four
// CTAs (32 warps) share an SM.  Per-CTA loss sums and |grad| maxima are
// reduced by a single-block kernel in a fixed order, so the scalar results
// are deterministic.
#include <atomic>
#include <cstdio>
#include <mutex>

#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr int kTW = 32, kTH = 16, kR = 5, kTaps = 2 * kR + 1;
constexpr int kThreads = 256;
constexpr int kSW = kTW + 2 * kR, kSH = kTH + 2 * kR;  // 42 x 26 statistics region
constexpr int kPW = kTW + 4 * kR, kPH = kTH + 4 * kR;  // 52 x 36 staged patch
constexpr int kRun1 = 7, kRuns1 = 4;          // pass 1: 26 rows as 4 runs of 7 (2 spare rows)
constexpr int kRun2 = 6, kRuns2 = kSW / kRun2;  // pass 2: 42 columns as 7 runs of 6
constexpr int kRun3 = 4, kRuns3 = kTH / kRun3;  // pass 3: 16 rows as 4 runs of 4
constexpr int kRun4 = 4, kRuns4 = kTW / kRun4;  // pass 4: 32 columns as 8 runs of 4
constexpr int kPRows = kRuns1 * kRun1 + 2 * kR;  // 38 staged rows (the 2 spare ones feed discarded outputs)
static_assert(kPRows >= kPH, "patch rows");
constexpr int kPStride = kPW + 1, kVStride = kPW + 1, kQStride = kSW + 1;
static_assert(kRuns1 * kRun1 >= kSH && kRuns2 * kRun2 == kSW, "run cover");
static_assert(kRuns1 * kPW <= kThreads && kRuns2 * kSH <= kThreads, "pass items");
static_assert(kRuns3 * kSW <= kThreads && kRuns4 * kTH <= kThreads, "pass items");

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

__device__ __forceinline__ float2 tap2(int t) { return make_float2(tap(t), tap(t)); }

struct LossSmem {
    float2 patch[kPRows][kPStride];  // (x, y) of this channel; x clipped when requested
    union {
        float4 v[kRuns1 * kRun1][kVStride];  // pass 1: (mu_x, mu_y, E[x^2+y^2], E[xy]) column sums
        struct {
            float2 q01[kTH][kQStride];  // pass 3: vertically blurred partials (p0, p1)
            float q2[kTH][kQStride];    //         and p2
        } q;
    } u;
    union {
        struct {
            float2 p01[kSH][kQStride];  // pass 2: partials (p0, p1)
            float p2[kSH][kQStride];    //         and p2
        } p;
        float g[kTH][kTW + 1];  // pass 4: gradient tile
    } w;
};

__device__ __forceinline__ float clip01(float v) { return fminf(fmaxf(v, 0.0f), 1.0f); }

// d clip(v, 0, 1) / dv with jnp.maximum/minimum tie semantics (1/2 at a bound).
__device__ __forceinline__ float clip_grad(float v)
{
    if (v > 0.0f && v < 1.0f) return 1.0f;
    if (v == 0.0f || v == 1.0f) return 0.5f;
    return 0.0f;
}

template <bool U8, bool CLIP>
__global__ void __launch_bounds__(kThreads, 4) loss_kernel(int width, int height,
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
    const int c = blockIdx.z;
    const int x0 = blockIdx.x * kTW, y0 = blockIdx.y * kTH;
    const float inv_n = 1.0f / (3.0f * (float)width * (float)height);
    const float weight = -0.2f * inv_n;
    const uint8_t* t8 = static_cast<const uint8_t*>(target_raw);
    const float* tf = static_cast<const float*>(target_raw);

    // Stage the zero-padded (x, y) patch of channel c: 64-lane rows, 4 rows
    // per sweep.  Every load of the thread is issued before the first use so
    // the rows' memory latencies overlap.
    {
        constexpr int kSweeps = (kPRows + kThreads / 64 - 1) / (kThreads / 64);
        const int col = tid & 63, row0 = tid >> 6;
        const int gx = x0 - 2 * kR + col;
        const bool col_in = col < kPW && gx >= 0 && gx < width;
        float xv[kSweeps], yv[kSweeps];
#pragma unroll
        for (int k = 0; k < kSweeps; k++) {
            const int pr = row0 + k * (kThreads / 64);
            const int gy = y0 - 2 * kR + pr;
            xv[k] = 0.0f;
            yv[k] = 0.0f;
            if (col_in && pr < kPRows && gy >= 0 && gy < height) {
                const int64_t idx = ((int64_t)gy * width + gx) * 3 + c;
                xv[k] = __ldg(image + idx);
                yv[k] = U8 ? (float)__ldg(t8 + idx) : __ldg(tf + idx);
            }
        }
        if (col < kPW) {
#pragma unroll
            for (int k = 0; k < kSweeps; k++) {
                const int pr = row0 + k * (kThreads / 64);
                if (pr < kPRows) {
                    const float x = CLIP ? clip01(xv[k]) : xv[k];
                    const float y = U8 ? yv[k] * (float)(1.0 / 255.0) : yv[k];
                    S.patch[pr][col] = make_float2(x, y);
                }
            }
        }
    }
    __syncthreads();
    // 1. Vertical window sums of (x, y) and (x^2 + y^2, xy).
    if (tid < kRuns1 * kPW) {
        const int q = tid % kPW, r0 = (tid / kPW) * kRun1;
        float2 m[kRun1], s[kRun1];
#pragma unroll
        for (int o = 0; o < kRun1; o++) m[o] = s[o] = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < kRun1 + 2 * kR; j++) {
            const float2 v = S.patch[r0 + j][q];
            const float2 sq = __fmul2_rn(v, v);
            const float2 u = make_float2(sq.x + sq.y, v.x * v.y);
#pragma unroll
            for (int o = 0; o < kRun1; o++) {
                const int t = j - o;
                if (t >= 0 && t < kTaps) {
                    m[o] = __ffma2_rn(tap2(t), v, m[o]);
                    s[o] = __ffma2_rn(tap2(t), u, s[o]);
                }
            }
        }
#pragma unroll
        for (int o = 0; o < kRun1; o++)
            S.u.v[r0 + o][q] = make_float4(m[o].x, m[o].y, s[o].x, s[o].y);
    }
    __syncthreads();
    // 2. Horizontal sums -> statistics -> SSIM partials (zero outside the
    // image) and the SSIM part of the loss on the tile's own pixels.
    float loss = 0.0f;
    if (tid < kRuns2 * kSH) {
        const int r = tid % kSH, c0 = (tid / kSH) * kRun2;
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
                    m[o] = __ffma2_rn(tap2(t), a, m[o]);
                    s[o] = __ffma2_rn(tap2(t), b, s[o]);
                }
            }
        }
        const int gy = y0 - kR + r;
        const bool row_in = gy >= 0 && gy < height;
        const bool row_own = r >= kR && r < kR + kTH;
#pragma unroll
        for (int o = 0; o < kRun2; o++) {
            const int cc = c0 + o;
            const int gx = x0 - kR + cc;
            float p0 = 0.0f, p1 = 0.0f, p2 = 0.0f;
            if (row_in && gx >= 0 && gx < width) {
                const float mx = m[o].x, my = m[o].y;
                const float mxy = mx * my;
                const float mm = fmaf(mx, mx, my * my);
                const float A = mm + 1e-4f;
                const float B = (s[o].x - mm) + 9e-4f;
                const float Cc = fmaf(2.0f, mxy, 1e-4f);
                const float D = fmaf(2.0f, s[o].y - mxy, 9e-4f);
                const float inv_a = __fdividef(1.0f, A), inv_b = __fdividef(1.0f, B);
                const float inv_ab = inv_a * inv_b;
                const float ssim = Cc * D * inv_ab;
                p0 = (my * (D - Cc) * inv_ab + mx * ssim * (inv_b - inv_a)) * (2.0f * weight);
                p1 = -ssim * inv_b * weight;
                p2 = 2.0f * Cc * inv_ab * weight;
                if (row_own && cc >= kR && cc < kR + kTW) loss += 0.2f * (1.0f - ssim);
            }
            S.w.p.p01[r][cc] = make_float2(p0, p1);
            S.w.p.p2[r][cc] = p2;
        }
    }
    __syncthreads();
    // 3. Vertical blur of the partials onto the tile rows.
    if (tid < kRuns3 * kSW) {
        const int cc = tid % kSW, r0 = (tid / kSW) * kRun3;
        float2 a[kRun3];
        float b[kRun3];
#pragma unroll
        for (int o = 0; o < kRun3; o++) {
            a[o] = make_float2(0.0f, 0.0f);
            b[o] = 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kRun3 + 2 * kR; j++) {
            const float2 u = S.w.p.p01[r0 + j][cc];
            const float v = S.w.p.p2[r0 + j][cc];
#pragma unroll
            for (int o = 0; o < kRun3; o++) {
                const int t = j - o;
                if (t >= 0 && t < kTaps) {
                    a[o] = __ffma2_rn(tap2(t), u, a[o]);
                    b[o] = fmaf(tap(t), v, b[o]);
                }
            }
        }
#pragma unroll
        for (int o = 0; o < kRun3; o++) {
            S.u.q.q01[r0 + o][cc] = a[o];
            S.u.q.q2[r0 + o][cc] = b[o];
        }
    }
    __syncthreads();
    // 4. Horizontal blur -> image gradient; the L1 part of the loss.
    if (tid < kRuns4 * kTH) {
        const int r = tid % kTH, c0 = (tid / kTH) * kRun4;
        float2 a[kRun4];
        float b[kRun4];
#pragma unroll
        for (int o = 0; o < kRun4; o++) {
            a[o] = make_float2(0.0f, 0.0f);
            b[o] = 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kRun4 + 2 * kR; j++) {
            const float2 u = S.u.q.q01[r][c0 + j];
            const float v = S.u.q.q2[r][c0 + j];
#pragma unroll
            for (int o = 0; o < kRun4; o++) {
                const int t = j - o;
                if (t >= 0 && t < kTaps) {
                    a[o] = __ffma2_rn(tap2(t), u, a[o]);
                    b[o] = fmaf(tap(t), v, b[o]);
                }
            }
        }
        const bool row_in = y0 + r < height;
#pragma unroll
        for (int o = 0; o < kRun4; o++) {
            const int col = c0 + o;
            const float2 xy = S.patch[r + 2 * kR][col + 2 * kR];
            const float sign = xy.x > xy.y ? 1.0f : (xy.x < xy.y ? -1.0f : 0.0f);
            S.w.g[r][col] = a[o].x + 2.0f * xy.x * a[o].y + xy.y * b[o] + 0.8f * sign * inv_n;
            if (row_in && x0 + col < width) loss += 0.8f * fabsf(xy.x - xy.y);
        }
    }
    __syncthreads();
    // Write the gradient tile (and its |max| for the scale).
    uint32_t scale_bits = 0;
    for (int k = tid; k < kTH * kTW; k += kThreads) {
        const int r = k / kTW, col = k % kTW;
        const int px = x0 + col, py = y0 + r;
        if (px < width && py < height) {
            const int64_t idx = ((int64_t)py * width + px) * 3 + c;
            float value = S.w.g[r][col];
            if (CLIP) value *= clip_grad(__ldg(image + idx));
            grad[idx] = value;
            scale_bits = max(scale_bits, __float_as_uint(value) & 0x7fffffffu);
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


// 32x16 output tiles of one channel; the kernel runs one CTA per tile and channel.
int64_t loss_tiles(const gsb_loss_params& p)
{
    return (int64_t)ceil_div(p.width, kTW) * ceil_div(p.height, kTH);
}

bool loss_shape_ok(const gsb_loss_params& p)
{
    return p.width > 0 && p.height > 0 && ceil_div(p.height, kTH) <= 65535 &&
           loss_tiles(p) <= (int64_t)1 << 28;
}

// The kernels need more than 48 KB of dynamic shared memory: opt in once per
// device (a host-side function attribute; it never enters a graph capture).
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
// per (tile, channel).
int launch_loss(cudaStream_t s, const gsb_loss_params& p, const float* image, const void* target,
                float* loss, float* grad, float* scale, float* block_loss, uint32_t* block_scale)
{
    dim3 grid(ceil_div(p.width, kTW), ceil_div(p.height, kTH), 3);
    const size_t smem = sizeof(LossSmem);
    auto launch = [&](auto kernel) {
        gsb::launch(kernel, grid, kThreads, smem, s, p.width, p.height, image, target, grad, block_loss,
                                            block_scale);
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
    gsb::launch(loss_finish_kernel, 1, 1024, 0, s, (int)(3 * loss_tiles(p)), inv_n, block_loss, block_scale,
                                          loss, scale);
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
// callee nowhere to put a workspace.  gsb_loss needs 2 x 4 bytes per 32x16
// tile and channel of temporaries (loss sums and |grad| maxima).  Here they
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
constexpr int kNoallocSlots = 3 * kNoallocMaxTiles;  // one per tile and channel
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
