// Fused L1(0.8) + SSIM(0.2) loss, image gradient and gradient scale (sm_100a).
//
// Semantics: reference/loss.py:6-43 (11x11 Gaussian window, sigma 1.5, SAME
// zero padding, C1 = 0.01^2, C2 = 0.03^2) with the per-pixel gradient of
// kernels/fused_loss.py:229-288: for every pixel the SSIM partials
// dS/dmu_x, dS/dE[x^2], dS/dE[xy] are formed from the window statistics and
// blurred once more, grad = blur(p0) + 2x blur(p1) + y blur(p2)
// + 0.8 sign(x - y) / (3HW).
//
// One CTA per 32x16 output tile.  The CTA stages the 52x36 zero-padded patch
// (10-pixel halo) of all three channels of image and target with coalesced
// row loads, then per channel runs four separable 11-tap passes in shared
// memory, each thread producing a run of consecutive outputs from one
// sliding window held in registers:
//   1. horizontal window sums of x, x^2, y, y^2, xy    (36 rows x 42 columns)
//   2. vertical sums -> statistics -> SSIM partials, loss (26 x 42)
//   3. horizontal blur of the partials                   (26 x 32)
//   4. vertical blur -> image gradient                   (16 x 32)
// The gradient tile is written back coalesced after the third channel.  The
// loss map and the partials never reach global memory.  Per-CTA loss sums
// and |grad| maxima are reduced by a single-block kernel in a fixed order, so
// the scalar results are deterministic.
#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr int kTW = 32, kTH = 16, kR = 5;
constexpr int kSW = kTW + 2 * kR, kSH = kTH + 2 * kR;  // 42 x 26 statistics region
constexpr int kPW = kSW + 2 * kR, kPH = kSH + 2 * kR;  // 52 x 36 staged patch
constexpr int kThreads = 256;
// Pass shapes: runs of consecutive outputs per thread.
constexpr int kRunH = 6;   // pass 1: 42 = 7 x 6 columns, 36 rows -> 252 items
constexpr int kRunV = 5;   // pass 2: 26 rows in 6 runs of 5, 42 columns -> 252 items
constexpr int kRunHB = 4;  // pass 3: 32 = 8 x 4 columns, 26 rows -> 208 items
constexpr int kRunVB = 2;  // pass 4: 16 = 8 x 2 rows, 32 columns -> 256 items
constexpr int kHRows = 6 * kRunV + 2 * kR;  // 40 rows (4 padding rows feed discarded outputs)

// exp(-(d/1.5)^2 / 2) normalised, correctly rounded to float32.
__constant__ float kTaps[11] = {0.001028380123898387f, 0.0075987582094967365f,
                                0.036000773310661316f, 0.10936068743467331f,
                                0.21300554275512695f,  0.26601171493530273f,
                                0.21300554275512695f,  0.10936068743467331f,
                                0.036000773310661316f, 0.0075987582094967365f,
                                0.001028380123898387f};

struct LossSmem {
    float x[kPH][kPW * 3];        // image patch, HWC
    float y[kPH][kPW * 3];        // target patch, HWC (normalised)
    float h[5][kHRows][kSW];      // horizontal sums; reused for blurred partials
    float part[3][kSH + 6][kSW];  // partials p0, p1, p2 (+ padding rows)
    float g[kTH][kTW * 3];        // gradient tile, HWC
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
__global__ void __launch_bounds__(kThreads) loss_kernel(int width, int height,
                                                        const float* __restrict__ image,
                                                        const void* __restrict__ target_raw,
                                                        float* __restrict__ grad,
                                                        float* __restrict__ block_loss,
                                                        uint32_t* __restrict__ block_scale)
{
    extern __shared__ float4 smem_raw[];
    LossSmem& S = *reinterpret_cast<LossSmem*>(smem_raw);
    float(*hp)[kSH + 6][kTW + 1] = reinterpret_cast<float(*)[kSH + 6][kTW + 1]>(&S.h[0][0][0]);
    __shared__ float warp_loss[kThreads / 32];
    __shared__ uint32_t warp_scale[kThreads / 32];
    const int tid = threadIdx.x;
    const int x0 = blockIdx.x * kTW, y0 = blockIdx.y * kTH;
    const float inv_n = 1.0f / (3.0f * (float)width * (float)height);
    const float weight = -0.2f * inv_n;
    const uint8_t* t8 = static_cast<const uint8_t*>(target_raw);
    const float* tf = static_cast<const float*>(target_raw);

    // Stage the zero-padded patch, all channels (rows are contiguous in HWC).
    for (int k = tid; k < kPH * kPW * 3; k += kThreads) {
        int r = k / (kPW * 3), q = k % (kPW * 3);
        int gx = x0 - 2 * kR + q / 3, gy = y0 + r - 2 * kR;
        float xv = 0.0f, yv = 0.0f;
        if (gx >= 0 && gx < width && gy >= 0 && gy < height) {
            int64_t idx = ((int64_t)gy * width + x0 - 2 * kR) * 3 + q;
            xv = image[idx];
            if (CLIP) xv = clip01(xv);
            yv = U8 ? (float)t8[idx] * (float)(1.0 / 255.0) : tf[idx];
        }
        S.x[r][q] = xv;
        S.y[r][q] = yv;
    }
    float loss = 0.0f;
    for (int c = 0; c < 3; c++) {
        __syncthreads();
        // 1. Horizontal window sums (run of kRunH columns per thread).
        if (tid < kPH * (kSW / kRunH)) {
            const int r = tid / (kSW / kRunH), q0 = (tid % (kSW / kRunH)) * kRunH;
            float xs[kRunH + 10], ys[kRunH + 10];
#pragma unroll
            for (int t = 0; t < kRunH + 10; t++) {
                xs[t] = S.x[r][(q0 + t) * 3 + c];
                ys[t] = S.y[r][(q0 + t) * 3 + c];
            }
#pragma unroll
            for (int o = 0; o < kRunH; o++) {
                float sx = 0.f, sxx = 0.f, sy = 0.f, syy = 0.f, sxy = 0.f;
#pragma unroll
                for (int t = 0; t < 11; t++) {
                    const float w = kTaps[t], a = xs[o + t], b = ys[o + t];
                    const float wa = w * a, wb = w * b;
                    sx += wa;
                    sxx = fmaf(wa, a, sxx);
                    sy += wb;
                    syy = fmaf(wb, b, syy);
                    sxy = fmaf(wa, b, sxy);
                }
                S.h[0][r][q0 + o] = sx;
                S.h[1][r][q0 + o] = sxx;
                S.h[2][r][q0 + o] = sy;
                S.h[3][r][q0 + o] = syy;
                S.h[4][r][q0 + o] = sxy;
            }
        }
        __syncthreads();
        // 2. Vertical sums -> statistics -> partials and loss (run of kRunV rows).
        if (tid < (kSH + kRunV - 1) / kRunV * kSW) {
            const int q = tid % kSW, r0 = (tid / kSW) * kRunV;
            float m[5][kRunV];
#pragma unroll
            for (int s = 0; s < 5; s++) {
                float col[kRunV + 10];
#pragma unroll
                for (int t = 0; t < kRunV + 10; t++) col[t] = S.h[s][r0 + t][q];
#pragma unroll
                for (int o = 0; o < kRunV; o++) {
                    float acc = 0.f;
#pragma unroll
                    for (int t = 0; t < 11; t++) acc = fmaf(kTaps[t], col[o + t], acc);
                    m[s][o] = acc;
                }
            }
            const int gx = x0 + q - kR;
#pragma unroll
            for (int o = 0; o < kRunV; o++) {
                const int r = r0 + o;
                const int gy = y0 + r - kR;
                float p0 = 0.f, p1 = 0.f, p2 = 0.f;
                if (r < kSH && gx >= 0 && gx < width && gy >= 0 && gy < height) {
                    const float mx = m[0][o], xx = m[1][o], my = m[2][o], yy = m[3][o], xy = m[4][o];
                    const float A = mx * mx + my * my + 1e-4f;
                    const float B = (xx - mx * mx) + (yy - my * my) + 9e-4f;
                    const float Cc = 2.0f * mx * my + 1e-4f;
                    const float D = 2.0f * (xy - mx * my) + 9e-4f;
                    const float inv_a = 1.0f / A, inv_b = 1.0f / B;
                    const float inv_ab = inv_a * inv_b;
                    const float ssim = Cc * D * inv_ab;
                    p0 = (2.0f * my * (D - Cc) * inv_ab + 2.0f * mx * ssim * (inv_b - inv_a)) * weight;
                    p1 = -ssim * inv_b * weight;
                    p2 = 2.0f * Cc * inv_ab * weight;
                    if (r >= kR && r < kR + kTH && q >= kR && q < kR + kTW) {
                        const float xv = S.x[r + kR][(q + kR) * 3 + c];
                        const float yv = S.y[r + kR][(q + kR) * 3 + c];
                        loss += 0.2f * (1.0f - ssim) + 0.8f * fabsf(xv - yv);
                    }
                }
                S.part[0][r][q] = p0;
                S.part[1][r][q] = p1;
                S.part[2][r][q] = p2;
            }
        }
        __syncthreads();
        // 3. Horizontal blur of the partials onto the tile columns.
        if (tid < kSH * (kTW / kRunHB)) {
            const int r = tid / (kTW / kRunHB), q0 = (tid % (kTW / kRunHB)) * kRunHB;
#pragma unroll
            for (int k = 0; k < 3; k++) {
                float row[kRunHB + 10];
#pragma unroll
                for (int t = 0; t < kRunHB + 10; t++) row[t] = S.part[k][r][q0 + t];
#pragma unroll
                for (int o = 0; o < kRunHB; o++) {
                    float acc = 0.f;
#pragma unroll
                    for (int t = 0; t < 11; t++) acc = fmaf(kTaps[t], row[o + t], acc);
                    hp[k][r][q0 + o] = acc;
                }
            }
        }
        __syncthreads();
        // 4. Vertical blur -> image gradient (run of kRunVB rows).
        {
            const int q = tid % kTW, r0 = (tid / kTW) * kRunVB;
            float acc[3][kRunVB];
#pragma unroll
            for (int k = 0; k < 3; k++) {
                float col[kRunVB + 10];
#pragma unroll
                for (int t = 0; t < kRunVB + 10; t++) col[t] = hp[k][r0 + t][q];
#pragma unroll
                for (int o = 0; o < kRunVB; o++) {
                    float a = 0.f;
#pragma unroll
                    for (int t = 0; t < 11; t++) a = fmaf(kTaps[t], col[o + t], a);
                    acc[k][o] = a;
                }
            }
#pragma unroll
            for (int o = 0; o < kRunVB; o++) {
                const int r = r0 + o;
                const float xv = S.x[r + 2 * kR][(q + 2 * kR) * 3 + c];
                const float yv = S.y[r + 2 * kR][(q + 2 * kR) * 3 + c];
                const float sign = xv > yv ? 1.0f : (xv < yv ? -1.0f : 0.0f);
                S.g[r][q * 3 + c] = acc[0][o] + 2.0f * xv * acc[1][o] + yv * acc[2][o] +
                                    0.8f * sign * inv_n;
            }
        }
    }
    __syncthreads();
    // Coalesced write of the gradient tile (and its |max| for the scale).
    uint32_t scale_bits = 0;
    for (int k = tid; k < kTH * kTW * 3; k += kThreads) {
        const int r = k / (kTW * 3), q = k % (kTW * 3);
        const int px = x0 + q / 3, py = y0 + r;
        if (px < width && py < height) {
            const int64_t idx = ((int64_t)py * width + x0) * 3 + q;
            float value = S.g[r][q];
            if (CLIP) value *= clip_grad(image[idx]);
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
        const int b = blockIdx.y * gridDim.x + blockIdx.x;
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
    __shared__ double partial[32];
    __shared__ uint32_t pscale[32];
    double s = 0.0;
    uint32_t m = 0;
    for (int b = threadIdx.x; b < blocks; b += blockDim.x) {
        s += (double)block_loss[b];
        m = max(m, block_scale[b]);
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

int loss_blocks(const gsb_loss_params& p) { return ceil_div(p.width, kTW) * ceil_div(p.height, kTH); }

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" size_t gsb_loss_workspace_size(const gsb_loss_params* p)
{
    if (!p || p->width <= 0 || p->height <= 0) return 0;
    return 2 * (((size_t)loss_blocks(*p) * 4 + 255) & ~size_t(255));
}

extern "C" int gsb_loss(gsb_stream_t stream, const gsb_loss_params* p, void* workspace,
                        size_t workspace_bytes, const float* image, const void* target, float* loss,
                        float* grad, float* scale)
{
    if (!p) return GSB_ERR_NULL;
    if (p->width <= 0 || p->height <= 0) return GSB_ERR_INVALID;
    if (!workspace || workspace_bytes < gsb_loss_workspace_size(p)) return GSB_ERR_WORKSPACE;
    if (!image || !target || !loss || !grad) return GSB_ERR_NULL;
    cudaStream_t s = as_stream(stream);
    int blocks = loss_blocks(*p);
    size_t half = ((size_t)blocks * 4 + 255) & ~size_t(255);
    float* block_loss = static_cast<float*>(workspace);
    uint32_t* block_scale = reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) + half);
    dim3 grid(ceil_div(p->width, kTW), ceil_div(p->height, kTH));
    size_t smem = sizeof(LossSmem);
    // The shared-memory opt-in is set once per process (one device per
    // process); it is a host-side attribute, so graph captures never see it.
    static bool configured[4] = {false, false, false, false};
    auto launch = [&](auto kernel, int which) {
        if (!configured[which]) {
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            configured[which] = true;
        }
        kernel<<<grid, kThreads, smem, s>>>(p->width, p->height, image, target, grad, block_loss,
                                            block_scale);
    };
    if (p->target_u8) {
        if (p->clip_input) launch(loss_kernel<true, true>, 0);
        else launch(loss_kernel<true, false>, 1);
    } else {
        if (p->clip_input) launch(loss_kernel<false, true>, 2);
        else launch(loss_kernel<false, false>, 3);
    }
    if (int e = check_launch()) return e;
    float inv_n = 1.0f / (3.0f * (float)p->width * (float)p->height);
    loss_finish_kernel<<<1, 1024, 0, s>>>(blocks, inv_n, block_loss, block_scale, loss, scale);
    return check_launch();
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
// output tile of temporaries (per-tile loss sums and |grad| maxima).  Here
// they live in the fixed array below, part of this library's device image.
//
// Limits and sharing:
//  * kNoallocMaxTiles tiles of 32x16 pixels (4096 x 2048 pixels, or any
//    image with ceil(W/32) * ceil(H/16) <= 16384); larger images are
//    rejected with GSB_ERR_INVALID and a message in gsb_last_error().
//  * The array takes 128 KiB on every GPU on which this library's device
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
#include <atomic>
#include <cstdio>
#include <mutex>

namespace gsb {
namespace {

constexpr int kNoallocMaxTiles = GSB_LOSS_NOALLOC_MAX_TILES;
constexpr int kNoallocMaxDevices = 64;

// [0, max) per-tile loss sums (float bits), [max, 2 max) per-tile |grad| maxima.
static __device__ __align__(256) uint32_t g_loss_scratch[2 * kNoallocMaxTiles];

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
    const int64_t tiles = (int64_t)ceil_div(p->width, kTW) * ceil_div(p->height, kTH);
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
    float* block_loss = static_cast<float*>(scratch);
    uint32_t* block_scale = static_cast<uint32_t*>(scratch) + kNoallocMaxTiles;
    cudaStream_t s = as_stream(stream);
    const int blocks = (int)tiles;
    dim3 grid(ceil_div(p->width, kTW), ceil_div(p->height, kTH));
    const size_t smem = sizeof(LossSmem);
    auto launch = [&](auto kernel) {
        kernel<<<grid, kThreads, smem, s>>>(p->width, p->height, image, target, grad, block_loss,
                                            block_scale);
    };
    if (p->target_u8) {
        if (p->clip_input) launch(loss_kernel<true, true>);
        else launch(loss_kernel<true, false>);
    } else {
        if (p->clip_input) launch(loss_kernel<false, true>);
        else launch(loss_kernel<false, false>);
    }
    if (int e = check_launch()) return e;
    float inv_n = 1.0f / (3.0f * (float)p->width * (float)p->height);
    loss_finish_kernel<<<1, 1024, 0, s>>>(blocks, inv_n, block_loss, block_scale, loss, scale);
    return check_launch();
}
