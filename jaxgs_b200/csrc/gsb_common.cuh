// Shared device helpers for the sm_100a kernels of libgsb200.so.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gsb200.h"

#define GSB_FULL_MASK 0xffffffffu

namespace gsb {

// Records the last CUDA error string for gsb_last_error().
void set_error(cudaError_t err);
// Records a library message (not a CUDA error) for gsb_last_error().
void set_error_text(const char* msg);
// Adds to the process-wide count of kernels this library has launched.
void count_launch();

// Counts the launch just issued; returns GSB_ERR_LAUNCH (and records the
// error) if it failed.
inline int check_launch()
{
    count_launch();
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
        set_error(err);
        return GSB_ERR_LAUNCH;
    }
    return GSB_OK;
}

inline cudaStream_t as_stream(gsb_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Programmatic dependent launch.  Every kernel of this library is launched
// with programmatic stream serialization and starts with pdl_begin(): it
// waits until the previous kernel on the stream has completed and its
// memory is visible (griddepcontrol.wait; a no-op without a programmatic
// predecessor), then lets the next kernel's blocks be scheduled as soon as
// all of its own blocks have started (griddepcontrol.launch_dependents).  The
// next kernel's blocks thus take the SMs that this kernel's last blocks
// leave idle, and launch latency overlaps the tail; no kernel reads another
// kernel's output before that kernel has finished.
__device__ __forceinline__ void pdl_begin()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// kernel<<<grid, block, smem, stream>>>(args...) with the programmatic
// serialization attribute; errors surface through check_launch().
template <typename... Params, typename... Args>
inline void launch(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                   Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

// Workspace carving: 256-byte aligned sub-buffers.
struct Carver {
    char* base;
    size_t used;
    size_t cap;
    template <typename T>
    T* take(size_t count)
    {
        size_t bytes = (count * sizeof(T) + 255) & ~size_t(255);
        T* out = reinterpret_cast<T*>(base ? base + used : nullptr);
        used += bytes;
        return out;
    }
};

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// NVLS multicast access (symmetric memory bound to a multicast object):
// the switch sums one 16-byte chunk over every GPU's copy, or writes it to
// every copy.
__device__ __forceinline__ float4 multimem_ld_reduce_add_v4(const float* mc)
{
    float4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(mc)
                 : "memory");
    return v;
}

__device__ __forceinline__ void multimem_st_v4(float* mc, float4 v)
{
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
                 "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// ---------------------------------------------------------------------------
// Explicitly rounded float32 arithmetic.  These never contract into a
// neighbouring FMA, so the binning's fixed roundings are identical to the
// host oracle's (kernels/half2.py:296-317 describes the same discipline).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float ffma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float fsqrt(float a) { return __fsqrt_rn(a); }

// PTX cvt.rzi.s32.f32: truncation toward zero, saturating, NaN -> 0.
__device__ __forceinline__ int32_t trunc_i32(float x) { return __float2int_rz(x); }

// Project-written natural logarithm (same operation sequence as the host
// oracle's gs_logf): Cody & Waite reduction x = 2^e m, m in [sqrt(1/2),
// sqrt(2)], log(m) = 2 atanh((m-1)/(m+1)) by its Taylor series to s^11/11,
// ln 2 split into an exact high part and a low remainder.  Only IEEE
// round-to-nearest operations, hence bit-identical on host and device.
// Callers pass finite x > 0.
__device__ __forceinline__ float gs_logf(float x)
{
    if (!(x > 0.0f)) return x == 0.0f ? -__int_as_float(0x7f800000) : __int_as_float(0x7fffffff);
    if (isinf(x)) return x;
    uint32_t bits = __float_as_uint(x);
    int e = 0;
    if (bits < 0x00800000u) {
        x = fmul(x, 8388608.0f);
        bits = __float_as_uint(x);
        e = -23;
    }
    e += (int)(bits >> 23) - 127;
    float m = __uint_as_float((bits & 0x007FFFFFu) | 0x3F800000u);
    if (m > 1.41421356f) {
        m = fmul(m, 0.5f);
        e += 1;
    }
    float f = fsub(m, 1.0f);
    float s = fdiv(f, fadd(m, 1.0f));
    float z = fmul(s, s);
    float p = ffma(z, 1.0f / 11.0f, 1.0f / 9.0f);
    p = ffma(z, p, 1.0f / 7.0f);
    p = ffma(z, p, 1.0f / 5.0f);
    p = ffma(z, p, 1.0f / 3.0f);
    float sz = fmul(s, z);
    float tail = ffma(sz, p, s);
    float lm = fmul(tail, 2.0f);
    float ef = (float)e;
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.42860682030941723212e-6f;
    return ffma(ef, ln2_hi, ffma(ef, ln2_lo, lm));
}

__device__ __forceinline__ unsigned lanemask_lt()
{
    unsigned mask;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(mask));
    return mask;
}

template <typename T>
__device__ __forceinline__ T warp_inclusive_scan(T v, int lane)
{
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        T n = __shfl_up_sync(GSB_FULL_MASK, v, d);
        if (lane >= d) v += n;
    }
    return v;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v)
{
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(GSB_FULL_MASK, v, d);
    return v;
}

}  // namespace gsb
