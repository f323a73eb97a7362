// View-sharded gradient exchange over NVLink 5 / NVSwitch (sm_100a).
//
// The ranks of the view-sharded step (one process per GPU) hold their
// gradient buffers in symmetric memory: the same allocation on every GPU,
// mapped into one NVLS multicast object and into each peer's address space.
//   * gsb_exchange_barrier: every rank stores an epoch into every peer's flag
//     slot (release, system scope) and waits until all ranks' flags reach the
//     epoch (acquire).  Each wait is bounded; on expiry the kernel records an
//     error word and returns, so a missing peer can never hang the GPU.
//   * gsb_nvls_allreduce: rank r owns the r-th shard of the buffer; for each
//     16-byte chunk of it, multimem.ld_reduce makes the switch fetch and sum
//     the chunk of every GPU, and multimem.st writes the sum into every GPU's
//     copy.  Each GPU sends and receives about one buffer's worth of bytes.
//   * gsb_multicast_nonzero is the all-gather of the colour rows: each rank
//     stores the non-zero 16-byte chunks of its own row (written locally by
//     the pullback) through the multicast address into every GPU's copy.
//     A few hundred blocks do it, each with one system-scope fence at its
//     end, so the pullback itself never waits for NVLink acknowledgements.
//   * gsb_p2p_allreduce: the same sum with plain peer loads and stores: rank
//     r reads shard r of every rank's buffer (its own locally), adds them in
//     rank order and stores the sum into shard r of every buffer.  Each GPU
//     moves (world - 1) / world of the buffer in each direction, about what
//     the switch-reduced form moves, with ordinary loads that keep many
//     requests in flight.
// Callers put a barrier between a producer and these collectives and after
// them (the sum is complete on every GPU only once every shard is stored).
// No TMA and no cluster-multicast loads are used: peers' memory is touched
// only by multimem.* and plain st/ld with system-scope ordering.
#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr int kBarrierSpinLimit = 1 << 22;  // about a second of local polls

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One block, one thread per rank.  flags: this rank's slots [world] (each
// peer writes slot `rank` of it); peer_flags[q]: rank q's slots.
__global__ void exchange_barrier_kernel(int world, int rank, uint32_t* const* peer_flags,
                                        const uint32_t* flags, uint32_t* epoch, int32_t* error)
{
    pdl_begin();
    __shared__ uint32_t next;
    if (threadIdx.x == 0) {
        __threadfence_system();  // this rank's earlier writes precede its signal
        next = *epoch + 1;
    }
    __syncthreads();
    const int q = threadIdx.x;
    if (q < world) {
        st_release_sys(peer_flags[q] + rank, next);
        int spins = 0;
        while ((int32_t)(ld_acquire_sys(flags + q) - next) < 0) {
            if (++spins > kBarrierSpinLimit) {
                atomicExch(error, 1);
                break;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        *epoch = next;
        __threadfence_system();
    }
}

constexpr int kUnroll = 4;  // independent 16-byte chunks in flight per thread

// Shard [begin, end) of the multicast buffer, in float4 chunks.  Every
// collective returns at once when the exchange's error word is set (a
// barrier gave up waiting for a peer): its inputs are then not known to be
// complete, and the buffers are left as they are.
__global__ void nvls_allreduce_kernel(float* mc, int64_t begin4, int64_t end4,
                                      const int32_t* error)
{
    pdl_begin();
    if (error && *reinterpret_cast<const volatile int32_t*>(error)) return;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = begin4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < end4;
         i += stride * kUnroll) {
        float4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; u++)
            if (i + u * stride < end4) v[u] = multimem_ld_reduce_add_v4(mc + (i + u * stride) * 4);
#pragma unroll
        for (int u = 0; u < kUnroll; u++)
            if (i + u * stride < end4) multimem_st_v4(mc + (i + u * stride) * 4, v[u]);
    }
    // The stores precede the barrier that follows: one system-scope fence per
    // block, cumulative over the block's stores through the block barrier.
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
}

// Chunks that are all zero are not sent: the receiving copies hold zeros
// there (they are cleared after each use), and most of a view's colour
// cotangents are zero.
__global__ void multicast_nonzero_kernel(const float4* __restrict__ src, float* mc, int64_t n4,
                                         const int32_t* error)
{
    pdl_begin();
    if (error && *reinterpret_cast<const volatile int32_t*>(error)) return;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride * kUnroll) {
        float4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; u++)
            v[u] = i + u * stride < n4 ? src[i + u * stride] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < kUnroll; u++)
            if (v[u].x != 0.0f || v[u].y != 0.0f || v[u].z != 0.0f || v[u].w != 0.0f)
                multimem_st_v4(mc + (i + u * stride) * 4, v[u]);
    }
    // The stores precede the barrier that follows: one system-scope fence per
    // block, cumulative over the block's stores through the block barrier.
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
}

constexpr int kMaxPeers = 8;
struct PeerBuffers {
    float* p[kMaxPeers];
};
constexpr int kP2PUnroll = 2;

__global__ void p2p_allreduce_kernel(PeerBuffers peers, int world, int64_t begin4, int64_t end4,
                                     const int32_t* error)
{
    pdl_begin();
    if (error && *reinterpret_cast<const volatile int32_t*>(error)) return;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = begin4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < end4;
         i += stride * kP2PUnroll) {
        float4 v[kMaxPeers][kP2PUnroll];
        // Every load of the chunk is issued before the first add; .cv loads
        // fetch the peers' data afresh (written before the barrier).
#pragma unroll
        for (int q = 0; q < kMaxPeers; q++)
#pragma unroll
            for (int u = 0; u < kP2PUnroll; u++)
                if (q < world && i + u * stride < end4)
                    v[q][u] = __ldcv(reinterpret_cast<const float4*>(peers.p[q]) + i + u * stride);
#pragma unroll
        for (int u = 0; u < kP2PUnroll; u++) {
            if (i + u * stride >= end4) continue;
            float4 acc = v[0][u];
#pragma unroll
            for (int q = 1; q < kMaxPeers; q++) {
                if (q < world) {
                    acc.x += v[q][u].x;
                    acc.y += v[q][u].y;
                    acc.z += v[q][u].z;
                    acc.w += v[q][u].w;
                }
            }
#pragma unroll
            for (int q = 0; q < kMaxPeers; q++)
                if (q < world) reinterpret_cast<float4*>(peers.p[q])[i + u * stride] = acc;
        }
    }
    // The remote stores precede the barrier that follows.
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gsb_exchange_barrier(gsb_stream_t stream, const gsb_exchange_params* p,
                                    uint32_t* const* peer_flags, const uint32_t* flags,
                                    uint32_t* epoch, int32_t* error)
{
    if (!p) return GSB_ERR_NULL;
    if (p->world < 1 || p->world > 1024 || p->rank < 0 || p->rank >= p->world)
        return GSB_ERR_INVALID;
    if (!peer_flags || !flags || !epoch || !error) return GSB_ERR_NULL;
    gsb::launch(exchange_barrier_kernel, 1, ((p->world + 31) / 32) * 32, 0, as_stream(stream), 
        p->world, p->rank, peer_flags, flags, epoch, error);
    return check_launch();
}

extern "C" int gsb_nvls_allreduce(gsb_stream_t stream, const gsb_exchange_params* p,
                                  float* multicast, int64_t count, const int32_t* error)
{
    if (!p) return GSB_ERR_NULL;
    if (p->world < 1 || p->rank < 0 || p->rank >= p->world || count < 0 || (count & 3) != 0)
        return GSB_ERR_INVALID;
    if (!multicast) return GSB_ERR_NULL;
    if (!aligned16(multicast)) return GSB_ERR_INVALID;
    const int64_t n4 = count / 4;
    const int64_t per = (n4 + p->world - 1) / p->world;
    const int64_t begin = per * p->rank, end = begin + per < n4 ? begin + per : n4;
    if (begin >= end) return GSB_OK;
    // One block per SM: the 44 MB all-reduce alone measured 124 us at 8 ranks
    // against 140 us with two to eight blocks per SM (126 against 139 us at
    // 2 ranks); more requests in flight do not move more bytes through the
    // switch.
    const int64_t want = (end - begin + 256 * kUnroll - 1) / (256 * kUnroll);
    const int blocks = (int)(want < 148 ? want : 148);
    gsb::launch(nvls_allreduce_kernel, blocks, 256, 0, as_stream(stream), multicast, begin, end,
                error);
    return check_launch();
}

extern "C" int gsb_multicast_nonzero(gsb_stream_t stream, const float* src, float* multicast,
                                     int64_t count, const int32_t* error)
{
    if (count < 0 || (count & 3) != 0) return GSB_ERR_INVALID;
    if (count == 0) return GSB_OK;
    if (!src || !multicast) return GSB_ERR_NULL;
    if (!aligned16(src) || !aligned16(multicast)) return GSB_ERR_INVALID;
    const int64_t n4 = count / 4;
    const int64_t want = (n4 + 256 * kUnroll - 1) / (256 * kUnroll);
    const int blocks = (int)(want < 148 * 2 ? want : 148 * 2);
    gsb::launch(multicast_nonzero_kernel, blocks, 256, 0, as_stream(stream),
                reinterpret_cast<const float4*>(src), multicast, n4, error);
    return check_launch();
}

extern "C" int gsb_p2p_allreduce(gsb_stream_t stream, const gsb_exchange_params* p,
                                 float* const* buffers, int64_t count, const int32_t* error)
{
    if (!p) return GSB_ERR_NULL;
    if (p->world < 1 || p->world > kMaxPeers || p->rank < 0 || p->rank >= p->world || count < 0 ||
        (count & 3) != 0)
        return GSB_ERR_INVALID;
    if (!buffers) return GSB_ERR_NULL;
    PeerBuffers peers{};
    for (int q = 0; q < p->world; q++) {
        if (!buffers[q]) return GSB_ERR_NULL;
        if (!aligned16(buffers[q])) return GSB_ERR_INVALID;
        peers.p[q] = buffers[q];
    }
    const int64_t n4 = count / 4;
    const int64_t per = (n4 + p->world - 1) / p->world;
    const int64_t begin = per * p->rank, end = begin + per < n4 ? begin + per : n4;
    if (begin >= end) return GSB_OK;
    // One block per SM: 79 us at 2 ranks and 143 us at 8 for 44 MB, against
    // 86 and 157 us with four blocks per SM.
    const int64_t want = (end - begin + 256 * kP2PUnroll - 1) / (256 * kP2PUnroll);
    const int blocks = (int)(want < 148 ? want : 148);
    gsb::launch(p2p_allreduce_kernel, blocks, 256, 0, as_stream(stream), peers, p->world, begin,
                end, error);
    return check_launch();
}
