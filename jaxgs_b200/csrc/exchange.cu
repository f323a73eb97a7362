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
//   * gsb_colour_push_compact / gsb_colour_expand: the colour all-gather in
//     compact form.  Each rank appends (id, r, g, b) for every Gaussian with
//     a non-zero colour cotangent to its compact row through the multicast
//     address, a warp's entries at consecutive addresses (one atomic per
//     warp), so the switch carries whole lines instead of the scattered
//     16-byte chunks of gsb_multicast_nonzero; after the next barrier every
//     rank scatters each view's entries into its local dense rows.
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

// Compact row layout: [centre x, y, z, entry count (int bits) | entries of
// (id (int bits), r, g, b)], 4 + 4 * capacity floats.  The count is
// written by compact_header_kernel after every entry is stored.  Two tables
// alternate: *slot (a device word, advanced by the expand call) picks the
// one a call pushes into and expands, so a rank can push its next step's
// entries while a slower peer still expands the previous ones.
__global__ void compact_push_kernel(const float* __restrict__ row, int64_t capacity, float* mc0,
                                    float* mc1, const int32_t* slot, int32_t* counter,
                                    const int32_t* error)
{
    pdl_begin();
    if (error && *reinterpret_cast<const volatile int32_t*>(error)) return;
    float* mc = (__ldg(slot) & 1) ? mc1 : mc0;
    const int lane = threadIdx.x & 31;
    const float* colours = row + 4;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    // Every lane of a warp runs the same number of iterations (the bound is
    // rounded up to whole warps), so the ballots see full warps.
    const int64_t bound = (capacity + 31) & ~int64_t(31);
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < bound; g += stride) {
        float r = 0.0f, gg = 0.0f, b = 0.0f;
        if (g < capacity) {
            r = __ldg(colours + g * 3);
            gg = __ldg(colours + g * 3 + 1);
            b = __ldg(colours + g * 3 + 2);
        }
        const bool live = r != 0.0f || gg != 0.0f || b != 0.0f;
        const unsigned mask = __ballot_sync(GSB_FULL_MASK, live);
        if (mask == 0) continue;
        int base = 0;
        if (lane == 0) base = atomicAdd(counter, __popc(mask));
        base = __shfl_sync(GSB_FULL_MASK, base, 0);
        if (live) {
            const int at = base + __popc(mask & lanemask_lt());
            multimem_st_v4(mc + 4 + (int64_t)at * 4,
                           make_float4(__int_as_float((int)g), r, gg, b));
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
}

// One thread: the row's header (centre and entry count) after the entries.
__global__ void compact_header_kernel(const float* __restrict__ row, float* mc0, float* mc1,
                                      const int32_t* slot, const int32_t* counter,
                                      const int32_t* error)
{
    pdl_begin();
    if (error && *reinterpret_cast<const volatile int32_t*>(error)) return;
    float* mc = (*slot & 1) ? mc1 : mc0;
    multimem_st_v4(mc, make_float4(row[0], row[1], row[2], __int_as_float(*counter)));
    __threadfence_system();
}

// grid.y: view; each view's entries scattered into its dense row [centre,
// pad, capacity * 3 colours] (cleared beforehand), the centre copied.
__global__ void compact_expand_kernel(const float* __restrict__ table0,
                                      const float* __restrict__ table1, const int32_t* slot,
                                      int64_t capacity, int64_t compact_row, float* dense,
                                      int64_t dense_row, const int32_t* error)
{
    pdl_begin();
    if (error && *reinterpret_cast<const volatile int32_t*>(error)) return;
    const int v = blockIdx.y;
    const float* src = ((*slot & 1) ? table1 : table0) + (int64_t)v * compact_row;
    float* dst = dense + (int64_t)v * dense_row;
    const int64_t n = __float_as_int(__ldg(src + 3));
    const int64_t count = n < 0 ? 0 : (n > capacity ? capacity : n);
    if (blockIdx.x == 0 && threadIdx.x < 3) dst[threadIdx.x] = __ldg(src + threadIdx.x);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) {
        const float4 e = __ldg(reinterpret_cast<const float4*>(src + 4) + i);
        const int64_t g = __float_as_int(e.x);
        if (g < 0 || g >= capacity) continue;
        float* c = dst + 4 + g * 3;
        c[0] = e.y;
        c[1] = e.z;
        c[2] = e.w;
    }
}

// One thread, after the expand: the next call uses the other table.
__global__ void compact_flip_kernel(int32_t* slot, const int32_t* error)
{
    pdl_begin();
    if (error && *reinterpret_cast<const volatile int32_t*>(error)) return;
    *slot ^= 1;
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

extern "C" int gsb_colour_push_compact(gsb_stream_t stream, const float* row, int64_t capacity,
                                       float* multicast0, float* multicast1, const int32_t* slot,
                                       int32_t* counter, const int32_t* error)
{
    if (capacity < 0 || capacity >= ((int64_t)1 << 31)) return GSB_ERR_INVALID;
    if (!row || !multicast0 || !multicast1 || !slot || !counter) return GSB_ERR_NULL;
    if (!aligned16(row) || !aligned16(multicast0) || !aligned16(multicast1))
        return GSB_ERR_INVALID;
    cudaStream_t s = as_stream(stream);
    if (cudaMemsetAsync(counter, 0, sizeof(int32_t), s) != cudaSuccess) return check_launch();
    if (capacity > 0) {
        const int64_t want = (capacity + 255) / 256;
        const int blocks = (int)(want < 148 * 4 ? want : 148 * 4);
        gsb::launch(compact_push_kernel, blocks, 256, 0, s, row, capacity, multicast0, multicast1,
                    slot, counter, error);
    }
    gsb::launch(compact_header_kernel, 1, 1, 0, s, row, multicast0, multicast1, slot,
                static_cast<const int32_t*>(counter), error);
    return check_launch();
}

extern "C" int gsb_colour_expand(gsb_stream_t stream, const float* table0, const float* table1,
                                 int32_t* slot, int world, int64_t capacity, float* dense,
                                 int64_t dense_row, const int32_t* error)
{
    if (world < 1 || world > 65535 || capacity < 0 || capacity >= ((int64_t)1 << 31) ||
        dense_row < 4 + capacity * 3)
        return GSB_ERR_INVALID;
    if (!table0 || !table1 || !slot || !dense) return GSB_ERR_NULL;
    if (!aligned16(table0) || !aligned16(table1)) return GSB_ERR_INVALID;
    const int64_t compact_row = 4 + 4 * capacity;
    cudaStream_t s = as_stream(stream);
    gsb::launch(compact_expand_kernel, dim3(148, world), 256, 0, s, table0, table1,
                static_cast<const int32_t*>(slot), capacity, compact_row, dense, dense_row, error);
    gsb::launch(compact_flip_kernel, 1, 1, 0, s, slot, error);
    return check_launch();
}
