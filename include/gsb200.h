/*
 * gsb200.h — C ABI of the B200 (sm_100a) Gaussian-splatting render-and-loss
 * hot path (libgsb200.so).
 *
 * Conventions shared by every entry point:
 *  - All array arguments are DEVICE pointers to flat, dense buffers with the
 *    reference's layouts (documented per call).  Camera arrays (view[16],
 *    intrinsics[4], center[3]) and small scalars that the reference keeps on
 *    the device (cluster_count[1], pair_count[1], grad_scale[1]) are device
 *    pointers too, so no call ever synchronises with the host.
 *  - Launches are asynchronous on `stream`.  Return value: GSB_OK, or a
 *    GSB_ERR_* code for invalid parameters, a too-small workspace, or a
 *    launch failure.  Arena overflow is reported as data (overflow[1]).
 *  - Calls that need temporaries take (workspace, workspace_bytes); query
 *    the size with the matching *_workspace_size().  Workspace base must be
 *    256-byte aligned (cudaMalloc / torch allocations are).
 *  - Outputs are written in full where the reference defines them; the
 *    undefined regions are the reference's (arena tail past pair_count,
 *    compact-gradient tail, projected fields outside the listed clusters).
 *
 * Reference interfaces replaced (imgengineer/jax-gs, src/jaxgs/...):
 *  each declaration cites the cutlass_call launcher it replaces.
 */
#ifndef GSB200_H
#define GSB200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GSB_API __attribute__((visibility("default")))
#else
#define GSB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void* gsb_stream_t; /* a cudaStream_t */

enum {
    GSB_OK = 0,
    GSB_ERR_INVALID = 1,    /* bad shape / unsupported option */
    GSB_ERR_WORKSPACE = 2,  /* workspace too small or misaligned */
    GSB_ERR_LAUNCH = 3,     /* CUDA launch error */
    GSB_ERR_NULL = 4        /* required pointer is NULL */
};

#define GSB_ABI_VERSION 11

/* Library utilities.  No counterpart in the reference, whose boundary
 * (cutlass.jax.cutlass_call) reports errors by raising in Python before
 * launch; here the same checks return the codes above, and these three
 * calls expose the version, the last CUDA error and a launch counter.
 *
 * Library ABI version (GSB_ABI_VERSION). */
GSB_API int gsb_abi_version(void);
/* Last CUDA error string seen by the library (thread-local). */
GSB_API const char* gsb_last_error(void);
/* Number of kernels this library has launched in this process (host-side
 * counter, incremented once per launch it issues). */
GSB_API unsigned long long gsb_launch_count(void);

/* ------------------------------------------------------------------------
 * Cluster culling + compaction.
 * Replaces scene/cluster.py:40-67 (frustum_cluster_mask) and
 * kernels/cluster_compact.py:31-44 (compact_visible_clusters; XLA cumsum +
 * CuTe _scatter), as called by render/pipeline.py:18-44.
 * center/extent: [num_clusters,3]; valid: [num_clusters] u8;
 * planes: [6,4] device floats (a,b,c,d).  Outputs: ids[num_clusters] (stable
 * ascending visible cluster ids; tail undefined), count[1],
 * visible_slots[capacity] u8 (slot mask, repeat of the cluster mask).
 * ------------------------------------------------------------------------ */
typedef struct {
    int num_clusters;
    int cluster_size;
    int capacity;
} gsb_cluster_params;

GSB_API size_t gsb_cluster_compact_workspace_size(const gsb_cluster_params* p);
GSB_API int gsb_cluster_compact(gsb_stream_t stream, const gsb_cluster_params* p, void* workspace,
                        size_t workspace_bytes, const float* center, const float* extent,
                        const uint8_t* valid, const float* planes, int32_t* ids,
                        int32_t* count, uint8_t* visible_slots);

/* ------------------------------------------------------------------------
 * Projection forward.
 * Replaces kernels/projector.py:17-100 (_project_gaussian_arrays ->
 * cutlass_call(launch_projection), kernels/projection.py:213-285).
 * Inputs: xyz[C*3], log_scale[C*3], rotation[C*4] (wxyz), opacity[C] (logit),
 * sh[C*sh_dim*3], alive[C] u8, view[16] (row-major world-to-camera),
 * intrinsics[4] (fx,fy,cx,cy), center[3]; cluster_ids / cluster_count used
 * when compacted.  Outputs: mean[C*2], depth[C], conic[C*4], radius[C],
 * color[C*3], alpha[C], visible[C] i8.
 * ------------------------------------------------------------------------ */
typedef struct {
    int capacity;
    int sh_dim;            /* coefficients stored per Gaussian (1,4,9,16) */
    int degree;            /* active SH degree, 0..3, (degree+1)^2 <= sh_dim */
    int width, height;
    float near_plane, far_plane;
    int cluster_size;
    int compacted;          /* 1: only the listed clusters' slots */
    int clear_invisible;    /* compacted only: zero the other slots' fields */
    int visible_color_only; /* culled slots get colour 0 instead of SH */
} gsb_project_params;

GSB_API int gsb_project_fwd(gsb_stream_t stream, const gsb_project_params* p, const float* xyz,
                    const float* log_scale, const float* rotation, const float* opacity,
                    const float* sh, const uint8_t* alive, const float* view,
                    const float* intrinsics, const float* center, const int32_t* cluster_ids,
                    const int32_t* cluster_count, float* mean, float* depth, float* conic,
                    float* radius, float* color, float* alpha, int8_t* visible);

/* ------------------------------------------------------------------------
 * Projection pullback (parameter gradients).
 * Replaces kernels/projector.py:240-307 (_compute_projection_gradients ->
 * cutlass_call(launch_projection_backward), projection_backward.py:393-472).
 * Cotangents: gmean[C*2], gdepth[C] (unused if rgb_only), gconic[C*4],
 * gradius[C] (unused if rgb_only), gcolor[C*3], galpha[C].
 * Outputs (compact visible-cluster order when compact_gradients, else pool
 * order, where every slot is written and unlisted clusters' rows are zero):
 * gxyz[C*3], glog_scale[C*3], grotation[C*4], gopacity[C],
 * gsh[C*sh_gradient_dim*3].
 * ------------------------------------------------------------------------ */
typedef struct {
    int capacity;
    int sh_dim;
    int sh_gradient_dim;   /* sh_dim, (degree+1)^2 (active only) or 1 (colour only) */
    int degree;
    float near_plane;
    int cluster_size;
    int compacted;
    int compact_gradients;
    int rgb_only;
    int sh_color_only;
} gsb_project_bwd_params;

GSB_API int gsb_project_bwd(gsb_stream_t stream, const gsb_project_bwd_params* p, const float* xyz,
                    const float* log_scale, const float* rotation, const float* opacity,
                    const float* sh, const float* view, const float* intrinsics,
                    const float* center, const float* color, const int32_t* cluster_ids,
                    const int32_t* cluster_count, const float* gmean, const float* gdepth,
                    const float* gconic, const float* gradius, const float* gcolor,
                    const float* galpha, float* gxyz, float* glog_scale, float* grotation,
                    float* gopacity, float* gsh);

/* ------------------------------------------------------------------------
 * Visible-cluster sparse Adam, one parameter field per call.
 * Replaces kernels/sparse_adam.py:98-136 (update_field -> cutlass_call of
 * _launch/_update, used by training/optimizer.py:276-341 sparse_adam_update
 * with compacted clusters): LiteGS Adam without bias correction,
 *   m = 0.9 m + 0.1 g;  v = 0.999 v + 0.001 g^2;
 *   value -= lr * m / (sqrt(v) + 1e-15),  lr = rate[0] (x10 for the first
 *   three channels of each row when is_sh, the SH DC coefficient),
 * on every channel of every alive slot of the listed clusters; every other
 * element is left as it was.  value/mean/variance[capacity * channels] are
 * updated in place (pool order); gradient is [capacity * channels] in pool
 * order, or (compact_gradients) the visible-cluster prefix
 * [count * cluster_size * channels].  rate is a device scalar, so a
 * schedule needs no new launch parameters.
 * ------------------------------------------------------------------------ */
typedef struct {
    int capacity;
    int channels;          /* floats per slot of this field (3, 3, 4, 1, sh_dim * 3) */
    int cluster_size;
    int is_sh;
    int compact_gradients;
} gsb_adam_params;

GSB_API int gsb_sparse_adam(gsb_stream_t stream, const gsb_adam_params* p, float* value,
                    float* mean, float* variance, const float* gradient, const int8_t* alive,
                    const int32_t* cluster_ids, const int32_t* cluster_count,
                    const float* rate);

/* ------------------------------------------------------------------------
 * Sparse Adam of the SH field with the SH gradient rebuilt inside the update.
 * Replaces the deferred SH pullback of training/optimizer.py:180-261
 * (optax_update with sh_pullback_center, which wraps the update in
 * training/sh_pullback.py:18-53 with_sh_pullback) fused with the "sh" field
 * of kernels/sparse_adam.py:98-136 update_field.  For every alive slot of
 * the listed clusters the gradient
 *   g[k][c] = sum over views v of Y_k(dir_v) * colour_v[c]
 * (k below (degree + 1)^2; zero for the bands above) is formed in shared
 * memory with the arithmetic of gsb_sh_from_colors, and the LiteGS update of
 * gsb_sparse_adam (is_sh) is applied to all sh_dim * 3 channels, so the
 * [C, sh_dim, 3] gradient is never written or read.
 * colors + v * view_stride: view v's masked colour cotangents (the
 * sh_color_only output of gsb_project_bwd), [C*3] in pool order or, with
 * compact_colors, the visible-cluster prefix [count * cluster_size * 3];
 * centers + v * center_stride: view v's camera centre; strides in floats,
 * 0 = dense.  sh/mean/variance[C * sh_dim * 3] are updated in place.
 * ------------------------------------------------------------------------ */
typedef struct {
    int capacity;
    int sh_dim;          /* coefficients per slot, 1..16 */
    int degree;          /* active SH degree, 0..3 */
    int cluster_size;
    int views;
    int compact_colors;
    int64_t view_stride;
    int64_t center_stride;
} gsb_adam_sh_params;

GSB_API int gsb_sparse_adam_sh(gsb_stream_t stream, const gsb_adam_sh_params* p, float* sh,
                       float* mean, float* variance, const float* xyz, const float* centers,
                       const float* colors, const int8_t* alive, const int32_t* cluster_ids,
                       const int32_t* cluster_count, const float* rate);

/* ------------------------------------------------------------------------
 * Density-control consumers of the fragment statistics.
 * gsb_densify_scores replaces training/densify.py:20-35
 * (compute_densification_scores): stats[C*4] = (count, weight, alpha
 * cotangent sum, squared sum) per slot (16-byte aligned), opacity[C] logits,
 * alive[C] -> scores[C] = max(sq/(n+1) - (sum/(n+1))^2, 0) * n *
 * sigmoid(opacity)^2 (0 for dead slots and non-finite values), prune[C] =
 * alive & weight == 0.
 * gsb_decay_opacity replaces the pool half of training/densify.py:158-165
 * (decay_opacity): alive slots' logits become logit(max(sigmoid / 2,
 * 1/128)); the caller clears the Adam moments.
 * ------------------------------------------------------------------------ */
GSB_API int gsb_densify_scores(gsb_stream_t stream, int64_t capacity, const float* stats,
                       const float* opacity, const int8_t* alive, float* scores,
                       int8_t* prune);
GSB_API int gsb_decay_opacity(gsb_stream_t stream, int64_t capacity, float* opacity,
                      const int8_t* alive);

/* ------------------------------------------------------------------------
 * SH coefficient cotangents from colour cotangents, summed over views.
 * Replaces training/sh_pullback.py:18-53 (with_sh_pullback: one view's
 * masked colour cotangent expanded on the SH basis of its direction from
 * the camera centre), summed over `views` cameras so that view-sharded ranks
 * can exchange 3 floats per Gaussian and view instead of sh_dim * 3.
 * Inputs: xyz[C*3]; view v's centre at centers + v * center_stride (3
 * floats) and its colour cotangents at colors + v * view_stride (C*3 floats,
 * the sh_color_only output of gsb_project_bwd in pool order); strides in
 * floats, 0 = dense (3 and C*3), so one gathered buffer of [colours | centre]
 * rows can be read in place.
 * Output: gsh[C*sh_dim*3] (bands above degree zero).
 * ------------------------------------------------------------------------ */
typedef struct {
    int capacity;
    int sh_dim;
    int degree;
    int views;
    int64_t view_stride;
    int64_t center_stride;
} gsb_sh_params;

GSB_API int gsb_sh_from_colors(gsb_stream_t stream, const gsb_sh_params* p, const float* xyz,
                       const float* centers, const float* colors, float* gsh);

/* ------------------------------------------------------------------------
 * Tile binning (AccuTile count, depth sort, scan, emission, stable tile sort,
 * tile ranges) in one call.
 * Replaces kernels/sorted_binning.py:9-117 (build_sorted_visibility_table_cute:
 * launch_count_pairs, jax.lax.sort, launch_pair_offsets, launch_emit_pairs,
 * pair_sort.sort_pairs_by_tile, launch_tile_ranges).
 * Inputs: mean[C*2], conic[C*4], alpha[C], depth[C], visible[C] i8.
 * Outputs: point_counts[C], gaussian_ids[max_pairs] (valid prefix ends at
 * min(pair_count, max_pairs)), tile_offsets[T+1], pair_count[1] (unclamped),
 * overflow[1]: bit 0 = pair_count > max_pairs (the reference's overflow);
 * bit 1 = an internal sort look-back gave up waiting (bounded spin; the table
 * is then invalid).  T = ceil(W/tile_w)*ceil(H/tile_h).
 * ------------------------------------------------------------------------ */
typedef struct {
    int capacity;
    int width, height;
    int tile_w, tile_h;    /* reference tile_size (width) and tile_height */
    int64_t max_pairs;     /* arena capacity, < 2^30 */
} gsb_bin_params;

GSB_API size_t gsb_bin_workspace_size(const gsb_bin_params* p);
/* Stable tile-sort digit plan (passes, bits per digit) for keys below
 * num_tiles: replaces kernels/pair_sort.py:33-37 (digit_plan).  Host-only. */
GSB_API int gsb_tile_sort_plan(int64_t num_tiles, int* passes, int* bits);
GSB_API int gsb_bin(gsb_stream_t stream, const gsb_bin_params* p, void* workspace,
            size_t workspace_bytes, const float* mean, const float* conic, const float* alpha,
            const float* depth, const int8_t* visible, int32_t* point_counts,
            int32_t* gaussian_ids, int32_t* tile_offsets, int32_t* pair_count,
            int32_t* overflow);

/* ------------------------------------------------------------------------
 * fp32 rasterization forward.
 * Replaces kernels/sorted_rasterizer.py:15-70 (_forward_arrays ->
 * cutlass_call(launch_forward_sorted), sorted_rasterize.py:28-88), extended to
 * the rectangular tiles of the packed path (tile_w a multiple of 8, tile_h a
 * multiple of 4, at most 16 x 16).
 * Inputs: mean[C*2], conic[C*4], depth[C], color[C*3], alpha[C] (opacity
 * after sigmoid), visible[C] i8 (only visible Gaussians are staged; the table
 * must reference no other), gaussian_ids, tile_offsets[T+1], background[3].
 * Outputs: rgb[H*W*3], out_depth[H*W] (may be NULL), out_alpha[H*W] (may be
 * NULL), final_t[H*W], last[H*W] (one past the last composited pair),
 * backward_work[T] (max over the tile's pixels of last - tile start),
 * splats[C*12] (48-byte staged records), contribution_bits
 * [gsb_raster_bit_words()] (per 32-pair batch and pixel block, which pairs
 * gave at least one pixel of the block a composited fragment; only words of
 * batches the forward reached are written), fragment_stats[C*2] (may be
 * NULL = not collected; not with GSB_RASTER_RGB_ONLY): per Gaussian the
 * number of composited fragments and the sum of their compositing weights
 * T*alpha, interleaved, zeroed then accumulated by the call -- the forward
 * statistics of kernels/packed_rasterize.py:363-377.
 * ------------------------------------------------------------------------ */
typedef struct {
    int capacity;
    int width, height;
    int tile_w, tile_h;
    int64_t max_pairs;     /* arena capacity of the table (sizes the bit words) */
    int flags;             /* GSB_RASTER_SPLATS_READY: splats already written by gsb_raster_pack;
                              GSB_RASTER_RGB_ONLY: the inference forward, which
                              writes no final_t / last / backward_work /
                              contribution_bits (they may be NULL); the
                              reference's record_contributions = False,
                              kernels/packed_rasterizer.py:219-232;
                              GSB_RASTER_CLAMP_RGB: write min(rgb, 1), the
                              packed rasterizer's output
                              (kernels/packed_rasterize.py:396) */
} gsb_raster_params;

#define GSB_RASTER_SPLATS_READY 1
#define GSB_RASTER_RGB_ONLY 2
#define GSB_RASTER_CLAMP_RGB 4

GSB_API size_t gsb_raster_workspace_size(const gsb_raster_params* p);
GSB_API size_t gsb_raster_bit_words(const gsb_raster_params* p);
GSB_API int gsb_raster_fwd(gsb_stream_t stream, const gsb_raster_params* p, void* workspace,
                   size_t workspace_bytes, const float* mean, const float* conic,
                   const float* depth, const float* color, const float* alpha,
                   const int8_t* visible, const int32_t* gaussian_ids,
                   const int32_t* tile_offsets, const float* background, float* rgb,
                   float* out_depth, float* out_alpha, float* final_t, int32_t* last,
                   int32_t* backward_work, float* splats, uint32_t* contribution_bits,
                   float* fragment_stats);

/* The first stage of gsb_raster_fwd on its own: write the splat records of
 * every visible Gaussian.  It depends on the projection only, so a caller
 * can run it on a second stream while the table is built, then call
 * gsb_raster_fwd with GSB_RASTER_SPLATS_READY in p->flags (that call then
 * skips the stage and its mean/conic/color/alpha/visible may be NULL).
 * Splitting of the launcher inside kernels/sorted_rasterizer.py:15-70. */
GSB_API int gsb_raster_pack(gsb_stream_t stream, const gsb_raster_params* p, const float* mean,
                    const float* conic, const float* color, const float* alpha,
                    const int8_t* visible, float* splats);

/* ------------------------------------------------------------------------
 * fp32 rasterization backward.
 * Replaces kernels/sorted_rasterizer.py:165-236 (the launch_backward_sorted
 * call inside rasterize_loss_and_grad; kernel sorted_rasterize.py:91-236).
 * Inputs: the forward's splats / final_t / last / backward_work /
 * contribution_bits, depth[C] (for the depth cotangent), gaussian_ids,
 * tile_offsets, background[3], drgb[H*W*3], ddepth[H*W] and dalpha[H*W] (may
 * be NULL = zero).  cluster_ids/count: when non-NULL only the listed
 * clusters' cotangents are zeroed (the table must reference no other
 * Gaussian, kernels/packed_rasterize.py:753-758) and gdepth is not written;
 * otherwise the whole pool is zeroed.
 * Outputs (accumulated): gmean[C*2], gconic[C*4], gdepth[C], gcolor[C*3],
 * galpha[C].
 * fragment_stats[C*3] (may be NULL = not collected; collect_stats of
 * kernels/sorted_rasterize.py:155-203): per Gaussian the number of
 * composited fragments (alpha >= 1/256, before the pixel's last index), the
 * sum of their compositing weights T*alpha, and the sum over fragments of
 * the squared per-pixel opacity cotangent (zero where alpha saturates at
 * 255/256).  With it galpha is zeroed over the whole pool, also when
 * cluster_ids is given, so that galpha is the fourth statistic everywhere
 * (kernels/packed_rasterize.py:753-766).
 * ------------------------------------------------------------------------ */
typedef struct {
    int capacity;
    int width, height;
    int tile_w, tile_h;
    int cluster_size;
    int64_t max_pairs;
    int flags;             /* GSB_RASTER_BWD_PREPARED: gsb_raster_bwd_prepare already ran;
                              GSB_RASTER_BWD_SYMMETRIC_CONIC: the packed
                              backward's symmetric_conic convention
                              (kernels/packed_rasterizer.py:98-177): gconic[1]
                              takes both off-diagonal contributions and
                              gconic[2] is left as zeroed */
} gsb_raster_bwd_params;

#define GSB_RASTER_BWD_PREPARED 1
#define GSB_RASTER_BWD_SYMMETRIC_CONIC 2

GSB_API int gsb_raster_bwd(gsb_stream_t stream, const gsb_raster_bwd_params* p, void* workspace,
                   size_t workspace_bytes, const float* splats, const float* depth,
                   const int32_t* gaussian_ids, const int32_t* tile_offsets,
                   const float* background, const float* final_t, const int32_t* last,
                   const int32_t* backward_work, const uint32_t* contribution_bits,
                   const float* drgb, const float* ddepth, const float* dalpha,
                   const int32_t* cluster_ids, const int32_t* cluster_count, float* gmean,
                   float* gconic, float* gdepth, float* gcolor, float* galpha,
                   float* fragment_stats);

/* The preparation stages of gsb_raster_bwd on their own: zero the cotangents
 * (the listed clusters' slots, or the whole pool; fragment_stats and galpha
 * over the whole pool when fragment_stats is non-NULL) and order the tiles by
 * backward_work into the workspace.  They need only the forward's
 * backward_work, so a caller can run them on a second stream during the
 * loss, then call gsb_raster_bwd with the same workspace and
 * GSB_RASTER_BWD_PREPARED in p->flags.
 * Splitting of the backward launch inside kernels/sorted_rasterizer.py:165-236. */
GSB_API int gsb_raster_bwd_prepare(gsb_stream_t stream, const gsb_raster_bwd_params* p,
                           void* workspace, size_t workspace_bytes,
                           const int32_t* backward_work, const int32_t* cluster_ids,
                           const int32_t* cluster_count, float* gmean, float* gconic,
                           float* gdepth, float* gcolor, float* galpha, float* fragment_stats);

/* ------------------------------------------------------------------------
 * Fused L1(0.8) + SSIM(0.2) loss and image gradient.
 * Replaces kernels/fused_loss.py:333-352 (fused_loss_and_grad /
 * _fused_loss_and_grad_with_scale -> cutlass_call(_launch)).
 * image[H*W*3] f32; target[H*W*3] u8 (target_u8=1) or f32 in [0,1].
 * clip_input=1 evaluates the loss on clip(image,0,1) and multiplies the
 * gradient by the clip's derivative (1 inside, 1/2 at 0 or 1, 0 outside),
 * as kernels/sorted_rasterizer.py:206-209 does with jax.vjp(jnp.clip).
 * Outputs: loss[1] (mean over 3HW), grad[H*W*3], scale[1] = max(max|grad|,
 * 1e-12) (may be NULL).
 * ------------------------------------------------------------------------ */
typedef struct {
    int width, height;
    int target_u8;
    int clip_input;
} gsb_loss_params;

GSB_API size_t gsb_loss_workspace_size(const gsb_loss_params* p);
GSB_API int gsb_loss(gsb_stream_t stream, const gsb_loss_params* p, void* workspace,
             size_t workspace_bytes, const float* image, const void* target, float* loss,
             float* grad, float* scale);

/* ------------------------------------------------------------------------
 * Allocation-free fused loss.  No counterpart in the reference (jax-gs lets
 * XLA allocate every temporary of its loss kernel).
 * For callers that cannot allocate device memory when they need the loss: a
 * JAX/XLA host whose allocator holds most of the GPU and gives a custom call
 * only planned buffers, a server with a fixed memory plan, a latency-bound
 * caller that cannot afford cudaMalloc's device synchronisation, or a plugin
 * ABI that passes only inputs and outputs.  Same arguments and results as
 * gsb_loss without the workspace; the per-CTA temporaries live in a fixed
 * 384 KiB device array inside the library, held on every GPU that loads the
 * library's device code until the process exits.  The call allocates nothing.
 *  - Size limit: ceil(W/32) * ceil(H/16) <= GSB_LOSS_NOALLOC_MAX_TILES
 *    (e.g. 4096 x 2048); larger images return GSB_ERR_INVALID and
 *    gsb_last_error() says why.
 *  - The first call on a device (with it current) looks up the array's
 *    address and sets the kernels' shared-memory limit; make it before any
 *    stream capture begins.
 *  - All calls on a device share the array (each call overwrites what it
 *    reads, so no clearing is needed); calls that overlap on the GPU race
 *    and must be ordered by the caller.
 * ------------------------------------------------------------------------ */
#define GSB_LOSS_NOALLOC_MAX_TILES 16384
GSB_API int gsb_loss_noalloc(gsb_stream_t stream, const gsb_loss_params* p, const float* image,
                     const void* target, float* loss, float* grad, float* scale);

/* ------------------------------------------------------------------------
 * View-sharded gradient exchange over NVLink / NVSwitch (NVLS multicast).
 * No single counterpart in the reference: it replaces the NCCL all-reduce of
 * the per-view gradients before the shared Adam update that the view-
 * sharded training step performs with collectives
 * written for symmetric memory (one allocation per GPU, mapped into an NVLS
 * multicast object and into every peer).  One process per GPU; every rank
 * makes the same calls in the same order.
 *  - gsb_exchange_barrier: every rank stores an epoch into slot `rank` of
 *    every peer's flags (peer_flags[q] = rank q's flags, a device array of
 *    world pointers) and waits for all world slots of its own flags to reach
 *    it.  epoch[1] and flags[world] start at zero on every rank.  A wait that
 *    gives up (a peer missing for seconds) sets error[0] = 1 and returns.
 *  - gsb_nvls_allreduce: sums count floats (a multiple of 4, 16-byte
 *    aligned) over all ranks' copies through the multicast address: rank r
 *    reduces and stores shard r.  Put a barrier before (inputs written) and
 *    after (sum complete everywhere).
 *  - gsb_p2p_allreduce: gsb_nvls_allreduce with plain peer loads and
 *    stores instead of the multicast object: buffers[q] is rank q's copy
 *    (host array of world <= 8 device pointers, each 16-byte aligned); rank
 *    r reads shard r of every copy, adds them in rank order and stores the
 *    sum into shard r of every copy.  Same barriers before and after.
 *  - gsb_multicast_nonzero: the all-gather of the colour cotangents.  Each
 *    rank's pullback (gsb_project_bwd, colour-only, pool order) writes its
 *    row of a symmetric row table locally, row = [centre x, y, z, 0 |
 *    colours C*3 | pad]; this call stores the row's non-zero 16-byte chunks
 *    (count floats, a multiple of 4, both addresses 16-byte aligned)
 *    through the multicast address of that row into every GPU's copy.  The
 *    receiving copies must hold zeros where nothing is sent: clear them
 *    after each use.  A gsb_exchange_barrier afterwards publishes the rows.
 *  - error (the barrier's error word, may be NULL): the three data calls
 *    return at once on the device when it is set, leaving every buffer as
 *    it is, since after a barrier that gave up their inputs are not known
 *    to be complete.  The sums are then stale: check the word (on the host,
 *    between steps) before an optimizer consumes them.
 * ------------------------------------------------------------------------ */
typedef struct {
    int world;
    int rank;
} gsb_exchange_params;

GSB_API int gsb_exchange_barrier(gsb_stream_t stream, const gsb_exchange_params* p,
                         uint32_t* const* peer_flags, const uint32_t* flags, uint32_t* epoch,
                         int32_t* error);
GSB_API int gsb_nvls_allreduce(gsb_stream_t stream, const gsb_exchange_params* p, float* multicast,
                       int64_t count, const int32_t* error);
GSB_API int gsb_multicast_nonzero(gsb_stream_t stream, const float* src, float* multicast,
                          int64_t count, const int32_t* error);
GSB_API int gsb_p2p_allreduce(gsb_stream_t stream, const gsb_exchange_params* p,
                      float* const* buffers, int64_t count, const int32_t* error);

/* The colour all-gather in compact form (no reference counterpart; part of
 * the view-sharded exchange).  gsb_colour_push_compact appends an entry
 * (id as int bits, r, g, b) for every Gaussian whose colour cotangent in
 * row[4 + 3g .. 4 + 3g + 2] is non-zero to this rank's compact row through
 * its multicast address, then the header (row[0..2], the camera centre, and
 * the entry count as int bits); a compact row holds 4 + 4 * capacity floats
 * and the entry order is unspecified.  Two tables alternate: the device
 * word *slot picks multicast0/table0 (even) or multicast1/table1 (odd).
 * counter: one device int32 of scratch, set to zero by the call.
 * gsb_colour_expand scatters every view's entries of the slot's gathered
 * compact table [world][4 + 4 * capacity] into dense rows
 * [world][dense_row] (centre, pad, capacity * 3 colours), which the caller
 * clears beforehand, then advances *slot.  Both return at once when the
 * exchange's error word is set. */
GSB_API int gsb_colour_push_compact(gsb_stream_t stream, const float* row, int64_t capacity,
                            float* multicast0, float* multicast1, const int32_t* slot,
                            int32_t* counter, const int32_t* error);
GSB_API int gsb_colour_expand(gsb_stream_t stream, const float* table0, const float* table1,
                      int32_t* slot, int world, int64_t capacity, float* dense,
                      int64_t dense_row, const int32_t* error);

#ifdef __cplusplus
}
#endif

#endif /* GSB200_H */
