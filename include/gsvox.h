/*
 * gsvox.h - C ABI of the B200-native Gaussian voxelization path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as `void*`; NULL = legacy default stream) and returns a status
 * code (GSV_OK on success). Nothing here allocates device memory: callers
 * pass output buffers and, where a function needs scratch space, a
 * workspace whose size they query first with the matching
 * `*_workspace_bytes` function. All launches are asynchronous on `stream`.
 *
 * Conventions shared with the reference (PaPieta/gs-voxelizer):
 *   - Volume sizes are given as (z, y, x) = (depth, height, width), the
 *     order of the reference's Python tuples.
 *   - Tiles are 8x8x8 voxels; tile id = tz*Ty*Tx + ty*Tx + tx with
 *     Tx = ceil(X/8), Ty = ceil(Y/8), Tz = ceil(Z/8).
 *   - pos3d_radii is [N,4] float (voxel-space x, y, z, radius), conics is
 *     [N,6] float (inverse covariance a,b,c,d,e,f = Q00,Q01,Q02,Q11,Q12,Q22),
 *     tile_min / tile_max are [N,3] int32 (x,y,z), intensities [N,C] float,
 *     the volume is [Z,Y,X,C] float.
 *   - 1 <= C <= 4 channels.
 *
 * Each function names the reference interface it replaces (file:line in the
 * reference project).
 */
#ifndef GSVOX_H
#define GSVOX_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GSV_API __attribute__((visibility("default")))
#else
#define GSV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum gsv_status {
    GSV_OK = 0,
    GSV_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad dims   */
    GSV_ERR_UNSUPPORTED_CHANNELS = 2, /* C outside 1..4                      */
    GSV_ERR_WORKSPACE_TOO_SMALL = 3,
    GSV_ERR_SIZE_OVERFLOW = 4,    /* sizes beyond the 32-bit index formats    */
    GSV_ERR_CUDA = 5              /* a CUDA launch or runtime call failed     */
};

/* Human-readable text of the last error raised on the calling host thread. */
GSV_API const char *gsv_last_error(void);

/* Library version, e.g. "0.1.0". */
GSV_API const char *gsv_version(void);

/* Number of CUDA kernels this library has launched in this process (all
 * devices, all threads). Instrumentation for benchmarks; no reference
 * counterpart. */
GSV_API uint64_t gsv_launch_count(void);

/* Install CUDA events (cudaEvent_t, passed as void*) that later calls from any
 * host thread of the process record immediately before and after the main
 * voxelization
 * kernel of kind `which` (0 = forward, 1 = per-Gaussian backward,
 * 2 = per-voxel backward), on the call's stream; NULL, NULL removes them.
 * Instrumentation for benchmarks; no reference counterpart. */
GSV_API int gsv_profile_kernel(int32_t which, void *start_event,
                               void *stop_event);

/*
 * Projection forward: quaternion/scale -> voxel-space inverse covariance
 * (conic), cull radius, 3D tile bounding box and tile count per Gaussian.
 * Writes every output element (culled Gaussians get zeros).
 * Replaces optim_to_render_forward_torch, gs_voxelizer/cuda/bindings.cu:44
 * (kernel gs_voxelizer/cuda/optim_to_render.cu:48).
 *   vol_size_voxel[3] = (Z, Y, X); vol_size_world[3], vol_center_pos[3] in
 *   (z, y, x) order.
 */
GSV_API int gsv_optim_to_render_forward(
    int32_t num_gaussians, int32_t channels,
    const float *pos3d, const float *scale3d, const float *quat,
    const float *intensities,
    const int32_t vol_size_voxel[3], const float vol_size_world[3],
    const float vol_center_pos[3],
    float *pos3d_radii_out, float *conics_out,
    int32_t *tile_min_out, int32_t *tile_max_out, int32_t *num_tiles_hit_out,
    void *stream);

/*
 * Projection backward: conic / position gradients -> gradients of pos3d
 * [N,3], scale3d [N,3] and quat [N,4]. Writes every output element.
 * Replaces optim_to_render_backward_torch, gs_voxelizer/cuda/bindings.cu:201
 * (kernel gs_voxelizer/cuda/optim_to_render.cu:246).
 */
GSV_API int gsv_optim_to_render_backward(
    int32_t num_gaussians,
    const float *pos3d, const float *scale3d, const float *quat,
    const int32_t vol_size_voxel[3], const float vol_size_world[3],
    const float vol_center_pos[3],
    const float *pos3d_radii_grad_in, const float *conics_grad_in,
    const float *pos3d_radii_out,
    float *pos3d_grad_out, float *scale3d_grad_out, float *quat_grad_out,
    void *stream);

/*
 * Binning: expand each Gaussian's tile box into (tile, gaussian) pairs and
 * order them by tile id, then by gaussian id (the order of the reference's
 * stable radix sort), and write the per-tile [start, end) ranges. Tiles that
 * no Gaussian touches get (0, 0), as in the reference.
 * gaussian_ids_sorted_out holds num_intersects int32, tile_bins_out holds
 * 2*T int32. cum_tiles_hit (inclusive prefix sum of num_tiles_hit) is
 * accepted for interface parity; the result depends only on the tile boxes.
 * Replaces bin_and_sort_gaussians_torch, gs_voxelizer/cuda/bindings.cu:261
 * (kernels gs_voxelizer/cuda/bin_and_sort_gaussians.cu:11,40 and the CUB sort
 * at bindings.cu:316-345).
 */
GSV_API size_t gsv_bin_and_sort_workspace_bytes(
    int32_t num_gaussians, int64_t num_intersects,
    const int32_t vol_size_voxel[3]);

GSV_API int gsv_bin_and_sort_gaussians(
    int32_t num_gaussians, int64_t num_intersects,
    const int32_t *tile_min, const int32_t *tile_max,
    const int32_t *cum_tiles_hit,
    const int32_t vol_size_voxel[3],
    int32_t *gaussian_ids_sorted_out, int32_t *tile_bins_out,
    void *workspace, size_t workspace_bytes, void *stream);

/*
 * Slab variant of the binning used by z-slab sharding: only tiles with
 * tile_z_begin <= tz < tile_z_end are binned, and tile ids / tile_bins are
 * local to the slab (tile id minus tile_z_begin*Ty*Tx). The result equals the
 * full-volume binning restricted to the slab. num_intersects must be the
 * number of (tile, gaussian) pairs that fall inside the slab.
 * No single reference counterpart: extends bindings.cu:261 for sharding.
 */
GSV_API size_t gsv_bin_and_sort_slab_workspace_bytes(
    int32_t num_gaussians, int64_t num_intersects,
    const int32_t vol_size_voxel[3], int32_t tile_z_begin, int32_t tile_z_end);

GSV_API int gsv_bin_and_sort_gaussians_slab(
    int32_t num_gaussians, int64_t num_intersects,
    const int32_t *tile_min, const int32_t *tile_max,
    const int32_t vol_size_voxel[3], int32_t tile_z_begin, int32_t tile_z_end,
    int32_t *gaussian_ids_sorted_out, int32_t *tile_bins_out,
    void *workspace, size_t workspace_bytes, void *stream);

/*
 * Count the (tile, gaussian) pairs of a z-slab of tiles into *count_out
 * (one int64 in device memory). No reference counterpart (sharding only).
 */
GSV_API int gsv_count_slab_intersects(
    int32_t num_gaussians, const int32_t *tile_min, const int32_t *tile_max,
    int32_t tile_z_begin, int32_t tile_z_end, int64_t *count_out,
    void *stream);

/*
 * Forward voxelization: vol[z,y,x,c] = sum over the tile's Gaussians of
 * I_c * exp(-1/2 d^T Q d), with the reference's two culls (sigma > 0 or not
 * finite; alpha * mean(I) < 1e-6). out_vol holds Z*Y*X*C floats and is fully
 * written.
 * Replaces voxelize_forward_torch, gs_voxelizer/cuda/bindings.cu:362
 * (kernel gs_voxelizer/cuda/voxelize.cu:39).
 */
GSV_API size_t gsv_voxelize_workspace_bytes(
    int32_t num_gaussians, int32_t channels, int64_t num_intersects,
    const int32_t vol_size_voxel[3]);

GSV_API int gsv_voxelize_forward(
    const int32_t vol_size_voxel[3], int32_t channels,
    int32_t num_gaussians, int64_t num_intersects,
    const int32_t *gaussian_ids_sorted, const int32_t *tile_bins,
    const float *pos3d_radii, const float *conics, const float *intensities,
    float *out_vol,
    void *workspace, size_t workspace_bytes, void *stream);

/*
 * Backward voxelization, per-Gaussian work distribution (the reference's
 * default): reads dL/dvol [Z,Y,X,C], writes pos3d_grad [N,4] (w = 0),
 * conics_grad [N,6], intensities_grad [N,C]. Outputs are fully written.
 * Replaces voxelize_backward_per_gaussian_torch, bindings.cu:589
 * (kernel gs_voxelizer/cuda/voxelize.cu:368 and helpers :577-610).
 */
GSV_API int gsv_voxelize_backward_per_gaussian(
    const int32_t vol_size_voxel[3], int32_t channels,
    int32_t num_gaussians, int64_t num_intersects,
    const int32_t *gaussian_ids_sorted, const int32_t *tile_bins,
    const float *pos3d_radii, const float *conics, const float *intensities,
    const float *vol_grad_in,
    float *pos3d_grad_out, float *conics_grad_out, float *intensities_grad_out,
    void *workspace, size_t workspace_bytes, void *stream);

/*
 * Backward voxelization, per-voxel work distribution (reference's
 * use_per_gaussian_backward=False). Same outputs as above.
 * Replaces voxelize_backward_torch, bindings.cu:462
 * (kernel gs_voxelizer/cuda/voxelize.cu:170).
 */
GSV_API int gsv_voxelize_backward(
    const int32_t vol_size_voxel[3], int32_t channels,
    int32_t num_gaussians, int64_t num_intersects,
    const int32_t *gaussian_ids_sorted, const int32_t *tile_bins,
    const float *pos3d_radii, const float *conics, const float *intensities,
    const float *vol_grad_in,
    float *pos3d_grad_out, float *conics_grad_out, float *intensities_grad_out,
    void *workspace, size_t workspace_bytes, void *stream);

/*
 * Slab variants of the voxelization used by z-slab sharding: the volume
 * buffers cover only voxel z in [8*tile_z_begin, min(Z, 8*tile_z_end)),
 * tile_bins comes from gsv_bin_and_sort_gaussians_slab, positions stay in
 * full-volume voxel coordinates. No single reference counterpart.
 */
GSV_API size_t gsv_voxelize_slab_workspace_bytes(
    int32_t num_gaussians, int32_t channels, int64_t num_intersects,
    const int32_t vol_size_voxel[3], int32_t tile_z_begin, int32_t tile_z_end);

GSV_API int gsv_voxelize_forward_slab(
    const int32_t vol_size_voxel[3], int32_t tile_z_begin, int32_t tile_z_end,
    int32_t channels, int32_t num_gaussians, int64_t num_intersects,
    const int32_t *gaussian_ids_sorted, const int32_t *tile_bins,
    const float *pos3d_radii, const float *conics, const float *intensities,
    float *out_vol,
    void *workspace, size_t workspace_bytes, void *stream);

GSV_API int gsv_voxelize_backward_per_gaussian_slab(
    const int32_t vol_size_voxel[3], int32_t tile_z_begin, int32_t tile_z_end,
    int32_t channels, int32_t num_gaussians, int64_t num_intersects,
    const int32_t *gaussian_ids_sorted, const int32_t *tile_bins,
    const float *pos3d_radii, const float *conics, const float *intensities,
    const float *vol_grad_in,
    float *pos3d_grad_out, float *conics_grad_out, float *intensities_grad_out,
    void *workspace, size_t workspace_bytes, void *stream);

/*
 * L1 loss, standalone: loss_out[0] = sum |vol - target| / denom (one float
 * in device memory), and its gradient grad_vol = sign(vol - target) *
 * grad_loss[0] / denom (grad_loss: one float in device memory, the incoming
 * gradient of the loss). Deterministic reduction. No reference counterpart:
 * the reference leaves losses to PyTorch in its callers.
 */
GSV_API size_t gsv_l1_loss_workspace_bytes(int64_t n);

GSV_API int gsv_l1_loss_forward(int64_t n, const float *vol,
                                const float *target, float denom,
                                float *loss_out, void *workspace,
                                size_t workspace_bytes, void *stream);

GSV_API int gsv_l1_loss_backward(int64_t n, const float *vol,
                                 const float *target, const float *grad_loss,
                                 float denom, float *grad_vol, void *stream);

/*
 * One training step's voxelization with the L1 loss fused in (z-slab form;
 * the full volume is tile_z_begin = 0, tile_z_end = ceil(Z/8)), as two calls
 * sharing one workspace of gsv_voxelize_l1_workspace_bytes:
 *  - forward: bins the slab's (tile, gaussian) pairs from the tile boxes into
 *    gaussian_ids_sorted_out / tile_bins_out (as
 *    gsv_bin_and_sort_gaussians_slab), writes the volume and
 *    loss_out[0] = sum |vol - target| / denom, and leaves the per-Gaussian
 *    records and the backward's work plan in the workspace;
 *  - backward: with the same ids, tile_bins and unchanged workspace, forms
 *    dL/dvol = sign(out_vol - target) * grad_loss[0] / denom while staging
 *    each tile (no gradient volume is read or written) and writes the
 *    per-Gaussian gradients like gsv_voxelize_backward_per_gaussian.
 * num_intersects: the slab's pair count (gsv_count_slab_intersects), or any
 * upper bound of it (a capacity), so that a step needs no host read of the
 * count: ids past the true count stay unused. If the true count exceeds
 * num_intersects, the tile ranges are clamped to it (no access outside the
 * buffers) and the results are invalid; the caller re-runs with a larger
 * capacity. pair_count_out (nullable, device int64) receives the slab's true
 * pair count and overflow_out (nullable, device float) 1.0 when it exceeds
 * num_intersects, else 0.0, both computed during the binning. Both calls of
 * a step take the same num_intersects.
 * No reference counterpart (fuses bindings.cu:261, :362 and :589 with the
 * loss the reference's callers compute in PyTorch).
 */
GSV_API size_t gsv_voxelize_l1_workspace_bytes(
    int32_t num_gaussians, int32_t channels, int64_t num_intersects,
    const int32_t vol_size_voxel[3], int32_t tile_z_begin, int32_t tile_z_end);

GSV_API int gsv_voxelize_forward_l1(
    const int32_t vol_size_voxel[3], int32_t tile_z_begin, int32_t tile_z_end,
    int32_t channels, int32_t num_gaussians, int64_t num_intersects,
    const int32_t *tile_min, const int32_t *tile_max,
    const float *pos3d_radii, const float *conics, const float *intensities,
    const float *target, float denom, int32_t *gaussian_ids_sorted_out,
    int32_t *tile_bins_out, float *out_vol, float *loss_out,
    int64_t *pair_count_out, float *overflow_out,
    void *workspace, size_t workspace_bytes, void *stream);

GSV_API int gsv_voxelize_backward_per_gaussian_l1(
    const int32_t vol_size_voxel[3], int32_t tile_z_begin, int32_t tile_z_end,
    int32_t channels, int32_t num_gaussians, int64_t num_intersects,
    const int32_t *gaussian_ids_sorted, const int32_t *tile_bins,
    const float *pos3d_radii, const float *conics, const float *intensities,
    const float *out_vol, const float *target, const float *grad_loss,
    float denom, float *pos3d_grad_out, float *conics_grad_out,
    float *intensities_grad_out, void *workspace, size_t workspace_bytes,
    void *stream);

/*
 * 3D SSIM (Wang et al. 2004) of planar volumes [channels][D][H][W]: 11^3
 * separable Gaussian window (sigma 1.5), zero padding, constants c1, c2
 * (the usual 0.01^2 and 0.03^2). Forward: ssim_out[0] (device float) = the
 * mean of the SSIM map over all voxels and channels; the workspace (size
 * from gsv_ssim3d_workspace_bytes, dhw = {D, H, W}) keeps three gradient
 * maps for the backward. Backward (same inputs and workspace): grad_img1 =
 * grad_out[0] * d ssim / d img1 (img2 is treated as constant).
 * Replaces the external fused_ssim3d that the reference's tests and speed
 * benchmarks call on the voxelized volume (test/test_gs_voxelizer.py:62,
 * test/compare_speed.py:174); not part of the reference's sources.
 */
GSV_API size_t gsv_ssim3d_workspace_bytes(int32_t channels, const int32_t dhw[3]);
GSV_API int gsv_ssim3d_forward(int32_t channels, const int32_t dhw[3],
                               const float *img1, const float *img2, float c1,
                               float c2, float *ssim_out, void *workspace,
                               size_t workspace_bytes, void *stream);
GSV_API int gsv_ssim3d_backward(int32_t channels, const int32_t dhw[3],
                                const float *img1, const float *img2,
                                const float *grad_out, const void *workspace,
                                size_t workspace_bytes, float *grad_img1,
                                void *stream);

/*
 * 3D total variation of planar volumes [channels][D][H][W] with forward
 * differences d_a = x(v + e_a) - x(v) (0 across the far boundary):
 * isotropic != 0: mean sqrt(dx^2 + dy^2 + dz^2 + eps) (eps > 0), else
 * mean (|dx| + |dy| + |dz|). value_out (nullable): the value; grad_vol
 * (nullable, needs grad_out): grad_out[0] * dTV/dvol. Replaces the external
 * fused-3D-tv loss named beside the reference (README.md:10); not part of
 * the reference's sources.
 */
GSV_API size_t gsv_tv3d_workspace_bytes(int32_t channels, const int32_t dhw[3]);
GSV_API int gsv_tv3d(int32_t channels, const int32_t dhw[3], const float *vol,
                     int32_t isotropic, float eps, float *value_out,
                     const float *grad_out, float *grad_vol, void *workspace,
                     size_t workspace_bytes, void *stream);

/*
 * Backward engine of the fused-L1 step (gsv_voxelize_forward_l1 +
 * gsv_voxelize_backward_per_gaussian_l1) for one channel: enable != 0
 * accumulates the per-pair sums on the tensor cores (tcgen05, tensor
 * memory), 0 (the default) selects the CUDA-core kernel, which also serves
 * 2-4 channels and is the faster of the two on B200 at BASELINE
 * configuration 2. With the tensor-core engine the forward also writes its
 * inputs (a per-tile sign plane and the tile of every pair) into the
 * workspace, which gsv_voxelize_l1_workspace_bytes then sizes larger.
 * Process-wide; returns the previous setting. Change it only between steps
 * and query the workspace size after it: both calls of a step and the size
 * of their workspace must see the same setting. No reference counterpart.
 */
GSV_API int gsv_set_tensor_core_backward(int32_t enable);

/*
 * Device error flags of this library's kernels on the current device, as
 * bits: 1 after a tensor-core backward launch gave up waiting on one of its
 * internal barriers, 2 after a gsv_peer_barrier gave up waiting for a peer
 * (results of those launches are invalid); 0 if none. clear != 0 resets
 * them. Synchronises with the device. No reference counterpart.
 */
GSV_API int gsv_device_error(int32_t *flag_out, int32_t clear);

/*
 * Forward voxelization that allocates nothing, for callers that cannot
 * provide a workspace: code whose device memory belongs to another allocator
 * (a framework that reserves the GPU's memory up front) or host programs that
 * receive only ready-made input/output buffers through a foreign-function
 * interface. Same inputs, output and results as gsv_voxelize_forward; the
 * per-Gaussian scratch lives in a fixed 16 MiB array inside the library's
 * device image (held by every GPU that loads the library until exit), so
 * num_gaussians is limited to 349525 (1-2 channels) or 262144 (3-4
 * channels); larger inputs return GSV_ERR_WORKSPACE_TOO_SMALL. All calls
 * share that array: calls that overlap on the GPU race, so serialise them.
 * The first call on each device resolves the array's address (make it before
 * any stream capture). No counterpart in the reference.
 */
GSV_API int gsv_voxelize_forward_noalloc(
    const int32_t vol_size_voxel[3], int32_t channels,
    int32_t num_gaussians, int64_t num_intersects,
    const int32_t *gaussian_ids_sorted, const int32_t *tile_bins,
    const float *pos3d_radii, const float *conics, const float *intensities,
    float *out_vol, void *stream);

/*
 * Halo exchange for owner-sharded z-slabs (one process per GPU). No
 * reference counterpart: the reference is single-GPU. Every rank owns a
 * subset of the Gaussians and projects only those; an owned Gaussian whose
 * tile box reaches another rank's slab is sent there as a render record of
 * GSV_HALO_RECORD_FLOATS floats (pos3d_radii 4, conic 6, intensities 4,
 * tile_min/tile_max 6 as int bits), and the gradients of those records
 * (GSV_HALO_GRAD_FLOATS floats: pos3d_radii 4, conic 6, intensities 4, pad)
 * come back to the owner. A buffer holds one segment per peer rank: a
 * header record, then seg_slots[peer] record slots, starting at record
 * seg_off[peer] (the rank's own entry is ignored). The caller moves the
 * buffers between ranks (an all-to-all); slab_tz is [world][2] tile-z ranges
 * [begin, end) of every rank's slab; all per-peer arrays are host memory,
 * world <= 64.
 *
 * gsv_halo_pack: records of the n owned Gaussians into `send` (slots in
 * owner-index order, so deterministic; Gaussians past a segment's slots are
 * dropped and flagged in its header) and slot_map[n][world] = slot or -1;
 * counts_out (nullable, device int64[world]) = the unclamped number of
 * Gaussians for every peer (0 for the rank itself), for sizing segments.
 * gsv_halo_unpack: the received records into the local arrays at
 * n_own + (slots of the lower-ranked peers) + slot, unused slots as
 * Gaussians with an empty tile box; flags[1] = 1 if a sender overflowed.
 * gsv_halo_pack_grads: gradients of those local entries back into the
 * owners' segments (same slots), header = (loss[0], max(flags[0..1])).
 * gsv_halo_accumulate: the owner adds the received gradients to its n owned
 * entries in rank order; out[0] = sum of all ranks' losses in rank order,
 * out[1] = max of all ranks' flags.
 */
#define GSV_HALO_RECORD_FLOATS 20
#define GSV_HALO_GRAD_FLOATS 16

GSV_API size_t gsv_halo_workspace_bytes(int32_t num_gaussians, int32_t world);

GSV_API int gsv_halo_pack(int32_t num_gaussians, int32_t channels,
                          const float *pos3d_radii, const float *conics,
                          const float *intensities, const int32_t *tile_min,
                          const int32_t *tile_max, int32_t world, int32_t rank,
                          const int32_t *slab_tz, const int64_t *seg_off,
                          const int32_t *seg_slots, float *send,
                          int32_t *slot_map, int64_t *counts_out,
                          void *workspace, size_t workspace_bytes,
                          void *stream);

GSV_API int gsv_halo_unpack(int32_t n_own, int32_t channels, int32_t world,
                            int32_t rank, const int64_t *seg_off,
                            const int32_t *seg_slots, const float *recv,
                            float *pos3d_radii, float *conics,
                            float *intensities, int32_t *tile_min,
                            int32_t *tile_max, float *flags, void *stream);

GSV_API int gsv_halo_pack_grads(int32_t n_own, int32_t channels, int32_t world,
                                int32_t rank, const int64_t *seg_off,
                                const int32_t *seg_slots,
                                const float *pos3d_radii_grad,
                                const float *conics_grad,
                                const float *intensities_grad,
                                const float *loss, const float *flags,
                                float *send, void *stream);

/*
 * Device barrier across `world` ranks (one GPU each) on `stream`, for the
 * direct-write halo exchange: sig_ptrs[d] is the device address of rank d's
 * signal array of `world` int32 (zero-initialised memory that every rank
 * can write, e.g. a symmetric-memory buffer over NVLink), `epoch` a device
 * int32 of this rank (initially 0) that the call advances. After the call,
 * on every rank's stream, all writes of the kernels before every rank's call
 * are visible. Graph-capturable (the epochs only grow); every rank must make
 * the same sequence of calls. Waits are bounded (about two seconds per
 * peer): on timeout the kernel sets bit 2 of gsv_device_error and returns.
 * No reference counterpart.
 */
GSV_API int gsv_peer_barrier(int32_t world, int32_t rank, const int64_t *sig_ptrs,
                             int32_t *epoch, void *stream);

/*
 * gsv_halo_pack_peers / gsv_halo_pack_grads_peers: as gsv_halo_pack /
 * gsv_halo_pack_grads, but each segment is written straight into the
 * destination rank's receive buffer instead of a local send buffer:
 * seg_dst[d] (d != rank) is the device address, 16-byte aligned, where this
 * rank's segment starts in rank d's receive buffer (memory of another GPU
 * reached over NVLink, e.g. a peer's symmetric-memory buffer; plain stores,
 * no multicast). The caller makes every rank's writes visible to their
 * receivers (a device barrier across the ranks) before the unpack /
 * accumulate. seg_off and seg_slots describe the segments as for the other
 * calls. No reference counterpart.
 */
GSV_API int gsv_halo_pack_peers(int32_t num_gaussians, int32_t channels,
                                const float *pos3d_radii, const float *conics,
                                const float *intensities, const int32_t *tile_min,
                                const int32_t *tile_max, int32_t world,
                                int32_t rank, const int32_t *slab_tz,
                                const int64_t *seg_off, const int32_t *seg_slots,
                                const int64_t *seg_dst, int32_t *slot_map,
                                int64_t *counts_out, void *workspace,
                                size_t workspace_bytes, void *stream);

GSV_API int gsv_halo_pack_grads_peers(int32_t n_own, int32_t channels,
                                      int32_t world, int32_t rank,
                                      const int64_t *seg_off,
                                      const int32_t *seg_slots,
                                      const float *pos3d_radii_grad,
                                      const float *conics_grad,
                                      const float *intensities_grad,
                                      const float *loss, const float *flags,
                                      const int64_t *seg_dst, void *stream);

GSV_API int gsv_halo_accumulate(int32_t num_gaussians, int32_t channels,
                                int32_t world, int32_t rank,
                                const int64_t *seg_off, const int32_t *slot_map,
                                const float *recv, float *pos3d_radii_grad,
                                float *conics_grad, float *intensities_grad,
                                const float *loss, const float *flags,
                                float *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GSVOX_H */
