/*
 * r2s.h - C ABI of libr2s.so, the sm_100a implementation of the r2splat
 * Gaussian backend (cone-beam projection rendering, voxelization and their
 * first-order VJPs).
 *
 * The reference binds its operators through pybind11
 * (r2splat/cuda/csrc/ext.cpp:7-27, declarations r2splat/cuda/include/Ops.h:9-79).
 * This header exposes the same 18 operators as plain C functions: device
 * pointers, element counts, scalar parameters and a CUDA stream; no torch types.
 * The Python package r2splat (r2splat/cuda/_wrapper.py) binds them through
 * ctypes and keeps the reference's Python signatures.  Fused entry points used
 * by the r2splat.ops fast path follow the 18 operators.
 *
 * Conventions
 *   - Every function returns R2S_OK (0) or an error code; r2s_last_error()
 *     returns the message of the last failure on the calling thread.
 *   - All pointers are device pointers unless stated otherwise; all work is
 *     enqueued on `stream` and nothing synchronizes the host.
 *   - `dtype` selects float32 (R2S_F32) or float64 (R2S_F64) for every
 *     floating-point buffer of the call; integer buffers are int32 unless
 *     stated (isect ids are int64, as in the reference).
 *   - Outputs are written in full (callers need not zero them) unless the
 *     comment says "accumulated".
 *   - The library never allocates device memory: scratch space ("workspace")
 *     is passed in by the caller and sized by the matching *_workspace_bytes().
 */
#ifndef R2S_H
#define R2S_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define R2S_API __attribute__((visibility("default")))
#else
#define R2S_API
#endif

typedef struct CUstream_st* r2s_stream_t; /* == cudaStream_t */

enum { R2S_F32 = 0, R2S_F64 = 1 };
enum {
    R2S_OK = 0,
    R2S_ERR_ARG = 1,         /* invalid argument (maps to RuntimeError, like TORCH_CHECK) */
    R2S_ERR_CUDA = 2,        /* CUDA launch/runtime error */
    R2S_ERR_CAPACITY = 3,    /* an index space exceeds int32 (reference limit) */
    R2S_ERR_UNSUPPORTED = 4  /* shape outside what this build supports */
};

/* ------------------------------------------------------------------------
 * Training-step rows (after the rasterizer backward)
 * ---------------------------------------------------------------------- */

/* One Adam parameter group: float32 parameter, gradient and the two moment
 * buffers (same numel), its learning rate and the step count after this
 * update (torch.optim.Adam's state["step"] + 1). */
typedef struct r2s_adam_group {
    float* param;
    const float* grad;
    float* exp_avg;
    float* exp_avg_sq;
    int64_t numel;
    double lr;
    int64_t step;
} r2s_adam_group;

/* Adam update of up to 8 parameter groups in one launch, with
 * torch.optim.Adam's arithmetic (amsgrad off, no weight decay).  Replaces the
 * per-group optimizer.step() of the reference training loop
 * (src/trainers/binary_tree.py:204-206) over the optimizers built by
 * GaussianModel.build_optimizers (src/models/gaussian_model.py:514-530). */
R2S_API int r2s_adam_step_f32(const r2s_adam_group* groups, int n_groups, double beta1,
                              double beta2, double eps, r2s_stream_t stream);

/* Children of a binary-tree split (replaces the tensor arithmetic of split(),
 * src/strategies/binary_tree.py:92-149, for scalar sigmoid scale bounds).
 * For each of the S Gaussians whose indices are in sel [S] (int64): the
 * longest activated-scale axis k, offset R[:, k] s_k of its normalized
 * quaternion's rotation; child_means [2S,3] = mean + offset (rows 0..S-1) and
 * mean - offset (rows S..2S-1); child_scales [2S,3] = the raw scales of the
 * activated scales with s_k / 1.6 (inverse bounded sigmoid with scale_eps);
 * child_quats [2S,4] = the raw quaternion; child_opacities [2S] = the raw
 * opacity, or with revised_opacity != 0 softplus^-1(1 - sqrt(1 - min(
 * softplus(raw), 0.9999))).  Float operations round one by one, as the
 * reference's elementwise torch ops. */
R2S_API int r2s_split_children_f32(const float* means, const float* raw_scales,
                                   const float* quats, const float* raw_opacities,
                                   const int64_t* sel, int64_t S, double scale_min,
                                   double scale_max, double scale_eps, int revised_opacity,
                                   float* child_means, float* child_scales, float* child_quats,
                                   float* child_opacities, r2s_stream_t stream);

/* Densification statistics of one training step: for every (view, Gaussian)
 * with radius > 0, grad2d[g] += |(gx * scale_x, gy * scale_y)|, count[g] += 1,
 * and, when max_radii is not NULL, max_radii[g] = max(max_radii[g],
 * radius / extent).  grads2d [C,N,2] float32 (means2d.absgrad or .grad),
 * radii [C,N] int32 (the per-axis maximum).  Replaces
 * BinaryTreeStrategy._update_state (src/strategies/binary_tree.py:305-347,
 * non-packed path; scale_x = W/2 * C, scale_y = H/2 * C, extent = max(W, H)). */
R2S_API int r2s_densify_stats_f32(const float* grads2d, const int32_t* radii, int64_t C,
                                  int64_t N, double scale_x, double scale_y, double extent,
                                  float* grad2d, float* count, float* max_radii,
                                  r2s_stream_t stream);

/* Projection losses of the reference's BinaryTreeLossComputer
 * (src/utils/loss.py:125-172) on C single-channel H x W images:
 * sums[0] += sum |x - t|, sums[1] += sum of the SSIM map (11x11 Gaussian window,
 * sigma 1.5, zero padding; src/utils/metric.py:36-56), sums[2] += sum
 * mask |x - te| (edge terms only when edge_mask is not NULL); divide by C*H*W
 * for the means.  When grad is not NULL it receives
 * g_l1 d(mean l1)/dx + g_ssim d(mean ssim)/dx + g_edge d(mean edge)/dx with
 * (g_l1, g_ssim, g_edge) read from the device array weights[3] (so an
 * autograd backward needs no host sync).  window_size must be 11; window_1d
 * is NULL or a host array of the 11 float32 1-D window weights as the caller's
 * SSIM builds them (the 2-D window is their outer product).  sums is a device
 * array of 3 doubles the caller zeroes. */
R2S_API int r2s_projection_loss_f32(const float* renders, const float* targets,
                                    const float* edge_targets, const float* edge_mask,
                                    int64_t C, int64_t H, int64_t W, int window_size,
                                    const float* window_1d, const float* weights, float* grad,
                                    double* sums, r2s_stream_t stream);

/* grad = g_l1 d(mean l1)/dx + g_ssim dssim + g_edge d(mean edge)/dx over n
 * pixels, where dssim is the map r2s_projection_loss_f32 wrote with weights
 * (0, 1, 0) and (g_l1, g_ssim, g_edge) is the device array weights[3]: the
 * backward of a loss whose SSIM gradient was computed in the forward pass. */
R2S_API int r2s_projection_loss_combine_f32(const float* renders, const float* targets,
                                            const float* edge_targets, const float* edge_mask,
                                            const float* dssim, int64_t n, const float* weights,
                                            float* grad, r2s_stream_t stream);

/* Volume total variation of compute_tv_loss (src/utils/loss.py:10-21) on a
 * D0 x D1 x D2 float32 volume: *sum += sum of the absolute forward differences
 * along the three axes (divide by their count for the "mean" reduction); when
 * grad is not NULL it receives g_tv d(mean tv)/dv, g_tv read from the device
 * scalar *weight. */
R2S_API int r2s_tv_loss_f32(const float* volume, int64_t D0, int64_t D1, int64_t D2,
                            const float* weight, float* grad, double* sum, r2s_stream_t stream);

R2S_API const char* r2s_version(void);
/* Copies the last error message of this thread into buf (NUL-terminated,
 * truncated to len-1 bytes); returns the full message length. */
R2S_API size_t r2s_last_error(char* buf, size_t len);

/* Bounds-checked build (libr2s_debug.so: every source built with R2S_DEBUG;
 * no counterpart in the reference, whose contributor guide asks for a CUDA
 * sanitizer run instead, CONTRIBUTING.md:33-35).  In that build the
 * rasterizer, voxelizer and binning kernels test every tile record range
 * (within [0, n_isects)), record id (below C*N or N), pixel/voxel index and
 * binning output slot before using it; a failed test sets a bit in
 * *flags (1 tile range, 2 record id, 4 pixel/voxel, 8 binning slot) and
 * skips the access.  r2s_debug_build() is 1 in that build, 0 in the release
 * library, whose r2s_debug_flags() always reports 0.  r2s_debug_flags reads
 * (and with clear != 0 resets) the flags of all kernels; flags is a host
 * pointer and the call waits for the device. */
R2S_API int r2s_debug_build(void);
R2S_API int r2s_debug_flags(unsigned* flags, int clear);

/* Pipe calibration (measurement support; no counterpart in the reference).
 * `blocks` CTAs of 256 threads each run 8 independent chains of `iters`
 * FFMAs (2 FLOP each) or of `iters` FMUL + ex2.approx steps, and write one
 * float per thread to out [blocks * 256].  Timed with CUDA events they give
 * the FP32 and MUFU ex2 throughput of this GPU at its current clock, the
 * denominators of the rasterizer's roofline fractions. */
R2S_API int r2s_calib_ffma_f32(float* out, int64_t iters, int blocks, r2s_stream_t stream);
R2S_API int r2s_calib_ex2_f32(float* out, int64_t iters, int blocks, r2s_stream_t stream);

/* ------------------------------------------------------------------------
 * Parameter transform: quats [N,4] (w,x,y,z; normalized in-kernel), raw
 * scales [N,3] -> covars [N,6] upper triangle (00,01,02,11,12,22),
 * max_scales [N].  Replaces parameter_transform_fwd_tensor
 * (r2splat/cuda/include/Ops.h:9-10; csrc/ParameterTransform.cpp:33-83).
 */
R2S_API int r2s_parameter_transform_fwd(int dtype, const void* quats, const void* raw_scales,
                                double scale_min, double scale_max, void* covars,
                                void* max_scales, int64_t n, r2s_stream_t stream);
/* VJP of the above.  Replaces parameter_transform_bwd_tensor
 * (Ops.h:11-13; csrc/ParameterTransform.cpp:89-143). */
R2S_API int r2s_parameter_transform_bwd(int dtype, const void* quats, const void* raw_scales,
                                double scale_min, double scale_max, const void* v_covars,
                                void* v_quats, void* v_raw_scales, int64_t n,
                                r2s_stream_t stream);

/* ------------------------------------------------------------------------
 * World -> image cone-beam projection.  means [N,3], covars [N,6],
 * viewmats [C,4,4] row-major, Ks [C,3,3] -> means2d [C,N,2],
 * cov2d [C,N,6] (3x3 ray-space covariance, upper triangle), radii [C,N,2].
 * Replaces world_to_image_projection_fwd_tensor
 * (Ops.h:31-34; csrc/WorldToImageProjection.cpp:37-120).
 */
R2S_API int r2s_world_to_image_projection_fwd(int dtype, const void* means, const void* covars,
                                      const void* viewmats, const void* Ks, int64_t C,
                                      int64_t N, uint32_t width, uint32_t height,
                                      double eps2d, double radius_clip, void* means2d,
                                      void* cov2d, int32_t* radii, r2s_stream_t stream);
/* VJP: v_means2d [C,N,2], v_cov2d [C,N,6] -> v_means [N,3], v_covars [N,6]
 * (summed over views).  Replaces world_to_image_projection_bwd_tensor
 * (Ops.h:35-38; csrc/WorldToImageProjection.cpp:126-206). */
R2S_API int r2s_world_to_image_projection_bwd(int dtype, const void* means, const void* covars,
                                      const void* viewmats, const void* Ks, int64_t C,
                                      int64_t N, uint32_t width, uint32_t height,
                                      const void* v_means2d, const void* v_cov2d,
                                      void* v_means, void* v_covars, r2s_stream_t stream);

/* ------------------------------------------------------------------------
 * Conics and line-integral factor: cov2d [T,6] (T = C*N) -> conics [T,3],
 * mus [T].  Replaces conics_mu_fwd_tensor (Ops.h:25-26; csrc/ConicsMu.cpp:34-80).
 */
R2S_API int r2s_conics_mu_fwd(int dtype, const void* cov2d, double eps, void* conics, void* mus,
                      int64_t total, r2s_stream_t stream);
/* Replaces conics_mu_bwd_tensor (Ops.h:27-29; csrc/ConicsMu.cpp:86-159). */
R2S_API int r2s_conics_mu_bwd(int dtype, const void* cov2d, double eps, const void* conics,
                      const void* mus, const void* v_conics, const void* v_mus,
                      void* v_cov2d, int64_t total, r2s_stream_t stream);

/* ------------------------------------------------------------------------
 * World -> volume mapping.  means [N,3], covars [N,6], ranges [3], centers [3]
 * (device) -> means3d [N,3], conics [N,6], radii [N,3].  max_scales is
 * accepted for interface parity and unused, as in the reference.
 * Replaces world_to_volume_mapping_fwd_tensor
 * (Ops.h:40-44; csrc/WorldToVolumeMapping.cpp:36-112).
 */
R2S_API int r2s_world_to_volume_mapping_fwd(int dtype, const void* means, const void* covars,
                                    const void* max_scales, const void* ranges,
                                    const void* centers, int64_t N, uint32_t dim2,
                                    uint32_t dim1, uint32_t dim0, double eps3d,
                                    double radius_clip, void* means3d, void* conics,
                                    int32_t* radii, r2s_stream_t stream);
/* Replaces world_to_volume_mapping_bwd_tensor
 * (Ops.h:45-48; csrc/WorldToVolumeMapping.cpp:118-192). */
R2S_API int r2s_world_to_volume_mapping_bwd(int dtype, const void* means, const void* covars,
                                    const void* ranges, const void* centers, int64_t N,
                                    uint32_t dim2, uint32_t dim1, uint32_t dim0,
                                    double eps3d, const void* v_means3d,
                                    const void* v_conics, void* v_means, void* v_covars,
                                    r2s_stream_t stream);

/* ------------------------------------------------------------------------
 * Tile binning.  The reference's isect_tiles (Ops.h:15-16;
 * csrc/IsectTiles.cpp:30-170) counts tiles per (view, Gaussian), scans,
 * emits (key = view*n_tiles + tile, value = view*N + g) and radix-sorts the
 * keys stably.  Here the same sorted arrays are produced by a stable
 * counting placement in two calls with one host read of n_isects between
 * them (the reference syncs at the same point, IsectTiles.cpp:100):
 *
 *   r2s_isect_tiles_prepare  -> tiles_per_gauss [C,N], rects [C*N] (8 B
 *                               each), tile_offsets [C,nty,ntx] (int32),
 *                               *n_isects_dev (one int64, device)
 *   r2s_bin_place            -> flatten_ids [n_isects] (int32) and, if
 *                               isect_ids != NULL, isect_ids [n_isects]
 *                               (int64), bit-identical to the reference's
 *                               sorted outputs.
 *
 * radii is [C,N,2] when radii_is_rect, else [C,N].  `workspace` must hold
 * r2s_bin_workspace_bytes(C, N, nty*ntx, 0) bytes.
 */
R2S_API int64_t r2s_bin_workspace_bytes(int64_t n_segments, int64_t n_items,
                                int64_t tiles_per_segment, int layered);
R2S_API int r2s_isect_tiles_prepare(int dtype, const void* means2d, const int32_t* radii,
                            int radii_is_rect, int64_t C, int64_t N, uint32_t tile_size,
                            uint32_t n_tiles_w, uint32_t n_tiles_h,
                            int32_t* tiles_per_gauss, void* rects, void* workspace,
                            int64_t workspace_bytes, int32_t* tile_offsets,
                            int64_t* n_isects_dev, r2s_stream_t stream);
/* 3D counterpart of the above for isect_tiles_3d (Ops.h:20-21;
 * csrc/IsectTiles3D.cpp:31-162): means3d [N,3], radii [N,3] ->
 * tiles_per_gauss [N], rects [N] (16 B each), tile_offsets [nt0,nt1,nt2],
 * *n_isects_dev.  The 3D key space is handled as nt0 layers of nt1*nt2 tiles,
 * so the workspace is r2s_bin_workspace_bytes(nt0, N, nt1*nt2, 1). */
R2S_API int r2s_isect_tiles_3d_prepare(int dtype, const void* means3d, const int32_t* radii,
                               int64_t N, uint32_t tile_size, uint32_t nt2, uint32_t nt1,
                               uint32_t nt0, int32_t* tiles_per_gauss, void* rects,
                               void* workspace, int64_t workspace_bytes,
                               int32_t* tile_offsets, int64_t* n_isects_dev,
                               r2s_stream_t stream);
/* Places the records after a *_prepare call.  layered = 0 for the 2D path
 * (segments = views, items = C*N) and 1 for the 3D path (segments = z
 * layers, items = N Gaussians).  key_base/segment_base let a caller bin a
 * contiguous range of segments (z-slab sharding); pass 0 for the full key
 * space. */
R2S_API int r2s_bin_place(const void* rects, int64_t n_segments, int64_t n_items,
                  int64_t tiles_per_segment, uint32_t tiles_x, int layered,
                  int64_t segment_base, const void* workspace, int64_t workspace_bytes,
                  const int32_t* tile_offsets, int64_t n_isects, int32_t* flatten_ids,
                  int64_t* isect_ids, r2s_stream_t stream);
/* Per-tile start offsets of a sorted key array.  Replaces
 * isect_offset_encode_tensor (Ops.h:17-18; csrc/IsectTiles.cpp:176-215) and
 * isect_offset_encode_3d_tensor (Ops.h:22-23; csrc/IsectTiles3D.cpp:168-204):
 * offsets[k] = first index i with isect_ids[i] >= k, k in [0, n_keys). */
R2S_API int r2s_isect_offset_encode(const int64_t* isect_ids, int64_t n_isects, int64_t n_keys,
                            int32_t* offsets, r2s_stream_t stream);

/* ------------------------------------------------------------------------
 * Additive X-ray rasterization (no alpha compositing):
 * image[c,i,j] = sum over the tile's list of w*mu*exp(-sigma), skipping
 * sigma < 0 and |alpha| < 1e-5.  Inputs are [C,N,...] flattened
 * (means2d 2, conics 3, opacities 1, mus 1), tile_offsets [C,nty,ntx],
 * flatten_ids [n_isects]; output image [C,H,W].  `splat_scratch` (nullable,
 * C*N*32 bytes) lets float32 inputs with 16-pixel tiles take the packed-record
 * kernel; without it a generic kernel runs.  Replaces
 * rasterize_to_pixels_fwd_tensor (Ops.h:50-53; csrc/RasterizeToPixels.cpp:25-115).
 */
R2S_API int r2s_rasterize_to_pixels_fwd(int dtype, const void* means2d, const void* conics,
                                const void* opacities, const void* mus,
                                const int32_t* tile_offsets, const int32_t* flatten_ids,
                                int64_t C, int64_t N, int64_t n_isects, uint32_t width,
                                uint32_t height, uint32_t tile_size, uint32_t n_tiles_w,
                                uint32_t n_tiles_h, void* splat_scratch, void* image,
                                r2s_stream_t stream);
/* VJP w.r.t. means2d, conics, opacities, mus (+ |d means2d| summed per
 * pixel when v_means2d_abs != NULL).  Both reference modes map here:
 * mode 0 = "pixel" (rasterize_to_pixels_bwd_tensor, Ops.h:54-58;
 * RasterizeToPixels.cpp:121-223) and mode 1 = "primitive"
 * (rasterize_to_pixels_bwd_per_gaussian_tensor, Ops.h:59-64;
 * RasterizeToPixels.cpp:225-317).  The modes differ only in the precision
 * of exp for float64 inputs, as in the reference.  `stats` is caller
 * scratch of C*N*8 elements of dtype; `splat_scratch` as for the forward. */
R2S_API int r2s_rasterize_to_pixels_bwd(int dtype, int mode, const void* means2d,
                                const void* conics, const void* opacities, const void* mus,
                                const int32_t* tile_offsets, const int32_t* flatten_ids,
                                const void* v_image, int64_t C, int64_t N, int64_t n_isects,
                                uint32_t width, uint32_t height, uint32_t tile_size,
                                uint32_t n_tiles_w, uint32_t n_tiles_h, void* splat_scratch,
                                void* stats, void* v_means2d_abs, void* v_means2d,
                                void* v_conics, void* v_opacities, void* v_mus,
                                r2s_stream_t stream);

/* Rasterizer backward that allocates nothing and takes no scratch (float32).
 * No counterpart in the reference.  For host programs that cannot hand this
 * library scratch memory -- their device memory belongs to an allocator the
 * plugin may not call (a fixed arena, or a framework that forbids cudaMalloc
 * inside its operators) and their binding passes only inputs and outputs.
 * Same arguments and results as r2s_rasterize_to_pixels_bwd without
 * splat_scratch/stats; the scratch is a static 8 MiB device array of the
 * library, so C*N is limited to 131072 (view, Gaussian) pairs (larger calls
 * return R2S_ERR_UNSUPPORTED).  Works on the current device; its first call
 * on each device looks the array up with cudaGetSymbolAddress and should come
 * before any stream capture (the address is cached per device together with
 * the id of the device's context, so after cudaDeviceReset the next call
 * looks it up again).  Every call reuses the same array: calls that
 * overlap on the GPU (other streams, other threads) race and must be
 * serialized by the caller. */
R2S_API int r2s_rasterize_to_pixels_bwd_noalloc_f32(
    int mode, const float* means2d, const float* conics, const float* opacities, const float* mus,
    const int32_t* tile_offsets, const int32_t* flatten_ids, const float* v_image, int64_t C,
    int64_t N, int64_t n_isects, uint32_t width, uint32_t height, uint32_t tile_size,
    uint32_t n_tiles_w, uint32_t n_tiles_h, float* v_means2d_abs, float* v_means2d,
    float* v_conics, float* v_opacities, float* v_mus, r2s_stream_t stream);

/* ------------------------------------------------------------------------
 * Voxelization: vol[z,y,x] = sum over the brick's list of w*exp(-sigma)
 * (6-term quadratic), skipping sigma < 0 and |alpha| < 1e-6.  means3d [N,3],
 * conics [N,6], opacities [N], tile_offsets [nt0,nt1,nt2] -> vol
 * [dim0,dim1,dim2].  Replaces voxelize_to_voxels_fwd_tensor
 * (Ops.h:66-69; csrc/VoxelizeToVoxels.cpp:31-108).
 */
R2S_API int r2s_voxelize_to_voxels_fwd(int dtype, const void* means3d, const void* conics,
                               const void* opacities, const int32_t* tile_offsets,
                               const int32_t* flatten_ids, int64_t N, int64_t n_isects,
                               uint32_t dim2, uint32_t dim1, uint32_t dim0,
                               uint32_t tile_size, uint32_t nt2, uint32_t nt1, uint32_t nt0,
                               void* volume, r2s_stream_t stream);
/* VJP -> v_means3d [N,3], v_conics [N,6], v_opacities [N].  mode 0 =
 * voxelize_to_voxels_bwd_tensor (Ops.h:70-74; VoxelizeToVoxels.cpp:114-192),
 * mode 1 = voxelize_to_voxels_bwd_per_gaussian_tensor (Ops.h:75-79;
 * VoxelizeToVoxels.cpp:194-278).  `stats` is caller scratch of N*12
 * elements of dtype. */
R2S_API int r2s_voxelize_to_voxels_bwd(int dtype, int mode, const void* means3d, const void* conics,
                               const void* opacities, const int32_t* tile_offsets,
                               const int32_t* flatten_ids, const void* v_volume, int64_t N,
                               int64_t n_isects, uint32_t dim2, uint32_t dim1, uint32_t dim0,
                               uint32_t tile_size, uint32_t nt2, uint32_t nt1, uint32_t nt0,
                               void* stats, void* v_means3d, void* v_conics,
                               void* v_opacities, r2s_stream_t stream);

/* ========================================================================
 * Fused float32 entry points used by r2splat.ops (the training/inference
 * fast path).  Each replaces a chain of reference calls in
 * r2splat/ops/direct.py and r2splat/ops/explicit.py with fewer launches and
 * fewer [C,N] intermediates; results equal the chain's.
 * ====================================================================== */

/* Parameter transform + softplus(raw_opacities) in one pass
 * (direct.py:93-117: parameter_transform_fwd + torch softplus). */
R2S_API int r2s_prepare_gaussians_f32(const float* quats, const float* raw_scales,
                              const float* raw_opacities, double scale_min,
                              double scale_max, float* covars, float* max_scales,
                              float* opacities, int64_t n, r2s_stream_t stream);

/* Projection + conics/mu + tile rectangle for all (view, Gaussian) pairs
 * (direct.py:170-187: world_to_image_projection_fwd, conics_mu_fwd, the
 * opacity expand and the first pass of isect_tiles).  Writes means2d
 * [C,N,2], radii [C,N,2], splats [C,N,8] (x, y, conic a, b, c, w*mu,
 * cull extent x, cull extent y), rects [C*N] (8 B) and tiles_per_gauss
 * [C,N] (nullable). */
R2S_API int r2s_project_splats_f32(const float* means, const float* covars,
                           const float* opacities, const float* viewmats, const float* Ks,
                           int64_t C, int64_t N, uint32_t width, uint32_t height,
                           uint32_t tile_size, uint32_t n_tiles_w, uint32_t n_tiles_h,
                           double eps2d, double radius_clip, float* means2d, int32_t* radii,
                           float* splats, void* rects, int32_t* tiles_per_gauss,
                           r2s_stream_t stream);
/* Counting phase of the binning from precomputed rects (both layouts). */
R2S_API int r2s_bin_prepare(const void* rects, int64_t n_segments, int64_t n_items,
                    int64_t tiles_per_segment, uint32_t tiles_x, int layered,
                    int64_t segment_base, void* workspace, int64_t workspace_bytes,
                    int32_t* tile_offsets, int64_t* n_isects_dev, r2s_stream_t stream);
/* Rasterize from splat records (float32, any tile size).  With 16-pixel
 * tiles, `cull_ranges` (nullable, [n_isects] uint16) receives each record's
 * culling ranges inside its tile (first/last column, first/last row, 4 bits
 * each; this build's culling, the reference has no such table) for the
 * backward of the same binning to read instead of recomputing them. */
R2S_API int r2s_raster_splats_fwd_f32(const float* splats, const int32_t* tile_offsets,
                              const int32_t* flatten_ids, int64_t C, int64_t N,
                              int64_t n_isects, uint32_t width, uint32_t height,
                              uint32_t tile_size, uint32_t n_tiles_w, uint32_t n_tiles_h,
                              float* image, uint16_t* cull_ranges, r2s_stream_t stream);
/* Backward sufficient statistics per (view, Gaussian), accumulated over
 * tiles (`cull_ranges`: the table the forward of the same binning wrote, or
 * NULL): stats [C*N, 8] = (S0, Sx, Sy, Sxx, Sxy, Syy, Ax, Ay) with
 * S* = sum over contributing pixels of v*exp(-sigma) * moments of the pixel
 * offset, A* = sum of |v*exp(-sigma)*(conic . d)|.  Zeroes `stats` first. */
R2S_API int r2s_raster_splats_bwd_f32(const float* splats, const int32_t* tile_offsets,
                              const int32_t* flatten_ids, const float* v_image, int64_t C,
                              int64_t N, int64_t n_isects, uint32_t width, uint32_t height,
                              uint32_t tile_size, uint32_t n_tiles_w, uint32_t n_tiles_h,
                              int with_abs, const uint16_t* cull_ranges, float* stats,
                              r2s_stream_t stream);

/* Volume mapping + voxel splat records + brick rectangles
 * (direct.py:289-314: world_to_volume_mapping_fwd and the first pass of
 * isect_tiles_3d).  Writes means3d [N,3], conics [N,6], radii [N,3],
 * vsplats [N,16] (x, y, z, c00, c01, c02, c11, c12, c22, w, ex, ey, ez, band, 0,
 * 0): the conic, opacity, culling half-extents and the voxel backward's
 * cut-off band (the log2-unit distance from the cut-off inside which its fast
 * test is re-checked against the reference's),
 * rects3 [N] (16 B), tiles_per_gauss [N] (nullable). */
R2S_API int r2s_map_vsplats_f32(const float* means, const float* covars, const float* opacities,
                        const float* ranges, const float* centers, int64_t N, uint32_t dim2,
                        uint32_t dim1, uint32_t dim0, uint32_t tile_size, uint32_t nt2,
                        uint32_t nt1, uint32_t nt0, double eps3d, double radius_clip,
                        float* means3d, float* conics, int32_t* radii, float* vsplats,
                        void* rects3, int32_t* tiles_per_gauss, r2s_stream_t stream);
/* Row table of the (record, brick) pairs of a 3D binning with 8-voxel bricks
 * (the voxel path of VoxelizeToVoxelsFwd.cu / VoxelizeToVoxelsBwd.cu has no
 * such table; it is this build's culling): rows[2 i], rows[2 i + 1] = for
 * record i, byte k = first row | last row << 4 of z-slice k of its brick that
 * its ellipsoid can reach, 0x0f for none.  Read by the two entry points
 * below, which then skip their own culling of those records. */
R2S_API int r2s_voxel_rows_f32(const float* vsplats, const int32_t* tile_offsets,
                             const int32_t* flatten_ids, int64_t N, int64_t n_isects,
                             uint32_t dim2, uint32_t dim1, uint32_t dim0, uint32_t tile_size,
                             uint32_t nt2, uint32_t nt1, uint32_t nt0, uint32_t layer_begin,
                             uint32_t layer_end, const int32_t* brick_order, uint32_t* rows,
                             r2s_stream_t stream);
/* Launch order of the bricks of a 3D binning (this build's scheduling; the
 * reference launches bricks in key order): order [n_keys] = the brick keys
 * (0 .. n_keys-1 of the binning's tile_offsets) grouped by floor(log2 of
 * their record count), largest group first, empty bricks last -- an
 * approximate longest-first order.  The three per-brick entry points take it
 * as `brick_order` (NULL: key order); results do not depend on it. */
R2S_API int r2s_brick_order(const int32_t* tile_offsets, int64_t n_keys, int64_t n_isects,
                            int32_t* order, r2s_stream_t stream);
/* Voxelize bricks [z_begin/8 .. ) from voxel splat records; `volume` points
 * at voxel row z_begin of a [dim0,dim1,dim2] grid (z-slab output).  `rows`:
 * the row table of the same binning, or NULL. */
R2S_API int r2s_voxel_splats_fwd_f32(const float* vsplats, const int32_t* tile_offsets,
                             const int32_t* flatten_ids, const uint32_t* rows, int64_t N,
                             int64_t n_isects, uint32_t dim2, uint32_t dim1, uint32_t dim0,
                             uint32_t tile_size, uint32_t nt2, uint32_t nt1, uint32_t nt0,
                             uint32_t layer_begin, uint32_t layer_end,
                             const int32_t* brick_order, float* volume, r2s_stream_t stream);
/* Voxel backward statistics [N, 12] float64 = (S0, Sx, Sy, Sz, Sxx, Sxy, Sxz,
 * Syy, Syz, Szz, 0, 0): each brick's float moments added into float64
 * per-Gaussian sums, so that the result does not depend on the order of the
 * additions (runs, brick orders and z-slab splits agree to ~1e-16);
 * zeroes `stats` first.  `rows`: the row table of the same binning, or
 * NULL. */
R2S_API int r2s_voxel_splats_bwd_f32(const float* vsplats, const int32_t* tile_offsets,
                             const int32_t* flatten_ids, const uint32_t* rows,
                             const float* v_volume, int64_t N,
                             int64_t n_isects, uint32_t dim2, uint32_t dim1, uint32_t dim0,
                             uint32_t tile_size, uint32_t nt2, uint32_t nt1, uint32_t nt0,
                             uint32_t layer_begin, uint32_t layer_end,
                             const int32_t* brick_order, double* stats, r2s_stream_t stream);

/* Whole explicit backward per Gaussian (explicit.py:233-385): converts the
 * raster statistics of every view to the reference's per-view gradients
 * (written to v_means2d / v_means2d_abs [C,N,2] when non-NULL), applies
 * conics_mu_bwd and world_to_image_projection_bwd, sums over views, adds the
 * voxel path (world_to_volume_mapping_bwd of the voxel statistics), then
 * parameter_transform_bwd and the softplus chain for opacities.  Outputs
 * v_means [N,3], v_quats [N,4], v_raw_scales [N,3], v_raw_opacities [N];
 * with accumulate != 0 they are added to the existing contents.
 * raster_stats / vox_stats may be NULL (that path had no upstream gradient);
 * vox_stats is the float64 output of r2s_voxel_splats_bwd_f32. */
R2S_API int r2s_explicit_backward_f32(
    const float* means, const float* quats, const float* raw_scales,
    const float* raw_opacities, double scale_min, double scale_max, const float* viewmats,
    const float* Ks, int64_t C, int64_t N, uint32_t width, uint32_t height, double eps2d,
    const float* raster_stats, float* v_means2d, float* v_means2d_abs, const float* ranges,
    const float* centers, uint32_t dim2, uint32_t dim1, uint32_t dim0, double eps3d,
    const double* vox_stats, int accumulate, float* v_means, float* v_quats,
    float* v_raw_scales, float* v_raw_opacities, r2s_stream_t stream);

/* Densification statistics of BinaryTreeStrategy._update_state
 * (src/strategies/binary_tree.py:305-347, unpacked renders) fused into the
 * explicit backward: for every view c where max(radii[c,n,0], radii[c,n,1])
 * > 0, with g = the view's v_means2d_abs (absgrad != 0) or v_means2d row,
 *   grad2d[n] += sqrt((g_x scale_x)^2 + (g_y scale_y)^2),  count[n] += 1,
 *   max_radii[n] = max(max_radii[n], max radius / extent)   (max_radii non-NULL)
 * in the same float32 operations as r2s_densify_stats_f32, whose [C,N] radii
 * input is the amax of these [C,N,2] radii.  scale_x = width/2 * n_cameras,
 * scale_y = height/2 * n_cameras, extent = max(width, height). */
typedef struct r2s_densify_args {
    const int32_t* radii; /* [C,N,2] */
    double scale_x, scale_y, extent;
    int absgrad;
    float* grad2d;    /* [N] */
    float* count;     /* [N] */
    float* max_radii; /* [N] or NULL */
} r2s_densify_args;

/* r2s_explicit_backward_f32 plus the densification statistics of the same
 * views in the same kernel (replaces the strategy's pass over
 * means2d.absgrad after BinaryTreeTrainer's backward_explicit,
 * src/trainers/binary_tree.py:159-194).  v_means2d / v_means2d_abs may be NULL:
 * the statistics do not need them stored. */
R2S_API int r2s_explicit_backward_densify_f32(
    const float* means, const float* quats, const float* raw_scales,
    const float* raw_opacities, double scale_min, double scale_max, const float* viewmats,
    const float* Ks, int64_t C, int64_t N, uint32_t width, uint32_t height, double eps2d,
    const float* raster_stats, float* v_means2d, float* v_means2d_abs, const float* ranges,
    const float* centers, uint32_t dim2, uint32_t dim1, uint32_t dim0, double eps3d,
    const double* vox_stats, int accumulate, float* v_means, float* v_quats,
    float* v_raw_scales, float* v_raw_opacities, const r2s_densify_args* densify,
    r2s_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* R2S_H */
