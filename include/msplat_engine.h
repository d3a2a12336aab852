/*
 * msplat_engine.h -- C-ABI of the B200 engine: the backend seam that
 * msplat's Metal engine exposes in core/metal/bindings.h, re-expressed with
 * plain pointers and sizes (no C++ or torch types), plus the few calls a
 * host needs that Metal's unified memory made implicit (stream, copies,
 * last error).
 *
 * Memory: every "device" pointer below is CUDA device memory on the current
 * device (cudaMalloc, msplat_gpu_alloc, or a torch CUDA tensor's data_ptr).
 * Small per-step values the reference kept in GPU tensors (view/projection
 * matrices, background colour) are passed as host arrays; the engine copies
 * them into a per-step parameter block on its stream.
 *
 * Errors: functions that can fail return 0 on success and a negative code
 * otherwise; msplat_last_error() describes the last failure.  Nothing here
 * falls back to the CPU: without a usable CUDA device every compute entry
 * point fails with MSPLAT_ERR_CUDA.
 *
 * Threading: one engine per process and device, used from one host thread
 * at a time (the reference's single global context and serial dispatch
 * queue, msplat_metal.mm:179, have the same rule).
 */
#ifndef MSPLAT_ENGINE_H
#define MSPLAT_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MSPLAT_OK 0
#define MSPLAT_ERR_ARG (-1)      /* invalid argument */
#define MSPLAT_ERR_CUDA (-2)     /* CUDA runtime error / no device */
#define MSPLAT_ERR_OVERFLOW (-3) /* intersection buffer overflow */

#define MSPLAT_N_ADAM_GROUPS 6   /* means, scales, quats, features_dc, features_rest, opacities */

/* ---- lifecycle and memory (bindings.h:8-27) ---------------------------- */

/* Last error message of this thread ("" when none). */
const char *msplat_last_error(void);

/* Use `cuda_stream` (a cudaStream_t) for all engine work; NULL selects the
 * engine's own stream.  No reference counterpart (Metal used one queue). */
int msplat_set_stream(void *cuda_stream);
void *msplat_get_stream(void);

/* Replaces msplat_device() (bindings.h:11-15): returns a pointer to the
 * CUDA device ordinal the engine runs on, or NULL if there is no device. */
void *msplat_device(void);

/* Replaces gpu_zeros / gpu_empty (bindings.h:17-18): device allocation of
 * `bytes`, zero-filled when `zero` != 0.  Free with msplat_gpu_free. */
void *msplat_gpu_alloc(size_t bytes, int zero);
void msplat_gpu_free(void *ptr);
/* Memory that the host and the engine's kernels both address (CUDA managed
 * memory): the counterpart of the MTLResourceStorageModeShared buffers
 * behind the reference's MTensor (metal_tensor.hpp:43-55), for hosts that
 * read and write tensors in place as the reference's Model does.  Before
 * an engine call reads a range the host has touched, move it to the device
 * with msplat_shared_prefetch (queued on the engine stream; the host must
 * not touch the range until msplat_gpu_sync).  Zeroed on the host when
 * `zero` != 0.  Free with msplat_shared_free. */
void *msplat_shared_alloc(size_t bytes, int zero);
void msplat_shared_free(void *ptr);
int msplat_shared_prefetch(const void *ptr, size_t bytes);
/* Host<->device copies on the engine stream (Metal's shared storage made
 * these implicit); `kind` 0 = host to device, 1 = device to host,
 * 2 = device to device.  Synchronous when `sync` != 0. */
int msplat_copy(void *dst, const void *src, size_t bytes, int kind, int sync);

/* msplat_commit (bindings.h:21): work is already queued on the stream;
 * this records a commit point (for GPU timing) and returns immediately. */
void msplat_commit(void);
/* msplat_gpu_sync (bindings.h:24): block until all queued work is done. */
void msplat_gpu_sync(void);
/* cleanup_msplat_metal (bindings.h:8): free every cached buffer. */
void cleanup_msplat_metal(void);
void cleanup_msplat_cuda(void);
/* msplat_set_metallib_path (msplat_metal.mm:168): accepted and ignored. */
void msplat_set_metallib_path(const char *path);

/* GPU timing (bindings.h:27-33).  Times are ms per committed step measured
 * with CUDA events on the engine stream. */
void msplat_enable_gpu_timing(int enable);
int msplat_drain_gpu_times(double *out, int max_out);
/* Per-stage times: fills stage_times[max_stages*max_samples] row-major by
 * stage and stage_names; returns the number of stages. */
int msplat_drain_stage_times(double *stage_times, int max_stages, int max_samples,
                             int *n_samples, const char **stage_names);

/* ---- the hot path ------------------------------------------------------- */

/*
 * One full training iteration: projection + SH, tile binning and per-tile
 * depth sort, forward raster, L1 + SSIM loss, backward raster, projection
 * backward, Adam for all six groups (SH groups only for visible Gaussians)
 * and the densification statistics.
 * Replaces std::tuple<MTensor,float> msplat_train_step(...) (bindings.h:50-67;
 * implementation msplat_metal.mm:771-1330) argument for argument:
 *   means3d (N,3), scales (N,3, log), quats (N,4, w x y z), features_dc (N,3),
 *   features_rest (N,features_rest_bases,3), opacities (N, logit),
 *   gt (H,W,3), vis_counts/xys_grad_norm/max_2d_size (N): device pointers;
 *   viewmat, projmat (16, row-major), cam_pos (3), background (3),
 *   tile_bounds (3), adam_step_sizes/adam_bc2_sqrts (num_adam_groups): host;
 *   adam_params/adam_exp_avg/adam_exp_avg_sq: host arrays of device pointers
 *   in group order means, scales, quats, features_dc, features_rest,
 *   opacities (params alias the tensors above, as in Model::fullIteration).
 *   window2d is accepted and unused (the loss uses the separable window).
 * On return *radii_out (if non-NULL) aliases the engine's radii buffer (N,
 * int32, device), valid until the next call, and *loss_out (if non-NULL) is
 * the loss of the most recent step whose value has reached the host
 * without a wait (the reference likewise reads its loss without syncing).
 */
int msplat_train_step(
    int num_points, float *means3d, float *scales, float glob_scale, float *quats,
    const float *viewmat, const float *projmat, float fx, float fy, float cx, float cy,
    unsigned img_height, unsigned img_width, const int *tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, const float *cam_pos,
    float *features_dc, float *features_rest, float *opacities, const float *background,
    const float *gt, const float *window2d, float ssim_weight, float loss_inv_n,
    int features_rest_bases, int num_adam_groups, float *const *adam_params,
    float *const *adam_exp_avg, float *const *adam_exp_avg_sq,
    const float *adam_step_sizes, const float *adam_bc2_sqrts, float adam_beta1,
    float adam_beta2, float adam_eps, float *vis_counts, float *xys_grad_norm,
    float *max_2d_size, float inv_max_dim, const int32_t **radii_out, float *loss_out);

/*
 * Data-parallel training, gradient half.  No counterpart in the reference
 * (which trains one view on one device); it is msplat_train_step with the
 * fused optimiser replaced by a gradient output, so that ranks training
 * different views of the same Gaussians can sum their gradients before
 * Adam.  Same arguments as msplat_train_step up to features_rest_bases,
 * then grad_out: a device buffer of (15 + 3*features_rest_bases) * N floats
 * holding, one after another, the gradients of means [N,3], scales [N,3],
 * quats [N,4], features_dc [N,3], features_rest [N,features_rest_bases*3]
 * and opacities [N], then a visibility flag per Gaussian (1 = radius > 0 in
 * this view).  Every element is written.  Parameters and moments are not
 * touched; the densification statistics are accumulated as in
 * msplat_train_step.
 */
int msplat_train_step_grads(
    int num_points, float *means3d, float *scales, float glob_scale, float *quats,
    const float *viewmat, const float *projmat, float fx, float fy, float cx, float cy,
    unsigned img_height, unsigned img_width, const int *tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, const float *cam_pos,
    float *features_dc, float *features_rest, float *opacities, const float *background,
    const float *gt, float ssim_weight, float loss_inv_n, int features_rest_bases,
    float *grad_out, float *vis_counts, float *xys_grad_norm, float *max_2d_size,
    float inv_max_dim, const int32_t **radii_out, float *loss_out);

/*
 * The gradient half in compact form, for msplat_dp_reduce_adam(compact=1).
 * No counterpart in the reference.  Same arguments as
 * msplat_train_step_grads; grad_out holds 15 * N + 4 floats: the gradients
 * of means [N,3], scales [N,3], quats [N,4], then v_rgb [N,3] (the colour
 * gradient of each visible Gaussian, 0 for the others), the gradient of
 * opacities [N], the visibility flags [N] and the camera position (3 floats).
 * Every SH coefficient's gradient is v_rgb times a basis value of the view
 * direction, so the optimiser rebuilds them from v_rgb and the camera.
 */
int msplat_train_step_grads_compact(
    int num_points, float *means3d, float *scales, float glob_scale, float *quats,
    const float *viewmat, const float *projmat, float fx, float fy, float cx, float cy,
    unsigned img_height, unsigned img_width, const int *tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, const float *cam_pos,
    float *features_dc, float *features_rest, float *opacities, const float *background,
    const float *gt, float ssim_weight, float loss_inv_n, int features_rest_bases,
    float *grad_out, float *vis_counts, float *xys_grad_norm, float *max_2d_size,
    float inv_max_dim, const int32_t **radii_out, float *loss_out);

/*
 * The gradient half for a batch of several views per step.  No counterpart
 * in the reference (one view per step).  Same arguments and buffer layout as
 * msplat_train_step_grads, but this view's gradients are ADDED to what
 * grad_out holds (the previous views of the step, written by
 * msplat_train_step_grads for the first one) and each visible Gaussian's
 * visibility entry grows by 1; Gaussians this view culls are neither read
 * nor written.  For the mean loss over a batch of V views pass loss_inv_n =
 * 1 / (H * W * 3 * V) to every view's call.
 */
int msplat_train_step_grads_accumulate(
    int num_points, float *means3d, float *scales, float glob_scale, float *quats,
    const float *viewmat, const float *projmat, float fx, float fy, float cx, float cy,
    unsigned img_height, unsigned img_width, const int *tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, const float *cam_pos,
    float *features_dc, float *features_rest, float *opacities, const float *background,
    const float *gt, float ssim_weight, float loss_inv_n, int features_rest_bases,
    float *grad_out, float *vis_counts, float *xys_grad_norm, float *max_2d_size,
    float inv_max_dim, const int32_t **radii_out, float *loss_out);

/*
 * Data-parallel training, optimiser half: Adam on Gaussians [begin, end)
 * from a gradient buffer in the msplat_train_step_grads layout (typically
 * summed over ranks), each gradient multiplied by grad_scale.  The update,
 * the per-group step sizes and the rule that features_dc/features_rest
 * only move for Gaussians whose visibility entry is > 0 (and features_rest
 * only for the SH degrees in use) are those of msplat_train_step's fused
 * Adam (msplat_metal.metal:1666-1689 and :1915-1985).  With one rank and
 * grad_scale = 1 the two halves give msplat_train_step's result bit for bit.
 */
int msplat_adam_apply(
    int num_points, int features_rest_bases, unsigned degree, unsigned degrees_to_use,
    const float *grads, float grad_scale, int begin, int end, int num_adam_groups,
    float *const *adam_params, float *const *adam_exp_avg, float *const *adam_exp_avg_sq,
    const float *adam_step_sizes, const float *adam_bc2_sqrts, float adam_beta1,
    float adam_beta2, float adam_eps);

/*
 * Data-parallel optimiser over peer memory.  No counterpart in the reference.
 * Replaces the all-reduce + msplat_adam_apply pair of the data-parallel step
 * when every rank's gradient buffer, parameter arrays and flag array are
 * mapped into every process (msplat_ipc_*): rank `rank` of `world` (<= 8)
 * sums the world gradient buffers (msplat_train_step_grads layout) for its
 * 1/world of the Gaussians, applies Adam with grad_scale 1/world using its
 * own moments (only its shard of them is ever used), and stores the updated
 * parameters into every rank's arrays.  rank_grads[world] and
 * rank_flags[world] (2*world unsigned each, zeroed once at allocation) and
 * rank_params[world*6] (group order as in msplat_train_step) are this
 * process's pointers to every rank's buffers.  `epoch` must grow by one per
 * step (from 1).  Queued on the engine stream: returns before the work
 * finishes; the step's cross-GPU waits give up after timeout_s seconds and
 * set bits read by msplat_dp_errors (1: gradients of a peer missing,
 * 2: updated shards of a peer missing).  With `compact` != 0 the gradient
 * buffers are in the msplat_train_step_grads_compact layout (4x smaller).
 */
int msplat_dp_reduce_adam(
    int rank, int world, int num_points, int features_rest_bases, unsigned degree,
    unsigned degrees_to_use, const float *const *rank_grads, float *const *rank_params,
    float *const *exp_avg, float *const *exp_avg_sq, unsigned *const *rank_flags,
    unsigned epoch, const float *adam_step_sizes, const float *adam_bc2_sqrts,
    float adam_beta1, float adam_beta2, float adam_eps, int compact, double timeout_s);
/* Error bits of the peer-memory steps on this device (waits until the
 * engine stream is idle); clears them when `reset` != 0.  -1 on failure. */
int msplat_dp_errors(int reset);
/* CUDA IPC: the 64-byte handle of an allocation made by msplat_gpu_alloc
 * (pass the pointer it returned), the mapping of a peer's handle into this
 * process (each handle is mapped once and cached), and the release of every
 * mapping.  No counterpart in the reference (a single-device engine). */
int msplat_ipc_get_handle(const void *dev_ptr, void *handle_out);
int msplat_ipc_open_handle(const void *handle, void **dev_ptr_out);
int msplat_ipc_close_all(void);

/*
 * Forward-only render.  Replaces MTensor msplat_render(...) (bindings.h:37-46;
 * implementation msplat_metal.mm:752-769).  *out_img receives a device
 * pointer to the engine's (H,W,3) float image, valid until the next call
 * (the reference returns an alias of its cached out_img the same way).
 */
int msplat_render(
    int num_points, const float *means3d, const float *scales, float glob_scale,
    const float *quats, const float *viewmat, const float *projmat, float fx, float fy,
    float cx, float cy, unsigned img_height, unsigned img_width, const int *tile_bounds,
    float clip_thresh, unsigned degree, unsigned degrees_to_use, const float *cam_pos,
    const float *features_dc, const float *features_rest, const float *opacities,
    const float *background, float **out_img);

/*
 * Forward-only render that allocates nothing.  No counterpart in the
 * reference: it exists for callers that must not allocate device memory
 * while rendering (a frame loop that cannot take the device-wide stall of
 * cudaMalloc/cudaFree, or a host that budgets all device memory up front).
 * Same arguments and the same image as msplat_render, but the image goes
 * into the caller's device buffer out_img (H*W*3 floats) and every
 * intermediate lives in one static device array of
 * MSPLAT_NOALLOC_SCRATCH_BYTES per device.
 *
 * Limit: the call is rejected with MSPLAT_ERR_ARG, before any CUDA call,
 * when 56 bytes per Gaussian + 8 per pixel + 20 per depth-chunk pixel
 * (chunked path only) + 132 per tile + 16 intersections of 20 bytes per
 * Gaussian do not fit the array (about 160k Gaussians at 1280x720).  Spare
 * bytes become extra intersection slots; more intersections than slots
 * return MSPLAT_ERR_OVERFLOW.  The first call on a device (with it current)
 * does the set-up and should precede any stream capture.  Calls on one
 * device share the array: overlapping calls race and must be serialised.
 * Synchronous on cuda_stream (NULL = the legacy default stream).
 */
#define MSPLAT_NOALLOC_SCRATCH_BYTES (64ull << 20)
int msplat_render_noalloc(
    int num_points, const float *means3d, const float *scales, float glob_scale,
    const float *quats, const float *viewmat, const float *projmat, float fx, float fy,
    float cx, float cy, unsigned img_height, unsigned img_width, const int *tile_bounds,
    float clip_thresh, unsigned degree, unsigned degrees_to_use, const float *cam_pos,
    const float *features_dc, const float *features_rest, const float *opacities,
    const float *background, float *out_img, void *cuda_stream);

/* ---- densification (follows the training step) ------------------------- */

/*
 * Densification.  Replaces int msplat_densify(...) (bindings.h:69-84;
 * implementation msplat_metal.mm:1337-1592) argument for argument, MTensor
 * replaced by device pointers: classify every Gaussian as split / duplicate
 * (average screen-space gradient above grad_thresh, largest scale above or
 * below size_thresh, screen size above screen_thresh when check_screen),
 * append two children per split (offsets R(q) * (sample * exp(scale)),
 * scale - ln 1.6, zero Adam state; random_samples [2N,3] standard normals)
 * and one copy per duplicate, cull (opacity below cull_alpha_thresh, split
 * parents, and with check_huge: largest scale above cull_scale_thresh or
 * screen size above cull_screen_size), and compact all 18 buffers (the six
 * parameter arrays and their two Adam moments, group order as in
 * msplat_train_step, each with room for 3N rows: buf_capacity) in order.
 * The scratch arrays may be NULL, in which case the engine provides them.
 * Synchronous; returns the new number of Gaussians, or a negative code.
 */
int msplat_densify(
    int N, int buf_capacity, float grad_thresh, float size_thresh, float screen_thresh,
    int check_screen, float cull_alpha_thresh, float cull_scale_thresh, float cull_screen_size,
    int check_huge, const float *xys_grad_norm, const float *vis_counts,
    const float *max_2d_size, float half_max_dim, float *means_buf, float *scales_buf,
    float *quats_buf, float *features_dc_buf, float *features_rest_buf, float *opacities_buf,
    int fr_stride, float *const *adam_exp_avg_buf, float *const *adam_exp_avg_sq_buf,
    int *split_flag, int *dup_flag, int *split_prefix, int *dup_prefix, int *keep_flag,
    int *keep_prefix, int *block_totals, float *compact_scratch, const float *random_samples);

/*
 * The opacity reset of Model::afterTrain (model.cpp:280-290), on the GPU
 * instead of the host: every opacity logit above logit(0.2) is lowered to
 * it and the opacity group's Adam moments are zeroed (n Gaussians).
 */
int msplat_reset_opacity(float *opacities, float *exp_avg, float *exp_avg_sq, int n);

/* ---- per-step host inputs ---------------------------------------------------
 * msplat_stage_input: copy `bytes` of host memory (pinned, for the copy to
 * overlap compute) into one of two engine-owned device buffers on a
 * separate copy stream, and return that buffer to pass as this step's
 * input (e.g. msplat_train_step's gt).  The copy waits only for the step
 * that read the same buffer two stagings ago, and the kernels queued next
 * on the engine stream wait for the copy, so with one staging per step the
 * upload of step s runs under the kernels of step s-1.  The buffer is valid
 * until the next-but-one staging.  No counterpart in the reference (its
 * images are host-visible to the GPU). */
int msplat_stage_input(const void *host, size_t bytes, const void **dev_out);

/* ---- model files ----------------------------------------------------------
 * Every array below may be device memory (the engine's buffers; a save first
 * waits for the engine's queued work, as msplat_gpu_sync does) or host
 * memory.  `params`, `exp_avg`, `exp_avg_sq`: six pointers in group order
 * means [N,3], scales [N,3], quats [N,4], features_dc [N,3], features_rest
 * [N,B,3], opacities [N,1], B = features_rest_bases.  keep_crs/scale/
 * translation are the model's CRS fields (keepCrs, scale, translation[3]).
 */

/* Writes a .msplat checkpoint, byte for byte Model::saveCheckpoint
 * (core/src/model.cpp:361-399): magic 0x4C50534D, version 1, step,
 * num_active, shDegree, adam_step_count (u32 each), adam_lr[6],
 * means_lr_init, means_lr_final (f32), then 18 tensors (the six parameter
 * groups, six exp_avg, six exp_avg_sq), each u32 ndim, i64 shape[ndim],
 * u64 byte count, raw f32. */
int msplat_save_checkpoint(const char *path, int step, int num_active, int sh_degree,
                           int adam_step_count, const float *adam_lr, float means_lr_init,
                           float means_lr_final, int features_rest_bases,
                           const float *const *params, const float *const *exp_avg,
                           const float *const *exp_avg_sq);

/* Reads the scalar state of a checkpoint (model.cpp:401-422) and the SH-rest
 * basis count B from its features_rest tensor, so the caller can size the
 * buffers before msplat_load_checkpoint.  NULL outputs are skipped; adam_lr
 * receives 6 floats.  0 or MSPLAT_ERR_ARG (bad magic or version: the
 * reference's "Not a valid msplat checkpoint file" / "Unsupported checkpoint
 * version"). */
int msplat_read_checkpoint_header(const char *path, int *step, int *num_active, int *sh_degree,
                                  int *adam_step_count, float *adam_lr, float *means_lr_init,
                                  float *means_lr_final, int *features_rest_bases);

/* Loads the 18 tensors of a checkpoint (model.cpp:424-435) into arrays with
 * room for `capacity` rows each (the backing buffers; the reference
 * allocates 4 * num_active of them, model.cpp:441-470).  Every tensor's
 * shape is checked.  Returns the checkpoint's step (>= 0) or a negative
 * code. */
int msplat_load_checkpoint(const char *path, int capacity, float *const *params,
                           float *const *exp_avg, float *const *exp_avg_sq);

/* Writes a PLY of n Gaussians, byte for byte saveGaussianPly
 * (core/src/loaders/save_gaussians.cpp:10-54): header comment
 * "msplat v<step>", per vertex x y z, zero normals, f_dc_*, f_rest_* in
 * [3, B] order, opacity, scale_0..2, rot_0..3; with keep_crs the means
 * become m / scale + translation and the log-scales log(exp(s) / scale). */
int msplat_save_ply(const char *path, int step, int n, int features_rest_bases,
                    const float *const *params, int keep_crs, float scale,
                    const float *translation);

/* Writes a .splat file, byte for byte saveGaussianSplat
 * (save_gaussians.cpp:56-97): 32-byte records (f32 position, f32 scale,
 * u8 rgba, u8 quaternion) sorted by size * sigmoid(opacity), largest
 * first.  params[4] (features_rest) is not read and may be NULL. */
int msplat_save_splat(const char *path, int n, const float *const *params, int keep_crs,
                      float scale, const float *translation);

/* The header of loadGaussianPly (save_gaussians.cpp:99-130): vertex count,
 * step (from a "comment Generated by msplat at iteration <k>" line, else 0)
 * and B (f_rest properties / 3).  MSPLAT_ERR_ARG for a file that is not a
 * PLY or has no vertices, as the reference throws. */
int msplat_read_ply_header(const char *path, int *n, int *step, int *features_rest_bases);

/* loadGaussianPly (save_gaussians.cpp:99-184) into arrays of >= capacity
 * rows (group order as above; features_rest back to [N, B, 3]); with
 * keep_crs the inverse CRS transform.  Returns the step or a negative
 * code. */
int msplat_load_ply(const char *path, int capacity, float *const *params, int keep_crs,
                    float scale, const float *translation);

/* ---- training images on the device ----------------------------------------
 * The reference prepares ground truth on the host (core/src/loaders/
 * image_io.cpp, core/src/input_data.cpp:17-75) and uploads it; these run on
 * the engine's stream over device buffers, float RGB interleaved (H, W, 3).
 */

/* Bytes (1 = grey, 3 = RGB, 4 = RGBA with alpha ignored) -> floats v / 255,
 * the conversion of imreadRGB (image_io.cpp:46-51). */
int msplat_bytes_to_rgb(const unsigned char *src, int width, int height, int channels, float *dst);

/* resizeArea (image_io.cpp:93-139): box-filter downscale, each output the
 * area-weighted mean of the source pixels it covers.  Bit-identical. */
int msplat_resize_area(const float *src, int src_w, int src_h, float *dst, int dst_w, int dst_h);

/* The crop rectangle of undistortImage (image_io.cpp:203-270), on the host:
 * roi = {x, y, width, height} of the inner rectangle of the undistorted
 * border (the whole image when that rectangle is empty). */
int msplat_undistort_roi(int w, int h, float fx, float fy, float cx, float cy, float k1, float k2,
                         float p1, float p2, float k3, int *roi);

/* undistortImage's resampling (image_io.cpp:141-201, 272-300): for each
 * pixel of the roi, Brown-Conrady distortion of its ray and a bilinear,
 * edge-clamped sample of `src` (w x h).  dst is roi[2] x roi[3].  The new
 * intrinsics are fx, fy, cx - roi[0], cy - roi[1]. */
int msplat_undistort(const float *src, int w, int h, float fx, float fy, float cx, float cy,
                     float k1, float k2, float p1, float p2, float k3, const int *roi, float *dst);

/* imreadRGB (image_io.cpp:12-56) into device memory: JPEG decoded by
 * nvJPEG on the GPU, PNG (any bit depth, colour type, interlacing) on the
 * host; RGBA composited over black.  msplat_image_info reads the size
 * only.  dst holds capacity_floats floats (>= 3 W H).  Synchronous. */
int msplat_image_info(const char *path, int *width, int *height);
int msplat_image_decode(const char *path, float *dst, long long capacity_floats, int *width,
                        int *height);

/* ---- datasets -------------------------------------------------------------
 * InputData (core/include/input_data.hpp) with its images resident in HBM.
 * Not thread-safe; one caller per dataset.
 */
typedef struct MsplatData MsplatData;

typedef struct MsplatCameraInfo {
    int width, height;
    float fx, fy, cx, cy;
    float k1, k2, k3, p1, p2;
    float cam_to_world[16]; /* row-major, OpenGL axes (y up, z back) */
} MsplatCameraInfo;

/* inputDataFromX (input_data.cpp:195-217): Nerfstudio (transforms.json),
 * COLMAP (cameras.bin / sparse/0/cameras.bin; loadColmap,
 * load_colmap.cpp:121-164) or Polycam (keyframes/corrected_cameras or
 * cameras.json), then autoScaleAndCenter (input_data.cpp:79-123).  No
 * images are read.  MSPLAT_ERR_ARG with the reference's message for an
 * unknown layout, an unsupported COLMAP camera model or a bad file. */
int msplat_dataset_open(const char *path, const char *colmap_image_path, MsplatData **out);
void msplat_dataset_close(MsplatData *ds);
int msplat_dataset_num_cameras(const MsplatData *ds);
int msplat_dataset_camera(const MsplatData *ds, int index, MsplatCameraInfo *out);
/* Camera::filePath; valid while the dataset is open. */
const char *msplat_dataset_camera_path(const MsplatData *ds, int index);
/* InputData::points (host memory owned by the dataset); returns the count. */
long long msplat_dataset_points(const MsplatData *ds, const float **xyz,
                                const unsigned char **rgb);
/* InputData::scale and translation[3]. */
int msplat_dataset_transform(const MsplatData *ds, float *scale, float *translation);
/* splitTrainTest (input_data.cpp:148-158): index i is a test camera when
 * i % test_every == 0.  The index arrays may be NULL (counts only). */
int msplat_dataset_split(const MsplatData *ds, int test_every, int *train_idx, int *n_train,
                         int *test_idx, int *n_test);
/* getCameras(validate = true) (input_data.cpp:127-146): the held-out
 * camera, std::mt19937(42)() % n for "random", else the first path that
 * contains val_image, else 0. */
int msplat_dataset_validation_camera(const MsplatData *ds, const char *val_image);
/* Camera::loadImage (input_data.cpp:17-52) for every camera / one camera:
 * decode, fit intrinsics to the decoded size, downscale by the factor (when
 * > 1), undistort and crop; the image stays in HBM and the camera's
 * intrinsics are updated. */
int msplat_dataset_load_images(MsplatData *ds, float downscale_factor);
int msplat_dataset_load_image(MsplatData *ds, int index, float downscale_factor);
/* Camera::getGPUImage (input_data.cpp:54-75): the resident image, or its
 * W/k x H/k area-downscaled copy (made on first use, then cached). */
int msplat_dataset_gt(MsplatData *ds, int index, int downscale, const float **dev_rgb,
                      int *width, int *height);
/* Device bytes held by the dataset's images. */
long long msplat_dataset_device_bytes(const MsplatData *ds);

/* Bridges from the trainer-level C API (include/msplat_c_api.h), no
 * counterpart in the reference: the engine dataset behind an MsplatDataset
 * handle (owned by it), and the dataset indices of its training (test = 0)
 * or held-out (test = 1) cameras (up to max_out; returns the count). */
MsplatData *msplat_dataset_data(void *c_api_dataset);
/* msplat_trainer_load_checkpoint with the camera re-shuffle optional: the
 * C++ Trainer re-shuffles on resume (msplat_api.mm:250-255), the Python
 * binding's load_checkpoint (python/bindings.cpp:273-275) does not. */
int msplat_trainer_load_checkpoint_ex(void *trainer, const char *path, int reshuffle);
int msplat_dataset_indices(void *c_api_dataset, int test, int *out, int max_out);

/* ---- initialisation from a point cloud ------------------------------------- */

/* PointsTensor::scales (core/include/kdtree_tensor.hpp:27-41, a nanoflann
 * k-d tree on the host) on the GPU: out[i] = mean of the square roots of
 * the k-1 smallest squared distances from point i to the others (the k
 * nearest include the point itself), by an exact grid search.  xyz (n,3)
 * and out (n) are host arrays; 2 <= k <= 8.  Synchronous. */
int msplat_knn_mean_distance(const float *xyz, long long n, int k, float *out);

/* The initial Gaussians of Model::Model (core/src/model.cpp:42-118) from a
 * point cloud (host xyz (n,3), 8-bit rgb (n,3)) into device arrays of >= n
 * rows: means = xyz; scales = log(mean distance to the 3 nearest
 * neighbours), repeated; random unit quaternions from std::mt19937(42);
 * features_dc from the colours; features_rest zero ((n, (sh_degree+1)^2-1,
 * 3)); opacities logit(0.1).  Synchronous. */
int msplat_init_gaussians(const float *xyz, const unsigned char *rgb, long long n, int sh_degree,
                          float *means, float *scales, float *quats, float *features_dc,
                          float *features_rest, float *opacities);

/* ---- evaluation ------------------------------------------------------------
 * The held-out metrics of evaluate() (python/bindings.cpp:186-216) on the
 * device: ssim_eval (core/src/ssim.cpp:61-123; Gaussian window of
 * window_size <= 11 taps and sigma, separable, edge-clamped), psnr and
 * l1_loss (core/src/model.cpp:24-40) of two (H, W, 3) float images in
 * device memory.  Synchronous; NULL outputs are skipped.
 */
int msplat_eval_metrics(const float *rendered, const float *gt, int height, int width,
                        int window_size, float sigma, float *psnr, float *ssim, float *l1);

/* ---- introspection (tests and benchmarks) ------------------------------- */

/* Loss of the last step; waits for it when `sync` != 0, else returns the
 * latest value already on the host. */
float msplat_last_loss(int sync);
/* Intersections of the last step (waits for the step). */
long long msplat_num_intersections(void);
/* Device error word of the last step (waits); bit 1 = intersection overflow. */
int msplat_device_errors(void);
/* Device pointer and element count of a named engine buffer: "xy", "depth",
 * "radii", "conic_op", "rgb", "tile_offset", "tile_sorted", "sorted_ids",
 * "out_img", "final_T", "final_idx", "v_rendered", "grad_acc", "chunk_idx".
 * "tile_sorted" is the length of each tile's sorted prefix in "sorted_ids"
 * (a tile of more than 8,192 keys may sort only its nearest keys; the
 * positions past the prefix are never read).  Returns 0 or MSPLAT_ERR_ARG
 * for an unknown name. */
int msplat_debug_buffer(const char *name, void **dev_ptr, long long *count);
/* Number of kernel launches the engine issued since the last reset. */
long long msplat_kernel_launches(int reset);
/* Binning modes of the last forward, for tests and benchmarks: bit 0, long
 * tile lists sorted their nearest keys only; bit 1, dense binning (large
 * rects counted by the corners of a 2D difference array).  Neither changes
 * any result. */
int msplat_last_binning(void);
/* Raster work of the last forward (render or training step), for
 * benchmarks; no counterpart in the reference.  Replays the reference's
 * per-pixel loop (nd_rasterize_forward_kernel, msplat_metal.metal:472-585)
 * over the engine's sorted lists and writes four sums over the image:
 * out[0] list positions visited before termination, out[1] pairs whose
 * sigma passes (0 <= sigma < 5.55), out[2] pairs blended into the pixel
 * (E, the contributing pixel.Gaussian evaluations), out[3] positions the
 * backward walks (rasterize_backward_kernel, :898-1099).  Synchronous.
 * MSPLAT_ERR_ARG when no forward ran yet or the last one was depth-chunked. */
int msplat_count_raster_work(unsigned long long *out);

#ifdef __cplusplus
}
#endif
#endif
