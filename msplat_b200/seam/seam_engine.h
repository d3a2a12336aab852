// seam_engine.h -- the CUDA engine as seen from the reference's backend seam.
//
// The reference's bindings.h declares C++ functions whose names the engine's
// C-ABI (include/msplat_engine.h) also uses with C linkage (msplat_render,
// msplat_commit, ...), so no translation unit can include both headers.
// bindings_cuda.cpp (reference types: MTensor, Image) calls the engine only
// through the functions below, and seam_engine.cpp (engine header) defines
// them.  Every call returns 0 or an engine error code; seam::last_error()
// holds the message.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace seam {

const char* last_error();

// memory the host and the engine both address (CUDA managed memory)
void* shared_alloc(size_t bytes, bool zero);
int prefetch(const void* ptr, size_t bytes);   // to the device, on the engine stream
int copy_device(void* dst, const void* src, size_t bytes);

void* device();
void commit();
void sync();
void cleanup();
void enable_timing(bool on);
int drain_times(std::vector<double>& out);
int drain_stage_times(std::vector<double>* stage_times, int max_stages, int& n_stages,
                      const char** stage_names);

// The engine's hot path; pointer arguments are device-addressable.
int render(int num_points, const float* means3d, const float* scales, float glob_scale,
           const float* quats, const float* viewmat, const float* projmat, float fx, float fy,
           float cx, float cy, unsigned img_height, unsigned img_width, const int* tile_bounds,
           float clip_thresh, unsigned degree, unsigned degrees_to_use, const float* cam_pos,
           const float* features_dc, const float* features_rest, const float* opacities,
           const float* background, float** out_img);

int train_step(int num_points, float* means3d, float* scales, float glob_scale, float* quats,
               const float* viewmat, const float* projmat, float fx, float fy, float cx, float cy,
               unsigned img_height, unsigned img_width, const int* tile_bounds, float clip_thresh,
               unsigned degree, unsigned degrees_to_use, const float* cam_pos, float* features_dc,
               float* features_rest, float* opacities, const float* background, const float* gt,
               float ssim_weight, float loss_inv_n, int features_rest_bases,
               int num_adam_groups, float* const* adam_params, float* const* adam_exp_avg,
               float* const* adam_exp_avg_sq, const float* adam_step_sizes,
               const float* adam_bc2_sqrts, float beta1, float beta2, float eps,
               float* vis_counts, float* xys_grad_norm, float* max_2d_size, float inv_max_dim,
               const int32_t** radii, float* loss);

int densify(int N, int buf_capacity, float grad_thresh, float size_thresh, float screen_thresh,
            int check_screen, float cull_alpha_thresh, float cull_scale_thresh,
            float cull_screen_size, int check_huge, const float* xys_grad_norm,
            const float* vis_counts, const float* max_2d_size, float half_max_dim,
            float* const* bufs, int fr_stride, float* const* exp_avg, float* const* exp_avg_sq,
            int* split_flag, int* dup_flag, int* split_prefix, int* dup_prefix, int* keep_flag,
            int* keep_prefix, int* block_totals, float* compact_scratch,
            const float* random_samples);

// PointsTensor::scales on the GPU (host arrays)
int knn_mean_distance(const float* xyz, long long n, int k, float* out);

// Image I/O of the loaders on the engine (host float RGB arrays)
int image_read(const std::string& path, std::vector<float>& rgb, int& width, int& height);
int resize_area(const float* src, int src_w, int src_h, float* dst, int dst_w, int dst_h);
int undistort(const float* src, int w, int h, float fx, float fy, float cx, float cy, float k1,
              float k2, float p1, float p2, float k3, int roi[4], std::vector<float>& dst);

}  // namespace seam
