// seam_engine.cpp -- seam::* (seam_engine.h) on the engine's C-ABI.
//
// The half of the CUDA backend seam that may include the engine header; see
// bindings_cuda.cpp for the half that implements the reference's bindings.h.
#include "seam_engine.h"

#include <cstring>

#include "msplat_engine.h"

namespace seam {

const char* last_error() { return msplat_last_error(); }

void* shared_alloc(size_t bytes, bool zero) { return msplat_shared_alloc(bytes, zero ? 1 : 0); }

int prefetch(const void* ptr, size_t bytes) { return msplat_shared_prefetch(ptr, bytes); }

int copy_device(void* dst, const void* src, size_t bytes)
{
    return msplat_copy(dst, src, bytes, 2, 0);
}

void* device() { return msplat_device(); }
void commit() { msplat_commit(); }
void sync() { msplat_gpu_sync(); }
void cleanup() { cleanup_msplat_cuda(); }
void enable_timing(bool on) { msplat_enable_gpu_timing(on ? 1 : 0); }

int drain_times(std::vector<double>& out)
{
    out.assign(1 << 16, 0.0);
    const int got = msplat_drain_gpu_times(out.data(), (int)out.size());
    out.resize((size_t)(got > 0 ? got : 0));
    return 0;
}

int drain_stage_times(std::vector<double>* stage_times, int max_stages, int& n_stages,
                      const char** stage_names)
{
    constexpr int kMaxSamples = 1 << 14;
    std::vector<double> flat((size_t)max_stages * kMaxSamples);
    int n_samples = 0;
    const char* names[16] = {};
    n_stages = msplat_drain_stage_times(flat.data(), max_stages, kMaxSamples, &n_samples, names);
    if (n_stages < 0) {
        n_stages = 0;
        return -1;
    }
    for (int s = 0; s < n_stages; s++) {
        stage_times[s].assign(flat.begin() + (size_t)s * kMaxSamples,
                              flat.begin() + (size_t)s * kMaxSamples + n_samples);
        if (stage_names) stage_names[s] = names[s];
    }
    return 0;
}

int render(int num_points, const float* means3d, const float* scales, float glob_scale,
           const float* quats, const float* viewmat, const float* projmat, float fx, float fy,
           float cx, float cy, unsigned img_height, unsigned img_width, const int* tile_bounds,
           float clip_thresh, unsigned degree, unsigned degrees_to_use, const float* cam_pos,
           const float* features_dc, const float* features_rest, const float* opacities,
           const float* background, float** out_img)
{
    return msplat_render(num_points, means3d, scales, glob_scale, quats, viewmat, projmat, fx, fy,
                         cx, cy, img_height, img_width, tile_bounds, clip_thresh, degree,
                         degrees_to_use, cam_pos, features_dc, features_rest, opacities,
                         background, out_img);
}

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
               const int32_t** radii, float* loss)
{
    return msplat_train_step(num_points, means3d, scales, glob_scale, quats, viewmat, projmat, fx,
                             fy, cx, cy, img_height, img_width, tile_bounds, clip_thresh, degree,
                             degrees_to_use, cam_pos, features_dc, features_rest, opacities,
                             background, gt, nullptr, ssim_weight, loss_inv_n, features_rest_bases,
                             num_adam_groups, adam_params, adam_exp_avg, adam_exp_avg_sq,
                             adam_step_sizes, adam_bc2_sqrts, beta1, beta2, eps, vis_counts,
                             xys_grad_norm, max_2d_size, inv_max_dim, radii, loss);
}

int densify(int N, int buf_capacity, float grad_thresh, float size_thresh, float screen_thresh,
            int check_screen, float cull_alpha_thresh, float cull_scale_thresh,
            float cull_screen_size, int check_huge, const float* xys_grad_norm,
            const float* vis_counts, const float* max_2d_size, float half_max_dim,
            float* const* bufs, int fr_stride, float* const* exp_avg, float* const* exp_avg_sq,
            int* split_flag, int* dup_flag, int* split_prefix, int* dup_prefix, int* keep_flag,
            int* keep_prefix, int* block_totals, float* compact_scratch,
            const float* random_samples)
{
    return msplat_densify(N, buf_capacity, grad_thresh, size_thresh, screen_thresh, check_screen,
                          cull_alpha_thresh, cull_scale_thresh, cull_screen_size, check_huge,
                          xys_grad_norm, vis_counts, max_2d_size, half_max_dim, bufs[0], bufs[1],
                          bufs[2], bufs[3], bufs[4], bufs[5], fr_stride, exp_avg, exp_avg_sq,
                          split_flag, dup_flag, split_prefix, dup_prefix, keep_flag, keep_prefix,
                          block_totals, compact_scratch, random_samples);
}

int knn_mean_distance(const float* xyz, long long n, int k, float* out)
{
    return msplat_knn_mean_distance(xyz, n, k, out);
}

namespace {

// A device buffer for the image helpers, freed on scope exit.
struct DevBuf {
    void* p = nullptr;
    explicit DevBuf(size_t bytes) : p(msplat_gpu_alloc(bytes, 0)) {}
    ~DevBuf() { msplat_gpu_free(p); }
    float* f() const { return static_cast<float*>(p); }
};

}  // namespace

int image_read(const std::string& path, std::vector<float>& rgb, int& width, int& height)
{
    int rc = msplat_image_info(path.c_str(), &width, &height);
    if (rc) return rc;
    const long long n = 3LL * width * height;
    DevBuf d((size_t)n * sizeof(float));
    if (!d.p) return MSPLAT_ERR_CUDA;
    if ((rc = msplat_image_decode(path.c_str(), d.f(), n, &width, &height))) return rc;
    rgb.resize((size_t)n);
    return msplat_copy(rgb.data(), d.p, (size_t)n * sizeof(float), 1, 1);
}

int resize_area(const float* src, int src_w, int src_h, float* dst, int dst_w, int dst_h)
{
    const size_t sb = (size_t)src_w * src_h * 3 * sizeof(float);
    const size_t db = (size_t)dst_w * dst_h * 3 * sizeof(float);
    DevBuf s(sb), d(db);
    if (!s.p || !d.p) return MSPLAT_ERR_CUDA;
    int rc = msplat_copy(s.p, src, sb, 0, 0);
    if (!rc) rc = msplat_resize_area(s.f(), src_w, src_h, d.f(), dst_w, dst_h);
    if (!rc) rc = msplat_copy(dst, d.p, db, 1, 1);
    return rc;
}

int undistort(const float* src, int w, int h, float fx, float fy, float cx, float cy, float k1,
              float k2, float p1, float p2, float k3, int roi[4], std::vector<float>& dst)
{
    int rc = msplat_undistort_roi(w, h, fx, fy, cx, cy, k1, k2, p1, p2, k3, roi);
    if (rc) return rc;
    const size_t sb = (size_t)w * h * 3 * sizeof(float);
    const size_t db = (size_t)roi[2] * roi[3] * 3 * sizeof(float);
    DevBuf s(sb), d(db);
    if (!s.p || !d.p) return MSPLAT_ERR_CUDA;
    rc = msplat_copy(s.p, src, sb, 0, 0);
    if (!rc) rc = msplat_undistort(s.f(), w, h, fx, fy, cx, cy, k1, k2, p1, p2, k3, roi, d.f());
    dst.resize((size_t)roi[2] * roi[3] * 3);
    if (!rc) rc = msplat_copy(dst.data(), d.p, db, 1, 1);
    return rc;
}

}  // namespace seam
