// ref_backend.cpp -- the reference's backend seam (core/metal/bindings.h)
// implemented on the host over the reference's own kernels built through
// the MSL shim (libmsplat_ref.so: ref_render, ref_train_step, ref_densify),
// so that the reference's Model (core/src/model.cpp) and Trainer / C API
// (core/src/msplat_api.mm, compiled as C++) run unmodified on the CPU:
// oracle/_ref/libmsplat_ref_trainer.so (build_ref.py build_trainer).
//
// TEST INFRASTRUCTURE ONLY: the end-to-end checker for the engine's native
// trainer (msplat_b200/csrc/trainer.cu).  Images come from "<path>.rgb8"
// sidecars (the reference decodes with CoreGraphics), as in ref_data.cpp.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <fstream>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

// MTensor keeps the storage of a shared (Metal) buffer in private fields that
// views alias; host allocations here fill the same fields, so that views of
// the Model's backing buffers alias host memory as they alias Metal buffers.
#define private public
#include "loaders.hpp"
#include "msplat.hpp"
#undef private
#include "msplat_oracle.h"

extern "C" {
int ref_render(const orc_params* P, orc_state* S, const float* params[6]);
int ref_train_step(const orc_params* P, orc_state* S, float* params[6], float* exp_avg[6],
                   float* exp_avg_sq[6], const float* gt, float* vis_counts, float* xys_grad_norm,
                   float* max_2d_size);
int ref_densify(int N, int buf_capacity, float grad_thresh, float size_thresh, float screen_thresh,
                int check_screen, float cull_alpha_thresh, float cull_scale_thresh,
                float cull_screen_size, int check_huge, const float* xys_grad_norm,
                const float* vis_counts, const float* max_2d_size, float half_max_dim,
                float* bufs[6], int fr_stride, float* exp_avg[6], float* exp_avg_sq[6],
                const float* random_samples, int* split_flag_out, int* dup_flag_out,
                int* keep_flag_out);
}

// Zero-filled host memory in the fields a Metal allocation would fill.  Never
// freed: MTensor has no owner count outside Objective-C (test runs are short).
MTensor gpu_zeros(std::vector<int64_t> shape, DType dtype)
{
    MTensor t;
    t._shape = std::move(shape);
    t._dtype = dtype;
    t._numel = 1;
    for (auto s : t._shape) t._numel *= s;
    const size_t bytes = std::max<size_t>((size_t)t._numel * dtypeSize(dtype), 4);
    void* p = std::calloc(bytes, 1);
    if (!p) throw std::bad_alloc();
    t._buffer = p;
    t._data = p;
    return t;
}

MTensor gpu_empty(std::vector<int64_t> shape, DType dtype) { return gpu_zeros(std::move(shape), dtype); }

void cleanup_msplat_metal() {}
void* msplat_device() { return nullptr; }
void msplat_commit() {}
void msplat_gpu_sync() {}
void msplat_enable_gpu_timing(bool) {}
void msplat_drain_gpu_times(std::vector<double>& out) { out.clear(); }
void msplat_drain_stage_times(std::vector<double>[], int, int& n_stages, const char**) { n_stages = 0; }

Image imreadRGB(const std::string& path)
{
    std::ifstream f(path + ".rgb8", std::ios::binary);
    if (!f.is_open()) throw std::runtime_error("Failed to load image: " + path);
    int w = 0, h = 0;
    f >> w >> h;
    f.get();
    std::vector<unsigned char> px((size_t)w * h * 3);
    f.read(reinterpret_cast<char*>(px.data()), (std::streamsize)px.size());
    if (!f) throw std::runtime_error("Failed to decode image: " + path);
    Image img;
    img.width = w;
    img.height = h;
    img.data.resize(px.size());
    for (size_t i = 0; i < px.size(); i++) img.data[i] = px[i] / 255.0f;
    return img;
}

void imwriteRGB(const std::string&, const Image&) { throw std::runtime_error("imwriteRGB: not built"); }

namespace {

struct StateBuffers {
    std::vector<float> xys, depths, conics, colors, aabb, out_img, final_T, v_rendered, v_xy, v_conic,
        v_rgb, v_opacity, v_mean3d, v_scale, v_quat;
    std::vector<int32_t> radii, tiles_hit, tile_bins, final_idx;
    orc_state S{};

    StateBuffers(int n, int tiles, size_t px)
    {
        auto f = [](std::vector<float>& v, size_t k) { v.assign(k, 0.f); return v.data(); };
        auto i = [](std::vector<int32_t>& v, size_t k) { v.assign(k, 0); return v.data(); };
        S.xys = f(xys, 2 * (size_t)n);
        S.depths = f(depths, n);
        S.radii = i(radii, n);
        S.conics = f(conics, 3 * (size_t)n);
        S.num_tiles_hit = i(tiles_hit, n);
        S.colors = f(colors, 3 * (size_t)n);
        S.aabb = f(aabb, 2 * (size_t)n);
        S.tile_bins = i(tile_bins, 2 * (size_t)tiles);
        S.isect_capacity = 0;
        S.out_img = f(out_img, 3 * px);
        S.final_T = f(final_T, px);
        S.final_idx = i(final_idx, px);
        S.v_rendered = f(v_rendered, 3 * px);
        S.v_xy = f(v_xy, 2 * (size_t)n);
        S.v_conic = f(v_conic, 3 * (size_t)n);
        S.v_rgb = f(v_rgb, 3 * (size_t)n);
        S.v_opacity = f(v_opacity, n);
        S.v_mean3d = f(v_mean3d, 3 * (size_t)n);
        S.v_scale = f(v_scale, 3 * (size_t)n);
        S.v_quat = f(v_quat, 4 * (size_t)n);
    }
};

orc_params make_params(int n, MTensor& viewmat, MTensor& projmat, float fx, float fy, float cx,
                       float cy, unsigned h, unsigned w, const std::tuple<int, int, int>& tb,
                       float glob_scale, float clip, unsigned degree, unsigned dtu,
                       const float cam_pos[3], const float* bg)
{
    orc_params P{};
    P.num_points = n;
    P.img_w = (int)w;
    P.img_h = (int)h;
    P.tiles_x = std::get<0>(tb);
    P.tiles_y = std::get<1>(tb);
    P.degree = (int)degree;
    P.degrees_to_use = (int)dtu;
    P.k_max = 1;
    std::memcpy(P.viewmat, viewmat.data<float>(), sizeof(P.viewmat));
    std::memcpy(P.projmat, projmat.data<float>(), sizeof(P.projmat));
    P.fx = fx;
    P.fy = fy;
    P.cx = cx;
    P.cy = cy;
    P.glob_scale = glob_scale;
    P.clip_thresh = clip;
    std::memcpy(P.cam_pos, cam_pos, sizeof(P.cam_pos));
    std::memcpy(P.background, bg, sizeof(P.background));
    return P;
}

}  // namespace

MTensor msplat_render(int num_points, MTensor& means3d, MTensor& scales, float glob_scale,
                      MTensor& quats, MTensor& viewmat, MTensor& projmat, float fx, float fy,
                      float cx, float cy, unsigned img_height, unsigned img_width,
                      const std::tuple<int, int, int> tile_bounds, float clip_thresh,
                      unsigned degree, unsigned degrees_to_use, float cam_pos[3],
                      MTensor& features_dc, MTensor& features_rest, MTensor& opacities,
                      MTensor& background)
{
    orc_params P = make_params(num_points, viewmat, projmat, fx, fy, cx, cy, img_height, img_width,
                               tile_bounds, glob_scale, clip_thresh, degree, degrees_to_use, cam_pos,
                               background.data<float>());
    const size_t px = (size_t)img_width * img_height;
    StateBuffers sb(num_points, P.tiles_x * P.tiles_y, px);
    const float* params[6] = {means3d.data<float>(), scales.data<float>(), quats.data<float>(),
                              features_dc.data<float>(), features_rest.data<float>(),
                              opacities.data<float>()};
    ref_render(&P, &sb.S, params);
    MTensor out({(int64_t)img_height, (int64_t)img_width, 3}, DType::Float32);
    std::memcpy(out.data_ptr(), sb.out_img.data(), px * 3 * sizeof(float));
    return out;
}

std::tuple<MTensor, float> msplat_train_step(
    int num_points, MTensor& means3d, MTensor& scales, float glob_scale, MTensor& quats,
    MTensor& viewmat, MTensor& projmat, float fx, float fy, float cx, float cy, unsigned img_height,
    unsigned img_width, const std::tuple<int, int, int> tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, float cam_pos[3], MTensor& features_dc,
    MTensor& features_rest, MTensor& opacities, MTensor& background, MTensor& gt, MTensor&,
    float ssim_weight, float loss_inv_n, int, int num_adam_groups, MTensor adam_params[],
    MTensor adam_exp_avg[], MTensor adam_exp_avg_sq[], float adam_step_sizes[],
    float adam_bc2_sqrts[], float adam_beta1, float adam_beta2, float adam_eps, MTensor& vis_counts,
    MTensor& xys_grad_norm, MTensor& max_2d_size, float inv_max_dim)
{
    orc_params P = make_params(num_points, viewmat, projmat, fx, fy, cx, cy, img_height, img_width,
                               tile_bounds, glob_scale, clip_thresh, degree, degrees_to_use, cam_pos,
                               background.data<float>());
    P.ssim_weight = ssim_weight;
    P.loss_inv_n = loss_inv_n;
    P.inv_max_dim = inv_max_dim;
    for (int g = 0; g < num_adam_groups && g < 6; g++) {
        P.adam_step_size[g] = adam_step_sizes[g];
        P.adam_bc2_sqrt[g] = adam_bc2_sqrts[g];
    }
    P.beta1 = adam_beta1;
    P.beta2 = adam_beta2;
    P.eps = adam_eps;
    const size_t px = (size_t)img_width * img_height;
    StateBuffers sb(num_points, P.tiles_x * P.tiles_y, px);
    float* params[6];
    float* m[6];
    float* v[6];
    for (int g = 0; g < 6; g++) {
        params[g] = adam_params[g].data<float>();
        m[g] = adam_exp_avg[g].data<float>();
        v[g] = adam_exp_avg_sq[g].data<float>();
    }
    (void)means3d;
    (void)scales;
    (void)quats;
    (void)features_dc;
    (void)features_rest;
    (void)opacities;
    ref_train_step(&P, &sb.S, params, m, v, gt.data<float>(), vis_counts.data<float>(),
                   xys_grad_norm.data<float>(), max_2d_size.data<float>());
    MTensor radii({(int64_t)num_points}, DType::Int32);
    std::memcpy(radii.data_ptr(), sb.radii.data(), sizeof(int32_t) * num_points);
    return {radii, (float)sb.S.loss};
}

int msplat_densify(int N, int buf_capacity, float grad_thresh, float size_thresh,
                   float screen_thresh, int check_screen, float cull_alpha_thresh,
                   float cull_scale_thresh, float cull_screen_size, int check_huge,
                   MTensor& xys_grad_norm, MTensor& vis_counts, MTensor& max_2d_size,
                   float half_max_dim, MTensor& means_buf, MTensor& scales_buf, MTensor& quats_buf,
                   MTensor& featuresDc_buf, MTensor& featuresRest_buf, MTensor& opacities_buf,
                   int fr_stride, MTensor adam_exp_avg_buf[], MTensor adam_exp_avg_sq_buf[],
                   MTensor&, MTensor&, MTensor&, MTensor&, MTensor&, MTensor&, MTensor&, MTensor&,
                   MTensor& random_samples)
{
    float* bufs[6] = {means_buf.data<float>(), scales_buf.data<float>(), quats_buf.data<float>(),
                      featuresDc_buf.data<float>(), featuresRest_buf.data<float>(),
                      opacities_buf.data<float>()};
    float* m[6];
    float* v[6];
    for (int g = 0; g < 6; g++) {
        m[g] = adam_exp_avg_buf[g].data<float>();
        v[g] = adam_exp_avg_sq_buf[g].data<float>();
    }
    std::vector<int> split(buf_capacity), dup(buf_capacity), keep(buf_capacity);
    return ref_densify(N, buf_capacity, grad_thresh, size_thresh, screen_thresh, check_screen,
                       cull_alpha_thresh, cull_scale_thresh, cull_screen_size, check_huge,
                       xys_grad_norm.data<float>(), vis_counts.data<float>(),
                       max_2d_size.data<float>(), half_max_dim, bufs, fr_stride, m, v,
                       random_samples.data<float>(), split.data(), dup.data(), keep.data());
}
