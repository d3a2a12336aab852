// bindings_cuda.cpp -- the reference's backend seam (core/metal/bindings.h)
// on the CUDA engine, so that the reference's own Model (core/src/model.cpp),
// Trainer and C API (core/src/msplat_api.mm) and data front end run
// unmodified with the B200 kernels in place of msplat_metal.mm.
//
// Memory.  The reference's MTensor wraps an MTLResourceStorageModeShared
// buffer: one address the host reads and writes in place (initialisation,
// opacity reset, checkpoints, PLY, ground-truth upload, render readback) and
// the GPU reads in its kernels.  Here gpu_zeros/gpu_empty return CUDA managed
// memory (msplat_shared_alloc), which has the same single-address semantics.
// Before each engine call the ranges that call reads or writes are moved to
// the device (msplat_shared_prefetch, on the engine stream); the reference
// calls msplat_gpu_sync before any host access to data the GPU wrote
// (msplat_api.mm:150,176,200,223; model.cpp:281,362), after which the host
// may touch them again.
//
// MTensor (core/include/metal_tensor.hpp) keeps its buffer handle and data
// pointer in private fields that views alias, and has no constructor for a
// shared allocation outside Objective-C.  In the reference tree the CUDA
// build would add one (MTensor(SharedAlloc, shape, dtype), filling the two
// fields); to compile against the header unchanged, this file fills the
// same two fields directly.  Compiled as C++ the header keeps no owner count
// (Objective-C releases the Metal buffer), so, as in the reference's C++
// build, tensors are never freed before exit.
//
// Errors: the reference has no status codes across this seam (asserts and
// exceptions); an engine failure here throws std::runtime_error with the
// engine's message.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <tuple>
#include <unordered_map>
#include <vector>

#define private public
#include "bindings.h"
#include "loaders.hpp"
#undef private

#include "seam_engine.h"

namespace {

[[noreturn]] void fail(const char* who)
{
    throw std::runtime_error(std::string(who) + ": " + seam::last_error());
}

void check(int rc, const char* who)
{
    if (rc != 0) fail(who);
}

MTensor shared_tensor(std::vector<int64_t> shape, DType dtype, bool zero)
{
    MTensor t;
    t._shape = std::move(shape);
    t._dtype = dtype;
    t._numel = 1;
    for (auto s : t._shape) t._numel *= s;
    const size_t bytes = std::max<size_t>((size_t)t._numel * dtypeSize(dtype), 4);
    void* p = seam::shared_alloc(bytes, zero);
    if (!p) fail("gpu_empty/gpu_zeros");
    t._buffer = p;
    t._data = p;
    return t;
}

// The range of `t` the next engine call touches, moved to the device.
void to_device(const MTensor& t, const char* who)
{
    if (!t.defined() || t.nbytes() == 0) return;
    if (!t._buffer) throw std::runtime_error(std::string(who) + ": a host-only tensor was passed "
                                             "where the engine needs a GPU tensor");
    check(seam::prefetch(t.data_ptr(), t.nbytes()), who);
}

// A grow-only shared buffer that engine outputs are copied into for the host
// (the reference returns aliases of its own cached buffers the same way,
// valid until the next call).
struct SharedCache {
    void* p = nullptr;
    size_t bytes = 0;
    void* get(size_t need)
    {
        if (need > bytes) {
            p = seam::shared_alloc(need, false);   // the old block stays valid for old aliases
            if (!p) fail("seam output buffer");
            bytes = need;
        }
        return p;
    }
};

SharedCache g_render_out, g_radii;

MTensor alias(void* p, std::vector<int64_t> shape, DType dtype)
{
    MTensor t;
    t._shape = std::move(shape);
    t._dtype = dtype;
    t._numel = 1;
    for (auto s : t._shape) t._numel *= s;
    t._buffer = p;
    t._data = p;
    return t;
}

}  // namespace

// ---- bindings.h: lifecycle, memory, timing --------------------------------

void cleanup_msplat_metal() { seam::cleanup(); }

void* msplat_device() { return seam::device(); }

MTensor gpu_zeros(std::vector<int64_t> shape, DType dtype)
{
    return shared_tensor(std::move(shape), dtype, true);
}

MTensor gpu_empty(std::vector<int64_t> shape, DType dtype)
{
    return shared_tensor(std::move(shape), dtype, false);
}

void msplat_commit() { seam::commit(); }

void msplat_gpu_sync() { seam::sync(); }

void msplat_enable_gpu_timing(bool enable) { seam::enable_timing(enable); }

void msplat_drain_gpu_times(std::vector<double>& out) { seam::drain_times(out); }

void msplat_drain_stage_times(std::vector<double> stage_times[], int max_stages, int& n_stages,
                              const char** stage_names)
{
    seam::drain_stage_times(stage_times, max_stages, n_stages, stage_names);
}

// ---- bindings.h: the hot path -------------------------------------------

MTensor msplat_render(int num_points, MTensor& means3d, MTensor& scales, float glob_scale,
                      MTensor& quats, MTensor& viewmat, MTensor& projmat, float fx, float fy,
                      float cx, float cy, unsigned img_height, unsigned img_width,
                      const std::tuple<int, int, int> tile_bounds, float clip_thresh,
                      unsigned degree, unsigned degrees_to_use, float cam_pos[3],
                      MTensor& features_dc, MTensor& features_rest, MTensor& opacities,
                      MTensor& background)
{
    for (MTensor* t : {&means3d, &scales, &quats, &features_dc, &features_rest, &opacities})
        to_device(*t, "msplat_render");
    const int tb[3] = {std::get<0>(tile_bounds), std::get<1>(tile_bounds),
                       std::get<2>(tile_bounds)};
    float* img = nullptr;
    check(seam::render(num_points, means3d.data<float>(), scales.data<float>(), glob_scale,
                       quats.data<float>(), viewmat.data<float>(), projmat.data<float>(), fx, fy,
                       cx, cy, img_height, img_width, tb, clip_thresh, degree, degrees_to_use,
                       cam_pos, features_dc.data<float>(), features_rest.data<float>(),
                       opacities.data<float>(), background.data<float>(), &img),
          "msplat_render");
    const size_t bytes = (size_t)img_height * img_width * 3 * sizeof(float);
    void* out = g_render_out.get(bytes);
    check(seam::copy_device(out, img, bytes), "msplat_render");
    return alias(out, {(int64_t)img_height, (int64_t)img_width, 3}, DType::Float32);
}

std::tuple<MTensor, float> msplat_train_step(
    int num_points, MTensor& means3d, MTensor& scales, float glob_scale, MTensor& quats,
    MTensor& viewmat, MTensor& projmat, float fx, float fy, float cx, float cy,
    unsigned img_height, unsigned img_width, const std::tuple<int, int, int> tile_bounds,
    float clip_thresh, unsigned degree, unsigned degrees_to_use, float cam_pos[3],
    MTensor& features_dc, MTensor& features_rest, MTensor& opacities, MTensor& background,
    MTensor& gt, MTensor& window2d, float ssim_weight, float loss_inv_n, int features_rest_bases,
    int num_adam_groups, MTensor adam_params[], MTensor adam_exp_avg[],
    MTensor adam_exp_avg_sq[], float adam_step_sizes[], float adam_bc2_sqrts[],
    float adam_beta1, float adam_beta2, float adam_eps, MTensor& vis_counts,
    MTensor& xys_grad_norm, MTensor& max_2d_size, float inv_max_dim)
{
    (void)window2d;   // the engine's loss uses the reference kernels' separable window
    const int groups = std::min(num_adam_groups, 6);
    float* p[6] = {};
    float* m[6] = {};
    float* v[6] = {};
    for (int g = 0; g < groups; g++) {
        for (MTensor* t : {&adam_params[g], &adam_exp_avg[g], &adam_exp_avg_sq[g]})
            to_device(*t, "msplat_train_step");
        p[g] = adam_params[g].data<float>();
        m[g] = adam_exp_avg[g].data<float>();
        v[g] = adam_exp_avg_sq[g].data<float>();
    }
    for (MTensor* t : {&means3d, &scales, &quats, &features_dc, &features_rest, &opacities, &gt,
                       &vis_counts, &xys_grad_norm, &max_2d_size})
        to_device(*t, "msplat_train_step");
    const int tb[3] = {std::get<0>(tile_bounds), std::get<1>(tile_bounds),
                       std::get<2>(tile_bounds)};
    const int32_t* radii = nullptr;
    float loss = 0.f;
    check(seam::train_step(num_points, means3d.data<float>(), scales.data<float>(), glob_scale,
                           quats.data<float>(), viewmat.data<float>(), projmat.data<float>(), fx,
                           fy, cx, cy, img_height, img_width, tb, clip_thresh, degree,
                           degrees_to_use, cam_pos, features_dc.data<float>(),
                           features_rest.data<float>(), opacities.data<float>(),
                           background.data<float>(), gt.data<float>(), ssim_weight, loss_inv_n,
                           features_rest_bases, groups, p, m, v, adam_step_sizes, adam_bc2_sqrts,
                           adam_beta1, adam_beta2, adam_eps, vis_counts.data<float>(),
                           xys_grad_norm.data<float>(), max_2d_size.data<float>(), inv_max_dim,
                           &radii, &loss),
          "msplat_train_step");
    const size_t bytes = (size_t)num_points * sizeof(int32_t);
    void* out = g_radii.get(bytes);
    if (bytes) check(seam::copy_device(out, radii, bytes), "msplat_train_step");
    return {alias(out, {(int64_t)num_points}, DType::Int32), loss};
}

int msplat_densify(int N, int buf_capacity, float grad_thresh, float size_thresh,
                   float screen_thresh, int check_screen, float cull_alpha_thresh,
                   float cull_scale_thresh, float cull_screen_size, int check_huge,
                   MTensor& xys_grad_norm, MTensor& vis_counts, MTensor& max_2d_size,
                   float half_max_dim, MTensor& means_buf, MTensor& scales_buf, MTensor& quats_buf,
                   MTensor& featuresDc_buf, MTensor& featuresRest_buf, MTensor& opacities_buf,
                   int fr_stride, MTensor adam_exp_avg_buf[], MTensor adam_exp_avg_sq_buf[],
                   MTensor& split_flag, MTensor& dup_flag, MTensor& split_prefix,
                   MTensor& dup_prefix, MTensor& keep_flag, MTensor& keep_prefix,
                   MTensor& block_totals, MTensor& compact_scratch, MTensor& random_samples)
{
    MTensor* bufs[6] = {&means_buf, &scales_buf, &quats_buf, &featuresDc_buf, &featuresRest_buf,
                        &opacities_buf};
    float* b[6];
    float* m[6];
    float* v[6];
    for (int g = 0; g < 6; g++) {
        for (MTensor* t : {bufs[g], &adam_exp_avg_buf[g], &adam_exp_avg_sq_buf[g]})
            to_device(*t, "msplat_densify");
        b[g] = bufs[g]->data<float>();
        m[g] = adam_exp_avg_buf[g].data<float>();
        v[g] = adam_exp_avg_sq_buf[g].data<float>();
    }
    for (MTensor* t : {&xys_grad_norm, &vis_counts, &max_2d_size, &split_flag, &dup_flag,
                       &split_prefix, &dup_prefix, &keep_flag, &keep_prefix, &block_totals,
                       &compact_scratch, &random_samples})
        to_device(*t, "msplat_densify");
    const int n = seam::densify(
        N, buf_capacity, grad_thresh, size_thresh, screen_thresh, check_screen, cull_alpha_thresh,
        cull_scale_thresh, cull_screen_size, check_huge, xys_grad_norm.data<float>(),
        vis_counts.data<float>(), max_2d_size.data<float>(), half_max_dim, b, fr_stride, m, v,
        split_flag.data<int32_t>(), dup_flag.data<int32_t>(), split_prefix.data<int32_t>(),
        dup_prefix.data<int32_t>(), keep_flag.data<int32_t>(), keep_prefix.data<int32_t>(),
        block_totals.data<int32_t>(), compact_scratch.data<float>(), random_samples.data<float>());
    if (n < 0) fail("msplat_densify");
    return n;
}

// ---- loaders.hpp: image I/O on the engine ---------------------------------
// (image_io.cpp decodes and encodes with CoreGraphics on Apple platforms.)

Image imreadRGB(const std::string& path)
{
    Image img;
    if (seam::image_read(path, img.data, img.width, img.height) != 0)
        throw std::runtime_error("Failed to load image: " + path + " (" + seam::last_error() + ")");
    return img;
}

Image resizeArea(const Image& src, int dstW, int dstH)
{
    Image out;
    out.width = dstW;
    out.height = dstH;
    out.data.resize((size_t)dstW * dstH * 3);
    check(seam::resize_area(src.ptr(), src.width, src.height, out.ptr(), dstW, dstH), "resizeArea");
    return out;
}

UndistortResult undistortImage(const Image& src, float fx, float fy, float cx, float cy,
                               float k1, float k2, float p1, float p2, float k3)
{
    int roi[4] = {0, 0, src.width, src.height};
    UndistortResult r;
    check(seam::undistort(src.ptr(), src.width, src.height, fx, fy, cx, cy, k1, k2, p1, p2, k3,
                          roi, r.image.data),
          "undistortImage");
    r.image.width = r.width = roi[2];
    r.image.height = r.height = roi[3];
    r.fx = fx;
    r.fy = fy;
    r.cx = cx - roi[0];
    r.cy = cy - roi[1];
    return r;
}

namespace {

// A PNG of 8-bit RGB rows in stored (uncompressed) deflate blocks: the
// format of imwriteRGB's output without a compression library.
uint32_t crc32_of(const uint8_t* p, size_t n, uint32_t c = 0xffffffffu)
{
    static uint32_t table[256];
    static bool init = false;
    if (!init) {
        for (uint32_t i = 0; i < 256; i++) {
            uint32_t x = i;
            for (int k = 0; k < 8; k++) x = (x & 1) ? 0xedb88320u ^ (x >> 1) : x >> 1;
            table[i] = x;
        }
        init = true;
    }
    for (size_t i = 0; i < n; i++) c = table[(c ^ p[i]) & 0xff] ^ (c >> 8);
    return c;
}

void put32(std::vector<uint8_t>& o, uint32_t v)
{
    for (int s = 24; s >= 0; s -= 8) o.push_back((uint8_t)(v >> s));
}

void chunk(std::vector<uint8_t>& o, const char* type, const std::vector<uint8_t>& data)
{
    put32(o, (uint32_t)data.size());
    const size_t at = o.size();
    o.insert(o.end(), type, type + 4);
    o.insert(o.end(), data.begin(), data.end());
    put32(o, crc32_of(o.data() + at, o.size() - at) ^ 0xffffffffu);
}

}  // namespace

void imwriteRGB(const std::string& path, const Image& img)
{
    const int w = img.width, h = img.height;
    std::vector<uint8_t> raw;   // filter byte 0 + one row of RGB8, per row
    raw.reserve((size_t)h * (1 + 3 * (size_t)w));
    for (int y = 0; y < h; y++) {
        raw.push_back(0);
        for (int i = 0; i < 3 * w; i++) {
            const float v = std::clamp(img.data[(size_t)y * 3 * w + i] * 255.0f, 0.0f, 255.0f);
            raw.push_back((uint8_t)(v + 0.5f));
        }
    }
    std::vector<uint8_t> z = {0x78, 0x01};   // zlib header, no compression
    uint32_t a = 1, b = 0;
    for (uint8_t c : raw) {
        a = (a + c) % 65521u;
        b = (b + a) % 65521u;
    }
    for (size_t off = 0; off < raw.size() || off == 0; off += 65535) {
        const size_t len = std::min<size_t>(65535, raw.size() - off);
        const bool last = off + len >= raw.size();
        z.push_back(last ? 1 : 0);
        z.push_back((uint8_t)(len & 0xff));
        z.push_back((uint8_t)(len >> 8));
        z.push_back((uint8_t)(~len & 0xff));
        z.push_back((uint8_t)((~len >> 8) & 0xff));
        z.insert(z.end(), raw.begin() + off, raw.begin() + off + len);
        if (last) break;
    }
    put32(z, (b << 16) | a);
    std::vector<uint8_t> png = {0x89, 'P', 'N', 'G', 0x0d, 0x0a, 0x1a, 0x0a};
    std::vector<uint8_t> ihdr;
    put32(ihdr, (uint32_t)w);
    put32(ihdr, (uint32_t)h);
    ihdr.insert(ihdr.end(), {8, 2, 0, 0, 0});   // 8-bit, RGB, deflate, no filter set, no interlace
    chunk(png, "IHDR", ihdr);
    chunk(png, "IDAT", z);
    chunk(png, "IEND", {});
    std::ofstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("Failed to write image: " + path);
    f.write(reinterpret_cast<const char*>(png.data()), (std::streamsize)png.size());
}
