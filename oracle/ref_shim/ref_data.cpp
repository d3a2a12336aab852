// ref_data.cpp -- C entry points over the reference's own data front end
// (msplat core/src/input_data.cpp, core/src/loaders/load_colmap.cpp,
// load_ply.cpp, load_nerfstudio.cpp, load_polycam.cpp, the resize /
// undistort half of image_io.cpp, ssim.cpp and psnr / l1_loss of
// model.cpp), compiled from the reference's sources into
// oracle/_ref/libmsplat_ref_data.so by build_ref.py build_data.
//
// TEST INFRASTRUCTURE ONLY: the checker for the engine's dataset loaders,
// device image preparation and evaluation metrics
// (msplat_b200/csrc/dataset.cu, kernels_image.cu, kernels_eval.cu).
//
// The reference decodes images with CoreGraphics (macOS only).  Here
// imreadRGB reads "<image path>.rgb8" instead -- a raw file the tests write
// beside each image: "<width> <height>\n" then width*height*3 bytes of the
// same pixels -- and converts each byte to v / 255.0f as the reference's
// imreadRGB does.  The allocation and sync calls of the Metal runtime are
// given host versions.
#include <cstdio>
#include <cstring>
#include <exception>
#include <fstream>
#include <string>
#include <vector>

#include "input_data.hpp"
#include "loaders.hpp"
#include "model.hpp"
#include "msplat.hpp"
#include "ssim.hpp"

MTensor gpu_empty(std::vector<int64_t> shape, DType dtype) { return MTensor(std::move(shape), dtype); }

MTensor gpu_zeros(std::vector<int64_t> shape, DType dtype)
{
    MTensor t(std::move(shape), dtype);
    t.zero();
    return t;
}

void msplat_gpu_sync() {}

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
thread_local std::string g_err;

Image host_image(const float* src, int w, int h)
{
    Image im;
    im.width = w;
    im.height = h;
    im.data.assign(src, src + (size_t)w * h * 3);
    return im;
}
}  // namespace

extern "C" {

const char* ref_data_last_error() { return g_err.c_str(); }

void* ref_dataset_open(const char* path, const char* image_path)
{
    try {
        return new InputData(inputDataFromX(path, image_path ? image_path : ""));
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void ref_dataset_close(void* d) { delete static_cast<InputData*>(d); }

int ref_dataset_num_cameras(void* d) { return (int)static_cast<InputData*>(d)->cameras.size(); }

// out: width, height (as floats), fx fy cx cy k1 k2 k3 p1 p2, c2w[16] -> 29 floats
void ref_dataset_camera(void* d, int i, float* out)
{
    const Camera& c = static_cast<InputData*>(d)->cameras[i];
    const float v[13] = {(float)c.width, (float)c.height, c.fx, c.fy, c.cx, c.cy,
                         c.k1, c.k2, c.k3, c.p1, c.p2, 0, 0};
    std::memcpy(out, v, 11 * sizeof(float));
    std::memcpy(out + 11, c.camToWorld, 16 * sizeof(float));
}

const char* ref_dataset_camera_path(void* d, int i)
{
    return static_cast<InputData*>(d)->cameras[i].filePath.c_str();
}

long long ref_dataset_points(void* d, float* xyz, unsigned char* rgb)
{
    const Points& p = static_cast<InputData*>(d)->points;
    if (xyz && p.count) std::memcpy(xyz, p.xyz.data(), p.xyz.size() * sizeof(float));
    if (rgb && p.count) std::memcpy(rgb, p.rgb.data(), p.rgb.size());
    return p.count;
}

void ref_dataset_transform(void* d, float* scale, float* translation)
{
    const InputData* in = static_cast<InputData*>(d);
    *scale = in->scale;
    std::memcpy(translation, in->translation, 3 * sizeof(float));
}

// indices of splitTrainTest's cameras, recovered by file path
int ref_dataset_split(void* d, int test_every, int* train, int* n_train, int* test, int* n_test)
{
    InputData* in = static_cast<InputData*>(d);
    auto split = in->splitTrainTest(test_every);
    auto index = [&](const Camera& c) {
        for (int i = 0; i < (int)in->cameras.size(); i++)
            if (in->cameras[i].filePath == c.filePath) return i;
        return -1;
    };
    *n_train = (int)std::get<0>(split).size();
    *n_test = (int)std::get<1>(split).size();
    for (int i = 0; i < *n_train; i++) train[i] = index(std::get<0>(split)[i]);
    for (int i = 0; i < *n_test; i++) test[i] = index(std::get<1>(split)[i]);
    return 0;
}

int ref_dataset_validation(void* d, const char* val_image)
{
    InputData* in = static_cast<InputData*>(d);
    auto got = in->getCameras(true, val_image);
    return (int)(std::get<1>(got) - in->cameras.data());
}

int ref_camera_load_image(void* d, int i, float downscale_factor)
{
    try {
        static_cast<InputData*>(d)->cameras[i].loadImage(downscale_factor);
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// Camera::getGPUImage(k) copied out (capacity in floats); *w, *h its size.
int ref_camera_gt(void* d, int i, int k, float* out, long long capacity, int* w, int* h)
{
    MTensor& t = static_cast<InputData*>(d)->cameras[i].getGPUImage(k);
    *h = (int)t.size(0);
    *w = (int)t.size(1);
    if ((long long)t.numel() > capacity) return -1;
    std::memcpy(out, t.data_ptr(), t.nbytes());
    return 0;
}

void ref_resize_area(const float* src, int sw, int sh, float* dst, int dw, int dh)
{
    Image r = resizeArea(host_image(src, sw, sh), dw, dh);
    std::memcpy(dst, r.data.data(), r.data.size() * sizeof(float));
}

// dst receives the cropped image (capacity w*h*3); intr_out = fx fy cx cy,
// size_out = width height
void ref_undistort(const float* src, int w, int h, float fx, float fy, float cx, float cy, float k1,
                   float k2, float p1, float p2, float k3, float* dst, float* intr_out, int* size_out)
{
    UndistortResult r = undistortImage(host_image(src, w, h), fx, fy, cx, cy, k1, k2, p1, p2, k3);
    std::memcpy(dst, r.image.data.data(), r.image.data.size() * sizeof(float));
    intr_out[0] = r.fx;
    intr_out[1] = r.fy;
    intr_out[2] = r.cx;
    intr_out[3] = r.cy;
    size_out[0] = r.width;
    size_out[1] = r.height;
}

// ssim_eval, psnr and l1_loss of the evaluation (bindings.cpp:199-201) on
// host copies of two (H, W, 3) images: out = {psnr, ssim, l1}
void ref_eval(const float* rendered, const float* gt, int H, int W, int window, float sigma,
              float* out)
{
    MTensor r({H, W, 3}, DType::Float32), g({H, W, 3}, DType::Float32);
    std::memcpy(r.data_ptr(), rendered, r.nbytes());
    std::memcpy(g.data_ptr(), gt, g.nbytes());
    out[0] = psnr(r, g);
    out[1] = ssim_eval(r, g, window, sigma);
    out[2] = l1_loss(r, g);
}

}  // extern "C"
