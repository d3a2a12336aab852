// msplat_api.hpp -- the reference's C++ API (core/include/msplat_api.hpp:
// namespace msplat: Config, Stats, EvalMetrics, PixelBuffer, Dataset,
// Trainer, sync, cleanup), header-only over the native trainer C API
// (include/msplat_c_api.h, implemented in libmsplat_b200.so).
//
// Same class names, members and method signatures, so C++ (and Swift C++
// interop) code written against the reference's header compiles against
// this one.  Where the reference would fail inside its engine, these throw
// std::runtime_error carrying msplat_last_error().
#pragma once

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>

#include "msplat_c_api.h"
#include "msplat_engine.h"

namespace msplat {

struct Config {
    int iterations = 30000;
    int shDegree = 3;
    int shDegreeInterval = 1000;
    float ssimWeight = 0.2f;
    int numDownscales = 2;
    int resolutionSchedule = 3000;
    int refineEvery = 100;
    int warmupLength = 500;
    int resetAlphaEvery = 30;
    float densifyGradThresh = 0.0002f;
    float densifySizeThresh = 0.01f;
    int stopScreenSizeAt = 4000;
    float splitScreenSize = 0.05f;
    bool keepCrs = false;
    float downscaleFactor = 1.0f;
    float bgColor[3] = {0.6130f, 0.0101f, 0.3984f};
};

struct Stats {
    int iteration = 0;
    int splatCount = 0;
    float msPerStep = 0.0f;
};

struct EvalMetrics {
    float psnr = 0.0f;
    float ssim = 0.0f;
    float l1 = 0.0f;
    int numTest = 0;
    int numGaussians = 0;
};

// Rendered RGB float32 HWC image; owns its malloc'd pixels.
struct PixelBuffer {
    float* data = nullptr;
    int width = 0;
    int height = 0;

    PixelBuffer() = default;
    PixelBuffer(float* d, int w, int h) : data(d), width(w), height(h) {}
    PixelBuffer(const PixelBuffer&) = delete;
    PixelBuffer& operator=(const PixelBuffer&) = delete;
    PixelBuffer(PixelBuffer&& o) noexcept : data(o.data), width(o.width), height(o.height)
    {
        o.data = nullptr;
    }
    PixelBuffer& operator=(PixelBuffer&& o) noexcept
    {
        if (this != &o) {
            std::free(data);
            data = o.data;
            width = o.width;
            height = o.height;
            o.data = nullptr;
        }
        return *this;
    }
    ~PixelBuffer() { std::free(data); }
};

namespace detail {
[[noreturn]] inline void fail(const char* what)
{
    throw std::runtime_error(std::string(what) + ": " + msplat_last_error());
}
inline MsplatConfig to_c(const Config& c)
{
    MsplatConfig o = msplat_default_config();
    o.iterations = c.iterations;
    o.shDegree = c.shDegree;
    o.shDegreeInterval = c.shDegreeInterval;
    o.ssimWeight = c.ssimWeight;
    o.numDownscales = c.numDownscales;
    o.resolutionSchedule = c.resolutionSchedule;
    o.refineEvery = c.refineEvery;
    o.warmupLength = c.warmupLength;
    o.resetAlphaEvery = c.resetAlphaEvery;
    o.densifyGradThresh = c.densifyGradThresh;
    o.densifySizeThresh = c.densifySizeThresh;
    o.stopScreenSizeAt = c.stopScreenSizeAt;
    o.splitScreenSize = c.splitScreenSize;
    o.keepCrs = c.keepCrs;
    o.downscaleFactor = c.downscaleFactor;
    std::memcpy(o.bgColor, c.bgColor, sizeof(o.bgColor));
    return o;
}
inline PixelBuffer take(MsplatPixelBuffer b) { return PixelBuffer(b.data, b.width, b.height); }
}  // namespace detail

class Dataset {
public:
    Dataset(const std::string& path, float downscaleFactor, bool evalMode, int testEvery)
        : h_(msplat_dataset_create(path.c_str(), downscaleFactor, evalMode, testEvery))
    {
        if (!h_) detail::fail("msplat::Dataset");
    }
    ~Dataset()
    {
        if (h_) msplat_dataset_destroy(h_);
    }
    Dataset(const Dataset&) = delete;
    Dataset& operator=(const Dataset&) = delete;
    Dataset(Dataset&& o) noexcept : h_(o.h_) { o.h_ = nullptr; }
    Dataset& operator=(Dataset&& o) noexcept
    {
        if (this != &o) {
            if (h_) msplat_dataset_destroy(h_);
            h_ = o.h_;
            o.h_ = nullptr;
        }
        return *this;
    }

    int numTrain() const { return msplat_dataset_num_train(h_); }
    int numTest() const { return msplat_dataset_num_test(h_); }
    void cameraPose(int index, float camToWorld[16]) const
    {
        msplat_dataset_camera_pose(h_, index, camToWorld);
    }
    void* _handle() const { return h_; }

private:
    MsplatDataset h_ = nullptr;
};

class Trainer {
public:
    Trainer(Dataset& dataset, const Config& config)
        : t_(msplat_trainer_create(dataset._handle(), detail::to_c(config))), iterations_(config.iterations)
    {
        if (!t_) detail::fail("msplat::Trainer");
    }
    ~Trainer()
    {
        if (t_) msplat_trainer_destroy(t_);
    }
    Trainer(const Trainer&) = delete;
    Trainer& operator=(const Trainer&) = delete;

    Stats step()
    {
        const MsplatStats s = msplat_trainer_step(t_);
        if (s.iteration == 0) detail::fail("msplat::Trainer::step");
        return Stats{s.iteration, s.splatCount, s.msPerStep};
    }
    // Steps until config.iterations (callbacks are the caller's: poll iteration()).
    void train(int /*callbackEvery*/)
    {
        while (iteration() < iterations_) step();
    }
    EvalMetrics evaluate()
    {
        const MsplatEvalMetrics m = msplat_trainer_evaluate(t_);
        return EvalMetrics{m.psnr, m.ssim, m.l1, m.numTest, m.numGaussians};
    }
    PixelBuffer render(int cameraIndex, bool useTest)
    {
        return detail::take(msplat_trainer_render(t_, cameraIndex, useTest));
    }
    PixelBuffer renderFromPose(const float camToWorld[16], int refCameraIndex)
    {
        return detail::take(msplat_trainer_render_pose(t_, camToWorld, refCameraIndex));
    }
    void renderFromPoseToBuffer(const float camToWorld[16], int refCameraIndex, uint8_t* outRGBA,
                                int* outWidth, int* outHeight)
    {
        msplat_trainer_render_pose_to_buffer(t_, camToWorld, refCameraIndex, outRGBA, outWidth,
                                             outHeight);
    }
    void exportPly(const std::string& path) { msplat_trainer_export_ply(t_, path.c_str()); }
    void exportSplat(const std::string& path) { msplat_trainer_export_splat(t_, path.c_str()); }
    void saveCheckpoint(const std::string& path) { msplat_trainer_save_checkpoint(t_, path.c_str()); }
    int loadCheckpoint(const std::string& path)
    {
        const int step = msplat_trainer_load_checkpoint(t_, path.c_str());
        if (step < 0) detail::fail("msplat::Trainer::loadCheckpoint");
        return step;
    }
    int splatCount() const { return msplat_trainer_splat_count(t_); }
    int iteration() const { return msplat_trainer_iteration(t_); }

private:
    MsplatTrainer t_ = nullptr;
    int iterations_ = 0;
};

inline void sync() { msplat_sync(); }
inline void cleanup() { msplat_cleanup(); }

}  // namespace msplat
