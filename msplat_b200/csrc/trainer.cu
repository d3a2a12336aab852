// trainer.cu -- the trainer-level API (include/msplat_c_api.h) natively on
// the engine: a Model with its parameters, Adam moments and densification
// statistics in device buffers, the per-step host work around
// msplat_train_step, the refinement schedule, evaluation, rendering and
// model files.
//
// Reference counterparts (behaviour kept step for step):
//   msplat::Dataset / Trainer and the C API   core/src/msplat_api.mm:14-395
//   Model::Model / setupOptimizers            core/src/model.cpp:42-165
//   ensureCapacity / getDownscaleFactor       core/src/model.cpp:197-234
//   afterTrain                                core/src/model.cpp:236-296
//   prepareCam / render / fullIteration       core/src/model.cpp:490-597
//   schedulersStep                            core/src/model.cpp:179-182
//
// The host arithmetic (camera matrices, Adam bias corrections, learning-rate
// schedule, the split samples from std::mt19937 / normal_distribution, the
// camera order from std::shuffle) is the reference's, operation for
// operation, so a run makes the same decisions as the reference's trainer
// given the same data.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <numeric>
#include <random>
#include <string>
#include <vector>

#include "../../include/msplat_c_api.h"
#include "../../include/msplat_engine.h"
#include "engine.h"

namespace msp {
namespace {

constexpr int kGroupsC = 6;
constexpr float kLrInit[kGroupsC] = {0.00016f, 0.005f, 0.001f, 0.0025f, 0.000125f, 0.05f};

int num_sh_bases(int degree)
{
    switch (degree) {
        case 0: return 1;
        case 1: return 4;
        case 2: return 9;
        case 3: return 16;
        default: return 25;
    }
}

struct TDataset {
    MsplatData* data = nullptr;
    std::vector<int> train, test;  // indices into the dataset's cameras
    ~TDataset()
    {
        if (data) msplat_dataset_close(data);
    }
};

struct CamSetup {
    float fx, fy, cx, cy;
    int height, width, degree, degrees_to_use;
    int tiles[3];
    float cam_pos[3];
    float viewmat[16], projmat[16];
};

// RGB float -> RGBA8 as renderFromPoseToBuffer converts
// (msplat_api.mm:226-232): clamp to [0, 1], scale by 255, truncate.
__global__ void rgba8_kernel(const float* __restrict__ rgb, long long n, uint8_t* __restrict__ out)
{
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        uchar4 o;
        o.x = (uint8_t)(fminf(fmaxf(rgb[i * 3 + 0], 0.f), 1.f) * 255.f);
        o.y = (uint8_t)(fminf(fmaxf(rgb[i * 3 + 1], 0.f), 1.f) * 255.f);
        o.z = (uint8_t)(fminf(fmaxf(rgb[i * 3 + 2], 0.f), 1.f) * 255.f);
        o.w = 255;
        reinterpret_cast<uchar4*>(out)[i] = o;
    }
}

struct Model {
    // schedule configuration
    int numCameras = 0, numDownscales = 0, resolutionSchedule = 1, shDegree = 3;
    int shDegreeInterval = 1000, refineEvery = 100, warmupLength = 500, resetAlphaEvery = 30;
    float densifyGradThresh = 0.0002f, densifySizeThresh = 0.01f;
    int stopScreenSizeAt = 4000;
    float splitScreenSize = 0.05f;
    int maxSteps = 30000, stopSplitAt = 15000;
    bool keepCrs = false;
    float scale = 1.f, translation[3] = {0, 0, 0}, bg[3] = {0.6130f, 0.0101f, 0.3984f};

    // device state
    int rest_bases = 15;
    int num_active = 0, capacity = 0;
    float* buf[kGroupsC] = {};
    float* m[kGroupsC] = {};
    float* v[kGroupsC] = {};
    float* stats[3] = {};  // vis_counts, xys_grad_norm, max_2d_size
    float* samples = nullptr;
    bool radii_defined = false;
    int lastHeight = 0, lastWidth = 0;

    // optimiser
    int adam_step_count = 0;
    float adam_lr[kGroupsC] = {};
    float beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f;
    float means_lr_init = 0.00016f, means_lr_final = 0.0000016f;

    ~Model() { release(); }

    size_t width(int g) const
    {
        static const int w[kGroupsC] = {3, 3, 4, 3, 0, 1};
        return g == 4 ? (size_t)rest_bases * 3 : (size_t)w[g];
    }

    void release()
    {
        for (int g = 0; g < kGroupsC; g++) {
            for (float** p : {&buf[g], &m[g], &v[g]})
                if (*p) cudaFree(*p), *p = nullptr;
        }
        for (auto& s : stats)
            if (s) cudaFree(s), s = nullptr;
        if (samples) cudaFree(samples), samples = nullptr;
        capacity = 0;
    }

    // Zeroed device buffers with room for `cap` Gaussians; the first `keep`
    // rows of every array are carried over when growing.
    int allocate(int cap, int keep)
    {
        float* nb[kGroupsC] = {};
        float* nm[kGroupsC] = {};
        float* nv[kGroupsC] = {};
        float* ns[3] = {};
        float* nsmp = nullptr;
        bool ok = true;
        cudaStream_t s = engine_stream();
        cudaStreamSynchronize(s);  // queued steps still use the old buffers
        auto alloc = [&](float*& p, size_t floats) {
            if (!ok) return;
            if (cudaMalloc(&p, std::max<size_t>(floats, 1) * sizeof(float)) != cudaSuccess ||
                cudaMemsetAsync(p, 0, std::max<size_t>(floats, 1) * sizeof(float), s) != cudaSuccess) {
                cudaGetLastError();
                ok = false;
            }
        };
        for (int g = 0; g < kGroupsC; g++) {
            alloc(nb[g], (size_t)cap * width(g));
            alloc(nm[g], (size_t)cap * width(g));
            alloc(nv[g], (size_t)cap * width(g));
        }
        for (auto& st : ns) alloc(st, (size_t)cap);
        alloc(nsmp, (size_t)cap * 3);
        if (!ok) {
            for (int g = 0; g < kGroupsC; g++)
                for (float* p : {nb[g], nm[g], nv[g]})
                    if (p) cudaFree(p);
            for (float* p : ns)
                if (p) cudaFree(p);
            if (nsmp) cudaFree(nsmp);
            set_error("out of device memory for %d Gaussians", cap);
            return MSPLAT_ERR_CUDA;
        }
        if (keep > 0) {
            for (int g = 0; g < kGroupsC; g++) {
                const size_t bytes = (size_t)keep * width(g) * sizeof(float);
                cudaMemcpyAsync(nb[g], buf[g], bytes, cudaMemcpyDeviceToDevice, s);
                cudaMemcpyAsync(nm[g], m[g], bytes, cudaMemcpyDeviceToDevice, s);
                cudaMemcpyAsync(nv[g], v[g], bytes, cudaMemcpyDeviceToDevice, s);
            }
            for (int k = 0; k < 3; k++)
                cudaMemcpyAsync(ns[k], stats[k], (size_t)keep * sizeof(float), cudaMemcpyDeviceToDevice, s);
        }
        if (cudaStreamSynchronize(s) != cudaSuccess) {
            set_error("growing the model buffers failed: %s", cudaGetErrorString(cudaGetLastError()));
            return MSPLAT_ERR_CUDA;
        }
        release();
        for (int g = 0; g < kGroupsC; g++) {
            buf[g] = nb[g];
            m[g] = nm[g];
            v[g] = nv[g];
        }
        for (int k = 0; k < 3; k++) stats[k] = ns[k];
        samples = nsmp;
        capacity = cap;
        return MSPLAT_OK;
    }

    void setup_optimizers()
    {
        for (int g = 0; g < kGroupsC; g++) adam_lr[g] = kLrInit[g];
        adam_step_count = 0;
        means_lr_init = 0.00016f;
        means_lr_final = 0.0000016f;
    }

    // Model::Model: Gaussians from the dataset's point cloud.
    int init(const TDataset& ds, const MsplatConfig& c, int num_cameras)
    {
        numCameras = num_cameras;
        numDownscales = c.numDownscales;
        resolutionSchedule = c.resolutionSchedule;
        shDegree = c.shDegree;
        shDegreeInterval = c.shDegreeInterval;
        refineEvery = c.refineEvery;
        warmupLength = c.warmupLength;
        resetAlphaEvery = c.resetAlphaEvery;
        densifyGradThresh = c.densifyGradThresh;
        densifySizeThresh = c.densifySizeThresh;
        stopScreenSizeAt = c.stopScreenSizeAt;
        splitScreenSize = c.splitScreenSize;
        maxSteps = c.iterations;
        stopSplitAt = c.iterations / 2;
        keepCrs = c.keepCrs;
        std::memcpy(bg, c.bgColor, sizeof(bg));
        msplat_dataset_transform(ds.data, &scale, translation);
        const float* xyz = nullptr;
        const unsigned char* rgb = nullptr;
        const long long n = msplat_dataset_points(ds.data, &xyz, &rgb);
        if (n <= 0) {
            set_error("the dataset has no point cloud to initialise Gaussians from");
            return MSPLAT_ERR_ARG;
        }
        rest_bases = num_sh_bases(shDegree) - 1;
        int rc = allocate((int)(4 * n), 0);
        if (rc) return rc;
        num_active = (int)n;
        rc = msplat_init_gaussians(xyz, rgb, n, shDegree, buf[0], buf[1], buf[2], buf[3], buf[4],
                                   buf[5]);
        if (rc) return rc;
        setup_optimizers();
        return MSPLAT_OK;
    }

    void ensure_capacity(int needed)
    {
        if (needed <= capacity) return;
        allocate(std::max(needed, capacity * 2), num_active);
    }

    int downscale_factor(int step) const
    {
        const int remaining = numDownscales - step / resolutionSchedule;
        return 1 << std::max(remaining, 0);
    }

    int degree() const
    {
        const int b = rest_bases + 1;
        return b <= 1 ? 0 : b <= 4 ? 1 : b <= 9 ? 2 : b <= 16 ? 3 : 4;
    }

    // Model::prepareCam
    CamSetup prepare_cam(const MsplatCameraInfo& cam, int step) const
    {
        const float sf = (float)downscale_factor(step);
        CamSetup s{};
        s.fx = cam.fx / sf;
        s.fy = cam.fy / sf;
        s.cx = cam.cx / sf;
        s.cy = cam.cy / sf;
        s.height = static_cast<int>(cam.height / sf);
        s.width = static_cast<int>(cam.width / sf);
        const float fovX = 2.0f * std::atan(s.width / (2.0f * s.fx));
        const float fovY = 2.0f * std::atan(s.height / (2.0f * s.fy));
        const float* d = cam.cam_to_world;
        float R[3][3], Rinv[3][3], T[3], Tinv[3];
        for (int i = 0; i < 3; i++) {
            R[i][0] = d[i * 4 + 0];
            R[i][1] = -d[i * 4 + 1];
            R[i][2] = -d[i * 4 + 2];
            T[i] = d[i * 4 + 3];
        }
        for (int i = 0; i < 3; i++)
            for (int j = 0; j < 3; j++) Rinv[i][j] = R[j][i];
        for (int i = 0; i < 3; i++) Tinv[i] = -(Rinv[i][0] * T[0] + Rinv[i][1] * T[1] + Rinv[i][2] * T[2]);
        const float vm[16] = {Rinv[0][0], Rinv[0][1], Rinv[0][2], Tinv[0],
                              Rinv[1][0], Rinv[1][1], Rinv[1][2], Tinv[1],
                              Rinv[2][0], Rinv[2][1], Rinv[2][2], Tinv[2],
                              0,          0,          0,          1};
        const float t_p = 0.001f * std::tan(0.5f * fovY), r_p = 0.001f * std::tan(0.5f * fovX);
        const float pm[16] = {0.001f / r_p, 0, 0, 0,
                              0, 0.001f / t_p, 0, 0,
                              0, 0, (1000.0f + 0.001f) / (1000.0f - 0.001f), -1000.0f * 0.001f / (1000.0f - 0.001f),
                              0, 0, 1, 0};
        float pvm[16] = {};
        for (int i = 0; i < 4; i++)
            for (int j = 0; j < 4; j++)
                for (int k = 0; k < 4; k++) pvm[i * 4 + j] += pm[i * 4 + k] * vm[k * 4 + j];
        std::memcpy(s.viewmat, vm, sizeof(vm));
        std::memcpy(s.projmat, pvm, sizeof(pvm));
        s.degrees_to_use = std::min<int>(step / shDegreeInterval, shDegree);
        s.degree = degree();
        s.tiles[0] = (s.width + 15) / 16;
        s.tiles[1] = (s.height + 15) / 16;
        s.tiles[2] = 1;
        s.cam_pos[0] = T[0];
        s.cam_pos[1] = T[1];
        s.cam_pos[2] = T[2];
        return s;
    }

    int render(const MsplatCameraInfo& cam, int step, float** out, int* w, int* h)
    {
        const CamSetup s = prepare_cam(cam, step);
        *w = s.width;
        *h = s.height;
        return msplat_render(num_active, buf[0], buf[1], 1.0f, buf[2], s.viewmat, s.projmat, s.fx,
                             s.fy, s.cx, s.cy, (unsigned)s.height, (unsigned)s.width, s.tiles,
                             0.01f, (unsigned)s.degree, (unsigned)s.degrees_to_use, s.cam_pos,
                             buf[3], buf[4], buf[5], bg, out);
    }

    // Model::fullIteration
    int full_iteration(const MsplatCameraInfo& cam, int step, const float* gt, float ssim_weight)
    {
        const CamSetup s = prepare_cam(cam, step);
        lastHeight = s.height;
        lastWidth = s.width;
        adam_step_count++;
        const float bc1 = 1.0f - std::pow(beta1, adam_step_count);
        const float bc2 = 1.0f - std::pow(beta2, adam_step_count);
        float ss[kGroupsC], bc2s[kGroupsC];
        for (int i = 0; i < kGroupsC; i++) {
            ss[i] = adam_lr[i] / bc1;
            bc2s[i] = std::sqrt(bc2);
        }
        const float inv_max_dim = 1.0f / static_cast<float>(std::max(lastHeight, lastWidth));
        const float loss_inv_n = 1.0f / (float)(s.height * s.width * 3);
        const int32_t* radii = nullptr;
        float loss = 0;
        const int rc = msplat_train_step(
            num_active, buf[0], buf[1], 1.0f, buf[2], s.viewmat, s.projmat, s.fx, s.fy, s.cx, s.cy,
            (unsigned)s.height, (unsigned)s.width, s.tiles, 0.01f, (unsigned)s.degree,
            (unsigned)s.degrees_to_use, s.cam_pos, buf[3], buf[4], buf[5], bg, gt, nullptr,
            ssim_weight, loss_inv_n, rest_bases, kGroupsC, buf, m, v, ss, bc2s, beta1, beta2, eps,
            stats[0], stats[1], stats[2], inv_max_dim, &radii, &loss);
        if (!rc) radii_defined = true;
        return rc;
    }

    // Model::schedulersStep
    void schedulers_step(int step)
    {
        const float t = std::clamp((float)step / (float)maxSteps, 0.f, 1.f);
        adam_lr[0] = std::exp(std::log(means_lr_init) * (1.f - t) + std::log(means_lr_final) * t);
    }

    void reset_stats()
    {
        for (auto s : stats) cudaMemsetAsync(s, 0, (size_t)capacity * sizeof(float), engine_stream());
    }

    // Model::afterTrain
    int after_train(int step)
    {
        if (!radii_defined) return MSPLAT_OK;
        if (!(step % refineEvery == 0 && step > warmupLength)) return MSPLAT_OK;
        const int reset_interval = resetAlphaEvery * refineEvery;
        const bool densify = step < stopSplitAt && step % reset_interval > numCameras + refineEvery;
        if (densify) {
            ensure_capacity(3 * num_active);
            if (3 * num_active > capacity) {
                set_error("out of device memory growing to %d Gaussians", 3 * num_active);
                return MSPLAT_ERR_CUDA;
            }
            // split samples: std::normal_distribution<float> on mt19937(step)
            std::vector<float> smp((size_t)2 * num_active * 3);
            std::mt19937 rng(step);
            std::normal_distribution<float> dist(0.0f, 1.0f);
            for (auto& x : smp) x = dist(rng);
            if (cudaMemcpyAsync(samples, smp.data(), smp.size() * sizeof(float),
                                cudaMemcpyHostToDevice, engine_stream()) != cudaSuccess) {
                set_error("uploading the split samples failed");
                return MSPLAT_ERR_CUDA;
            }
            const float half_max_dim = 0.5f * static_cast<float>(std::max(lastWidth, lastHeight));
            const int check_screen = step < stopScreenSizeAt ? 1 : 0;
            const bool check_huge = step > refineEvery * resetAlphaEvery;
            const int n = msplat_densify(
                num_active, capacity, densifyGradThresh, densifySizeThresh, splitScreenSize,
                check_screen, 0.1f, 0.5f, 0.15f, check_huge ? 1 : 0, stats[1], stats[0], stats[2],
                half_max_dim, buf[0], buf[1], buf[2], buf[3], buf[4], buf[5], (int)width(4), m, v,
                nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, samples);
            if (n < 0) return n;
            num_active = n;
        }
        if (step < stopSplitAt && step % reset_interval == refineEvery) {
            const int rc = msplat_reset_opacity(buf[5], m[5], v[5], num_active);
            if (rc) return rc;
        }
        reset_stats();
        return MSPLAT_OK;
    }

    int save_checkpoint(const char* path, int step)
    {
        msplat_gpu_sync();
        return msplat_save_checkpoint(path, step, num_active, shDegree, adam_step_count, adam_lr,
                                      means_lr_init, means_lr_final, rest_bases, buf, m, v);
    }

    // Model::loadCheckpoint: buffers of 4N rows, optimiser state restored
    int load_checkpoint(const char* path)
    {
        int step = 0, n = 0, deg = 0, adam_steps = 0, rb = 0;
        float lr[kGroupsC], lr0 = 0, lr1 = 0;
        int rc = msplat_read_checkpoint_header(path, &step, &n, &deg, &adam_steps, lr, &lr0, &lr1, &rb);
        if (rc) return rc;
        msplat_gpu_sync();
        rest_bases = rb;
        if ((rc = allocate(std::max(4 * n, 1), 0))) return rc;
        rc = msplat_load_checkpoint(path, capacity, buf, m, v);
        if (rc < 0) return rc;
        num_active = n;
        adam_step_count = adam_steps;
        std::memcpy(adam_lr, lr, sizeof(lr));
        means_lr_init = lr0;
        means_lr_final = lr1;
        return step;
    }
};

struct TTrainer {
    Model model;
    MsplatConfig cfg{};
    TDataset* ds = nullptr;
    int current = 0;
    std::vector<size_t> order;
    size_t pos = 0;
    std::mt19937 rng{42};

    void shuffle()
    {
        std::shuffle(order.begin(), order.end(), rng);
        pos = 0;
    }
    size_t next_camera()
    {
        if (pos >= order.size()) shuffle();
        return order[pos++];
    }
    bool camera(bool test, int index, MsplatCameraInfo* info, int* dataset_index) const
    {
        const auto& list = test ? ds->test : ds->train;
        if (index < 0 || index >= (int)list.size()) return false;
        *dataset_index = list[index];
        return msplat_dataset_camera(ds->data, list[index], info) == MSPLAT_OK;
    }
};

MsplatPixelBuffer download_rgb(const float* dev, int w, int h)
{
    MsplatPixelBuffer pb{nullptr, 0, 0};
    if (!dev || w <= 0 || h <= 0) return pb;
    const size_t bytes = (size_t)w * h * 3 * sizeof(float);
    float* host = (float*)std::malloc(bytes);
    if (!host) return pb;
    if (msplat_copy(host, dev, bytes, 1, 1) != MSPLAT_OK) {
        std::free(host);
        return pb;
    }
    pb.data = host;
    pb.width = w;
    pb.height = h;
    return pb;
}

}  // namespace
}  // namespace msp

using namespace msp;

extern "C" {

MsplatDataset msplat_dataset_create(const char* path, float downscaleFactor, bool evalMode,
                                    int testEvery)
{
    auto ds = std::make_unique<TDataset>();
    if (msplat_dataset_open(path, nullptr, &ds->data) != MSPLAT_OK) return nullptr;
    if (msplat_dataset_load_images(ds->data, downscaleFactor) != MSPLAT_OK) return nullptr;
    const int n = msplat_dataset_num_cameras(ds->data);
    if (evalMode) {
        if (testEvery <= 0) {
            set_error("msplat_dataset_create: testEvery must be positive");
            return nullptr;
        }
        for (int i = 0; i < n; i++) (i % testEvery == 0 ? ds->test : ds->train).push_back(i);
    } else {
        ds->train.resize(n);
        std::iota(ds->train.begin(), ds->train.end(), 0);
    }
    return ds.release();
}

void msplat_dataset_destroy(MsplatDataset ds) { delete static_cast<TDataset*>(ds); }

int msplat_dataset_num_train(MsplatDataset ds)
{
    return ds ? (int)static_cast<TDataset*>(ds)->train.size() : 0;
}

int msplat_dataset_num_test(MsplatDataset ds)
{
    return ds ? (int)static_cast<TDataset*>(ds)->test.size() : 0;
}

void msplat_dataset_camera_pose(MsplatDataset ds, int cameraIndex, float camToWorld[16])
{
    auto* d = static_cast<TDataset*>(ds);
    if (!d || cameraIndex < 0 || cameraIndex >= (int)d->train.size()) return;
    MsplatCameraInfo info;
    if (msplat_dataset_camera(d->data, d->train[cameraIndex], &info) == MSPLAT_OK)
        std::memcpy(camToWorld, info.cam_to_world, sizeof(info.cam_to_world));
}

MsplatTrainer msplat_trainer_create(MsplatDataset ds, MsplatConfig config)
{
    auto* d = static_cast<TDataset*>(ds);
    if (!d) {
        set_error("msplat_trainer_create: no dataset");
        return nullptr;
    }
    {
        std::lock_guard<std::mutex> lk(engine_mutex());
        if (engine_init() != MSPLAT_OK) return nullptr;
    }
    auto t = std::make_unique<TTrainer>();
    t->cfg = config;
    t->ds = d;
    if (t->model.init(*d, config, (int)d->train.size()) != MSPLAT_OK) return nullptr;
    t->order.resize(d->train.size());
    std::iota(t->order.begin(), t->order.end(), 0);
    t->shuffle();
    return t.release();
}

void msplat_trainer_destroy(MsplatTrainer t)
{
    if (!t) return;
    msplat_gpu_sync();
    delete static_cast<TTrainer*>(t);
}

MsplatStats msplat_trainer_step(MsplatTrainer tp)
{
    MsplatStats st{0, 0, 0.f};
    auto* t = static_cast<TTrainer*>(tp);
    if (!t || t->order.empty()) {
        set_error("msplat_trainer_step: no trainer or no training cameras");
        return st;
    }
    t->current++;
    const size_t ci = t->next_camera();
    const int dsi = t->ds->train[ci];
    MsplatCameraInfo cam;
    msplat_dataset_camera(t->ds->data, dsi, &cam);
    const int factor = t->model.downscale_factor(t->current);
    const float* gt = nullptr;
    int gw = 0, gh = 0;
    if (msplat_dataset_gt(t->ds->data, dsi, factor, &gt, &gw, &gh) != MSPLAT_OK) return st;
    const auto t0 = std::chrono::high_resolution_clock::now();
    if (t->model.full_iteration(cam, t->current, gt, t->cfg.ssimWeight) != MSPLAT_OK) return st;
    t->model.schedulers_step(t->current);
    if (t->model.after_train(t->current) != MSPLAT_OK) return st;
    msplat_commit();
    const auto t1 = std::chrono::high_resolution_clock::now();
    st.iteration = t->current;
    st.splatCount = t->model.num_active;
    st.msPerStep = std::chrono::duration_cast<std::chrono::microseconds>(t1 - t0).count() / 1000.0f;
    return st;
}

void msplat_trainer_train(MsplatTrainer tp)
{
    auto* t = static_cast<TTrainer*>(tp);
    if (!t) return;
    while (t->current < t->cfg.iterations) {
        const MsplatStats s = msplat_trainer_step(tp);
        if (s.iteration == 0) break;  // failed: msplat_last_error says why
    }
}

MsplatEvalMetrics msplat_trainer_evaluate(MsplatTrainer tp)
{
    MsplatEvalMetrics out{0.f, 0.f, 0.f, 0, 0};
    auto* t = static_cast<TTrainer*>(tp);
    if (!t || t->ds->test.empty()) return out;
    double sp = 0, ss = 0, sl = 0;
    const int n = (int)t->ds->test.size();
    const int step = t->cfg.iterations;
    for (int i = 0; i < n; i++) {
        MsplatCameraInfo cam;
        int dsi = 0;
        if (!t->camera(true, i, &cam, &dsi)) return out;
        float* img = nullptr;
        int w = 0, h = 0;
        if (t->model.render(cam, step, &img, &w, &h) != MSPLAT_OK) return out;
        const float* gt = nullptr;
        int gw = 0, gh = 0;
        if (msplat_dataset_gt(t->ds->data, dsi, t->model.downscale_factor(step), &gt, &gw, &gh) !=
            MSPLAT_OK)
            return out;
        if (gw != w || gh != h) {
            set_error("evaluate: render %dx%d vs ground truth %dx%d", w, h, gw, gh);
            return out;
        }
        float p = 0, s = 0, l = 0;
        if (msplat_eval_metrics(img, gt, h, w, 11, 1.5f, &p, &s, &l) != MSPLAT_OK) return out;
        sp += p;
        ss += s;
        sl += l;
    }
    out.psnr = (float)(sp / n);
    out.ssim = (float)(ss / n);
    out.l1 = (float)(sl / n);
    out.numTest = n;
    out.numGaussians = t->model.num_active;
    return out;
}

MsplatPixelBuffer msplat_trainer_render(MsplatTrainer tp, int cameraIndex, bool useTest)
{
    auto* t = static_cast<TTrainer*>(tp);
    MsplatCameraInfo cam;
    int dsi = 0;
    if (!t || !t->camera(useTest, cameraIndex, &cam, &dsi)) return MsplatPixelBuffer{nullptr, 0, 0};
    float* img = nullptr;
    int w = 0, h = 0;
    if (t->model.render(cam, t->current, &img, &w, &h) != MSPLAT_OK) return MsplatPixelBuffer{nullptr, 0, 0};
    return download_rgb(img, w, h);
}

MsplatPixelBuffer msplat_trainer_render_pose(MsplatTrainer tp, const float camToWorld[16],
                                             int refCameraIndex)
{
    auto* t = static_cast<TTrainer*>(tp);
    MsplatCameraInfo cam;
    int dsi = 0;
    if (!t || !camToWorld || !t->camera(false, refCameraIndex, &cam, &dsi))
        return MsplatPixelBuffer{nullptr, 0, 0};
    std::memcpy(cam.cam_to_world, camToWorld, sizeof(cam.cam_to_world));
    float* img = nullptr;
    int w = 0, h = 0;
    if (t->model.render(cam, t->current, &img, &w, &h) != MSPLAT_OK) return MsplatPixelBuffer{nullptr, 0, 0};
    return download_rgb(img, w, h);
}

void msplat_trainer_render_pose_to_buffer(MsplatTrainer tp, const float camToWorld[16],
                                          int refCameraIndex, uint8_t* outRGBA, int* outWidth,
                                          int* outHeight)
{
    auto* t = static_cast<TTrainer*>(tp);
    MsplatCameraInfo cam;
    int dsi = 0;
    if (!t || !camToWorld || !t->camera(false, refCameraIndex, &cam, &dsi)) {
        if (outWidth) *outWidth = 0;
        if (outHeight) *outHeight = 0;
        return;
    }
    std::memcpy(cam.cam_to_world, camToWorld, sizeof(cam.cam_to_world));
    float* img = nullptr;
    int w = 0, h = 0;
    if (t->model.render(cam, t->current, &img, &w, &h) != MSPLAT_OK) {
        w = h = 0;
    }
    if (outWidth) *outWidth = w;
    if (outHeight) *outHeight = h;
    if (!outRGBA || !img || w <= 0 || h <= 0) return;
    const long long px = (long long)w * h;
    uint8_t* dev = nullptr;
    std::lock_guard<std::mutex> lk(engine_mutex());
    cudaStream_t s = engine_stream();
    if (cudaMallocAsync(&dev, (size_t)px * 4, s) != cudaSuccess) {
        cudaGetLastError();
        set_error("render_pose_to_buffer: out of device memory");
        return;
    }
    rgba8_kernel<<<(int)std::min<long long>((px + 255) / 256, 148 * 16), 256, 0, s>>>(img, px, dev);
    engine_add_launches(1);
    cudaMemcpyAsync(outRGBA, dev, (size_t)px * 4, cudaMemcpyDeviceToHost, s);
    cudaFreeAsync(dev, s);
    cudaStreamSynchronize(s);
}

void msplat_trainer_export_ply(MsplatTrainer tp, const char* path)
{
    auto* t = static_cast<TTrainer*>(tp);
    if (!t) return;
    Model& md = t->model;
    msplat_save_ply(path, t->current, md.num_active, md.rest_bases, md.buf, md.keepCrs ? 1 : 0,
                    md.scale, md.translation);
}

void msplat_trainer_export_splat(MsplatTrainer tp, const char* path)
{
    auto* t = static_cast<TTrainer*>(tp);
    if (!t) return;
    Model& md = t->model;
    msplat_save_splat(path, md.num_active, md.buf, md.keepCrs ? 1 : 0, md.scale, md.translation);
}

void msplat_trainer_save_checkpoint(MsplatTrainer tp, const char* path)
{
    auto* t = static_cast<TTrainer*>(tp);
    if (t) t->model.save_checkpoint(path, t->current);
}

int msplat_trainer_load_checkpoint_ex(MsplatTrainer tp, const char* path, int reshuffle)
{
    auto* t = static_cast<TTrainer*>(tp);
    if (!t) return -1;
    const int step = t->model.load_checkpoint(path);
    if (step < 0) return -1;
    t->current = step;
    if (reshuffle) t->shuffle();
    return step;
}

// msplat::Trainer::loadCheckpoint re-shuffles the camera order on resume
// (msplat_api.mm:250-255); the Python binding's load_checkpoint does not.
int msplat_trainer_load_checkpoint(MsplatTrainer tp, const char* path)
{
    return msplat_trainer_load_checkpoint_ex(tp, path, 1);
}

int msplat_trainer_splat_count(MsplatTrainer tp)
{
    auto* t = static_cast<TTrainer*>(tp);
    return t ? t->model.num_active : 0;
}

int msplat_trainer_iteration(MsplatTrainer tp)
{
    auto* t = static_cast<TTrainer*>(tp);
    return t ? t->current : 0;
}

MsplatData* msplat_dataset_data(void* c_api_dataset)
{
    return c_api_dataset ? static_cast<TDataset*>(c_api_dataset)->data : nullptr;
}

int msplat_dataset_indices(void* c_api_dataset, int test, int* out, int max_out)
{
    auto* d = static_cast<TDataset*>(c_api_dataset);
    if (!d) return MSPLAT_ERR_ARG;
    const auto& list = test ? d->test : d->train;
    for (int i = 0; i < (int)list.size() && i < max_out && out; i++) out[i] = list[i];
    return (int)list.size();
}

void msplat_sync(void) { msplat_gpu_sync(); }

void msplat_cleanup(void) { cleanup_msplat_cuda(); }

}  // extern "C"
