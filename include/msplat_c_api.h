/*
 * msplat_c_api.h -- the trainer-level C API, the same names, structs and
 * argument meaning as the reference's core/include/msplat_c_api.h (its
 * Swift-facing wrapper of msplat::Trainer, core/src/msplat_api.mm:279-395),
 * implemented natively on the CUDA engine (msplat_b200/csrc/trainer.cu).
 *
 * A program written against the reference's C API links against
 * libmsplat_b200.so instead and runs unchanged.  Differences, all additive:
 * a failure returns NULL / zeroed results and sets msplat_last_error()
 * (include/msplat_engine.h) where the reference would throw through the C
 * boundary; images stay resident in device memory.
 */
#ifndef MSPLAT_C_API_H
#define MSPLAT_C_API_H

#include <stdbool.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* TrainingConfig (python/bindings.cpp:24-43, msplat_api.hpp:14-31). */
typedef struct {
    int iterations;
    int shDegree;
    int shDegreeInterval;
    float ssimWeight;
    int numDownscales;
    int resolutionSchedule;
    int refineEvery;
    int warmupLength;
    int resetAlphaEvery;
    float densifyGradThresh;
    float densifySizeThresh;
    int stopScreenSizeAt;
    float splitScreenSize;
    bool keepCrs;
    float downscaleFactor;
    float bgColor[3];
} MsplatConfig;

/* The reference's defaults (msplat_c_api.h msplat_default_config). */
static inline MsplatConfig msplat_default_config(void)
{
    MsplatConfig c;
    c.iterations = 30000;
    c.shDegree = 3;
    c.shDegreeInterval = 1000;
    c.ssimWeight = 0.2f;
    c.numDownscales = 2;
    c.resolutionSchedule = 3000;
    c.refineEvery = 100;
    c.warmupLength = 500;
    c.resetAlphaEvery = 30;
    c.densifyGradThresh = 0.0002f;
    c.densifySizeThresh = 0.01f;
    c.stopScreenSizeAt = 4000;
    c.splitScreenSize = 0.05f;
    c.keepCrs = false;
    c.downscaleFactor = 1.0f;
    c.bgColor[0] = 0.6130f;
    c.bgColor[1] = 0.0101f;
    c.bgColor[2] = 0.3984f;
    return c;
}

typedef struct {
    int iteration;
    int splatCount;
    float msPerStep; /* host wall time of the step's enqueue, as the reference measures */
} MsplatStats;

typedef struct {
    float psnr;
    float ssim;
    float l1;
    int numTest;
    int numGaussians;
} MsplatEvalMetrics;

/* RGB float32 HWC; the caller free()s data. */
typedef struct {
    float *data;
    int width;
    int height;
} MsplatPixelBuffer;

typedef void *MsplatDataset;
typedef void *MsplatTrainer;

/* Dataset(path, downscaleFactor, evalMode, testEvery): load the layout
 * (COLMAP, Nerfstudio, Polycam), every image into device memory, and split
 * (every testEvery-th camera held out when evalMode).  NULL on failure. */
MsplatDataset msplat_dataset_create(const char *path, float downscaleFactor, bool evalMode,
                                    int testEvery);
void msplat_dataset_destroy(MsplatDataset ds);
int msplat_dataset_num_train(MsplatDataset ds);
int msplat_dataset_num_test(MsplatDataset ds);
/* Camera-to-world pose of training camera `cameraIndex` (row-major 4x4). */
void msplat_dataset_camera_pose(MsplatDataset ds, int cameraIndex, float camToWorld[16]);

/* Trainer over a dataset (which must outlive it): Gaussians initialised
 * from the dataset's point cloud as Model::Model does.  NULL on failure. */
MsplatTrainer msplat_trainer_create(MsplatDataset ds, MsplatConfig config);
void msplat_trainer_destroy(MsplatTrainer t);

MsplatStats msplat_trainer_step(MsplatTrainer t);
/* Steps until config.iterations. */
void msplat_trainer_train(MsplatTrainer t);
/* Mean PSNR / SSIM / L1 over the held-out cameras (zeros when none). */
MsplatEvalMetrics msplat_trainer_evaluate(MsplatTrainer t);
MsplatPixelBuffer msplat_trainer_render(MsplatTrainer t, int cameraIndex, bool useTest);
MsplatPixelBuffer msplat_trainer_render_pose(MsplatTrainer t, const float camToWorld[16],
                                             int refCameraIndex);
/* Render into caller-provided RGBA8 (width*height*4 bytes); outRGBA = NULL
 * returns the dimensions only. */
void msplat_trainer_render_pose_to_buffer(MsplatTrainer t, const float camToWorld[16],
                                          int refCameraIndex, uint8_t *outRGBA, int *outWidth,
                                          int *outHeight);
void msplat_trainer_export_ply(MsplatTrainer t, const char *path);
void msplat_trainer_export_splat(MsplatTrainer t, const char *path);
void msplat_trainer_save_checkpoint(MsplatTrainer t, const char *path);
/* Returns the checkpoint's iteration (-1 on failure). */
int msplat_trainer_load_checkpoint(MsplatTrainer t, const char *path);
int msplat_trainer_splat_count(MsplatTrainer t);
int msplat_trainer_iteration(MsplatTrainer t);

void msplat_set_metallib_path(const char *path); /* accepted and ignored */
void msplat_sync(void);
void msplat_cleanup(void);

#ifdef __cplusplus
}
#endif

#endif
