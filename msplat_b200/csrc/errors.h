// errors.h -- the device error word and how a render call reports it.
//
// Kernels OR bits into one int in device memory; the host reads it back
// after the work finishes.  This header has no CUDA dependency so the
// decoding can be compiled and checked on a machine without a GPU.
#pragma once

#include "../../include/msplat_engine.h"

namespace msp {

// Device error word bits.
enum ErrorBits : int {
    kErrIsectOverflow = 1,   // intersections exceeded the key buffer
    kErrStageTimeout = 2,    // a bulk copy into shared memory did not complete in time
};

// Status of a synchronous render whose error word read back as `err`.
// Any bit makes the image incomplete, so every nonzero word is a failure:
//  * a shared-memory copy that timed out left its block's Gaussians
//    culled -> MSPLAT_ERR_CUDA (a device-side failure);
//  * an intersection overflow alone -> MSPLAT_ERR_OVERFLOW (fewer Gaussians
//    or a smaller image fit);
//  * bits this build does not know -> MSPLAT_ERR_CUDA.
// `what` receives a sentence for the error message (nullptr when err == 0).
inline int render_status(int err, const char** what)
{
    *what = nullptr;
    if (err == 0) return MSPLAT_OK;
    if (err & kErrStageTimeout) {
        *what = (err & kErrIsectOverflow)
                    ? "a shared-memory bulk copy timed out and the intersections overflowed"
                    : "a shared-memory bulk copy timed out and its Gaussians were dropped";
        return MSPLAT_ERR_CUDA;
    }
    if (err == kErrIsectOverflow) {
        *what = "the tile intersections overflowed the key buffer";
        return MSPLAT_ERR_OVERFLOW;
    }
    *what = "the device error word holds bits this build does not define";
    return MSPLAT_ERR_CUDA;
}

}  // namespace msp
