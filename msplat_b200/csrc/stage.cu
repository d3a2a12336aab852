// stage.cu -- per-step host inputs copied to the device behind the previous
// step's kernels.
//
// The reference's ground-truth image is host-visible memory the Metal
// kernels read in place (Apple unified memory).  A CUDA host that keeps its
// images in host memory has to copy each step's image to the device; on
// the engine's own stream that copy would sit between two steps' kernels.
// msplat_stage_input instead copies on a dedicated copy stream into one of
// two device staging buffers, so step s's upload runs while step s-1
// computes:
//   * the copy of slot k waits for the kernels of the step that last read
//     slot k (two stagings ago), not for the step in flight;
//   * the engine stream waits for the copy before the kernels queued next.
// No counterpart in the reference's interface.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "../../include/msplat_engine.h"
#include "engine.h"

namespace msp {
namespace {

struct Stage {
    bool ready = false;
    cudaStream_t copy = nullptr;
    void* buf[2] = {nullptr, nullptr};
    size_t bytes[2] = {0, 0};
    cudaEvent_t consumed[2] = {};  // engine stream: work queued up to the next staging
    cudaEvent_t copied[2] = {};    // copy stream: the slot's data has arrived
    bool consumed_recorded[2] = {false, false};
    int next = 0;
    long long stagings = 0;
};

Stage s_stage;

#define STAGE_CUDA(expr)                                                               \
    do {                                                                               \
        cudaError_t e_ = (expr);                                                       \
        if (e_ != cudaSuccess) {                                                       \
            set_error("msplat_stage_input: %s: %s", #expr, cudaGetErrorString(e_));   \
            return MSPLAT_ERR_CUDA;                                                    \
        }                                                                              \
    } while (0)

int stage_init()
{
    Stage& S = s_stage;
    if (S.ready) return MSPLAT_OK;
    STAGE_CUDA(cudaStreamCreateWithFlags(&S.copy, cudaStreamNonBlocking));
    for (int k = 0; k < 2; k++) {
        STAGE_CUDA(cudaEventCreateWithFlags(&S.consumed[k], cudaEventDisableTiming));
        STAGE_CUDA(cudaEventCreateWithFlags(&S.copied[k], cudaEventDisableTiming));
    }
    S.ready = true;
    return MSPLAT_OK;
}

}  // namespace

void stage_release()
{
    Stage& S = s_stage;
    if (!S.ready) return;
    cudaStreamSynchronize(S.copy);
    for (int k = 0; k < 2; k++) {
        if (S.buf[k]) cudaFree(S.buf[k]);
        S.buf[k] = nullptr;
        S.bytes[k] = 0;
        S.consumed_recorded[k] = false;
    }
    S.next = 0;
    S.stagings = 0;
}

}  // namespace msp

using namespace msp;

extern "C" {

int msplat_stage_input(const void* host, size_t bytes, const void** dev_out)
{
    if (!host || !dev_out || bytes == 0) {
        set_error("msplat_stage_input: invalid arguments");
        return MSPLAT_ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(engine_mutex());
    int rc = engine_init();
    if (rc) return rc;
    if ((rc = stage_init())) return rc;
    Stage& S = s_stage;
    const cudaStream_t es = engine_stream();
    const int k = S.next;
    const int other = k ^ 1;
    // everything queued so far on the engine stream includes the step that
    // read the other slot: it is the other slot's last reader
    if (S.stagings > 0) {
        STAGE_CUDA(cudaEventRecord(S.consumed[other], es));
        S.consumed_recorded[other] = true;
    }
    if (S.bytes[k] < bytes) {
        // growing: nothing may still read the old buffer
        if (S.consumed_recorded[k]) STAGE_CUDA(cudaEventSynchronize(S.consumed[k]));
        if (S.buf[k]) STAGE_CUDA(cudaFree(S.buf[k]));
        S.buf[k] = nullptr;
        S.bytes[k] = 0;
        STAGE_CUDA(cudaMalloc(&S.buf[k], bytes));
        S.bytes[k] = bytes;
    }
    if (S.consumed_recorded[k]) STAGE_CUDA(cudaStreamWaitEvent(S.copy, S.consumed[k], 0));
    STAGE_CUDA(cudaMemcpyAsync(S.buf[k], host, bytes, cudaMemcpyHostToDevice, S.copy));
    STAGE_CUDA(cudaEventRecord(S.copied[k], S.copy));
    STAGE_CUDA(cudaStreamWaitEvent(es, S.copied[k], 0));
    S.next = other;
    S.stagings++;
    *dev_out = S.buf[k];
    return MSPLAT_OK;
}

}  // extern "C"
