// engine.cu -- host driver of the CUDA engine and the C-ABI seam
// (include/msplat_engine.h).  Plays the role of msplat's Metal host driver
// (core/metal/msplat_metal.mm): a process-wide buffer cache reused across
// steps (FusedTensorCache, msplat_metal.mm:348-454), the dispatch order of
// msplat_train_step (:771-1330) and forward_pipeline (:462-750), and the
// depth-chunk rule (:873-889).  All work goes to one CUDA stream; per-step
// scalars travel in a parameter block copied from a pinned ring.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/msplat_engine.h"
#include "engine.h"

namespace msp {

static thread_local std::string t_last_error;

void set_error(const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
}

#define MSP_CUDA(expr)                                                                    \
    do {                                                                                  \
        cudaError_t e_ = (expr);                                                          \
        if (e_ != cudaSuccess) {                                                          \
            set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__,   \
                      __LINE__);                                                          \
            return MSPLAT_ERR_CUDA;                                                       \
        }                                                                                 \
    } while (0)

constexpr int kRing = 8;
constexpr unsigned kChunkHost = 512;  // depth chunk, as kChunk in msp_math.cuh
constexpr int kStages = 6;
static const char* kStageNames[kStages] = {"proj_sh_fwd", "bin_sort", "rast_fwd",
                                           "loss_fwd_bwd", "rast_bwd", "proj_bwd_adam"};

// The step's parameters and, after them, the step's counters: one upload per
// step sets the parameters and zeroes the counters, one readback returns
// them (loss sum, error bits, intersections, the largest tile).
struct alignas(64) ParamSlot {
    StepParams p;
    alignas(64) int counters[16];
};
constexpr int kCtrLoss = 0, kCtrErr = 4, kCtrIsect = 8, kCtrMaxTile = 9, kCtrRead = 12;
static_assert(offsetof(ParamSlot, p) == 0, "the parameters lead the slot");

struct Engine {
    bool ready = false;
    int device = -1;
    cudaStream_t own_stream = nullptr;
    cudaStream_t user_stream = nullptr;
    bool user_stream_set = false;
    // allocated sizes
    long long cap_N = 0, cap_grad_N = 0, cap_pix = 0, cap_T = 0, cap_isect = 0, cap_chunk = 0;
    Buffers B{};
    ParamSlot* d_slot = nullptr;
    StepParams* d_params = nullptr;  // &d_slot->p
    ParamSlot* h_ring = nullptr;
    cudaEvent_t ring_ev[kRing] = {};
    int ring_pos = 0;
    // readback: pinned copy of the counters (kCtrRead ints)
    int* h_ctr = nullptr;
    cudaEvent_t readback_ev = nullptr;
    SideStream side{};
    bool readback_pending = false;
    bool readback_has_loss = false;  // a training step's readback (a render has no loss)
    float last_loss = 0.f;
    double last_loss_scale = 1.0;
    long long growth_isect = 0;  // requested capacity after an overflow
    int last_k_max = 0;          // depth chunks of the last forward (0: none yet)
    int last_max_tile = 0;       // largest tile count of the last view read back
    long long last_isect = 0;    // its intersections
    long long last_isect_n = 0;  // and its Gaussians
    long long readback_n = 0;    // Gaussians of the view whose readback is queued
    bool last_prefix_sort = false;  // the last forward sorted long lists' fronts only
    bool last_dense_bins = false;   // the last forward used dense binning
    int last_num_tiles = 0;
    unsigned long long* d_work = nullptr;  // msplat_count_raster_work's counters
    // timing
    bool timing = false;
    cudaEvent_t st_ev[kStages + 1][kRing] = {};
    int st_pos = 0;
    std::vector<double> step_times;
    std::vector<double> stage_times[kStages];
    std::vector<int> pending_timing;  // ring slots with recorded events
    long long launches = 0;

    cudaStream_t stream() const { return user_stream_set ? user_stream : own_stream; }
};

static Engine g;
// Device address of the counters that follow the parameters in d_slot.
static int* d_counters()
{
    return reinterpret_cast<int*>(reinterpret_cast<char*>(g.d_slot) + offsetof(ParamSlot, counters));
}

static std::mutex g_mu;

static int init_engine()
{
    if (g.ready) return MSPLAT_OK;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n <= 0) {
        set_error("no CUDA device available (%s); the engine has no CPU path",
                  e == cudaSuccess ? "0 devices" : cudaGetErrorString(e));
        return MSPLAT_ERR_CUDA;
    }
    MSP_CUDA(cudaGetDevice(&g.device));
    // A blocking stream: ordered with the legacy default stream, so callers
    // that never pick a stream still see their own prior work completed.
    MSP_CUDA(cudaStreamCreateWithFlags(&g.own_stream, cudaStreamDefault));
    MSP_CUDA(cudaMalloc(&g.d_slot, sizeof(ParamSlot)));
    MSP_CUDA(cudaMemset(g.d_slot, 0, sizeof(ParamSlot)));
    g.d_params = reinterpret_cast<StepParams*>(g.d_slot);
    MSP_CUDA(cudaMallocHost(&g.h_ring, sizeof(ParamSlot) * kRing));
    for (int i = 0; i < kRing; i++) MSP_CUDA(cudaEventCreateWithFlags(&g.ring_ev[i], cudaEventDisableTiming));
    MSP_CUDA(cudaMallocHost(&g.h_ctr, sizeof(int) * kCtrRead));
    memset(g.h_ctr, 0, sizeof(int) * kCtrRead);
    MSP_CUDA(cudaEventCreateWithFlags(&g.readback_ev, cudaEventDisableTiming));
    MSP_CUDA(cudaStreamCreateWithFlags(&g.side.stream, cudaStreamNonBlocking));
    MSP_CUDA(cudaEventCreateWithFlags(&g.side.fork, cudaEventDisableTiming));
    MSP_CUDA(cudaEventCreateWithFlags(&g.side.join, cudaEventDisableTiming));
    for (int s = 0; s <= kStages; s++)
        for (int r = 0; r < kRing; r++) MSP_CUDA(cudaEventCreate(&g.st_ev[s][r]));
    g.B.loss_sum = reinterpret_cast<float*>(d_counters() + kCtrLoss);
    g.B.err = d_counters() + kCtrErr;
    g.B.isect_total = d_counters() + kCtrIsect;
    g.B.max_tile = d_counters() + kCtrMaxTile;
    MSP_CUDA(cudaDeviceSynchronize());
    g.ready = true;
    return MSPLAT_OK;
}

// Access for the other host files of the engine (dp_peer.cu).
std::mutex& engine_mutex() { return g_mu; }
int engine_init() { return init_engine(); }
cudaStream_t engine_stream() { return g.stream(); }
const SideStream& engine_side() { return g.side; }
void engine_add_launches(int n) { g.launches += n; }

template <typename T>
static int realloc_dev(T*& p, size_t count)
{
    if (p) cudaFree(p);
    p = nullptr;
    if (count == 0) count = 1;
    MSP_CUDA(cudaMalloc(&p, count * sizeof(T)));
    return MSPLAT_OK;
}

static void free_buffers()
{
    Buffers& B = g.B;
    void* ptrs[] = {B.proj.xy, B.proj.depth, B.proj.radii, B.proj.conic_op, B.proj.rgb, B.proj.rect,
                    B.proj.sh_mean, B.tile_count, B.tile_offset, B.tile_order, B.tile_sorted, B.tile_flag, B.keys, B.keys_alt,
                    B.sorted_ids, B.out_img,
                    B.final_T, B.final_idx, B.v_rendered, B.grad_acc,
                    B.chunk_T, B.chunk_C, B.chunk_idx, B.prefix_T, B.after_C};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    float* ls = B.loss_sum;
    int* er = B.err;
    int* it = B.isect_total;
    int* mt = B.max_tile;
    B = Buffers{};
    B.loss_sum = ls;
    B.err = er;
    B.isect_total = it;
    B.max_tile = mt;
    g.cap_N = g.cap_grad_N = g.cap_pix = g.cap_T = g.cap_isect = g.cap_chunk = 0;
}

// Buffer cache: grow-only, like FusedTensorCache::ensure_* (msplat_metal.mm:383-452).
static int ensure(long long N, long long W, long long H, long long T, int K, bool train)
{
    Buffers& B = g.B;
    int rc;
    if (N > g.cap_N) {
        long long n = std::max(N, g.cap_N + g.cap_N / 4);
        if ((rc = realloc_dev(B.proj.xy, n))) return rc;
        if ((rc = realloc_dev(B.proj.depth, n))) return rc;
        if ((rc = realloc_dev(B.proj.radii, n))) return rc;
        if ((rc = realloc_dev(B.proj.conic_op, n))) return rc;
        if ((rc = realloc_dev(B.proj.rgb, n))) return rc;
        if ((rc = realloc_dev(B.proj.rect, n))) return rc;
        g.cap_N = n;
    }
    if (train && N > g.cap_grad_N) {
        long long n = std::max(N, g.cap_N);
        if ((rc = realloc_dev(B.grad_acc, (size_t)n * kGradStride))) return rc;
        if ((rc = realloc_dev(B.proj.sh_mean, (size_t)n * 3))) return rc;
        g.cap_grad_N = n;
    }
    long long want_isect = std::max(16 * N, g.growth_isect);
    if (want_isect > g.cap_isect) {
        if ((rc = realloc_dev(B.keys, want_isect))) return rc;
        if ((rc = realloc_dev(B.keys_alt, want_isect))) return rc;
        if ((rc = realloc_dev(B.sorted_ids, want_isect))) return rc;
        g.cap_isect = want_isect;
    }
    const long long P = W * H;
    if (P > g.cap_pix) {
        if ((rc = realloc_dev(B.out_img, P * 3))) return rc;
        if ((rc = realloc_dev(B.final_T, P))) return rc;
        if ((rc = realloc_dev(B.final_idx, P))) return rc;
        if ((rc = realloc_dev(B.v_rendered, P * 3))) return rc;
        g.cap_pix = P;
    }
    if (T > g.cap_T) {
        if ((rc = realloc_dev(B.tile_count, T * kCountPitch))) return rc;
        if ((rc = realloc_dev(B.tile_offset, T + 1))) return rc;
        if ((rc = realloc_dev(B.tile_order, T))) return rc;
        if ((rc = realloc_dev(B.tile_sorted, T))) return rc;
        if ((rc = realloc_dev(B.tile_flag, T + 1))) return rc;
        MSP_CUDA(cudaMemsetAsync(B.tile_count, 0, sizeof(int) * T * kCountPitch, g.stream()));
        g.cap_T = T;
    }
    if (K > 1 && (long long)K * P > g.cap_chunk) {
        const long long n = (long long)K * P;
        if ((rc = realloc_dev(B.chunk_T, n))) return rc;
        if ((rc = realloc_dev(B.chunk_C, n * 3))) return rc;
        if ((rc = realloc_dev(B.chunk_idx, n))) return rc;
        if ((rc = realloc_dev(B.prefix_T, n))) return rc;
        if ((rc = realloc_dev(B.after_C, n * 3))) return rc;
        g.cap_chunk = n;
    }
    return MSPLAT_OK;
}

// Depth-chunk rule of msplat_metal.mm:873-889 (capacity = 16 * N, :809).
int chunk_k_max(long long N, int num_tiles)
{
    if (num_tiles >= 400) return 1;
    const long long capacity = N * 16;
    const unsigned avg = (unsigned)(capacity / std::max(1, num_tiles));
    const unsigned cons = avg * 6;
    unsigned k = (cons + kChunkHost - 1) / kChunkHost;
    if (k < 2) k = 2;
    const unsigned abs_max = (unsigned)((capacity + kChunkHost - 1) / kChunkHost);
    if (k > abs_max) k = abs_max;
    return (int)k;
}

// Consume the previous step's readback if it is already complete.
static void poll_readback(bool wait)
{
    if (!g.readback_pending) return;
    if (wait) {
        cudaEventSynchronize(g.readback_ev);
    } else if (cudaEventQuery(g.readback_ev) != cudaSuccess) {
        return;
    }
    g.readback_pending = false;
    if (g.readback_has_loss) {
        float loss_sum;
        memcpy(&loss_sum, &g.h_ctr[kCtrLoss], sizeof(float));
        g.last_loss = (float)((double)loss_sum * g.last_loss_scale);
    }
    g.last_max_tile = g.h_ctr[kCtrMaxTile];
    g.last_isect = g.h_ctr[kCtrIsect];
    g.last_isect_n = g.readback_n;
    const int err = g.h_ctr[kCtrErr];
    if (err & kErrStageTimeout)
        fprintf(stderr, "msplat: a shared-memory bulk copy timed out; the step is incomplete\n");
    if (err & kErrIsectOverflow) {
        const long long need = (long long)g.h_ctr[kCtrIsect];
        if (need > g.growth_isect) {
            g.growth_isect = need + need / 4;
            fprintf(stderr, "msplat: intersection buffer overflow (%lld > %lld); growing\n", need,
                    g.cap_isect);
        }
    }
}

static void drain_timing_slot(int slot)
{
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, g.st_ev[0][slot], g.st_ev[kStages][slot]) == cudaSuccess)
        g.step_times.push_back(ms);
    for (int s = 0; s < kStages; s++) {
        if (cudaEventElapsedTime(&ms, g.st_ev[s][slot], g.st_ev[s + 1][slot]) == cudaSuccess)
            g.stage_times[s].push_back(ms);
    }
}

struct StageMarks {
    bool on;
    int slot;
    void mark(int s, cudaStream_t st)
    {
        if (on) cudaEventRecord(g.st_ev[s][slot], st);
    }
};

static StageMarks begin_timing()
{
    StageMarks m{g.timing, 0};
    if (!m.on) return m;
    m.slot = g.st_pos;
    g.st_pos = (g.st_pos + 1) % kRing;
    // the slot's previous events must be complete before reuse
    for (size_t i = 0; i < g.pending_timing.size(); i++) {
        if (g.pending_timing[i] == m.slot) {
            cudaEventSynchronize(g.st_ev[kStages][m.slot]);
            drain_timing_slot(m.slot);
            g.pending_timing.erase(g.pending_timing.begin() + i);
            break;
        }
    }
    g.pending_timing.push_back(m.slot);
    return m;
}

// Fill the next pinned ring slot and queue its copy into the device block.
static int upload_params(const StepParams& p, cudaStream_t st)
{
    const int slot = g.ring_pos;
    g.ring_pos = (g.ring_pos + 1) % kRing;
    MSP_CUDA(cudaEventSynchronize(g.ring_ev[slot]));
    g.h_ring[slot].p = p;
    memset(g.h_ring[slot].counters, 0, sizeof(g.h_ring[slot].counters));
    MSP_CUDA(cudaMemcpyAsync(g.d_slot, &g.h_ring[slot], sizeof(ParamSlot), cudaMemcpyHostToDevice, st));
    MSP_CUDA(cudaEventRecord(g.ring_ev[slot], st));
    return MSPLAT_OK;
}

int fill_params(StepParams& p, const CamArgs& a)
{
    if (a.N < 0 || a.W == 0 || a.H == 0 || !a.viewmat || !a.projmat || !a.cam_pos || !a.background) {
        set_error("invalid arguments (num_points=%d, %ux%u)", a.N, a.W, a.H);
        return MSPLAT_ERR_ARG;
    }
    memset(&p, 0, sizeof(p));
    memcpy(p.viewmat, a.viewmat, sizeof(p.viewmat));
    memcpy(p.projmat, a.projmat, sizeof(p.projmat));
    p.fx = a.fx; p.fy = a.fy; p.cx = a.cx; p.cy = a.cy;
    // msplat_metal.metal:1746-1747 (same float operations on the host)
    p.tan_fovx = 0.5f * (float)a.W / a.fx;
    p.tan_fovy = 0.5f * (float)a.H / a.fy;
    p.glob_scale = a.glob_scale;
    p.clip_thresh = a.clip_thresh;
    memcpy(p.cam_pos, a.cam_pos, sizeof(p.cam_pos));
    memcpy(p.bg, a.background, sizeof(p.bg));
    p.num_points = a.N;
    p.img_w = (int)a.W;
    p.img_h = (int)a.H;
    p.tiles_x = a.tile_bounds ? a.tile_bounds[0] : (int)((a.W + 15) / 16);
    p.tiles_y = a.tile_bounds ? a.tile_bounds[1] : (int)((a.H + 15) / 16);
    if (p.tiles_x != (int)((a.W + 15) / 16) || p.tiles_y != (int)((a.H + 15) / 16)) {
        set_error("tile_bounds (%d,%d) do not cover %ux%u with 16x16 tiles", p.tiles_x, p.tiles_y,
                  a.W, a.H);
        return MSPLAT_ERR_ARG;
    }
    if (p.tiles_x > 65535 || p.tiles_y > 65535) {
        set_error("image too large");
        return MSPLAT_ERR_ARG;
    }
    p.num_tiles = p.tiles_x * p.tiles_y;
    p.degree = (int)a.degree;
    p.degrees_to_use = (int)std::min(a.degrees_to_use, a.degree);
    p.rest_stride = a.rest_stride;
    p.k_max = chunk_k_max(a.N, p.num_tiles);
    return MSPLAT_OK;
}

// Nearest-key sorting of long tile lists, when the last view whose counters
// were read back had a tile longer than kSortRun keys (single-pass raster
// only).  The readback is consumed only once complete, so a host running
// ahead of the device keeps an older view's answer: any answer is correct.
static int prefix_sort_for(const StepParams& p)
{
    return (p.k_max == 1 && g.last_max_tile > kSortRun) ? 1 : 0;
}

// Dense binning, when the last view whose counters were read back averaged
// more than kDenseRatio intersections per Gaussian (same rule as above for
// a host running ahead).
static int dense_bins_for(const StepParams& p)
{
    (void)p;
    return (g.last_isect_n > 0 && g.last_isect > (long long)kDenseRatio * g.last_isect_n) ? 1 : 0;
}

// Forward half shared by render and train (forward_pipeline, msplat_metal.mm:462-750).
static int run_forward(const StepParams& p, const float* means, const float* scales,
                       const float* quats, const float* dc, const float* rest, const float* opac,
                       bool train, StageMarks& tm, cudaStream_t st)
{
    const Buffers& B = g.B;
    tm.mark(0, st);
    launch_project_forward(g.d_params, p.num_points, means, scales, quats, dc, rest, opac, B, train,
                           p.degrees_to_use, p.rest_stride, st);
    tm.mark(1, st);
    launch_scan_tiles(g.d_params, p.num_tiles, p.dense_bins != 0, B, st);
    launch_scatter(g.d_params, p.num_points, B, st);
    // the sorts of tiles above kSortRun / kLargeRun keys only when the last
    // view read back (or none yet) had such a tile
    const bool large_sort = g.last_max_tile == 0 || g.last_max_tile > kSortRun;
    const bool huge_sort = g.last_max_tile > kLargeRun;
    const int sort_launches = launch_sort_tiles(g.d_params, p.num_tiles, p.prefix_sort != 0,
                                                large_sort, huge_sort, B, st);
    tm.mark(2, st);
    launch_raster_forward(g.d_params, p.num_tiles, p.k_max, p.prefix_sort != 0, p.img_w, p.img_h, B,
                          st);
    g.last_k_max = p.k_max;
    g.last_num_tiles = p.num_tiles;
    g.last_prefix_sort = p.prefix_sort != 0;
    g.last_dense_bins = p.dense_bins != 0;
    g.launches += 3 + sort_launches + (p.k_max > 1 ? 2 : p.prefix_sort ? 3 : 1);
    MSP_CUDA(cudaGetLastError());
    return MSPLAT_OK;
}

static int queue_readback(cudaStream_t st, const StepParams& p)
{
    MSP_CUDA(cudaMemcpyAsync(g.h_ctr, d_counters(), sizeof(int) * kCtrRead,
                             cudaMemcpyDeviceToHost, st));
    MSP_CUDA(cudaEventRecord(g.readback_ev, st));
    g.readback_pending = true;
    g.readback_has_loss = true;
    g.readback_n = p.num_points;
    g.last_loss_scale = 1.0 / (3.0 * (double)p.img_w * (double)p.img_h);
    return MSPLAT_OK;
}

}  // namespace msp

using namespace msp;

extern "C" {

const char* msplat_last_error(void) { return t_last_error.c_str(); }

int msplat_set_stream(void* cuda_stream)
{
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = init_engine();
    if (rc) return rc;
    g.user_stream = (cudaStream_t)cuda_stream;
    g.user_stream_set = cuda_stream != nullptr;
    return MSPLAT_OK;
}

void* msplat_get_stream(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (init_engine()) return nullptr;
    return (void*)g.stream();
}

void* msplat_device(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (init_engine()) return nullptr;
    return (void*)&g.device;
}

void* msplat_gpu_alloc(size_t bytes, int zero)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (init_engine()) return nullptr;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 4) != cudaSuccess) {
        set_error("cudaMalloc(%zu) failed", bytes);
        return nullptr;
    }
    if (zero) cudaMemsetAsync(p, 0, bytes ? bytes : 4, g.stream());
    return p;
}

void msplat_gpu_free(void* ptr)
{
    if (!ptr) return;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g.ready) cudaStreamSynchronize(g.stream());
    cudaFree(ptr);
}

void* msplat_shared_alloc(size_t bytes, int zero)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (init_engine()) return nullptr;
    void* p = nullptr;
    const size_t n = bytes ? bytes : 4;
    cudaError_t e = cudaMallocManaged(&p, n, cudaMemAttachGlobal);
    if (e != cudaSuccess) {
        set_error("cudaMallocManaged(%zu) failed: %s", n, cudaGetErrorString(e));
        return nullptr;
    }
    // first touched by the host (the caller fills it), so zero it there too
    if (zero) memset(p, 0, n);
    return p;
}

void msplat_shared_free(void* ptr)
{
    if (!ptr) return;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g.ready) cudaStreamSynchronize(g.stream());
    cudaFree(ptr);
}

int msplat_shared_prefetch(const void* ptr, size_t bytes)
{
    if (!ptr || bytes == 0) return MSPLAT_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = init_engine();
    if (rc) return rc;
    MSP_CUDA(cudaMemPrefetchAsync(ptr, bytes, g.device, g.stream()));
    return MSPLAT_OK;
}

int msplat_copy(void* dst, const void* src, size_t bytes, int kind, int sync)
{
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = init_engine();
    if (rc) return rc;
    cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice
                     : kind == 1 ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
    MSP_CUDA(cudaMemcpyAsync(dst, src, bytes, k, g.stream()));
    if (sync) MSP_CUDA(cudaStreamSynchronize(g.stream()));
    return MSPLAT_OK;
}

void msplat_commit(void) {}

void msplat_gpu_sync(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.ready) return;
    cudaStreamSynchronize(g.stream());
    poll_readback(true);
}

void cleanup_msplat_cuda(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.ready) return;
    cudaStreamSynchronize(g.stream());
    poll_readback(true);  // consumed here, so no later call reads the old view's counters
    free_buffers();
    stage_release();
    if (g.d_work) cudaFree(g.d_work);
    g.d_work = nullptr;
    g.last_k_max = 0;
    g.last_max_tile = 0;
    g.last_isect = g.last_isect_n = 0;
    g.growth_isect = 0;
}

void cleanup_msplat_metal(void) { cleanup_msplat_cuda(); }

void msplat_set_metallib_path(const char* path) { (void)path; }

void msplat_enable_gpu_timing(int enable)
{
    std::lock_guard<std::mutex> lk(g_mu);
    g.timing = enable != 0;
}

static void drain_all_timing()
{
    for (int slot : g.pending_timing) {
        cudaEventSynchronize(g.st_ev[kStages][slot]);
        drain_timing_slot(slot);
    }
    g.pending_timing.clear();
}

int msplat_drain_gpu_times(double* out, int max_out)
{
    std::lock_guard<std::mutex> lk(g_mu);
    drain_all_timing();
    int n = (int)std::min<size_t>(g.step_times.size(), (size_t)std::max(0, max_out));
    for (int i = 0; i < n; i++) out[i] = g.step_times[i];
    g.step_times.clear();
    return n;
}

int msplat_drain_stage_times(double* stage_times, int max_stages, int max_samples, int* n_samples,
                             const char** stage_names)
{
    std::lock_guard<std::mutex> lk(g_mu);
    drain_all_timing();
    const int ns = std::min(max_stages, kStages);
    int m = 0;
    for (int s = 0; s < ns; s++) {
        const int cnt = (int)std::min<size_t>(g.stage_times[s].size(), (size_t)max_samples);
        for (int i = 0; i < cnt; i++) stage_times[s * max_samples + i] = g.stage_times[s][i];
        m = std::max(m, cnt);
        if (stage_names) stage_names[s] = kStageNames[s];
        g.stage_times[s].clear();
    }
    if (n_samples) *n_samples = m;
    return ns;
}

// Shared body of msplat_train_step (A = the optimiser, G unused) and
// msplat_train_step_grads (G = the gradient buffer, Adam left to the caller).
static int train_common(const char* who, int num_points, float* means3d, float* scales,
                        float glob_scale, float* quats, const float* viewmat,
                        const float* projmat, float fx, float fy, float cx, float cy,
                        unsigned img_height, unsigned img_width, const int* tile_bounds,
                        float clip_thresh, unsigned degree, unsigned degrees_to_use,
                        const float* cam_pos, float* features_dc, float* features_rest,
                        float* opacities, const float* background, const float* gt,
                        float ssim_weight, float loss_inv_n, int features_rest_bases,
                        StepParams& p, AdamPtrs& A, const GradOut* G, float* vis_counts,
                        float* xys_grad_norm, float* max_2d_size, float inv_max_dim,
                        const int32_t** radii_out, float* loss_out)
{
    int rc = init_engine();
    if (rc) return rc;
    if (!gt || !vis_counts || !xys_grad_norm || !max_2d_size) {
        set_error("%s: missing gt or statistics buffers", who);
        return MSPLAT_ERR_ARG;
    }
    poll_readback(false);
    CamArgs a{num_points, viewmat, projmat, fx, fy, cx, cy, glob_scale, clip_thresh, img_height,
              img_width, tile_bounds, degree, degrees_to_use, cam_pos, background,
              features_rest_bases * 3};
    const StepParams adam = p;
    if ((rc = fill_params(p, a))) return rc;
    p.prefix_sort = prefix_sort_for(p);
    p.dense_bins = dense_bins_for(p);
    memcpy(p.adam_step, adam.adam_step, sizeof(p.adam_step));
    memcpy(p.adam_bc2, adam.adam_bc2, sizeof(p.adam_bc2));
    p.beta1 = adam.beta1;
    p.beta2 = adam.beta2;
    p.eps = adam.eps;
    p.num_adam_groups = adam.num_adam_groups;
    p.ssim_weight = ssim_weight;
    p.loss_inv_n = loss_inv_n;
    p.inv_max_dim = inv_max_dim;
    const cudaStream_t st = g.stream();
    if ((rc = ensure(num_points, img_width, img_height, p.num_tiles, p.k_max, true))) return rc;
    p.capacity = g.cap_isect;
    StageMarks tm = begin_timing();
    if ((rc = upload_params(p, st))) return rc;
    if ((rc = run_forward(p, means3d, scales, quats, features_dc, features_rest, opacities, true,
                          tm, st)))
        return rc;
    tm.mark(3, st);
    launch_ssim(g.d_params, p.img_w, p.img_h, gt, g.B, st);
    tm.mark(4, st);
    launch_raster_backward(g.d_params, p.num_tiles, p.k_max, p.img_w, p.img_h, g.B, st);
    tm.mark(5, st);
    StatPtrs S{vis_counts, xys_grad_norm, max_2d_size};
    int bwd_launches = 1;
    if (G)
        bwd_launches = launch_project_backward_grads(g.d_params, num_points, p.degrees_to_use, p.rest_stride,
                                      g.B, A, S, *G, st);
    else
        bwd_launches = launch_project_backward_adam(g.d_params, num_points, p.degrees_to_use,
                                                    p.rest_stride, g.B, A, S, st);
    tm.mark(6, st);
    g.launches += 1 + (p.k_max > 1 ? 2 : 1) + bwd_launches;
    MSP_CUDA(cudaGetLastError());
    if ((rc = queue_readback(st, p))) return rc;
    if (radii_out) *radii_out = g.B.proj.radii;
    if (loss_out) *loss_out = g.last_loss;
    return MSPLAT_OK;
}

int msplat_train_step(
    int num_points, float* means3d, float* scales, float glob_scale, float* quats,
    const float* viewmat, const float* projmat, float fx, float fy, float cx, float cy,
    unsigned img_height, unsigned img_width, const int* tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, const float* cam_pos, float* features_dc,
    float* features_rest, float* opacities, const float* background, const float* gt,
    const float* window2d, float ssim_weight, float loss_inv_n, int features_rest_bases,
    int num_adam_groups, float* const* adam_params, float* const* adam_exp_avg,
    float* const* adam_exp_avg_sq, const float* adam_step_sizes, const float* adam_bc2_sqrts,
    float adam_beta1, float adam_beta2, float adam_eps, float* vis_counts, float* xys_grad_norm,
    float* max_2d_size, float inv_max_dim, const int32_t** radii_out, float* loss_out)
{
    (void)window2d;
    std::lock_guard<std::mutex> lk(g_mu);
    if (num_adam_groups < 0 || num_adam_groups > kGroups ||
        (num_adam_groups > 0 && (!adam_params || !adam_exp_avg || !adam_exp_avg_sq ||
                                 !adam_step_sizes || !adam_bc2_sqrts))) {
        set_error("msplat_train_step: missing optimiser arguments");
        return MSPLAT_ERR_ARG;
    }
    StepParams p;
    memset(&p, 0, sizeof(p));
    p.beta1 = adam_beta1;
    p.beta2 = adam_beta2;
    p.eps = adam_eps;
    p.num_adam_groups = num_adam_groups;
    AdamPtrs A{};
    for (int gi = 0; gi < num_adam_groups; gi++) {
        p.adam_step[gi] = adam_step_sizes[gi];
        p.adam_bc2[gi] = adam_bc2_sqrts[gi];
        A.param[gi] = adam_params[gi];
        A.exp_avg[gi] = adam_exp_avg[gi];
        A.exp_avg_sq[gi] = adam_exp_avg_sq[gi];
        A.numel[gi] = (A.param[gi] && A.exp_avg[gi] && A.exp_avg_sq[gi]) ? 1 : 0;
    }
    // The SH groups are only updated through the fused path when all of
    // them are present (msplat_metal.mm:1079-1087).
    if (num_adam_groups < 5) A.numel[3] = A.numel[4] = 0;
    return train_common("msplat_train_step", num_points, means3d, scales, glob_scale, quats,
                        viewmat, projmat, fx, fy, cx, cy, img_height, img_width, tile_bounds,
                        clip_thresh, degree, degrees_to_use, cam_pos, features_dc, features_rest,
                        opacities, background, gt, ssim_weight, loss_inv_n, features_rest_bases,
                        p, A, nullptr, vis_counts, xys_grad_norm, max_2d_size, inv_max_dim,
                        radii_out, loss_out);
}

static int train_grads_common(
    int mode, int num_points, float* means3d, float* scales, float glob_scale, float* quats,
    const float* viewmat, const float* projmat, float fx, float fy, float cx, float cy,
    unsigned img_height, unsigned img_width, const int* tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, const float* cam_pos, float* features_dc,
    float* features_rest, float* opacities, const float* background, const float* gt,
    float ssim_weight, float loss_inv_n, int features_rest_bases, float* grad_out,
    float* vis_counts, float* xys_grad_norm, float* max_2d_size, float inv_max_dim,
    const int32_t** radii_out, float* loss_out);

int msplat_train_step_grads(
    int num_points, float* means3d, float* scales, float glob_scale, float* quats,
    const float* viewmat, const float* projmat, float fx, float fy, float cx, float cy,
    unsigned img_height, unsigned img_width, const int* tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, const float* cam_pos, float* features_dc,
    float* features_rest, float* opacities, const float* background, const float* gt,
    float ssim_weight, float loss_inv_n, int features_rest_bases, float* grad_out,
    float* vis_counts, float* xys_grad_norm, float* max_2d_size, float inv_max_dim,
    const int32_t** radii_out, float* loss_out)
{
    return train_grads_common(0, num_points, means3d, scales, glob_scale, quats, viewmat,
                              projmat, fx, fy, cx, cy, img_height, img_width, tile_bounds,
                              clip_thresh, degree, degrees_to_use, cam_pos, features_dc,
                              features_rest, opacities, background, gt, ssim_weight, loss_inv_n,
                              features_rest_bases, grad_out, vis_counts, xys_grad_norm,
                              max_2d_size, inv_max_dim, radii_out, loss_out);
}

int msplat_train_step_grads_compact(
    int num_points, float* means3d, float* scales, float glob_scale, float* quats,
    const float* viewmat, const float* projmat, float fx, float fy, float cx, float cy,
    unsigned img_height, unsigned img_width, const int* tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, const float* cam_pos, float* features_dc,
    float* features_rest, float* opacities, const float* background, const float* gt,
    float ssim_weight, float loss_inv_n, int features_rest_bases, float* grad_out,
    float* vis_counts, float* xys_grad_norm, float* max_2d_size, float inv_max_dim,
    const int32_t** radii_out, float* loss_out)
{
    return train_grads_common(1, num_points, means3d, scales, glob_scale, quats, viewmat,
                              projmat, fx, fy, cx, cy, img_height, img_width, tile_bounds,
                              clip_thresh, degree, degrees_to_use, cam_pos, features_dc,
                              features_rest, opacities, background, gt, ssim_weight, loss_inv_n,
                              features_rest_bases, grad_out, vis_counts, xys_grad_norm,
                              max_2d_size, inv_max_dim, radii_out, loss_out);
}

int msplat_train_step_grads_accumulate(
    int num_points, float* means3d, float* scales, float glob_scale, float* quats,
    const float* viewmat, const float* projmat, float fx, float fy, float cx, float cy,
    unsigned img_height, unsigned img_width, const int* tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, const float* cam_pos, float* features_dc,
    float* features_rest, float* opacities, const float* background, const float* gt,
    float ssim_weight, float loss_inv_n, int features_rest_bases, float* grad_out,
    float* vis_counts, float* xys_grad_norm, float* max_2d_size, float inv_max_dim,
    const int32_t** radii_out, float* loss_out)
{
    return train_grads_common(2, num_points, means3d, scales, glob_scale, quats, viewmat,
                              projmat, fx, fy, cx, cy, img_height, img_width, tile_bounds,
                              clip_thresh, degree, degrees_to_use, cam_pos, features_dc,
                              features_rest, opacities, background, gt, ssim_weight, loss_inv_n,
                              features_rest_bases, grad_out, vis_counts, xys_grad_norm,
                              max_2d_size, inv_max_dim, radii_out, loss_out);
}

static int train_grads_common(
    int mode, int num_points, float* means3d, float* scales, float glob_scale, float* quats,
    const float* viewmat, const float* projmat, float fx, float fy, float cx, float cy,
    unsigned img_height, unsigned img_width, const int* tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, const float* cam_pos, float* features_dc,
    float* features_rest, float* opacities, const float* background, const float* gt,
    float ssim_weight, float loss_inv_n, int features_rest_bases, float* grad_out,
    float* vis_counts, float* xys_grad_norm, float* max_2d_size, float inv_max_dim,
    const int32_t** radii_out, float* loss_out)
{
    std::lock_guard<std::mutex> lk(g_mu);
    static const char* const kNames[3] = {"msplat_train_step_grads",
                                          "msplat_train_step_grads_compact",
                                          "msplat_train_step_grads_accumulate"};
    const bool compact = mode == 1;
    if (!grad_out || features_rest_bases < 0) {
        set_error("%s: missing gradient buffer", kNames[mode]);
        return MSPLAT_ERR_ARG;
    }
    StepParams p;
    memset(&p, 0, sizeof(p));
    AdamPtrs A{};
    A.param[0] = means3d;
    A.param[1] = scales;
    A.param[2] = quats;
    const size_t n = (size_t)std::max(num_points, 0);
    const size_t rs = (size_t)features_rest_bases * 3;
    GradOut G{};
    G.g[0] = grad_out;
    G.g[1] = G.g[0] + 3 * n;
    G.g[2] = G.g[1] + 3 * n;
    G.g[3] = G.g[2] + 4 * n;
    if (compact) {
        // means, scales, quats, v_rgb, opacities, visibility, camera position
        G.compact = 1;
        G.g[5] = G.g[3] + 3 * n;
        G.vis = G.g[5] + n;
        G.cam = G.vis + n;
    } else {
        G.g[4] = G.g[3] + 3 * n;
        G.g[5] = G.g[4] + rs * n;
        G.vis = G.g[5] + n;
        G.accumulate = mode == 2;
    }
    return train_common(kNames[mode], num_points, means3d, scales, glob_scale, quats,
                        viewmat, projmat, fx, fy, cx, cy, img_height, img_width, tile_bounds,
                        clip_thresh, degree, degrees_to_use, cam_pos, features_dc, features_rest,
                        opacities, background, gt, ssim_weight, loss_inv_n, features_rest_bases,
                        p, A, &G, vis_counts, xys_grad_norm, max_2d_size, inv_max_dim, radii_out,
                        loss_out);
}

int msplat_adam_apply(int num_points, int features_rest_bases, unsigned degree,
                      unsigned degrees_to_use, const float* grads, float grad_scale, int begin,
                      int end, int num_adam_groups, float* const* adam_params,
                      float* const* adam_exp_avg, float* const* adam_exp_avg_sq,
                      const float* adam_step_sizes, const float* adam_bc2_sqrts, float adam_beta1,
                      float adam_beta2, float adam_eps)
{
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = init_engine();
    if (rc) return rc;
    const long long rs = (long long)features_rest_bases * 3;
    if (!grads || num_points < 0 || features_rest_bases < 0 || begin < 0 || end > num_points ||
        begin > end || num_adam_groups < 0 || num_adam_groups > kGroups ||
        (num_adam_groups > 0 && (!adam_params || !adam_exp_avg || !adam_exp_avg_sq ||
                                 !adam_step_sizes || !adam_bc2_sqrts)) ||
        (long long)num_points * std::max(rs, 4LL) >= (1LL << 31) - (1LL << 21)) {
        set_error("msplat_adam_apply: invalid arguments (N=%d, range [%d,%d), groups %d)",
                  num_points, begin, end, num_adam_groups);
        return MSPLAT_ERR_ARG;
    }
    const size_t n = (size_t)num_points;
    ApplyArgs a{};
    const int strides[kGroups] = {3, 3, 4, 3, (int)rs, 1};
    const float* gp = grads;
    for (int gi = 0; gi < kGroups; gi++) {
        a.grad[gi] = gp;
        a.stride[gi] = strides[gi];
        gp += (size_t)strides[gi] * n;
    }
    a.vis = gp;
    for (int gi = 0; gi < num_adam_groups; gi++) {
        if (!adam_params[gi] || !adam_exp_avg[gi] || !adam_exp_avg_sq[gi] || strides[gi] == 0)
            continue;
        a.param[gi] = adam_params[gi];
        a.exp_avg[gi] = adam_exp_avg[gi];
        a.exp_avg_sq[gi] = adam_exp_avg_sq[gi];
        a.step[gi] = adam_step_sizes[gi];
        a.bc2[gi] = adam_bc2_sqrts[gi];
    }
    // The SH groups move together, as in the fused step.
    if (num_adam_groups < 5) a.param[3] = a.param[4] = nullptr;
    const int dtu = (int)std::min(degrees_to_use, degree);
    a.used_rest = rest_bases_updated(dtu, (int)rs) * 3;
    a.beta1 = adam_beta1;
    a.beta2 = adam_beta2;
    a.eps = adam_eps;
    a.scale = grad_scale;
    a.begin = begin;
    a.end = end;
    launch_adam_apply(a, g.stream());
    g.launches += 1;
    MSP_CUDA(cudaGetLastError());
    return MSPLAT_OK;
}

int msplat_render(int num_points, const float* means3d, const float* scales, float glob_scale,
                  const float* quats, const float* viewmat, const float* projmat, float fx,
                  float fy, float cx, float cy, unsigned img_height, unsigned img_width,
                  const int* tile_bounds, float clip_thresh, unsigned degree,
                  unsigned degrees_to_use, const float* cam_pos, const float* features_dc,
                  const float* features_rest, const float* opacities, const float* background,
                  float** out_img)
{
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = init_engine();
    if (rc) return rc;
    poll_readback(false);
    const int rest_stride = (num_sh_bases_host((int)degree) - 1) * 3;
    CamArgs a{num_points, viewmat, projmat, fx, fy, cx, cy, glob_scale, clip_thresh, img_height,
              img_width, tile_bounds, degree, degrees_to_use, cam_pos, background, rest_stride};
    StepParams p;
    if ((rc = fill_params(p, a))) return rc;
    p.prefix_sort = prefix_sort_for(p);
    p.dense_bins = dense_bins_for(p);
    const cudaStream_t st = g.stream();
    if ((rc = ensure(num_points, img_width, img_height, p.num_tiles, p.k_max, false))) return rc;
    p.capacity = g.cap_isect;
    StageMarks tm = begin_timing();
    if ((rc = upload_params(p, st))) return rc;
    if ((rc = run_forward(p, means3d, scales, quats, features_dc, features_rest, opacities, false,
                          tm, st)))
        return rc;
    for (int s = 3; s <= 6; s++) tm.mark(s, st);
    MSP_CUDA(cudaMemcpyAsync(g.h_ctr, d_counters(), sizeof(int) * kCtrRead,
                             cudaMemcpyDeviceToHost, st));
    MSP_CUDA(cudaEventRecord(g.readback_ev, st));
    g.readback_pending = true;
    g.readback_has_loss = false;
    g.readback_n = p.num_points;
    if (out_img) *out_img = g.B.out_img;
    return MSPLAT_OK;
}

float msplat_last_loss(int sync)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.ready) return 0.f;
    poll_readback(sync != 0);
    return g.last_loss;
}

long long msplat_num_intersections(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.ready) return 0;
    cudaStreamSynchronize(g.stream());
    poll_readback(true);
    return (long long)g.h_ctr[kCtrIsect];
}

int msplat_device_errors(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.ready) return 0;
    cudaStreamSynchronize(g.stream());
    poll_readback(true);
    return g.h_ctr[kCtrErr];
}

int msplat_debug_buffer(const char* name, void** dev_ptr, long long* count)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.ready || !name || !dev_ptr) {
        set_error("engine not initialised or bad arguments");
        return MSPLAT_ERR_ARG;
    }
    const Buffers& B = g.B;
    struct Ent { const char* n; void* p; long long c; };
    const Ent ents[] = {
        {"xy", B.proj.xy, g.cap_N}, {"depth", B.proj.depth, g.cap_N},
        {"radii", B.proj.radii, g.cap_N}, {"conic_op", B.proj.conic_op, g.cap_N},
        {"rgb", B.proj.rgb, g.cap_N}, {"tile_offset", B.tile_offset, g.cap_T + 1},
        {"tile_sorted", B.tile_sorted, g.cap_T},
        {"sorted_ids", B.sorted_ids, g.cap_isect}, {"out_img", B.out_img, g.cap_pix * 3},
        {"final_T", B.final_T, g.cap_pix}, {"final_idx", B.final_idx, g.cap_pix},
        {"v_rendered", B.v_rendered, g.cap_pix * 3},
        {"grad_acc", B.grad_acc, g.cap_grad_N * kGradStride},
        {"chunk_idx", B.chunk_idx, g.cap_chunk}};
    for (const Ent& e : ents) {
        if (strcmp(e.n, name) == 0) {
            if (e.p == B.tile_sorted && e.p && !g.last_prefix_sort && g.last_num_tiles > 0) {
                // a forward without prefix sorting leaves it unwritten: whole lists
                launch_whole_lists(g.d_params, g.last_num_tiles, B, g.stream());
                MSP_CUDA(cudaGetLastError());
                MSP_CUDA(cudaStreamSynchronize(g.stream()));
            }
            *dev_ptr = e.p;
            if (count) *count = e.c;
            return MSPLAT_OK;
        }
    }
    set_error("unknown buffer '%s'", name);
    return MSPLAT_ERR_ARG;
}

int msplat_count_raster_work(unsigned long long* out)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.ready || !out) {
        set_error("msplat_count_raster_work: engine not initialised or null output");
        return MSPLAT_ERR_ARG;
    }
    if (g.last_k_max != 1) {
        set_error("msplat_count_raster_work: the last forward was %s",
                  g.last_k_max == 0 ? "never run" : "depth-chunked (counts cover the single-pass "
                                                    "path only)");
        return MSPLAT_ERR_ARG;
    }
    cudaStream_t st = g.stream();
    if (!g.d_work) MSP_CUDA(cudaMalloc(&g.d_work, 4 * sizeof(unsigned long long)));
    MSP_CUDA(cudaMemsetAsync(g.d_work, 0, 4 * sizeof(unsigned long long), st));
    launch_count_raster_work(g.d_params, g.last_num_tiles, g.last_prefix_sort, g.B, g.d_work, st);
    MSP_CUDA(cudaGetLastError());
    MSP_CUDA(cudaMemcpyAsync(out, g.d_work, 4 * sizeof(unsigned long long),
                             cudaMemcpyDeviceToHost, st));
    MSP_CUDA(cudaStreamSynchronize(st));
    return MSPLAT_OK;
}

long long msplat_kernel_launches(int reset)
{
    std::lock_guard<std::mutex> lk(g_mu);
    long long n = g.launches;
    if (reset) g.launches = 0;
    return n;
}

int msplat_last_binning(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    return (g.last_prefix_sort ? 1 : 0) | (g.last_dense_bins ? 2 : 0);
}

}  // extern "C"
