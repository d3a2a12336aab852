// engine.h -- internal types of the CUDA engine (not part of the C-ABI).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include <mutex>

#include "errors.h"

namespace msp {

constexpr int kGroups = 6;        // means, scales, quats, features_dc, features_rest, opacities
constexpr int kGradStride = 9;    // per-Gaussian raster gradient: v_rgb[3], v_conic[3], v_xy[2], v_opacity
// Tile counters are spread one per 128-byte line: every visible Gaussian
// adds (and later subtracts) one per tile it covers, and counters sharing a
// line would serialise those atomics in a single L2 slice.
constexpr int kCountPitch = 32;

// Per-step scalars.  Written by the host into a pinned ring slot and copied
// into device memory on the step's stream, so every kernel reads the same
// block and a captured graph can be replayed with new cameras.
struct StepParams {
    float viewmat[16];
    float projmat[16];
    float fx, fy, cx, cy;
    float tan_fovx, tan_fovy;
    float glob_scale, clip_thresh;
    float cam_pos[3];
    float bg[3];
    float ssim_weight, loss_inv_n, inv_max_dim;
    float adam_step[kGroups];
    float adam_bc2[kGroups];
    float beta1, beta2, eps;
    int num_points;
    int img_w, img_h;
    int tiles_x, tiles_y, num_tiles;
    int degree, degrees_to_use, rest_stride;
    int k_max;
    int num_adam_groups;
    int prefix_sort;  // tiles of more than kSortRun keys sort their nearest keys only
    int dense_bins;   // binning for views of many tiles per Gaussian (kDenseArea)
    int pad0;
    long long capacity;
};

// Dense binning (StepParams::dense_bins, set by the host when the last view
// read back held more than kDenseRatio intersections per Gaussian).  The
// projection counts a rect of more than kDenseArea tiles as the four
// corners of a 2D difference array (slot 2 of the tiles' counter lines)
// instead of one atomic per tile, and the scan sums the corners back into
// counts.  The counts, and so every result, are the same.
constexpr int kDenseArea = 8;
constexpr int kDenseRatio = 16;

// Per-tile sorts: up to kSortRun keys in one CTA's registers or the
// 128-thread radix sort, up to kLargeRun in the 512-thread radix sort.
// With StepParams::prefix_sort set (single-pass raster only), a tile of
// more than kSortRun keys sorts only its nearest keys (about
// kPrefixTarget, at most kLargeRun of them), and the forward raster sorts
// it whole only when one of its pixels runs past them.  The host sets it
// when the largest tile of the last view whose counters it read back was
// above kSortRun, so scenes without such tiles launch exactly what they
// did without it.
constexpr int kSortRun = 2048;
constexpr int kLargeRun = 8192;
constexpr int kPrefixTarget = 1024;

// Per-Gaussian geometry written by the projection and read by binning and
// both rasterizers.
struct ProjOut {
    float2* xy;          // pixel centre
    float* depth;        // view-space z
    int* radii;          // 3-sigma radius, 0 = culled
    float4* conic_op;    // conic a, b, c and sigmoid(opacity)
    float4* rgb;         // raw SH colour (w unused)
    uint2* rect;         // tile rect: x0 | y0<<16, x1 | y1<<16 (exclusive max)
    float* sh_mean;      // [N*3] training only: the means as projected (SH-rest Adam reads
                         // them while the projection VJP updates the means)
};

struct Buffers {
    ProjOut proj;
    int* tile_count;       // [T * kCountPitch] zero between steps
    int* tile_offset;      // [T+1] exclusive scan
    int* tile_order;       // [T] tiles by intersection count, largest first (CTA order)
    unsigned long long* keys;      // [capacity]
    unsigned long long* keys_alt;  // [capacity] merge scratch for tiles longer than one register-sorted run
    int* sorted_ids;       // [capacity]
    // Tiles of more than kSortRun keys (with StepParams::prefix_sort) get
    // their nearest keys selected and sorted, not the whole list:
    // tile_sorted[t] is the length of tile t's sorted prefix (its key count
    // when the whole list is sorted).  The forward raster sets tile_flag[t] when a pixel
    // of tile t runs past the prefix without terminating, and
    // tile_flag[T] counts such tiles; those are then sorted whole and
    // rasterized again.  Both reset by the scan of the tile counts.
    int* tile_sorted;      // [T]
    int* tile_flag;        // [T+1]
    float* out_img;        // [H*W*3]
    float* final_T;        // [H*W]
    int* final_idx;        // [H*W]
    float* v_rendered;     // [H*W*3]
    float* grad_acc;       // [N*9]
    float* chunk_T;        // [K*H*W]
    float* chunk_C;        // [K*H*W*3]
    int* chunk_idx;        // [K*H*W]
    float* prefix_T;       // [K*H*W]
    float* after_C;        // [K*H*W*3]
    float* loss_sum;       // [1]
    int* err;              // [1]
    int* isect_total;      // [1] intersections of the view (scan output), or null
    int* max_tile;         // [1] the view's largest tile count (scan output), or null
};

// Device pointers of the optimiser, one entry per group.
struct AdamPtrs {
    float* param[kGroups];
    float* exp_avg[kGroups];
    float* exp_avg_sq[kGroups];
    long long numel[kGroups];
};

struct StatPtrs {
    float* vis_counts;
    float* grad_norm;
    float* max_2d;
};

// Planar per-group gradient output of the data-parallel step: group g's
// gradient has the layout of its parameter tensor ([N, per-Gaussian
// floats]); vis[i] is 1 for a Gaussian with radius > 0 in this view, else 0.
//
// Compact form (peer-memory data parallelism): g[3] holds v_rgb (the colour
// gradient, from which every SH coefficient's gradient follows with the view
// direction), g[4] is unused, and cam (3 floats) receives the camera
// position of the step.
//
// Accumulating form (several views per rank and step, full layout only):
// each visible Gaussian's gradients are added to what the buffer holds and
// its vis entry grows by 1; culled Gaussians are neither read nor written.
struct GradOut {
    float* g[kGroups];
    float* vis;
    float* cam;
    int compact;
    int accumulate;
    int rest_done;  // the SH-rest group is written by rest_grads_kernel
};

// Adam over a range of Gaussians [begin, end) from a gradient buffer laid
// out as GradOut; every gradient is multiplied by `scale` first.
struct ApplyArgs {
    float* param[kGroups];
    float* exp_avg[kGroups];
    float* exp_avg_sq[kGroups];
    const float* grad[kGroups];
    const float* vis;
    float step[kGroups];
    float bc2[kGroups];
    int stride[kGroups];       // floats per Gaussian of each group
    float beta1, beta2, eps, scale;
    int begin, end;
    int used_rest;             // SH-rest floats updated (degrees in use)
};

inline int num_sh_bases_host(int degree)
{
    return degree <= 0 ? 1 : degree == 1 ? 4 : degree == 2 ? 9 : degree == 3 ? 16 : 25;
}

// Per-device one-time set-up (kernel attributes such as the dynamic
// shared-memory limit are per device; entry points may be called from
// several host threads, some without the engine lock).  Runs f(dev) once for
// the current device and table; false when there is no usable device.
constexpr int kMaxDeviceSlots = 64;
template <class F>
inline bool once_per_device(std::once_flag (&flags)[kMaxDeviceSlots], F&& f)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDeviceSlots) return false;
    std::call_once(flags[dev], f, dev);
    return true;
}

// Camera arguments of one call, as passed through the C-ABI.
struct CamArgs {
    int N;
    const float* viewmat;
    const float* projmat;
    float fx, fy, cx, cy, glob_scale, clip_thresh;
    unsigned H, W;
    const int* tile_bounds;
    unsigned degree, degrees_to_use;
    const float* cam_pos;
    const float* background;
    int rest_stride;
};

// Engine state shared with the other host files (engine.cu).
std::mutex& engine_mutex();          // the engine's lock (take it in every entry point)
int engine_init();                   // idempotent; MSPLAT_OK or an error code
cudaStream_t engine_stream();
// Second stream for work that overlaps the engine stream within a step,
// with the events that fork it from and join it back to the engine stream.
struct SideStream {
    cudaStream_t stream;
    cudaEvent_t fork, join;
};
const SideStream& engine_side();        // stream all engine work goes to
void engine_add_launches(int n);     // for msplat_kernel_launches
void stage_release();                // frees msplat_stage_input's buffers (engine lock held)

// Host helpers shared by the entry points (engine.cu).
void set_error(const char* fmt, ...);                  // text for msplat_last_error()
int fill_params(StepParams& p, const CamArgs& a);      // validates, fills the block
int chunk_k_max(long long N, int num_tiles);           // depth chunks of one tile

// Kernel launchers (kernels_*.cu).
void launch_project_forward(const StepParams* P, int N, const float* means, const float* scales,
                            const float* quats, const float* dc, const float* rest,
                            const float* opac, const Buffers& B, bool zero_grads,
                            int degrees_to_use_host, int rest_stride_host, cudaStream_t s);
void launch_scan_tiles(const StepParams* P, int num_tiles, bool dense_bins, const Buffers& B,
                       cudaStream_t s);
void launch_scatter(const StepParams* P, int N, const Buffers& B, cudaStream_t s);
int launch_sort_tiles(const StepParams* P, int num_tiles, bool prefix_sort, bool large_sort,
                      bool huge_sort, const Buffers& B, cudaStream_t s);
void launch_whole_lists(const StepParams* P, int num_tiles, const Buffers& B, cudaStream_t s);
void launch_count_raster_work(const StepParams* P, int num_tiles, bool prefix_sort, const Buffers& B,
                              unsigned long long* d_out, cudaStream_t s);
void launch_raster_forward(const StepParams* P, int num_tiles, int k_max, bool prefix_sort, int W, int H,
                           const Buffers& B, cudaStream_t s);
void launch_ssim(const StepParams* P, int W, int H, const float* gt, const Buffers& B,
                 cudaStream_t s);
void launch_raster_backward(const StepParams* P, int num_tiles, int k_max, int W, int H,
                            const Buffers& B, cudaStream_t s);
// Returns the number of kernels launched (the SH-rest Adam runs as its own kernel).
int launch_project_backward_adam(const StepParams* P, int N, int degrees_to_use_host,
                                 int rest_stride_host, const Buffers& B, const AdamPtrs& A,
                                 const StatPtrs& St, cudaStream_t s);
int launch_project_backward_grads(const StepParams* P, int N, int degrees_to_use_host,
                                   int rest_stride_host, const Buffers& B, const AdamPtrs& A,
                                   const StatPtrs& St, const GradOut& G, cudaStream_t s);
int rest_bases_updated(int degrees_to_use, int rest_stride);
void launch_adam_apply(const ApplyArgs& a, cudaStream_t s);

}  // namespace msp
