// noalloc.cu -- msplat_render_noalloc: the forward render with every
// intermediate buffer carved out of one static device array.
//
// Some callers cannot allocate device memory while they render: a viewer
// whose frame loop must not stall (cudaMalloc and cudaFree can synchronise
// the whole device), an embedder that plans all device memory once at
// start-up and owns every byte after that, or a process whose free memory is
// held by another allocator's cache.  msplat_render grows its buffer cache
// with cudaMalloc on demand, so they cannot use it.  This entry point runs
// the same kernels as msplat_render, in the same order, but takes its
// scratch from a file-scope __device__ array and writes the image into a
// buffer the caller owns.  It calls no cudaMalloc/cudaFree and no library
// routine that allocates.
//
// The array is created by the driver when this file's module is loaded, one
// per device and process.  The first call on a device, made with that device
// current, looks up its address (cudaGetSymbolAddress, which also loads the
// module) and so does the set-up; it should come before any stream capture.
//
// Calls share the array, so two calls that overlap on one device (from two
// host threads) race on it: the caller must serialise them.  Each call is
// synchronous on its stream: it returns after the image is written and the
// overflow check is read.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "../../include/msplat_engine.h"
#include "engine.h"

namespace msp {
namespace {

constexpr size_t kScratchBytes = MSPLAT_NOALLOC_SCRATCH_BYTES;
constexpr size_t kAlign = 256;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_scratch[kScratchBytes];

std::once_flag g_once[kMaxDevices];
void* g_base[kMaxDevices];
cudaError_t g_setup_err[kMaxDevices];

inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Byte offsets of every buffer inside the array; capacity = intersections.
struct Layout {
    size_t params, err, xy, depth, radii, conic_op, rgb, rect, tile_count, tile_offset, tile_order;
    size_t tile_sorted, tile_flag;
    size_t final_T, final_idx, chunk_T, chunk_C, chunk_idx, keys, keys_alt, sorted_ids;
    size_t end;
    long long capacity;
};

// Lays out the buffers for N Gaussians, P pixels, T tiles and K depth
// chunks with `cap` intersection slots.
Layout layout(long long N, long long P, long long T, int K, long long cap)
{
    Layout L{};
    size_t o = 0;
    auto take = [&o](size_t bytes) {
        const size_t at = o;
        o = align_up(o + bytes);
        return at;
    };
    const size_t n = (size_t)N, px = (size_t)P;
    L.params = take(sizeof(StepParams));
    L.err = take(4 * sizeof(int));
    L.xy = take(n * sizeof(float2));
    L.depth = take(n * sizeof(float));
    L.radii = take(n * sizeof(int));
    L.conic_op = take(n * sizeof(float4));
    L.rgb = take(n * sizeof(float4));
    L.rect = take(n * sizeof(uint2));
    L.tile_count = take((size_t)T * kCountPitch * sizeof(int));
    L.tile_offset = take((size_t)(T + 1) * sizeof(int));
    L.tile_order = take((size_t)T * sizeof(int));
    L.tile_sorted = take((size_t)T * sizeof(int));
    L.tile_flag = take((size_t)(T + 1) * sizeof(int));
    L.final_T = take(px * sizeof(float));
    L.final_idx = take(px * sizeof(int));
    const size_t kp = K > 1 ? (size_t)K * px : 0;
    L.chunk_T = take(kp * sizeof(float));
    L.chunk_C = take(kp * 3 * sizeof(float));
    L.chunk_idx = take(kp * sizeof(int));
    L.keys = take((size_t)cap * sizeof(unsigned long long));
    L.keys_alt = take((size_t)cap * sizeof(unsigned long long));
    L.sorted_ids = take((size_t)cap * sizeof(int));
    L.end = o;
    L.capacity = cap;
    return L;
}

int scratch_base(void** base)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_error("msplat_render_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
        return MSPLAT_ERR_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("msplat_render_noalloc: device %d beyond the %d supported", dev, kMaxDevices);
        return MSPLAT_ERR_ARG;
    }
    std::call_once(g_once[dev], [dev] {
        g_setup_err[dev] = cudaGetSymbolAddress(&g_base[dev], g_scratch);
    });
    if (g_setup_err[dev] != cudaSuccess || !g_base[dev]) {
        set_error("msplat_render_noalloc: scratch set-up on device %d failed: %s", dev,
                  cudaGetErrorString(g_setup_err[dev]));
        return MSPLAT_ERR_CUDA;
    }
    *base = g_base[dev];
    return MSPLAT_OK;
}

#define NA_CUDA(expr)                                                                     \
    do {                                                                                  \
        cudaError_t e_ = (expr);                                                          \
        if (e_ != cudaSuccess) {                                                          \
            set_error("msplat_render_noalloc: %s failed: %s", #expr, cudaGetErrorString(e_)); \
            return MSPLAT_ERR_CUDA;                                                       \
        }                                                                                 \
    } while (0)

}  // namespace
}  // namespace msp

using namespace msp;

extern "C" int msplat_render_noalloc(
    int num_points, const float* means3d, const float* scales, float glob_scale,
    const float* quats, const float* viewmat, const float* projmat, float fx, float fy, float cx,
    float cy, unsigned img_height, unsigned img_width, const int* tile_bounds, float clip_thresh,
    unsigned degree, unsigned degrees_to_use, const float* cam_pos, const float* features_dc,
    const float* features_rest, const float* opacities, const float* background,
    float* out_img, void* cuda_stream)
{
    const int rest_stride = (num_sh_bases_host((int)degree) - 1) * 3;
    CamArgs a{num_points, viewmat, projmat, fx, fy, cx, cy, glob_scale, clip_thresh, img_height,
              img_width, tile_bounds, degree, degrees_to_use, cam_pos, background, rest_stride};
    StepParams p;
    int rc = fill_params(p, a);
    if (rc) return rc;
    // one synchronous call with no earlier view to go by: long lists sort
    // their nearest keys whenever the raster is single-pass
    p.prefix_sort = p.k_max == 1 ? 1 : 0;
    if (!out_img || (num_points > 0 && (!means3d || !scales || !quats || !features_dc ||
                                        !opacities || (rest_stride > 0 && !features_rest)))) {
        set_error("msplat_render_noalloc: null device pointer");
        return MSPLAT_ERR_ARG;
    }
    // Size check before any CUDA call: the reference's intersection budget
    // (16 per Gaussian, msplat_metal.mm:809) must fit beside the rest.
    const long long N = num_points;
    const long long P = (long long)img_width * img_height;
    const long long min_cap = std::max(16 * N, 1LL);
    const Layout need = layout(N, P, p.num_tiles, p.k_max, min_cap);
    if (need.end > kScratchBytes) {
        set_error("msplat_render_noalloc: %d Gaussians at %ux%u (%d depth chunks) need %zu bytes "
                  "of scratch; the static array holds %zu",
                  num_points, img_width, img_height, p.k_max, need.end, kScratchBytes);
        return MSPLAT_ERR_ARG;
    }
    // Whatever is left over becomes extra intersection slots.
    const size_t spare = kScratchBytes - need.end;
    long long cap = min_cap + (long long)(spare / 20);
    Layout L = layout(N, P, p.num_tiles, p.k_max, cap);
    while (L.end > kScratchBytes) L = layout(N, P, p.num_tiles, p.k_max, --cap);
    p.capacity = cap;

    void* vbase = nullptr;
    if ((rc = scratch_base(&vbase))) return rc;
    char* base = static_cast<char*>(vbase);
    Buffers B{};
    StepParams* d_params = reinterpret_cast<StepParams*>(base + L.params);
    B.err = reinterpret_cast<int*>(base + L.err);
    B.proj.xy = reinterpret_cast<float2*>(base + L.xy);
    B.proj.depth = reinterpret_cast<float*>(base + L.depth);
    B.proj.radii = reinterpret_cast<int*>(base + L.radii);
    B.proj.conic_op = reinterpret_cast<float4*>(base + L.conic_op);
    B.proj.rgb = reinterpret_cast<float4*>(base + L.rgb);
    B.proj.rect = reinterpret_cast<uint2*>(base + L.rect);
    B.tile_count = reinterpret_cast<int*>(base + L.tile_count);
    B.tile_offset = reinterpret_cast<int*>(base + L.tile_offset);
    B.tile_order = reinterpret_cast<int*>(base + L.tile_order);
    B.tile_sorted = reinterpret_cast<int*>(base + L.tile_sorted);
    B.tile_flag = reinterpret_cast<int*>(base + L.tile_flag);
    B.final_T = reinterpret_cast<float*>(base + L.final_T);
    B.final_idx = reinterpret_cast<int*>(base + L.final_idx);
    if (p.k_max > 1) {
        B.chunk_T = reinterpret_cast<float*>(base + L.chunk_T);
        B.chunk_C = reinterpret_cast<float*>(base + L.chunk_C);
        B.chunk_idx = reinterpret_cast<int*>(base + L.chunk_idx);
    }
    B.keys = reinterpret_cast<unsigned long long*>(base + L.keys);
    B.keys_alt = reinterpret_cast<unsigned long long*>(base + L.keys_alt);
    B.sorted_ids = reinterpret_cast<int*>(base + L.sorted_ids);
    B.out_img = out_img;

    const cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    // The parameter block goes from this stack frame; a copy from pageable
    // memory has been staged by the time cudaMemcpyAsync returns.
    NA_CUDA(cudaMemcpyAsync(d_params, &p, sizeof(StepParams), cudaMemcpyHostToDevice, st));
    // Only the tile counters and the error word must start at zero; every
    // other buffer is written before it is read.
    NA_CUDA(cudaMemsetAsync(B.err, 0, 4 * sizeof(int), st));
    NA_CUDA(cudaMemsetAsync(B.tile_count, 0, sizeof(int) * (size_t)p.num_tiles * kCountPitch, st));
    launch_project_forward(d_params, p.num_points, means3d, scales, quats, features_dc,
                           features_rest, opacities, B, false, p.degrees_to_use, p.rest_stride, st);
    launch_scan_tiles(d_params, p.num_tiles, false, B, st);
    launch_scatter(d_params, p.num_points, B, st);
    launch_sort_tiles(d_params, p.num_tiles, p.prefix_sort != 0, true, true, B, st);
    launch_raster_forward(d_params, p.num_tiles, p.k_max, p.prefix_sort != 0, p.img_w, p.img_h, B, st);
    NA_CUDA(cudaGetLastError());
    int h_check[2] = {0, 0};
    NA_CUDA(cudaMemcpyAsync(&h_check[0], B.err, sizeof(int), cudaMemcpyDeviceToHost, st));
    NA_CUDA(cudaMemcpyAsync(&h_check[1], B.tile_offset + p.num_tiles, sizeof(int),
                            cudaMemcpyDeviceToHost, st));
    NA_CUDA(cudaStreamSynchronize(st));
    const char* what = nullptr;
    rc = render_status(h_check[0], &what);
    if (rc == MSPLAT_ERR_OVERFLOW) {
        set_error("msplat_render_noalloc: %d tile intersections exceed the %lld slots of the "
                  "static scratch; the image is incomplete",
                  h_check[1], cap);
    } else if (rc != MSPLAT_OK) {
        set_error("msplat_render_noalloc: %s (error word 0x%x); the image is incomplete", what,
                  (unsigned)h_check[0]);
    }
    return rc;
}
