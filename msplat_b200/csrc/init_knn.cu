// init_knn.cu -- Gaussians from a point cloud: the initial state of
// Model::Model (core/src/model.cpp:42-118).
//
// The expensive part is the initial scale of every Gaussian: the mean
// distance to its three nearest neighbours (PointsTensor::scales,
// core/include/kdtree_tensor.hpp:27-41, a nanoflann v1.5.5 k-d tree search
// on the host).  Here it is an exact k-nearest-neighbour search on the GPU
// over a uniform grid: points are bucketed by cell (count, scan, scatter),
// then every point scans shells of cells around its own until no unvisited
// cell can hold a closer point than its current k-th.  Squared distances
// are formed as nanoflann's L2_Simple_Adaptor does ((dx^2 + dy^2) + dz^2,
// no fused multiply-add), so the k smallest values, and their square roots
// and means, are the ones the k-d tree finds.
//
// The rest of the initial state is host arithmetic in the reference's
// order (std::log of the mean distance, quaternions from std::mt19937(42)
// and std::uniform_real_distribution<float>, SH DC from the point colours,
// logit(0.1) opacities) and one upload per array.
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <random>
#include <vector>

#include <cub/device/device_scan.cuh>

#include "../../include/msplat_engine.h"
#include "engine.h"

namespace msp {
namespace {

constexpr int kKnnMax = 8;
constexpr long long kMaxCells = 1LL << 24;

struct Grid {
    float lox, loy, loz;
    float cell, inv_cell;
    int gx, gy, gz;
};

__device__ __forceinline__ int cell_axis(float v, float lo, float inv, int g)
{
    int c = (int)floorf((v - lo) * inv);
    return c < 0 ? 0 : (c >= g ? g - 1 : c);
}

__global__ void knn_count_kernel(const float* __restrict__ xyz, long long n, Grid G,
                                 int* __restrict__ cell_of, int* __restrict__ counts)
{
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int cx = cell_axis(xyz[i * 3 + 0], G.lox, G.inv_cell, G.gx);
        const int cy = cell_axis(xyz[i * 3 + 1], G.loy, G.inv_cell, G.gy);
        const int cz = cell_axis(xyz[i * 3 + 2], G.loz, G.inv_cell, G.gz);
        const int c = (cz * G.gy + cy) * G.gx + cx;
        cell_of[i] = c;
        atomicAdd(&counts[c], 1);
    }
}

__global__ void knn_scatter_kernel(const float* __restrict__ xyz, long long n,
                                   const int* __restrict__ cell_of, const int* __restrict__ start,
                                   int* __restrict__ cursor, float4* __restrict__ sorted)
{
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int c = cell_of[i];
        const int pos = start[c] + atomicAdd(&cursor[c], 1);
        sorted[pos] = make_float4(xyz[i * 3 + 0], xyz[i * 3 + 1], xyz[i * 3 + 2], __int_as_float((int)i));
    }
}

__device__ __forceinline__ void knn_insert(float* best, int k, float d)
{
    if (!(d < best[k - 1])) return;
    int j = k - 1;
    while (j > 0 && best[j - 1] > d) {
        best[j] = best[j - 1];
        j--;
    }
    best[j] = d;
}

// One thread per point, in cell order (neighbouring threads search
// neighbouring cells).  out[i] = (sqrt(d_1) + ... + sqrt(d_{k-1})) / (k-1)
// over the k smallest squared distances d_0 <= ... <= d_{k-1} (d_0 is the
// point itself).
__global__ void knn_query_kernel(const float4* __restrict__ sorted, long long n,
                                 const int* __restrict__ start, Grid G, int k,
                                 float* __restrict__ out)
{
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < n;
         t += (long long)gridDim.x * blockDim.x) {
        const float4 q = sorted[t];
        const int hx = cell_axis(q.x, G.lox, G.inv_cell, G.gx);
        const int hy = cell_axis(q.y, G.loy, G.inv_cell, G.gy);
        const int hz = cell_axis(q.z, G.loz, G.inv_cell, G.gz);
        float best[kKnnMax];
        for (int j = 0; j < kKnnMax; j++) best[j] = FLT_MAX;
        const int rmax = max(G.gx, max(G.gy, G.gz));
        for (int r = 0; r <= rmax; r++) {
            const int z0 = max(hz - r, 0), z1 = min(hz + r, G.gz - 1);
            const int y0 = max(hy - r, 0), y1 = min(hy + r, G.gy - 1);
            for (int cz = z0; cz <= z1; cz++) {
                for (int cy = y0; cy <= y1; cy++) {
                    const bool face = abs(cz - hz) == r || abs(cy - hy) == r;
                    // on a face every x of the shell; inside only its two ends
                    const int xs = face ? max(hx - r, 0) : hx - r;
                    const int xstep = face ? 1 : 2 * r;
                    for (int cx = xs; cx <= min(hx + r, G.gx - 1); cx += max(xstep, 1)) {
                        if (cx < 0) continue;
                        const int c = (cz * G.gy + cy) * G.gx + cx;
                        for (int p = start[c]; p < start[c + 1]; p++) {
                            const float4 o = sorted[p];
                            const float dx = q.x - o.x, dy = q.y - o.y, dz = q.z - o.z;
                            float d = 0.0f;
                            d = __fadd_rn(d, __fmul_rn(dx, dx));
                            d = __fadd_rn(d, __fmul_rn(dy, dy));
                            d = __fadd_rn(d, __fmul_rn(dz, dz));
                            knn_insert(best, k, d);
                        }
                        if (r == 0) break;
                    }
                }
            }
            // every point outside the (2r+1)^3 block is at least `reach` away
            float reach = FLT_MAX;
            bool all = true;
            if (hx - r > 0) { reach = fminf(reach, q.x - (G.lox + (float)(hx - r) * G.cell)); all = false; }
            if (hx + r < G.gx - 1) { reach = fminf(reach, (G.lox + (float)(hx + r + 1) * G.cell) - q.x); all = false; }
            if (hy - r > 0) { reach = fminf(reach, q.y - (G.loy + (float)(hy - r) * G.cell)); all = false; }
            if (hy + r < G.gy - 1) { reach = fminf(reach, (G.loy + (float)(hy + r + 1) * G.cell) - q.y); all = false; }
            if (hz - r > 0) { reach = fminf(reach, q.z - (G.loz + (float)(hz - r) * G.cell)); all = false; }
            if (hz + r < G.gz - 1) { reach = fminf(reach, (G.loz + (float)(hz + r + 1) * G.cell) - q.z); all = false; }
            if (all) break;
            // margin for the rounding of the cell assignment and the bounds
            reach -= 2e-3f * G.cell + 4e-7f * (fabsf(q.x) + fabsf(q.y) + fabsf(q.z) + fabsf(G.lox) +
                                                fabsf(G.loy) + fabsf(G.loz));
            if (best[k - 1] < FLT_MAX && reach > 0.f && best[k - 1] <= reach * reach) break;
        }
        float sum = 0.0f;
        for (int j = 1; j < k; j++) sum = __fadd_rn(sum, sqrtf(best[j]));
        out[__float_as_int(q.w)] = __fdiv_rn(sum, (float)(k - 1));
    }
}

#define KNN_CUDA(expr)                                                                  \
    do {                                                                                \
        cudaError_t e_ = (expr);                                                        \
        if (e_ != cudaSuccess) {                                                        \
            set_error("msplat_knn_mean_distance: %s: %s", #expr, cudaGetErrorString(e_)); \
            rc = MSPLAT_ERR_CUDA;                                                       \
            goto done;                                                                  \
        }                                                                               \
    } while (0)

Grid make_grid(const float* xyz, long long n)
{
    float lo[3] = {FLT_MAX, FLT_MAX, FLT_MAX}, hi[3] = {-FLT_MAX, -FLT_MAX, -FLT_MAX};
    for (long long i = 0; i < n; i++)
        for (int a = 0; a < 3; a++) {
            lo[a] = std::min(lo[a], xyz[i * 3 + a]);
            hi[a] = std::max(hi[a], xyz[i * 3 + a]);
        }
    double ext[3], vol = 1.0, emax = 0.0;
    for (int a = 0; a < 3; a++) {
        ext[a] = (double)hi[a] - (double)lo[a];
        vol *= ext[a];
        emax = std::max(emax, ext[a]);
    }
    // about four points per cell for a volume-filling cloud
    double cell = std::cbrt(vol * 4.0 / (double)std::max<long long>(n, 1));
    cell = std::max(cell, emax / 1024.0);
    if (!(cell > 0.0)) cell = 1.0;
    int g[3];
    for (;;) {
        long long total = 1;
        for (int a = 0; a < 3; a++) {
            g[a] = (int)std::max(1.0, std::ceil(ext[a] / cell));
            total *= g[a];
        }
        if (total <= kMaxCells) break;
        cell *= 1.25;
    }
    Grid G;
    G.lox = lo[0];
    G.loy = lo[1];
    G.loz = lo[2];
    G.cell = (float)cell;
    G.inv_cell = (float)(1.0 / cell);
    G.gx = g[0];
    G.gy = g[1];
    G.gz = g[2];
    return G;
}

}  // namespace
}  // namespace msp

using namespace msp;

extern "C" {

int msplat_knn_mean_distance(const float* xyz, long long n, int k, float* out)
{
    if (!xyz || !out || n < 1 || k < 2 || k > kKnnMax) {
        set_error("msplat_knn_mean_distance: invalid arguments");
        return MSPLAT_ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(engine_mutex());
    int rc = engine_init();
    if (rc) return rc;
    cudaStream_t s = engine_stream();
    const Grid G = make_grid(xyz, n);
    const long long cells = (long long)G.gx * G.gy * G.gz;
    float *d_xyz = nullptr, *d_out = nullptr;
    int *cell_of = nullptr, *counts = nullptr, *start = nullptr, *cursor = nullptr;
    float4* sorted = nullptr;
    void* tmp = nullptr;
    size_t tmp_bytes = 0;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 32);
    KNN_CUDA(cudaMallocAsync(&d_xyz, (size_t)n * 3 * sizeof(float), s));
    KNN_CUDA(cudaMallocAsync(&d_out, (size_t)n * sizeof(float), s));
    KNN_CUDA(cudaMallocAsync(&cell_of, (size_t)n * sizeof(int), s));
    KNN_CUDA(cudaMallocAsync(&counts, (size_t)(cells + 1) * sizeof(int), s));
    KNN_CUDA(cudaMallocAsync(&start, (size_t)(cells + 1) * sizeof(int), s));
    KNN_CUDA(cudaMallocAsync(&cursor, (size_t)cells * sizeof(int), s));
    KNN_CUDA(cudaMallocAsync(&sorted, (size_t)n * sizeof(float4), s));
    KNN_CUDA(cudaMemcpyAsync(d_xyz, xyz, (size_t)n * 3 * sizeof(float), cudaMemcpyHostToDevice, s));
    KNN_CUDA(cudaMemsetAsync(counts, 0, (size_t)(cells + 1) * sizeof(int), s));
    KNN_CUDA(cudaMemsetAsync(cursor, 0, (size_t)cells * sizeof(int), s));
    knn_count_kernel<<<blocks, 256, 0, s>>>(d_xyz, n, G, cell_of, counts);
    KNN_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, tmp_bytes, counts, start, (int)(cells + 1), s));
    KNN_CUDA(cudaMallocAsync(&tmp, tmp_bytes, s));
    KNN_CUDA(cub::DeviceScan::ExclusiveSum(tmp, tmp_bytes, counts, start, (int)(cells + 1), s));
    knn_scatter_kernel<<<blocks, 256, 0, s>>>(d_xyz, n, cell_of, start, cursor, sorted);
    knn_query_kernel<<<(int)((n + 127) / 128), 128, 0, s>>>(sorted, n, start, G, k, d_out);
    engine_add_launches(3);
    KNN_CUDA(cudaGetLastError());
    KNN_CUDA(cudaMemcpyAsync(out, d_out, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost, s));
    KNN_CUDA(cudaStreamSynchronize(s));
done:
    for (void* p : {(void*)d_xyz, (void*)d_out, (void*)cell_of, (void*)counts, (void*)start,
                    (void*)cursor, (void*)sorted, tmp})
        if (p) cudaFreeAsync(p, s);
    cudaStreamSynchronize(s);
    return rc;
}

int msplat_init_gaussians(const float* xyz, const unsigned char* rgb, long long n, int sh_degree,
                          float* means, float* scales, float* quats, float* features_dc,
                          float* features_rest, float* opacities)
{
    if (!xyz || !rgb || n < 1 || sh_degree < 0 || !means || !scales || !quats || !features_dc ||
        !opacities || (sh_degree > 0 && !features_rest)) {
        set_error("msplat_init_gaussians: invalid arguments");
        return MSPLAT_ERR_ARG;
    }
    // mean distance to the 3 nearest neighbours, then its log, repeated 3x
    std::vector<float> dist((size_t)n);
    int rc = msplat_knn_mean_distance(xyz, n, 4, dist.data());
    if (rc) return rc;
    std::vector<float> sc((size_t)n * 3), q((size_t)n * 4), dc((size_t)n * 3), op((size_t)n);
    for (long long i = 0; i < n; i++) {
        const float v = std::log(dist[i]);
        sc[i * 3] = sc[i * 3 + 1] = sc[i * 3 + 2] = v;
    }
    // uniformly random rotations (Shoemake), from mt19937(42)
    std::mt19937 rng(42);
    std::uniform_real_distribution<float> uni(0.0f, 1.0f);
    for (long long i = 0; i < n; i++) {
        const float u = uni(rng), v = uni(rng), w = uni(rng);
        q[i * 4 + 0] = std::sqrt(1 - u) * std::sin(2 * M_PI * v);
        q[i * 4 + 1] = std::sqrt(1 - u) * std::cos(2 * M_PI * v);
        q[i * 4 + 2] = std::sqrt(u) * std::sin(2 * M_PI * w);
        q[i * 4 + 3] = std::sqrt(u) * std::cos(2 * M_PI * w);
    }
    // SH DC from 8-bit colour: (c / 255 - 0.5) / C0, in double
    const double kC0 = 0.28209479177387814;
    for (long long i = 0; i < n * 3; i++) dc[i] = (float)((rgb[i] / 255.0 - 0.5) / kC0);
    const float logit01 = std::log(0.1f / 0.9f);
    std::fill(op.begin(), op.end(), logit01);
    const int dim_sh = sh_degree == 0 ? 1 : sh_degree == 1 ? 4 : sh_degree == 2 ? 9 : sh_degree == 3 ? 16 : 25;
    const size_t rest_floats = (size_t)n * (dim_sh - 1) * 3;
    std::lock_guard<std::mutex> lk(engine_mutex());
    cudaStream_t s = engine_stream();
    const struct {
        float* dst;
        const void* src;
        size_t bytes;
    } up[5] = {{means, xyz, (size_t)n * 12}, {scales, sc.data(), sc.size() * 4},
               {quats, q.data(), q.size() * 4}, {features_dc, dc.data(), dc.size() * 4},
               {opacities, op.data(), op.size() * 4}};
    for (auto& u : up)
        if (cudaMemcpyAsync(u.dst, u.src, u.bytes, cudaMemcpyHostToDevice, s) != cudaSuccess) {
            set_error("msplat_init_gaussians: upload failed");
            return MSPLAT_ERR_CUDA;
        }
    if (rest_floats && cudaMemsetAsync(features_rest, 0, rest_floats * 4, s) != cudaSuccess) {
        set_error("msplat_init_gaussians: memset failed");
        return MSPLAT_ERR_CUDA;
    }
    if (cudaStreamSynchronize(s) != cudaSuccess) {
        set_error("msplat_init_gaussians: %s", cudaGetErrorString(cudaGetLastError()));
        return MSPLAT_ERR_CUDA;
    }
    return MSPLAT_OK;
}

}  // extern "C"
