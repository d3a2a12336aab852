// ref_io.cpp -- C entry points over the reference's own Gaussian file I/O
// (msplat core/src/loaders/save_gaussians.cpp: saveGaussianPly,
// saveGaussianSplat, loadGaussianPly), compiled from the reference's source
// where it lies into oracle/_ref/libmsplat_ref_io.so by build_ref.py.
//
// TEST INFRASTRUCTURE ONLY: the checker for the engine's msplat_save_ply /
// msplat_save_splat / msplat_load_ply.  The reference's MTensor has a plain
// C++ (host memory) form; the three Metal runtime calls that file makes
// (msplat_gpu_sync, gpu_empty, gpu_zeros) are given host versions here.
#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>
#include <vector>

#include "loaders.hpp"
#include "msplat.hpp"

MTensor gpu_empty(std::vector<int64_t> shape, DType dtype) { return MTensor(std::move(shape), dtype); }

MTensor gpu_zeros(std::vector<int64_t> shape, DType dtype)
{
    MTensor t(std::move(shape), dtype);
    t.zero();
    return t;
}

void msplat_gpu_sync() {}

namespace {

MTensor host_tensor(const float* src, std::vector<int64_t> shape)
{
    MTensor t(std::move(shape), DType::Float32);
    if (t.nbytes()) std::memcpy(t.data_ptr(), src, t.nbytes());
    return t;
}

thread_local std::string g_err;

}  // namespace

extern "C" {

const char* ref_io_last_error() { return g_err.c_str(); }

// params: means [n,3], scales [n,3], quats [n,4], dc [n,3], rest [n,B,3], opacities [n,1]
static int save_common(int which, const char* path, int step, int n, int rest_bases,
                       const float* const* params, int keep_crs, float scale,
                       const float* translation)
{
    try {
        const int64_t N = n;
        MTensor m = host_tensor(params[0], {N, 3}), s = host_tensor(params[1], {N, 3}),
                q = host_tensor(params[2], {N, 4}), dc = host_tensor(params[3], {N, 3}),
                fr = host_tensor(params[4], {N, rest_bases, 3}), op = host_tensor(params[5], {N, 1});
        GaussianParams p{m, s, q, dc, fr, op, scale,
                         {translation[0], translation[1], translation[2]}, keep_crs != 0};
        if (which == 0)
            saveGaussianPly(path, p, step);
        else
            saveGaussianSplat(path, p);
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

int ref_save_ply(const char* path, int step, int n, int rest_bases, const float* const* params,
                 int keep_crs, float scale, const float* translation)
{
    return save_common(0, path, step, n, rest_bases, params, keep_crs, scale, translation);
}

int ref_save_splat(const char* path, int n, const float* const* params, int keep_crs, float scale,
                   const float* translation)
{
    return save_common(1, path, 0, n, 0, params, keep_crs, scale, translation);
}

// Loads with the reference and copies out up to `capacity` rows per group;
// *n, *rest_bases receive the sizes.  Returns the step or -1 (error text in
// ref_io_last_error: the reference throws for unreadable files).
int ref_load_ply(const char* path, int keep_crs, float scale, const float* translation,
                 int capacity, float* const* out, int* n, int* rest_bases)
{
    try {
        LoadedGaussians g = loadGaussianPly(path, scale, translation, keep_crs != 0);
        *n = (int)g.means.size(0);
        *rest_bases = (int)g.featuresRest.size(1);
        if (*n > capacity) {
            g_err = "capacity too small";
            return -1;
        }
        MTensor* src[6] = {&g.means, &g.scales, &g.quats, &g.featuresDc, &g.featuresRest,
                           &g.opacities};
        for (int k = 0; k < 6; k++)
            if (out[k] && src[k]->nbytes()) std::memcpy(out[k], src[k]->data_ptr(), src[k]->nbytes());
        return g.step;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

}  // extern "C"
