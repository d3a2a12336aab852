// kernels_eval.cu -- held-out image metrics on the device: SSIM with a
// separable, edge-clamped Gaussian window, PSNR and L1 of a rendered image
// against its ground truth, both (H, W, 3) float in HBM.
//
// Replaces the host metrics of the reference's evaluate()
// (python/bindings.cpp:186-216): ssim_eval (core/src/ssim.cpp:61-123),
// psnr and l1_loss (core/src/model.cpp:24-40), which need the rendered
// image and the ground truth copied to the host and take seconds per view
// at full resolution.
//
// One kernel pass: each 32 x 32 tile stages the channel's rows with a
// 5-pixel halo (indices clamped at the image border) in shared memory,
// blurs the five moment maps (x, y, x^2, y^2, xy) horizontally then
// vertically, forms the per-pixel SSIM and accumulates it, the squared and
// the absolute differences in double.  Compiled with --fmad=false: every
// per-pixel float is the reference's; only the order of the double sums
// differs, far below float resolution.
#include <cuda_runtime.h>

#include <cmath>
#include <vector>

#include "../../include/msplat_engine.h"
#include "engine.h"

namespace msp {
namespace {

constexpr int kTile = 32;
constexpr int kHalo = 5;  // window sizes up to 11
constexpr int kSpan = kTile + 2 * kHalo;
constexpr int kMaxWindow = 2 * kHalo + 1;
constexpr int kEvalThreads = 256;

__constant__ float c_window[kMaxWindow];

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

__global__ void __launch_bounds__(kEvalThreads)
eval_metrics_kernel(const float* __restrict__ r, const float* __restrict__ g, int H, int W, int ws,
                    double* __restrict__ partial)
{
    __shared__ float sr[kSpan][kSpan + 1];
    __shared__ float sg[kSpan][kSpan + 1];
    __shared__ float hs[5][kSpan][kTile + 1];
    __shared__ double red[3][kEvalThreads / 32];

    const int x0 = blockIdx.x * kTile, y0 = blockIdx.y * kTile;
    const int tid = threadIdx.x;
    const int pad = ws / 2;
    const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
    double acc_ssim = 0.0, acc_sq = 0.0, acc_abs = 0.0;

    for (int c = 0; c < 3; c++) {
        for (int idx = tid; idx < kSpan * kSpan; idx += kEvalThreads) {
            const int j = idx / kSpan, i = idx % kSpan;
            const int yy = clampi(y0 - kHalo + j, 0, H - 1), xx = clampi(x0 - kHalo + i, 0, W - 1);
            const size_t o = ((size_t)yy * W + xx) * 3 + c;
            sr[j][i] = r[o];
            sg[j][i] = g[o];
        }
        __syncthreads();
        // horizontal pass over every staged row, for the tile's columns
        for (int idx = tid; idx < kSpan * kTile; idx += kEvalThreads) {
            const int j = idx / kTile, i = idx % kTile;
            const int x = x0 + i;
            float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f, s4 = 0.f;
            for (int k = 0; k < ws; k++) {
                const int lx = clampi(x + k - pad, 0, W - 1) - (x0 - kHalo);
                const float a = sr[j][lx], b = sg[j][lx], wk = c_window[k];
                s0 += a * wk;
                s1 += b * wk;
                s2 += (a * a) * wk;
                s3 += (b * b) * wk;
                s4 += (a * b) * wk;
            }
            hs[0][j][i] = s0;
            hs[1][j][i] = s1;
            hs[2][j][i] = s2;
            hs[3][j][i] = s3;
            hs[4][j][i] = s4;
        }
        __syncthreads();
        // vertical pass, SSIM map and the difference sums
        for (int idx = tid; idx < kTile * kTile; idx += kEvalThreads) {
            const int row = idx / kTile, i = idx % kTile;
            const int x = x0 + i, y = y0 + row;
            if (x >= W || y >= H) continue;
            float m1 = 0.f, m2 = 0.f, s11 = 0.f, s22 = 0.f, s12 = 0.f;
            for (int k = 0; k < ws; k++) {
                const int lj = clampi(y + k - pad, 0, H - 1) - (y0 - kHalo);
                const float wk = c_window[k];
                m1 += hs[0][lj][i] * wk;
                m2 += hs[1][lj][i] * wk;
                s11 += hs[2][lj][i] * wk;
                s22 += hs[3][lj][i] * wk;
                s12 += hs[4][lj][i] * wk;
            }
            const float m1sq = m1 * m1, m2sq = m2 * m2, m12 = m1 * m2;
            const float sig1 = s11 - m1sq, sig2 = s22 - m2sq, sig12 = s12 - m12;
            const float num = (2.0f * m12 + C1) * (2.0f * sig12 + C2);
            const float den = (m1sq + m2sq + C1) * (sig1 + sig2 + C2);
            acc_ssim += (double)(num / den);
            const float d = sr[row + kHalo][i + kHalo] - sg[row + kHalo][i + kHalo];
            acc_sq += (double)d * (double)d;
            acc_abs += (double)fabsf(d);
        }
        __syncthreads();
    }
    // block reduction: warp shuffles, then the warps' partials in order
    for (int off = 16; off; off >>= 1) {
        acc_ssim += __shfl_down_sync(0xffffffffu, acc_ssim, off);
        acc_sq += __shfl_down_sync(0xffffffffu, acc_sq, off);
        acc_abs += __shfl_down_sync(0xffffffffu, acc_abs, off);
    }
    if ((tid & 31) == 0) {
        red[0][tid >> 5] = acc_ssim;
        red[1][tid >> 5] = acc_sq;
        red[2][tid >> 5] = acc_abs;
    }
    __syncthreads();
    if (tid < 3) {
        double s = 0.0;
        for (int w = 0; w < kEvalThreads / 32; w++) s += red[tid][w];
        partial[(size_t)(blockIdx.y * gridDim.x + blockIdx.x) * 3 + tid] = s;
    }
}

// Sums the per-tile partials in a fixed order (one block).
__global__ void eval_finish_kernel(const double* __restrict__ partial, int tiles, double* __restrict__ out)
{
    __shared__ double red[3][32];
    const int lane = threadIdx.x & 31, q = threadIdx.x >> 5;  // q: metric 0..2
    double s = 0.0;
    for (int t = lane; t < tiles; t += 32) s += partial[(size_t)t * 3 + q];
    red[q][lane] = s;
    __syncwarp();
    if (lane == 0) {
        double tot = 0.0;
        for (int l = 0; l < 32; l++) tot += red[q][l];
        out[q] = tot;
    }
}

}  // namespace
}  // namespace msp

using namespace msp;

extern "C" {

int msplat_eval_metrics(const float* rendered, const float* gt, int height, int width,
                        int window_size, float sigma, float* psnr, float* ssim, float* l1)
{
    if (!rendered || !gt || height <= 0 || width <= 0 || window_size < 1 ||
        window_size > kMaxWindow || !(sigma > 0.f)) {
        set_error("msplat_eval_metrics: invalid arguments");
        return MSPLAT_ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(engine_mutex());
    int rc = engine_init();
    if (rc) return rc;
    // the 1D Gaussian window of ssim_eval (ssim.cpp:69-76)
    std::vector<float> win(kMaxWindow, 0.f);
    float wsum = 0;
    for (int i = 0; i < window_size; i++) {
        const float x = (float)(i - window_size / 2);
        win[i] = std::exp(-(x * x) / (2.0f * sigma * sigma));
        wsum += win[i];
    }
    for (int i = 0; i < window_size; i++) win[i] /= wsum;
    cudaStream_t s = engine_stream();
    const dim3 grid((width + kTile - 1) / kTile, (height + kTile - 1) / kTile);
    const int tiles = (int)(grid.x * grid.y);
    double* dev = nullptr;
    if (cudaMallocAsync(&dev, ((size_t)tiles * 3 + 3) * sizeof(double), s) != cudaSuccess) {
        cudaGetLastError();
        set_error("msplat_eval_metrics: out of device memory");
        return MSPLAT_ERR_CUDA;
    }
    cudaMemcpyToSymbolAsync(c_window, win.data(), sizeof(float) * kMaxWindow, 0,
                            cudaMemcpyHostToDevice, s);
    eval_metrics_kernel<<<grid, kEvalThreads, 0, s>>>(rendered, gt, height, width, window_size, dev);
    eval_finish_kernel<<<1, 96, 0, s>>>(dev, tiles, dev + (size_t)tiles * 3);
    engine_add_launches(2);
    double sums[3] = {0, 0, 0};
    cudaMemcpyAsync(sums, dev + (size_t)tiles * 3, sizeof(sums), cudaMemcpyDeviceToHost, s);
    cudaFreeAsync(dev, s);
    const cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        set_error("msplat_eval_metrics: %s", cudaGetErrorString(e));
        return MSPLAT_ERR_CUDA;
    }
    const long long n = (long long)height * width * 3;
    // ssim_eval's count is an int; psnr and l1_loss divide by the int64 numel
    if (ssim) *ssim = (float)(sums[0] / (int)n);
    if (psnr) *psnr = (float)(10.0f * std::log10(1.0 / (sums[1] / (double)n)));
    if (l1) *l1 = (float)(sums[2] / (double)n);
    return MSPLAT_OK;
}

}  // extern "C"
