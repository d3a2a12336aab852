// kernels_densify.cu -- densification (split / duplicate / cull / compact)
// and the opacity reset of the training schedule, on the GPU.
//
// Reference: msplat_densify (core/metal/msplat_metal.mm:1337-1592) with its
// kernels (msplat_metal.metal:3466-3729, scans :2368-2439), and the CPU
// opacity reset of Model::afterTrain (core/src/model.cpp:280-290).  Compiled
// with --fmad=false: classification thresholds, the split children's
// positions and the cull decisions are bit-identical to the CPU oracle
// (same exp, IEEE sqrt and division, no contraction).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>

#include "../../include/msplat_engine.h"
#include "engine.h"
#include "msp_math.cuh"

namespace msp {
namespace {

constexpr int kScanBlock = 1024;

__device__ __forceinline__ float max_exp_scale(const float* s)
{
    return fmaxf(fmaxf(msp_expf(s[0]), msp_expf(s[1])), msp_expf(s[2]));
}

// densify_classify_kernel (msplat_metal.metal:3475-3509)
__global__ void classify_kernel(int N, const float* __restrict__ grad_norm,
                                const float* __restrict__ vis_counts,
                                const float* __restrict__ scales, const float* __restrict__ max_2d,
                                float half_max_dim, float grad_thresh, float size_thresh,
                                float screen_thresh, int check_screen, int* __restrict__ split,
                                int* __restrict__ dup)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N) return;
    const float vc = vis_counts[i];
    if (vc <= 0.0f) {
        split[i] = 0;
        dup[i] = 0;
        return;
    }
    const float avg_grad = __fmul_rn(__fdiv_rn(grad_norm[i], vc), half_max_dim);
    const bool high_grad = avg_grad > grad_thresh;
    const bool is_large = max_exp_scale(scales + 3 * (size_t)i) > size_thresh;
    bool do_split = is_large;
    if (check_screen && max_2d[i] > screen_thresh) do_split = true;
    split[i] = do_split && high_grad;
    dup[i] = !is_large && high_grad;
}

// Inclusive scan of n ints in three launches: per-block totals, one block
// scanning the totals (exclusive), per-block scan plus the block's offset.
__global__ void __launch_bounds__(kScanBlock)
block_totals_kernel(const int* __restrict__ in, int n, int* __restrict__ totals)
{
    __shared__ int s[kScanBlock / 32];
    const int i = blockIdx.x * kScanBlock + threadIdx.x;
    int v = i < n ? in[i] : 0;
    v = __reduce_add_sync(0xffffffffu, v);
    if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int w = 0; w < kScanBlock / 32; w++) t += s[w];
        totals[blockIdx.x] = t;
    }
}

__global__ void __launch_bounds__(kScanBlock)
scan_totals_kernel(int* __restrict__ totals, int nblocks)
{
    // one CTA; exclusive scan in chunks of kScanBlock
    __shared__ int s_warp[kScanBlock / 32];
    __shared__ int s_carry;
    if (threadIdx.x == 0) s_carry = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int base = 0; base < nblocks; base += kScanBlock) {
        const int i = base + threadIdx.x;
        const int v = i < nblocks ? totals[i] : 0;
        int incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += u;
        }
        if (lane == 31) s_warp[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const int wv = s_warp[lane];
            int wi = wv;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += u;
            }
            s_warp[lane] = wi - wv;
        }
        __syncthreads();
        const int carry = s_carry;
        if (i < nblocks) totals[i] = carry + s_warp[warp] + incl - v;
        __syncthreads();
        if (threadIdx.x == kScanBlock - 1) s_carry = carry + s_warp[warp] + incl;
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kScanBlock)
block_scan_kernel(const int* __restrict__ in, int n, const int* __restrict__ offsets,
                  int* __restrict__ out)
{
    __shared__ int s_warp[kScanBlock / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int i = blockIdx.x * kScanBlock + threadIdx.x;
    const int v = i < n ? in[i] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int wv = s_warp[lane];
        int wi = wv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += u;
        }
        s_warp[lane] = wi - wv;
    }
    __syncthreads();
    if (i < n) out[i] = offsets[blockIdx.x] + s_warp[warp] + incl;
}

void scan_inclusive(const int* in, int* out, int n, int* totals, cudaStream_t s)
{
    if (n <= 0) return;
    const int blocks = (n + kScanBlock - 1) / kScanBlock;
    block_totals_kernel<<<blocks, kScanBlock, 0, s>>>(in, n, totals);
    scan_totals_kernel<<<1, kScanBlock, 0, s>>>(totals, blocks);
    block_scan_kernel<<<blocks, kScanBlock, 0, s>>>(in, n, totals, out);
}

struct Groups {
    float* p[kGroups];
    float* m[kGroups];
    float* v[kGroups];
    int stride[kGroups];
};

// densify_append_split_kernel (msplat_metal.metal:3514-3600): two children
// at N + 2*ord and N + 2*ord + 1 around the parent, offsets R(q) * (sample *
// exp(scale)); children get scale - ln 1.6 and zero Adam state; the parent's
// scale is shrunk in place.
__global__ void split_kernel(int N, const int* __restrict__ split, const int* __restrict__ prefix,
                             const float* __restrict__ samples, float log_size_fac, Groups G)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N || split[i] == 0) return;
    const int ord = prefix[i] - 1;
    const float* q = G.p[2] + 4 * (size_t)i;
    float qw = q[0], qx = q[1], qy = q[2], qz = q[3];
    const float qlen = __fsqrt_rn(((qw * qw + qx * qx) + qy * qy) + qz * qz);
    qw = __fdiv_rn(qw, qlen);
    qx = __fdiv_rn(qx, qlen);
    qy = __fdiv_rn(qy, qlen);
    qz = __fdiv_rn(qz, qlen);
    float* sp = G.p[1] + 3 * (size_t)i;
    const float sx = msp_expf(sp[0]), sy = msp_expf(sp[1]), sz = msp_expf(sp[2]);
    for (int k = 0; k < 2; k++) {
        const size_t child = (size_t)N + 2 * (size_t)ord + k;
        const float* rs = samples + 3 * (size_t)(ord * 2 + k);
        const float r0 = rs[0] * sx, r1 = rs[1] * sy, r2 = rs[2] * sz;
        const float v0 = ((1.f - 2.f * (qy * qy + qz * qz)) * r0 + 2.f * (qx * qy - qw * qz) * r1) +
                         2.f * (qx * qz + qw * qy) * r2;
        const float v1 = (2.f * (qx * qy + qw * qz) * r0 + (1.f - 2.f * (qx * qx + qz * qz)) * r1) +
                         2.f * (qy * qz - qw * qx) * r2;
        const float v2 = (2.f * (qx * qz - qw * qy) * r0 + 2.f * (qy * qz + qw * qx) * r1) +
                         (1.f - 2.f * (qx * qx + qy * qy)) * r2;
        float* pm = G.p[0];
        pm[child * 3] = pm[(size_t)i * 3] + v0;
        pm[child * 3 + 1] = pm[(size_t)i * 3 + 1] + v1;
        pm[child * 3 + 2] = pm[(size_t)i * 3 + 2] + v2;
        for (int j = 0; j < 3; j++) G.p[1][child * 3 + j] = sp[j] - log_size_fac;
        for (int gi = 2; gi < kGroups; gi++) {
            const int S = G.stride[gi];
            for (int j = 0; j < S; j++) G.p[gi][child * S + j] = G.p[gi][(size_t)i * S + j];
        }
        for (int gi = 0; gi < kGroups; gi++) {
            const int S = G.stride[gi];
            for (int j = 0; j < S; j++) {
                G.m[gi][child * S + j] = 0.f;
                G.v[gi][child * S + j] = 0.f;
            }
        }
    }
    for (int j = 0; j < 3; j++) sp[j] -= log_size_fac;
}

// densify_append_dup_kernel (msplat_metal.metal:3604-3651): a copy at
// N + 2*nSplits + ord with zero Adam state (after the split stage, so a
// parent that also splits is copied with its shrunk scale).
__global__ void dup_kernel(int N, const int* __restrict__ dup, const int* __restrict__ dprefix,
                           const int* __restrict__ sprefix, Groups G)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N || dup[i] == 0) return;
    const int n_split = sprefix[N - 1];
    const size_t dst = (size_t)N + 2 * (size_t)n_split + dprefix[i] - 1;
    for (int gi = 0; gi < kGroups; gi++) {
        const int S = G.stride[gi];
        for (int j = 0; j < S; j++) {
            G.p[gi][dst * S + j] = G.p[gi][(size_t)i * S + j];
            G.m[gi][dst * S + j] = 0.f;
            G.v[gi][dst * S + j] = 0.f;
        }
    }
}

// densify_cull_classify_kernel (msplat_metal.metal:3656-3694) over 3N slots
__global__ void cull_kernel(int N, int worst, const int* __restrict__ sprefix,
                            const int* __restrict__ dprefix, const int* __restrict__ split,
                            const float* __restrict__ opac, const float* __restrict__ scales,
                            const float* __restrict__ max_2d, float cull_alpha, float cull_scale,
                            float cull_screen, int check_huge, int check_screen,
                            int* __restrict__ keep)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= worst) return;
    const int n_split = N > 0 ? sprefix[N - 1] : 0;
    const int n_dup = N > 0 ? dprefix[N - 1] : 0;
    const int n_new = N + 2 * n_split + n_dup;
    if (i >= n_new) {
        keep[i] = 0;
        return;
    }
    bool cull = sigmoid_ref(opac[i]) < cull_alpha;
    if (i < N && split[i] != 0) cull = true;
    if (check_huge) {
        if (max_exp_scale(scales + 3 * (size_t)i) > cull_scale) cull = true;
        if (check_screen && i < N && max_2d[i] > cull_screen) cull = true;
    }
    keep[i] = cull ? 0 : 1;
}

// compact_scatter_kernel / compact_copy_back_kernel (:3698-3729)
__global__ void compact_scatter_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                       const int* __restrict__ prefix, const int* __restrict__ keep,
                                       long long total, int stride)
{
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const long long e = t / stride;
        if (!keep[e]) continue;
        dst[(long long)(prefix[e] - 1) * stride + (t - e * stride)] = src[t];
    }
}

__global__ void copy_back_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                 const int* __restrict__ prefix, int last, int stride)
{
    const long long total = (long long)prefix[last] * stride;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x)
        dst[t] = src[t];
}

// The opacity reset of Model::afterTrain (model.cpp:280-290): logits above
// logit(0.2) are lowered to it; the opacity moments are zeroed.
__global__ void reset_opacity_kernel(float* __restrict__ opac, float* __restrict__ m,
                                     float* __restrict__ v, int n)
{
    const float reset_logit = -1.3862943611198906f;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        if (opac[i] > reset_logit) opac[i] = reset_logit;
        m[i] = 0.f;
        v[i] = 0.f;
    }
}

// Engine-owned scratch for callers that pass none (grow-only).
struct DensifyScratch {
    int* ints = nullptr;
    long long ints_cap = 0;
    float* floats = nullptr;
    long long floats_cap = 0;
};
DensifyScratch g_scratch;

int grow(void** p, long long& cap, long long want, size_t elem)
{
    if (want <= cap) return MSPLAT_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    cap = 0;
    if (cudaMalloc(p, (size_t)std::max(want, 1LL) * elem) != cudaSuccess) {
        set_error("msplat_densify: cudaMalloc of %lld scratch elements failed", want);
        return MSPLAT_ERR_CUDA;
    }
    cap = want;
    return MSPLAT_OK;
}

#define DN_CUDA(expr)                                                                     \
    do {                                                                                  \
        cudaError_t e_ = (expr);                                                          \
        if (e_ != cudaSuccess) {                                                          \
            set_error("msplat_densify: %s failed: %s", #expr, cudaGetErrorString(e_));    \
            return MSPLAT_ERR_CUDA;                                                       \
        }                                                                                 \
    } while (0)

}  // namespace
}  // namespace msp

using namespace msp;

extern "C" {

int msplat_densify(int N, int buf_capacity, float grad_thresh, float size_thresh,
                   float screen_thresh, int check_screen, float cull_alpha_thresh,
                   float cull_scale_thresh, float cull_screen_size, int check_huge,
                   const float* xys_grad_norm, const float* vis_counts, const float* max_2d_size,
                   float half_max_dim, float* means_buf, float* scales_buf, float* quats_buf,
                   float* features_dc_buf, float* features_rest_buf, float* opacities_buf,
                   int fr_stride, float* const* adam_exp_avg_buf,
                   float* const* adam_exp_avg_sq_buf, int* split_flag, int* dup_flag,
                   int* split_prefix, int* dup_prefix, int* keep_flag, int* keep_prefix,
                   int* block_totals, float* compact_scratch, const float* random_samples)
{
    std::lock_guard<std::mutex> lk(engine_mutex());
    int rc = engine_init();
    if (rc) return rc;
    const long long worst = 3LL * N;
    if (N < 0 || fr_stride < 0 || worst > buf_capacity || worst >= (1LL << 31) ||
        !xys_grad_norm || !vis_counts || !max_2d_size || !means_buf || !scales_buf ||
        !quats_buf || !features_dc_buf || !opacities_buf || (fr_stride > 0 && !features_rest_buf) ||
        !adam_exp_avg_buf || !adam_exp_avg_sq_buf || !random_samples) {
        set_error("msplat_densify: invalid arguments (N=%d, capacity %d, 3N must fit)", N,
                  buf_capacity);
        return MSPLAT_ERR_ARG;
    }
    Groups G{};
    float* params[kGroups] = {means_buf, scales_buf, quats_buf, features_dc_buf,
                              features_rest_buf, opacities_buf};
    const int strides[kGroups] = {3, 3, 4, 3, fr_stride, 1};
    for (int gi = 0; gi < kGroups; gi++) {
        G.p[gi] = params[gi];
        G.m[gi] = adam_exp_avg_buf[gi];
        G.v[gi] = adam_exp_avg_sq_buf[gi];
        G.stride[gi] = strides[gi];
        if (strides[gi] && (!G.m[gi] || !G.v[gi])) {
            set_error("msplat_densify: missing Adam buffer for group %d", gi);
            return MSPLAT_ERR_ARG;
        }
    }
    if (N == 0) return 0;
    // scratch: the caller's (the reference's argument list) or the engine's
    const long long nb = (worst + kScanBlock - 1) / kScanBlock + 1;
    if (!split_flag || !dup_flag || !split_prefix || !dup_prefix || !keep_flag || !keep_prefix ||
        !block_totals) {
        if ((rc = grow((void**)&g_scratch.ints, g_scratch.ints_cap, 4LL * N + 2 * worst + nb,
                       sizeof(int))))
            return rc;
        int* p = g_scratch.ints;
        split_flag = p; p += N;
        dup_flag = p; p += N;
        split_prefix = p; p += N;
        dup_prefix = p; p += N;
        keep_flag = p; p += worst;
        keep_prefix = p; p += worst;
        block_totals = p;
    }
    const int max_stride = std::max(4, fr_stride);
    if (!compact_scratch) {
        if ((rc = grow((void**)&g_scratch.floats, g_scratch.floats_cap, worst * max_stride,
                       sizeof(float))))
            return rc;
        compact_scratch = g_scratch.floats;
    }
    const cudaStream_t s = engine_stream();
    const int tb = 256;
    const int gN = (N + tb - 1) / tb;
    classify_kernel<<<gN, tb, 0, s>>>(N, xys_grad_norm, vis_counts, scales_buf, max_2d_size,
                                      half_max_dim, grad_thresh, size_thresh, screen_thresh,
                                      check_screen, split_flag, dup_flag);
    scan_inclusive(split_flag, split_prefix, N, block_totals, s);
    scan_inclusive(dup_flag, dup_prefix, N, block_totals, s);
    split_kernel<<<gN, tb, 0, s>>>(N, split_flag, split_prefix, random_samples, logf(1.6f), G);
    dup_kernel<<<gN, tb, 0, s>>>(N, dup_flag, dup_prefix, split_prefix, G);
    const int gW = (int)((worst + tb - 1) / tb);
    cull_kernel<<<gW, tb, 0, s>>>(N, (int)worst, split_prefix, dup_prefix, split_flag,
                                  opacities_buf, scales_buf, max_2d_size, cull_alpha_thresh,
                                  cull_scale_thresh, cull_screen_size, check_huge, check_screen,
                                  keep_flag);
    scan_inclusive(keep_flag, keep_prefix, (int)worst, block_totals, s);
    int launches = 1 + 3 * 3 + 3;
    for (int b = 0; b < 3 * kGroups; b++) {
        const int gi = b % kGroups;
        if (!strides[gi]) continue;
        float* buf = b < kGroups ? G.p[gi] : b < 2 * kGroups ? G.m[gi] : G.v[gi];
        const long long total = worst * strides[gi];
        const int grid = (int)std::min<long long>((total + tb - 1) / tb, 148LL * 16);
        compact_scatter_kernel<<<grid, tb, 0, s>>>(buf, compact_scratch, keep_prefix, keep_flag,
                                                   total, strides[gi]);
        copy_back_kernel<<<grid, tb, 0, s>>>(compact_scratch, buf, keep_prefix, (int)worst - 1,
                                             strides[gi]);
        launches += 2;
    }
    engine_add_launches(launches);
    DN_CUDA(cudaGetLastError());
    int new_count = 0;
    DN_CUDA(cudaMemcpyAsync(&new_count, keep_prefix + worst - 1, sizeof(int),
                            cudaMemcpyDeviceToHost, s));
    DN_CUDA(cudaStreamSynchronize(s));
    return new_count;
}

int msplat_reset_opacity(float* opacities, float* exp_avg, float* exp_avg_sq, int n)
{
    std::lock_guard<std::mutex> lk(engine_mutex());
    int rc = engine_init();
    if (rc) return rc;
    if (n < 0 || (n > 0 && (!opacities || !exp_avg || !exp_avg_sq))) {
        set_error("msplat_reset_opacity: invalid arguments");
        return MSPLAT_ERR_ARG;
    }
    if (n == 0) return MSPLAT_OK;
    reset_opacity_kernel<<<std::min((n + 255) / 256, 148 * 8), 256, 0, engine_stream()>>>(
        opacities, exp_avg, exp_avg_sq, n);
    engine_add_launches(1);
    DN_CUDA(cudaGetLastError());
    return MSPLAT_OK;
}

}  // extern "C"
