// kernels_fwd.cu -- forward half of the step: projection + SH, tile binning,
// per-tile depth sort and the forward rasterizer.  Compiled with
// --fmad=false (see msp_math.cuh): every value here is bit-identical to the
// CPU oracle.
#include "engine.h"
#include "msp_math.cuh"
#include "tma.cuh"

namespace msp {

constexpr int kProjThreads = 128;
#ifndef MSP_SORT_THREADS
#define MSP_SORT_THREADS 128
#endif
constexpr int kSortThreads = MSP_SORT_THREADS;
#ifndef MSP_SORT_RADIX
#define MSP_SORT_RADIX 1
#endif
#ifndef MSP_RADIX_SPLIT
#define MSP_RADIX_SPLIT 1
#endif
#ifndef MSP_FWD_MIN_BLOCKS
#define MSP_FWD_MIN_BLOCKS 6
#endif
#ifndef MSP_SCATTER_ROUNDS
#define MSP_SCATTER_ROUNDS 1
#endif
#ifndef MSP_SORT_MIN_BLOCKS
#define MSP_SORT_MIN_BLOCKS 8
#endif
constexpr int kSortKMax = kSortRun / kSortThreads;  // keys per thread at most

// ---------------------------------------------------------------------------
// Projection + SH colour + tile counting.
// Reference: project_and_sh_forward_kernel, msplat_metal.metal:1695-1787,
// with helpers :53-317 and sh_coeffs_to_color :587-654.  The per-tile
// counting of scatter_to_prealloc_bins_kernel (:2025-2059) is fused here:
// each visible Gaussian adds one to every tile of its rect.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void sh_to_color(int degree, float x, float y, float z,
                                            const float* dc, const float* r, float col[3])
{
    const float C1 = MSP_SH_C1;
    float xx = x * x, xy = x * y, xz = x * z, yy = y * y, yz = y * z, zz = z * z;
#pragma unroll
    for (int c = 0; c < 3; c++) {
        float v = MSP_SH_C0 * dc[c];
        if (degree >= 1) {
            v += C1 * ((-y * r[0 * 3 + c] + z * r[1 * 3 + c]) - x * r[2 * 3 + c]);
            if (degree >= 2) {
                v += ((((kSH_C2[0] * xy * r[3 * 3 + c] + kSH_C2[1] * yz * r[4 * 3 + c]) +
                        kSH_C2[2] * ((2.f * zz - xx) - yy) * r[5 * 3 + c]) +
                       kSH_C2[3] * xz * r[6 * 3 + c]) +
                      kSH_C2[4] * (xx - yy) * r[7 * 3 + c]);
                if (degree >= 3) {
                    v += ((((((kSH_C3[0] * y * (3.f * xx - yy) * r[8 * 3 + c] +
                               kSH_C3[1] * xy * z * r[9 * 3 + c]) +
                              kSH_C3[2] * y * ((4.f * zz - xx) - yy) * r[10 * 3 + c]) +
                             kSH_C3[3] * z * ((2.f * zz - 3.f * xx) - 3.f * yy) * r[11 * 3 + c]) +
                            kSH_C3[4] * x * ((4.f * zz - xx) - yy) * r[12 * 3 + c]) +
                           kSH_C3[5] * z * (xx - yy) * r[13 * 3 + c]) +
                          kSH_C3[6] * x * (xx - 3.f * yy) * r[14 * 3 + c]);
                    if (degree >= 4) {
                        v += ((((((((kSH_C4[0] * xy * (xx - yy) * r[15 * 3 + c] +
                                     kSH_C4[1] * yz * (3.f * xx - yy) * r[16 * 3 + c]) +
                                    kSH_C4[2] * xy * (7.f * zz - 1.f) * r[17 * 3 + c]) +
                                   kSH_C4[3] * yz * (7.f * zz - 3.f) * r[18 * 3 + c]) +
                                  kSH_C4[4] * (zz * (35.f * zz - 30.f) + 3.f) * r[19 * 3 + c]) +
                                 kSH_C4[5] * xz * (7.f * zz - 3.f) * r[20 * 3 + c]) +
                                kSH_C4[6] * (xx - yy) * (7.f * zz - 1.f) * r[21 * 3 + c]) +
                               kSH_C4[7] * xz * (xx - 3.f * yy) * r[22 * 3 + c]) +
                              kSH_C4[8] * (xx * (xx - 3.f * yy) - yy * (3.f * xx - yy)) *
                                  r[23 * 3 + c]);
                    }
                }
            }
        }
        col[c] = v;
    }
}

// Block layout of the staged inputs in shared memory (floats).
struct ProjStage {
    static constexpr int kMeans = 0;
    static constexpr int kScales = kMeans + 3 * kProjThreads;
    static constexpr int kQuats = kScales + 3 * kProjThreads;
    static constexpr int kOpac = kQuats + 4 * kProjThreads;
    static constexpr int kDc = kOpac + kProjThreads;
    static constexpr int kRest = kDc + 3 * kProjThreads;  // + kProjThreads * rest_stride
};

// All of a block's inputs (means, scales, quats, opacities, dc and the
// SH-rest rows, ~30 KB for 128 Gaussians at SH degree 3) are staged in
// shared memory first: by seven 1D bulk copies issued together when the
// block is full and the arrays are 16-byte aligned, else by plain loads.
// Every byte of the block is then in flight at once instead of in two
// dependent rounds (geometry, then the SH rows of the visible Gaussians).
template <bool ZERO_GRADS>
__global__ void __launch_bounds__(kProjThreads)
project_forward_kernel(const StepParams* __restrict__ P, int N, const float* __restrict__ means,
                       const float* __restrict__ scales, const float* __restrict__ quats,
                       const float* __restrict__ dc, const float* __restrict__ rest,
                       const float* __restrict__ opac, ProjOut out, int* __restrict__ tile_count,
                       float* __restrict__ grad_acc, int rest_stride, int bulk,
                       int* __restrict__ err)
{
    extern __shared__ __align__(16) float sm[];
    __shared__ unsigned long long s_bar;
    __shared__ int s_fail;
    const float* s_means = sm + ProjStage::kMeans;
    const float* s_scales = sm + ProjStage::kScales;
    const float* s_quats = sm + ProjStage::kQuats;
    const float* s_opac = sm + ProjStage::kOpac;
    const float* s_dc = sm + ProjStage::kDc;
    const float* s_rest = sm + ProjStage::kRest;
    const int tid = threadIdx.x;
    const int base = blockIdx.x * kProjThreads;
    const int i = base + tid;
    const int cnt = min(kProjThreads, N - base);
    const size_t gb = (size_t)base;

    if (bulk && cnt == kProjThreads) {
        if (tid == 0) mbar_init(&s_bar);
        __syncthreads();
        if (tid == 0) {
            const unsigned rs_bytes = (unsigned)(kProjThreads * rest_stride * 4);
            mbar_expect_tx(&s_bar, (unsigned)(ProjStage::kRest * 4) + rs_bytes);
            bulk_load(sm + ProjStage::kMeans, means + gb * 3, kProjThreads * 12, &s_bar);
            bulk_load(sm + ProjStage::kScales, scales + gb * 3, kProjThreads * 12, &s_bar);
            bulk_load(sm + ProjStage::kQuats, quats + gb * 4, kProjThreads * 16, &s_bar);
            bulk_load(sm + ProjStage::kOpac, opac + gb, kProjThreads * 4, &s_bar);
            bulk_load(sm + ProjStage::kDc, dc + gb * 3, kProjThreads * 12, &s_bar);
            if (rs_bytes) bulk_load(sm + ProjStage::kRest, rest + gb * rest_stride, rs_bytes, &s_bar);
            s_fail = !mbar_wait_bounded(&s_bar, 0);
            if (s_fail) {
                atomicOr(err, kErrStageTimeout);
                mbar_wait_bounded(&s_bar, 0);  // let copies still in flight land
            }
        }
        __syncthreads();
        if (s_fail) {  // leave the block's Gaussians culled
            out.radii[i] = 0;
            return;
        }
    } else {
        for (int e = tid; e < cnt * 3; e += kProjThreads) {
            sm[ProjStage::kMeans + e] = means[gb * 3 + e];
            sm[ProjStage::kScales + e] = scales[gb * 3 + e];
            sm[ProjStage::kDc + e] = dc[gb * 3 + e];
        }
        for (int e = tid; e < cnt * 4; e += kProjThreads) sm[ProjStage::kQuats + e] = quats[gb * 4 + e];
        if (tid < cnt) sm[ProjStage::kOpac + tid] = opac[gb + tid];
        for (int e = tid; e < cnt * rest_stride; e += kProjThreads)
            sm[ProjStage::kRest + e] = rest[gb * rest_stride + e];
        __syncthreads();
    }

    bool vis = false;
    float px_c = 0.f, py_c = 0.f;
    int x0 = 0, y0 = 0, x1 = 0, y1 = 0;
    float p[3] = {0.f, 0.f, 0.f};
    if (i < N) {
        out.radii[i] = 0;
        p[0] = s_means[3 * tid];
        p[1] = s_means[3 * tid + 1];
        p[2] = s_means[3 * tid + 2];
        const float* vm = P->viewmat;
        // clip_near_plane / transform_4x3 (:90-97, :134-145)
        float pv0 = ((vm[0] * p[0] + vm[1] * p[1]) + vm[2] * p[2]) + vm[3];
        float pv1 = ((vm[4] * p[0] + vm[5] * p[1]) + vm[6] * p[2]) + vm[7];
        float pv2 = ((vm[8] * p[0] + vm[9] * p[1]) + vm[10] * p[2]) + vm[11];
        if (!(pv2 <= P->clip_thresh)) {
            float s0 = msp_expf(s_scales[3 * tid]);
            float s1 = msp_expf(s_scales[3 * tid + 1]);
            float s2 = msp_expf(s_scales[3 * tid + 2]);
            const float4 q4 = make_float4(s_quats[4 * tid], s_quats[4 * tid + 1],
                                          s_quats[4 * tid + 2], s_quats[4 * tid + 3]);
            // quat_to_rotmat (:111-131): memory order w, x, y, z
            float qs = rsqrt_ieee(((q4.w * q4.w + q4.x * q4.x) + q4.y * q4.y) + q4.z * q4.z);
            float w = q4.x * qs, x = q4.y * qs, y = q4.z * qs, z = q4.w * qs;
            // R columns (Metal float3x3 is column-major)
            float R[3][3] = {{1.f - 2.f * (y * y + z * z), 2.f * (x * y + w * z), 2.f * (x * z - w * y)},
                             {2.f * (x * y - w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z + w * x)},
                             {2.f * (x * z + w * y), 2.f * (y * z - w * x), 1.f - 2.f * (x * x + y * y)}};
            float gsc = P->glob_scale;
            float sc[3] = {gsc * s0, gsc * s1, gsc * s2};
            float M[3][3];
#pragma unroll
            for (int c = 0; c < 3; c++)
#pragma unroll
                for (int r = 0; r < 3; r++) M[c][r] = R[c][r] * sc[c];
            // tmp = M * M^T, cov3d upper triangle (:157-172)
            float cv[6];
            {
                float t00 = (M[0][0] * M[0][0] + M[1][0] * M[1][0]) + M[2][0] * M[2][0];
                float t01 = (M[0][1] * M[0][0] + M[1][1] * M[1][0]) + M[2][1] * M[2][0];
                float t02 = (M[0][2] * M[0][0] + M[1][2] * M[1][0]) + M[2][2] * M[2][0];
                float t11 = (M[0][1] * M[0][1] + M[1][1] * M[1][1]) + M[2][1] * M[2][1];
                float t12 = (M[0][2] * M[0][1] + M[1][2] * M[1][1]) + M[2][2] * M[2][1];
                float t22 = (M[0][2] * M[0][2] + M[1][2] * M[1][2]) + M[2][2] * M[2][2];
                cv[0] = t00; cv[1] = t01; cv[2] = t02; cv[3] = t11; cv[4] = t12; cv[5] = t22;
            }
            // project_cov3d_ewa (:241-281)
            const float fx = P->fx, fy = P->fy;
            float lim_x = 1.3f * P->tan_fovx, lim_y = 1.3f * P->tan_fovy;
            float qx = pv2 * fminf(lim_x, fmaxf(-lim_x, pv0 / pv2));
            float qy = pv2 * fminf(lim_y, fmaxf(-lim_y, pv1 / pv2));
            float rz = 1.f / pv2;
            float rz2 = rz * rz;
            float j00 = fx * rz, j11 = fy * rz;
            float j20 = (-fx * qx) * rz2, j21 = (-fy * qy) * rz2;
            float t0[3], t1[3];
#pragma unroll
            for (int k = 0; k < 3; k++) {
                t0[k] = j00 * vm[k] + j20 * vm[8 + k];
                t1[k] = j11 * vm[4 + k] + j21 * vm[8 + k];
            }
            float tv0[3] = {(t0[0] * cv[0] + t0[1] * cv[1]) + t0[2] * cv[2],
                            (t0[0] * cv[1] + t0[1] * cv[3]) + t0[2] * cv[4],
                            (t0[0] * cv[2] + t0[1] * cv[4]) + t0[2] * cv[5]};
            float tv1[3] = {(t1[0] * cv[0] + t1[1] * cv[1]) + t1[2] * cv[2],
                            (t1[0] * cv[1] + t1[1] * cv[3]) + t1[2] * cv[4],
                            (t1[0] * cv[2] + t1[1] * cv[4]) + t1[2] * cv[5]};
            float c2x = ((tv0[0] * t0[0] + tv0[1] * t0[1]) + tv0[2] * t0[2]) + 0.3f;
            float c2y = (tv0[0] * t1[0] + tv0[1] * t1[1]) + tv0[2] * t1[2];
            float c2z = ((tv1[0] * t1[0] + tv1[1] * t1[1]) + tv1[2] * t1[2]) + 0.3f;
            // compute_cov2d_bounds (:283-305)
            float det = c2x * c2z - c2y * c2y;
            if (det != 0.f) {
                float inv_det = 1.f / det;
                float ca = c2z * inv_det, cb = -c2y * inv_det, cc = c2x * inv_det;
                float bb = 0.5f * (c2x + c2z);
                float disc = sqrtf(fmaxf(0.1f, bb * bb - det));
                float radius = ceilf(3.f * sqrtf(bb + disc));
                // project_pix (:308-317)
                const float* pm = P->projmat;
                float h0 = ((pm[0] * p[0] + pm[1] * p[1]) + pm[2] * p[2]) + pm[3];
                float h1 = ((pm[4] * p[0] + pm[5] * p[1]) + pm[6] * p[2]) + pm[7];
                float h3 = ((pm[12] * p[0] + pm[13] * p[1]) + pm[14] * p[2]) + pm[15];
                float rw = 1.f / (h3 + 1e-6f);
                float ndx = h0 * rw, ndy = h1 * rw;
                px_c = ((0.5f * (float)P->img_w) * ndx + P->cx) - 0.5f;
                py_c = ((0.5f * (float)P->img_h) * ndy + P->cy) - 0.5f;
                float ax = ceilf(3.0f * sqrtf(c2x));
                float ay = ceilf(3.0f * sqrtf(c2z));
                // get_tile_bbox (:57-87)
                float tcx = px_c / 16.f, tcy = py_c / 16.f;
                float trx = ax / 16.f, try_ = ay / 16.f;
                x0 = min(max(0, f2i(tcx - trx)), P->tiles_x);
                x1 = min(max(0, f2i((tcx + trx) + 1)), P->tiles_x);
                y0 = min(max(0, f2i(tcy - try_)), P->tiles_y);
                y1 = min(max(0, f2i((tcy + try_) + 1)), P->tiles_y);
                int area = (x1 - x0) * (y1 - y0);
                if (area > 0) {
                    vis = true;
                    out.radii[i] = f2i(radius);
                    out.depth[i] = pv2;
                    out.xy[i] = make_float2(px_c, py_c);
                    out.conic_op[i] = make_float4(ca, cb, cc, sigmoid_ref(s_opac[tid]));
                    out.rect[i] = make_uint2((unsigned)x0 | ((unsigned)y0 << 16),
                                             (unsigned)x1 | ((unsigned)y1 << 16));
                }
            }
        }
    }
    if (!vis) return;
    // SH colour (:1780-1786): viewdir = normalize(p - cam_pos)
    float d0 = p[0] - P->cam_pos[0], d1 = p[1] - P->cam_pos[1], d2 = p[2] - P->cam_pos[2];
    float dn = rsqrt_ieee((d0 * d0 + d1 * d1) + d2 * d2);
    float col[3];
    float dcv[3] = {s_dc[3 * tid], s_dc[3 * tid + 1], s_dc[3 * tid + 2]};
    sh_to_color(P->degrees_to_use, d0 * dn, d1 * dn, d2 * dn, dcv, s_rest + tid * rest_stride, col);
    out.rgb[i] = make_float4(col[0], col[1], col[2], 0.f);
    if (ZERO_GRADS) {  // training: the SH-rest Adam's copy of the mean
        out.sh_mean[3 * (size_t)i] = p[0];
        out.sh_mean[3 * (size_t)i + 1] = p[1];
        out.sh_mean[3 * (size_t)i + 2] = p[2];
    }
    const int tx_n = P->tiles_x;
    if (P->dense_bins && (x1 - x0) * (y1 - y0) > kDenseArea) {
        // corners of the rect in a 2D difference array; a corner past the
        // grid's last row or column changes no tile of the grid
        const int ty_n = P->tiles_y;
        atomicAdd(&tile_count[(y0 * tx_n + x0) * kCountPitch + 2], 1);
        if (x1 < tx_n) atomicAdd(&tile_count[(y0 * tx_n + x1) * kCountPitch + 2], -1);
        if (y1 < ty_n) atomicAdd(&tile_count[(y1 * tx_n + x0) * kCountPitch + 2], -1);
        if (x1 < tx_n && y1 < ty_n) atomicAdd(&tile_count[(y1 * tx_n + x1) * kCountPitch + 2], 1);
    } else {
        for (int ty = y0; ty < y1; ty++)
            for (int tx = x0; tx < x1; tx++) atomicAdd(&tile_count[(ty * tx_n + tx) * kCountPitch], 1);
    }
    if (ZERO_GRADS) {
        float* g = grad_acc + (size_t)i * kGradStride;
#pragma unroll
        for (int k = 0; k < kGradStride; k++) g[k] = 0.f;
    }
}

void launch_project_forward(const StepParams* P, int N, const float* means, const float* scales,
                            const float* quats, const float* dc, const float* rest,
                            const float* opac, const Buffers& B, bool zero_grads,
                            int degrees_to_use_host, int rest_stride_host, cudaStream_t s)
{
    (void)degrees_to_use_host;
    if (N <= 0) return;
    const size_t smem = (size_t)(ProjStage::kRest + kProjThreads * rest_stride_host) * sizeof(float);
    const uintptr_t mis = (uintptr_t)means | (uintptr_t)scales | (uintptr_t)quats |
                          (uintptr_t)dc | (uintptr_t)opac | (rest_stride_host ? (uintptr_t)rest : 0);
    const int bulk = (mis & 15) == 0 && smem <= 48 * 1024;
    const int grid = (N + kProjThreads - 1) / kProjThreads;
    if (zero_grads)
        project_forward_kernel<true><<<grid, kProjThreads, smem, s>>>(
            P, N, means, scales, quats, dc, rest, opac, B.proj, B.tile_count, B.grad_acc,
            rest_stride_host, bulk, B.err);
    else
        project_forward_kernel<false><<<grid, kProjThreads, smem, s>>>(
            P, N, means, scales, quats, dc, rest, opac, B.proj, B.tile_count, nullptr,
            rest_stride_host, bulk, B.err);
}

// ---------------------------------------------------------------------------
// Exclusive scan of per-tile counts (one CTA, warp-shuffle scans).  Plays the
// role of prefix_sum_kernel (msplat_metal.metal:2312-2364); ranges here are
// [offset[t], offset[t+1]) with no per-tile cap.
// ---------------------------------------------------------------------------
constexpr int kOrderBuckets = 1024;  // = the scan CTA's threads
__device__ __forceinline__ int order_bucket(int count) { return min(count >> 1, kOrderBuckets - 1); }

// Dense binning: the rows, then the columns, of the 2D difference array in
// slot 2 of the counter lines, summed in place (a warp per row or column,
// 32 entries a step); slot 0 then gets the whole count and slot 2 is zeroed
// for the next view.
__device__ void sum_difference_corners(int* count, int tx_n, int ty_n, int T)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int kWarps = 1024 / 32;
    for (int pass = 0; pass < 2; pass++) {
        const int lines = pass == 0 ? ty_n : tx_n;    // rows, then columns
        const int len = pass == 0 ? tx_n : ty_n;
        for (int l = warp; l < lines; l += kWarps) {
            int carry = 0;
            for (int k0 = 0; k0 < len; k0 += 32) {
                const int k = k0 + lane;
                const int t = pass == 0 ? l * tx_n + k : k * tx_n + l;
                int v = k < len ? count[t * kCountPitch + 2] : 0;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int u = __shfl_up_sync(0xffffffffu, v, o);
                    if (lane >= o) v += u;
                }
                v += carry;
                if (k < len) count[t * kCountPitch + 2] = v;
                carry = __shfl_sync(0xffffffffu, v, 31);
            }
        }
        __syncthreads();
    }
    for (int t = threadIdx.x; t < T; t += 1024) {
        count[t * kCountPitch] += count[t * kCountPitch + 2];
        count[t * kCountPitch + 2] = 0;
    }
    __syncthreads();
}

template <bool DENSE>
__global__ void __launch_bounds__(1024)
scan_tiles_kernel(const StepParams* __restrict__ P, int T, int* __restrict__ count,
                  int* __restrict__ offset, int* __restrict__ order, int* __restrict__ err,
                  int* __restrict__ isect_total, int* __restrict__ max_tile,
                  int* __restrict__ tile_sorted, int* __restrict__ tile_flag)
{
    __shared__ int s_warp[32];
    __shared__ int s_bucket[kOrderBuckets];
    const int tid = threadIdx.x;
    if (DENSE) sum_difference_corners(count, P->tiles_x, P->tiles_y, T);
    const int per = (T + 1023) / 1024;
    const int beg = min(tid * per, T), end = min(beg + per, T);
    int local = 0, lmax = 0;
    for (int i = beg; i < end; i++) {
        const int c = count[i * kCountPitch];
        local += c;
        lmax = max(lmax, c);
    }
    const int lane = tid & 31, warp = tid >> 5;
    if (max_tile) {
        // the largest tile, into a counter that starts the view at zero
        lmax = __reduce_max_sync(0xffffffffu, lmax);
        if (lane == 0 && lmax > 0) atomicMax(max_tile, lmax);
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int v = s_warp[lane];
        int wi = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int u = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += u;
        }
        s_warp[lane] = wi - v;  // exclusive
    }
    __syncthreads();
    int run = s_warp[warp] + incl - local;
    const bool prefix = P->prefix_sort != 0;
    for (int i = beg; i < end; i++) {
        offset[i] = run;
        const int c = count[i * kCountPitch];
        if (prefix) {
            tile_sorted[i] = c;  // whole lists unless the prefix sort selects the front
            tile_flag[i] = 0;
        }
        run += c;
    }
    if (prefix && tid == 0) tile_flag[T] = 0;
    if (tid == 1023) {
        offset[T] = run;
        if (isect_total) *isect_total = run;
        if ((long long)run > P->capacity) atomicOr(err, kErrIsectOverflow);
    }
    // CTA order of the per-tile kernels: tiles by intersection count, largest
    // first (a counting sort on count/2, capped), so the longest tiles start
    // in the first wave and the last wave holds short ones.  The order within
    // a bucket is arbitrary; no result depends on it.
    for (int b = tid; b < kOrderBuckets; b += 1024) s_bucket[b] = 0;
    __syncthreads();
    for (int i = beg; i < end; i++) atomicAdd(&s_bucket[order_bucket(count[i * kCountPitch])], 1);
    __syncthreads();
    {
        // exclusive scan of the buckets from the largest down: one bucket per thread
        const int b = kOrderBuckets - 1 - tid;
        const int c = s_bucket[b];
        int x = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += v;
        }
        if (lane == 31) s_warp[warp] = x;
        __syncthreads();
        if (warp == 0) {
            const int v = s_warp[lane];
            int wi = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += u;
            }
            s_warp[lane] = wi - v;
        }
        __syncthreads();
        s_bucket[b] = s_warp[warp] + x - c;
    }
    __syncthreads();
    for (int i = beg; i < end; i++)
        order[atomicAdd(&s_bucket[order_bucket(count[i * kCountPitch])], 1)] = i;
}

void launch_scan_tiles(const StepParams* P, int num_tiles, bool dense_bins, const Buffers& B,
                       cudaStream_t s)
{
    if (dense_bins)
        scan_tiles_kernel<true><<<1, 1024, 0, s>>>(P, num_tiles, B.tile_count, B.tile_offset,
                                                   B.tile_order, B.err, B.isect_total, B.max_tile,
                                                   B.tile_sorted, B.tile_flag);
    else
        scan_tiles_kernel<false><<<1, 1024, 0, s>>>(P, num_tiles, B.tile_count, B.tile_offset,
                                                    B.tile_order, B.err, B.isect_total, B.max_tile,
                                                    B.tile_sorted, B.tile_flag);
}

// ---------------------------------------------------------------------------
// Key scatter: every visible Gaussian writes (depth bits << 32 | id) into
// each tile of its rect.  The slot comes from counting the tile's counter
// back down, which also leaves the counters at zero for the next step.
// Reference key: scatter_to_prealloc_bins_kernel, msplat_metal.metal:2044-2056.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
scatter_kernel(const StepParams* __restrict__ P, int N, const int* __restrict__ radii,
               const float* __restrict__ depth, const uint2* __restrict__ rect,
               int* __restrict__ count, const int* __restrict__ offset,
               unsigned long long* __restrict__ keys)
{
    // Warp-cooperative: the warp's 32 Gaussians' (Gaussian, tile) pairs are
    // dealt out to all lanes, 32 at a time, so every lane has an atomic in
    // flight each round however unevenly the rects are sized.
    const int lane = threadIdx.x & 31;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    int x0 = 0, y0 = 0, w = 0, area = 0;
    unsigned long long key = 0;
    if (i < N && radii[i] > 0) {
        const uint2 r = rect[i];
        x0 = r.x & 0xffff;
        y0 = r.x >> 16;
        w = (r.y & 0xffff) - x0;
        area = w * ((r.y >> 16) - y0);
        key = ((unsigned long long)__float_as_uint(depth[i]) << 32) | (unsigned)i;
    }
    // inclusive prefix of the areas over the warp
    int incl = area;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    const long long cap = P->capacity;
    const int tx_n = P->tiles_x;
    // kRounds rounds of 32 pairs per iteration: their atomics are issued
    // together, so a lane waits for one atomic latency per kRounds pairs.
    // Measured at C1 (bin+sort): 1 round 0.195 ms, 2: 0.197, 3: 0.200,
    // 4: 0.202, 8: 0.206 -- fewer registers and more warps beat more
    // atomics in flight per warp.
    constexpr int kRounds = MSP_SCATTER_ROUNDS;
    for (int p0 = 0; p0 < total; p0 += 32 * kRounds) {
        int tile[kRounds];
        unsigned long long kv[kRounds];
#pragma unroll
        for (int u = 0; u < kRounds; u++) {
            const int pidx = p0 + 32 * u + lane;
            // owner = first lane whose inclusive prefix exceeds pidx
            int owner = 0;
#pragma unroll
            for (int step = 16; step > 0; step >>= 1) {
                const int probe = __shfl_sync(0xffffffffu, incl, owner + step - 1);
                if (probe <= pidx) owner += step;
            }
            const int o_incl = __shfl_sync(0xffffffffu, incl, owner);
            const int o_area = __shfl_sync(0xffffffffu, area, owner);
            const int o_x0 = __shfl_sync(0xffffffffu, x0, owner);
            const int o_y0 = __shfl_sync(0xffffffffu, y0, owner);
            const int o_w = __shfl_sync(0xffffffffu, w, owner);
            kv[u] = __shfl_sync(0xffffffffu, key, owner);
            tile[u] = -1;
            if (pidx < total) {
                const int k = pidx - (o_incl - o_area);
                tile[u] = (o_y0 + k / o_w) * tx_n + o_x0 + k % o_w;
            }
        }
        int pos[kRounds];
#pragma unroll
        for (int u = 0; u < kRounds; u++)
            if (tile[u] >= 0) pos[u] = atomicSub(&count[tile[u] * kCountPitch], 1) - 1;
#pragma unroll
        for (int u = 0; u < kRounds; u++) {
            if (tile[u] < 0) continue;
            const long long idx = (long long)offset[tile[u]] + pos[u];
            if (idx < cap) keys[idx] = kv[u];
        }
    }
}

void launch_scatter(const StepParams* P, int N, const Buffers& B, cudaStream_t s)
{
    if (N <= 0) return;
    scatter_kernel<<<(N + 255) / 256, 256, 0, s>>>(P, N, B.proj.radii, B.proj.depth, B.proj.rect,
                                                   B.tile_count, B.tile_offset, B.keys);
}

// ---------------------------------------------------------------------------
// Per-tile ascending sort of the 64-bit keys, then the Gaussian ids in that
// order.  Reference: bitonic_sort_per_tile_kernel, msplat_metal.metal:2064-2138
// (the fused pack is replaced by id gathers in the rasterizers).
// A tile of n <= kSortRun keys is padded with ~0 to npow = max(256, 2^ceil(log2 n))
// and sorted by a bitonic network whose element e = thread*K + r lives in
// register r of `thread` (K = npow / 256): compare-exchange distances below K
// stay in registers, distances below 32K use warp shuffles, larger ones go
// through shared memory.  Larger tiles that the radix sorts below do not take
// (more than kLargeRun keys, or refused) sort kSortRun runs that way and
// merge them pairwise along merge paths.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cmpx(unsigned long long& lo, unsigned long long& hi, bool up)
{
    const unsigned long long a = lo, b = hi;
    const bool swap = (a > b) == up;
    lo = swap ? b : a;
    hi = swap ? a : b;
}

template <int K>
__device__ __forceinline__ void bitonic_regs(unsigned long long (&v)[K], unsigned long long* s,
                                             int npow)
{
    const int t = threadIdx.x, lane = t & 31;
    for (int k = 2; k <= npow; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j < K) {
                // compile-time distance jj == j keeps v[] in registers
#pragma unroll
                for (int jj = K >> 1; jj >= 1; jj >>= 1) {
                    if (jj != j) continue;
#pragma unroll
                    for (int r = 0; r < K; r++) {
                        if (r & jj) continue;
                        const int e = t * K + r;
                        cmpx(v[r], v[r | jj], (e & k) == 0);
                    }
                }
            } else if (j < 32 * K) {
                const int lm = j / K;                   // partner lane offset
                const bool lower = (lane & lm) == 0;
#pragma unroll
                for (int r = 0; r < K; r++) {
                    const int e = t * K + r;
                    const bool up = (e & k) == 0;
                    const unsigned long long o = __shfl_xor_sync(0xffffffffu, v[r], lm);
                    const bool take_min = lower == up;
                    v[r] = take_min ? (o < v[r] ? o : v[r]) : (o > v[r] ? o : v[r]);
                }
            } else {
                // shared-memory exchange; index e is stored at e + e/16 so
                // that a warp's 64-bit accesses hit distinct banks
                __syncthreads();
#pragma unroll
                for (int r = 0; r < K; r++) {
                    const int e = t * K + r;
                    s[e + (e >> 4)] = v[r];
                }
                __syncthreads();
#pragma unroll
                for (int r = 0; r < K; r++) {
                    const int e = t * K + r;
                    const bool up = (e & k) == 0;
                    const int f = e ^ j;
                    const unsigned long long o = s[f + (f >> 4)];
                    const bool take_min = ((e & j) == 0) == up;
                    v[r] = take_min ? (o < v[r] ? o : v[r]) : (o > v[r] ? o : v[r]);
                }
            }
        }
    }
}

// Sort keys[0, n) (n <= kSortRun) in registers; write the sorted keys back to
// `out_keys` and/or their ids to `out_ids` (either may be null).
template <int K>
__device__ __forceinline__ void sort_run(const unsigned long long* keys, int n,
                                         unsigned long long* s, unsigned long long* out_keys,
                                         int* out_ids)
{
    const int npow = K * kSortThreads;
    unsigned long long v[K];
#pragma unroll
    for (int r = 0; r < K; r++) {
        const int e = threadIdx.x * K + r;
        v[r] = e < n ? keys[e] : ~0ull;
    }
    bitonic_regs<K>(v, s, npow);
#pragma unroll
    for (int r = 0; r < K; r++) {
        const int e = threadIdx.x * K + r;
        if (e < n) {
            if (out_keys) out_keys[e] = v[r];
            if (out_ids) out_ids[e] = (int)(unsigned)(v[r] & 0xffffffffull);
        }
    }
}

__device__ __forceinline__ void sort_small(const unsigned long long* keys, int n,
                                           unsigned long long* s, unsigned long long* out_keys,
                                           int* out_ids)
{
    if (n <= kSortThreads) sort_run<1>(keys, n, s, out_keys, out_ids);
    else if (n <= 2 * kSortThreads) sort_run<2>(keys, n, s, out_keys, out_ids);
    else if (n <= 4 * kSortThreads) sort_run<4>(keys, n, s, out_keys, out_ids);
    else if (kSortKMax == 8 || n <= 8 * kSortThreads) sort_run<8>(keys, n, s, out_keys, out_ids);
    else if constexpr (kSortKMax >= 16) sort_run<16>(keys, n, s, out_keys, out_ids);
}

__device__ __forceinline__ int merge_path(const unsigned long long* a, int la,
                                          const unsigned long long* b, int lb, int d)
{
    int lo = max(0, d - lb), hi = min(d, la);
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (a[mid] > b[d - 1 - mid]) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

// Per-tile LSD radix sort of the 32-bit depths (the ids ride along) for
// 2 <= n <= RUN keys with T threads: 8-bit digits, one pass per byte that
// is not the same for every key of the tile.  Each pass is stable: warp w
// ranks its contiguous share of the keys 32 at a time (__match_any_sync
// groups the lanes with equal digits), and the per-(digit, warp) counts are
// scanned digit-major, warp-minor.  Stability keeps equal depths in input
// order, which the scatter's atomics leave arbitrary, so each run of equal
// depths is then put in id order by one thread (insertion sort in shared
// memory); the result is the order of the 64-bit keys (depth << 32 | id).
// A tile whose depths are all equal, or that holds a run of more than
// kMaxTieRun equal depths, is reported and sorted by the bitonic / merge
// path on the full keys instead.
constexpr int kRadixSplit = MSP_RADIX_SPLIT;
constexpr int kMaxTieRun = 32;

template <int T, int RUN>
struct RadixSmemT {
    static constexpr int kWarps = T / 32;
    static constexpr int kChunks = RUN / T;  // 32-key chunks per warp at most
    static constexpr int kCols = kWarps * kRadixSplit;
    // Each warp's keys form kRadixSplit consecutive sub-ranges with their
    // own digit counters, so its scatter runs kRadixSplit independent chains
    // of counter reads and updates instead of one.
    static_assert(kChunks % kRadixSplit == 0, "sub-ranges of whole chunks");
    unsigned key[RUN];
    int val[RUN];
    // [column * 256 + digit], column = warp * split + sub-range: a warp's
    // lanes with different digits touch different banks
    int hist[256 * kCols];
    int wsum[kWarps];
    unsigned red[2 * kWarps];
};
using RadixSmem = RadixSmemT<kSortThreads, kSortRun>;

// Exclusive prefix sum of S.hist in place, over the counters in
// digit-major, column-minor order (256 * kCols counters).
template <int T, int RUN>
__device__ __forceinline__ int hist_at(int logical)
{
    constexpr int kCols = RadixSmemT<T, RUN>::kCols;
    return (logical % kCols) * 256 + logical / kCols;
}

template <int T, int RUN>
__device__ __forceinline__ void radix_scan(RadixSmemT<T, RUN>& S)
{
    using SM = RadixSmemT<T, RUN>;
    constexpr int kPer = 256 * SM::kCols / T;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int c[kPer];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < kPer; i++) {
        c[i] = S.hist[hist_at<T, RUN>(tid * kPer + i)];
        sum += c[i];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
    }
    if (lane == 31) S.wsum[warp] = incl;
    __syncthreads();
    int base = incl - sum;
#pragma unroll
    for (int w = 0; w < SM::kWarps; w++) base += w < warp ? S.wsum[w] : 0;
#pragma unroll
    for (int i = 0; i < kPer; i++) {
        S.hist[hist_at<T, RUN>(tid * kPer + i)] = base;
        base += c[i];
    }
}

// Returns false (and writes nothing) when the tile cannot be sorted here
// (all depths equal, or a run of equal depths longer than kMaxTieRun);
// otherwise writes the ids in ascending (depth, id) order.
// Register r of a lane holds element w0 + ((r % split) * cv + r / split) * 32
// + lane: sub-range r % split, its chunk r / split.
// FROM_SMEM: the n keys are in S.key (depths) and S.val (ids) instead of
// `keys` (which is then unused); every thread loads its share before the
// first write to either.
template <int T, int RUN, bool FROM_SMEM = false>
__device__ __forceinline__ bool radix_sort_tile(const unsigned long long* __restrict__ keys, int n,
                                                RadixSmemT<T, RUN>& S, int* __restrict__ out_ids)
{
    using SM = RadixSmemT<T, RUN>;
    constexpr int V = kRadixSplit;
    constexpr int kChunks = SM::kChunks;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned lt = (1u << lane) - 1u;
    const int C = (n + T - 1) / T;     // chunks per warp
    const int cv = (C + V - 1) / V;    // chunks per sub-range
    const int nr = cv * V;             // registers in use
    const int w0 = warp * nr * 32;     // this warp's first element
    auto elem = [&](int r) { return w0 + ((r % V) * cv + r / V) * 32 + lane; };
    unsigned k[kChunks];
    int v[kChunks];
    unsigned ko = 0u, ka = ~0u;
#pragma unroll
    for (int r = 0; r < kChunks; r++) {
        k[r] = ~0u;  // padding sorts last and stays behind equal real keys
        v[r] = 0;
        const int e = elem(r);
        if (r < nr && e < n) {
            if (FROM_SMEM) {
                k[r] = S.key[e];
                v[r] = S.val[e];
            } else {
                const unsigned long long kv = keys[e];
                k[r] = (unsigned)(kv >> 32);
                v[r] = (int)(unsigned)(kv & 0xffffffffull);
            }
            ko |= k[r];
            ka &= k[r];
        }
    }
    ko = __reduce_or_sync(0xffffffffu, ko);
    ka = __reduce_and_sync(0xffffffffu, ka);
    if (lane == 0) {
        S.red[warp] = ko;
        S.red[SM::kWarps + warp] = ka;
    }
    __syncthreads();
    unsigned all_or = 0u, all_and = ~0u;
#pragma unroll
    for (int w = 0; w < SM::kWarps; w++) {
        all_or |= S.red[w];
        all_and &= S.red[SM::kWarps + w];
    }
    const unsigned varying = all_or ^ all_and;
    if (varying == 0u) return false;  // n >= 2 equal depths
    for (int shift = 0; shift < 32; shift += 8) {
        if (((varying >> shift) & 0xffu) == 0u) continue;
        for (int i = lane; i < 256 * V; i += 32) S.hist[warp * V * 256 + i] = 0;
        __syncwarp();
        // counts need no order: shared-memory atomics, no chain between chunks
#pragma unroll
        for (int r = 0; r < kChunks; r++) {
            if (r >= nr) break;
            const unsigned d = (k[r] >> shift) & 0xffu;
            atomicAdd(&S.hist[(warp * V + r % V) * 256 + d], 1);
        }
        __syncthreads();
        radix_scan(S);
        __syncthreads();
        // V independent chains: chunk r0 / V of every sub-range at once
#pragma unroll
        for (int r0 = 0; r0 < kChunks; r0 += V) {
            if (r0 >= nr) break;
            unsigned peers[V];
            int slot[V], base[V];
#pragma unroll
            for (int u = 0; u < V; u++) {
                const unsigned d = (k[r0 + u] >> shift) & 0xffu;
                peers[u] = __match_any_sync(0xffffffffu, d);
                slot[u] = (warp * V + u) * 256 + d;
                base[u] = S.hist[slot[u]];
            }
            __syncwarp();
#pragma unroll
            for (int u = 0; u < V; u++) {
                if ((peers[u] & lt) == 0u) S.hist[slot[u]] = base[u] + __popc(peers[u]);
                const int pos = base[u] + __popc(peers[u] & lt);
                S.key[pos] = k[r0 + u];
                S.val[pos] = v[r0 + u];
            }
            __syncwarp();
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < kChunks; r++) {
            if (r >= nr) break;
            const int e = elem(r);
            k[r] = S.key[e];
            v[r] = S.val[e];
        }
    }
    // S.key holds the sorted depths (at least one pass ran): any equal
    // neighbours among the real keys?
    bool tie = false;
#pragma unroll
    for (int r = 0; r < kChunks; r++) {
        if (r >= nr) break;
        const int e = elem(r);
        if (e + 1 < n && k[r] == S.key[e + 1]) tie = true;
    }
    if (__syncthreads_or(tie)) {
        // each run of equal depths, in id order: the thread holding the
        // run's first element sorts its ids in place (runs are disjoint)
        bool too_long = false;
#pragma unroll
        for (int r = 0; r < kChunks; r++) {
            if (r >= nr) break;
            const int e = elem(r);
            if (e + 1 >= n || k[r] != S.key[e + 1] || (e > 0 && S.key[e - 1] == k[r])) continue;
            int end = e + 2;
            while (end < n && end - e <= kMaxTieRun && S.key[end] == k[r]) end++;
            if (end - e > kMaxTieRun) {
                too_long = true;
                continue;
            }
            for (int a = e + 1; a < end; a++) {
                const int x = S.val[a];
                int b = a - 1;
                while (b >= e && (unsigned)S.val[b] > (unsigned)x) {
                    S.val[b + 1] = S.val[b];
                    b--;
                }
                S.val[b + 1] = x;
            }
        }
        if (__syncthreads_or(too_long)) return false;
#pragma unroll
        for (int r = 0; r < kChunks; r++) {
            if (r >= nr) break;
            v[r] = S.val[elem(r)];
        }
    }
#pragma unroll
    for (int r = 0; r < kChunks; r++) {
        if (r >= nr) break;
        const int e = elem(r);
        if (e < n) out_ids[e] = v[r];
    }
    return true;
}

// Tiles of kSortRun + 1 .. kLargeRun keys: the same radix sort with 512
// threads and 80 KB of dynamic shared memory, two CTAs per SM, each CTA
// walking the tile list (largest first) and taking every gridDim.x-th tile.
// Slot 1 of a tile's counter line (slot 0 is the count) records whether the
// tile is left to sort_tiles_kernel (1) or done (0); it is written for every
// tile of more than kSortRun keys and read only for those.
//
// Tiles of more than kSortRun keys, when StepParams::prefix_sort is set
// (single-pass raster only; sort_tile_prefixes_kernel takes them all and
// sort_large_tiles_kernel is not launched): a pixel stops at the first
// Gaussian that takes its transmittance to 1e-4, and in a long list that
// is nearly always close to the front.  So only the front of the list is
// sorted: the keys whose depth is below a threshold that about
// kPrefixTarget (at most kLargeRun) keys pass.  Every key with a smaller
// depth passes too, so those keys are exactly the first m of the whole
// list's (depth, id) order, and a raster that stays inside them gives the
// result of the whole list bit for bit.  tile_sorted[t] = m; the forward
// raster flags a tile whose pixels run past the prefix, and the flagged
// tiles are then sorted whole and rasterized again.  The depths are
// compared as unsigned bits, the order of the keys.
constexpr int kLargeThreads = 512;
using LargeSmem = RadixSmemT<kLargeThreads, kLargeRun>;
// The selection histogram of a CTA of T threads over RadixSmemT<T, RUN>:
// as many buckets (at most 2048) as S.hist holds, in kCopies copies.
template <int T, int RUN>
struct SelShape {
    using Smem = RadixSmemT<T, RUN>;
    static constexpr int kHist = 256 * Smem::kCols;
    static constexpr int kBuckets = kHist >= 2048 ? 2048 : kHist;
    static constexpr int kCopies = kHist / kBuckets;
    static_assert(kBuckets % T == 0, "whole buckets per thread");
};

// Histogram of the depths depth(0 .. count-1) that lie in [lo, hi], in
// SelShape::kBuckets buckets of 2^shift values, then the bucket b at which
// base + the running count first exceeds `budget` (one must).  Returns b
// and, in *before, base + the count of the buckets before b.
template <int T, int RUN, typename DepthAt>
__device__ int crossing_bucket(DepthAt depth, int count, unsigned lo, unsigned hi, int shift,
                               int base, int budget, RadixSmemT<T, RUN>& S, int* before)
{
    using Sh = SelShape<T, RUN>;
    constexpr int kWarps = T / 32;
    constexpr int kPer = Sh::kBuckets / T;
    __shared__ int s_cross[2];  // crossing bucket, keys before it
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __syncthreads();  // earlier reads of S.hist, S.wsum and s_cross are done
    for (int i = tid; i < Sh::kBuckets * Sh::kCopies; i += T) S.hist[i] = 0;
    __syncthreads();
    int* h = S.hist + (warp % Sh::kCopies) * Sh::kBuckets;
    for (int i = tid; i < count; i += T) {
        const unsigned d = depth(i);
        if (d >= lo && d <= hi) atomicAdd(&h[(d - lo) >> shift], 1);
    }
    __syncthreads();
    int c[kPer], sum = 0;
#pragma unroll
    for (int r = 0; r < kPer; r++) {
        c[r] = 0;
#pragma unroll
        for (int q = 0; q < Sh::kCopies; q++) c[r] += S.hist[q * Sh::kBuckets + tid * kPer + r];
        sum += c[r];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
    }
    if (lane == 31) S.wsum[warp] = incl;
    __syncthreads();
    int run = base + incl - sum;
#pragma unroll
    for (int w = 0; w < kWarps; w++) run += w < warp ? S.wsum[w] : 0;
#pragma unroll
    for (int r = 0; r < kPer; r++) {
        if (run <= budget && run + c[r] > budget) {
            s_cross[0] = tid * kPer + r;
            s_cross[1] = run;
        }
        run += c[r];
    }
    __syncthreads();
    *before = s_cross[1];
    return s_cross[0];
}

// Smallest shift with span >> shift < B.
template <int B>
__device__ __forceinline__ int bucket_shift(unsigned span)
{
    int shift = 0;
    while ((span >> shift) >= (unsigned)B) shift++;
    return shift;
}

// Block-wide min and max of one value per thread.
template <int T, int RUN>
__device__ __forceinline__ void block_min_max(unsigned vmin, unsigned vmax, RadixSmemT<T, RUN>& S,
                                              unsigned* lo, unsigned* hi)
{
    constexpr int kWarps = T / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    vmin = __reduce_min_sync(0xffffffffu, vmin);
    vmax = __reduce_max_sync(0xffffffffu, vmax);
    __syncthreads();  // earlier reads of S.red are done
    if (lane == 0) {
        S.red[warp] = vmin;
        S.red[kWarps + warp] = vmax;
    }
    __syncthreads();
    unsigned a = ~0u, b = 0u;
#pragma unroll
    for (int w = 0; w < kWarps; w++) {
        a = min(a, S.red[w]);
        b = max(b, S.red[kWarps + w]);
    }
    *lo = a;
    *hi = b;
}

// The keys of depth < thr into S.key (depths) and S.val (ids), the first
// RUN of them; returns how many there are (possibly more).
template <int T, int RUN>
__device__ int compact_below(const unsigned long long* __restrict__ keys, int n,
                             unsigned long long thr, RadixSmemT<T, RUN>& S)
{
    __shared__ int s_m;
    const int tid = threadIdx.x, lane = tid & 31;
    __syncthreads();  // every thread has read what it needs of S.key
    if (tid == 0) s_m = 0;
    __syncthreads();
    const unsigned lt = (1u << lane) - 1u;
    // kU keys per thread loaded before any is placed: a long list is one
    // CTA's work, so its loads must overlap
    constexpr int kU = 8;
    for (int i0 = 0; i0 < n; i0 += T * kU) {
        unsigned long long kv[kU];
#pragma unroll
        for (int u = 0; u < kU; u++) {
            const int i = i0 + u * T + tid;
            kv[u] = i < n ? keys[i] : 0ull;
        }
#pragma unroll
        for (int u = 0; u < kU; u++) {
            const bool take = i0 + u * T + tid < n && (kv[u] >> 32) < thr;
            const unsigned bal = __ballot_sync(0xffffffffu, take);
            int at = 0;
            if (lane == 0 && bal) at = atomicAdd(&s_m, __popc(bal));
            at = __shfl_sync(0xffffffffu, at, 0) + __popc(bal & lt);
            if (take && at < RUN) {
                S.key[at] = (unsigned)(kv[u] >> 32);
                S.val[at] = (int)(unsigned)(kv[u] & 0xffffffffull);
            }
        }
    }
    __syncthreads();
    return s_m;
}

// The nearest keys of a tile of n > kSortRun keys, into S.key (depths) and
// S.val (ids) in no particular order, for a CTA of T threads; returns their
// count m, 1 <= m <= RUN, or 0 when none was found.
// First from a sample: kSelSample depths at even strides through the list
// give a threshold expected to pass about kPrefixTarget keys; one pass
// counts and gathers them.  When that passes none or more than RUN keys,
// the exact levels: histograms of all n depths, the last bucket that still
// fits RUN, and where that leaves less than half of it used, the next
// bucket split the same way (10 or 11 bits a level, down to single depth
// values; 0 when more than RUN keys share the smallest depth).
constexpr int kSelSample = 2048;
static_assert(kSelSample <= kSortRun, "the sample fits S.key of the smaller sort");
static_assert(kPrefixTarget < kSortRun, "the sample rank is below the sample size");

template <int T, int RUN>
__device__ int select_nearest(const unsigned long long* __restrict__ keys, int n,
                              RadixSmemT<T, RUN>& S)
{
    constexpr int kB = SelShape<T, RUN>::kBuckets;
    static_assert(kSelSample <= RUN && kSelSample % T == 0, "sample in S.key");
    const int tid = threadIdx.x;
    {
        constexpr int kPer = kSelSample / T;
        unsigned smin = ~0u, smax = 0u;
#pragma unroll
        for (int r = 0; r < kPer; r++) {
            const int j = tid + r * T;
            const unsigned d = (unsigned)(keys[(long long)j * n / kSelSample] >> 32);
            S.key[j] = d;
            smin = min(smin, d);
            smax = max(smax, d);
        }
        unsigned lo, hi;
        block_min_max(smin, smax, S, &lo, &hi);  // its barriers also publish S.key
        const int shift = bucket_shift<kB>(hi - lo);
        // sample rank of the target: q of kSelSample samples ~ kPrefixTarget of n keys
        const int q = max(1, (int)((long long)kPrefixTarget * kSelSample / n));
        int before = 0;
        const int b = crossing_bucket([&](int i) { return S.key[i]; }, kSelSample, lo, hi, shift, 0,
                                      q, S, &before);
        const unsigned long long thr = (unsigned long long)lo + ((unsigned long long)b << shift);
        const int m = compact_below(keys, n, thr, S);
        if (m >= 1 && m <= RUN) return m;
    }
    if (n <= RUN) return 0;  // no budget to cross: the caller sorts it whole
    unsigned dmin = ~0u, dmax = 0u;
    for (int i = tid; i < n; i += T) {
        const unsigned d = (unsigned)(keys[i] >> 32);
        dmin = min(dmin, d);
        dmax = max(dmax, d);
    }
    unsigned lo, hi;
    block_min_max(dmin, dmax, S, &lo, &hi);
    // keys with depth < lo are selected (`base` of them); [lo, hi] is split
    int base = 0;
    unsigned long long thr = lo;
    for (int level = 0; level < 4; level++) {
        const int shift = bucket_shift<kB>(hi - lo);
        // The keys in [lo, hi] plus base exceed RUN, so exactly one bucket
        // crosses the budget: all before it fit, it does not.
        int before = 0;
        const int b = crossing_bucket([&](int i) { return (unsigned)(keys[i] >> 32); }, n, lo, hi,
                                      shift, base, RUN, S, &before);
        const unsigned long long bucket_lo = (unsigned long long)lo + ((unsigned long long)b << shift);
        thr = bucket_lo;  // selects everything before bucket b
        base = before;
        if (before >= RUN / 2 || shift == 0) break;
        // split bucket b at the next level
        lo = (unsigned)bucket_lo;
        hi = (unsigned)min((unsigned long long)hi, bucket_lo + ((1ull << shift) - 1ull));
    }
    return min(compact_below(keys, n, thr, S), RUN);
}

__global__ void __launch_bounds__(kLargeThreads, 2)
sort_large_tiles_kernel(const StepParams* __restrict__ P, const int* __restrict__ offset,
                        const int* __restrict__ order, int num_tiles,
                        const unsigned long long* __restrict__ keys, int* __restrict__ ids,
                        int* __restrict__ tile_line)
{
    extern __shared__ __align__(16) unsigned char s_large[];
    LargeSmem& S = *reinterpret_cast<LargeSmem*>(s_large);
    const long long cap = P->capacity;
    for (int i = blockIdx.x; i < num_tiles; i += gridDim.x) {
        const int t = order[i];
        const long long start = min((long long)offset[t], cap);
        const long long end = min((long long)offset[t + 1], cap);
        const int n = (int)(end - start);
        if (n <= kSortRun || n > kLargeRun) continue;
        __syncthreads();  // the previous tile's last reads of S
        const bool ok = radix_sort_tile(keys + start, n, S, ids + start);
        if (threadIdx.x == 0) tile_line[t * kCountPitch + 1] = ok ? 0 : 1;
    }
}

// With StepParams::prefix_sort set (the only launches of these two
// kernels) the tiles of more than kSortRun keys sort their nearest keys,
// selected as in select_nearest, and record the prefix in tile_sorted and
// their flag in slot 1 of the counter line; a tile whose selection or
// sort fails is left to sort_tiles_kernel's merge path (flag 1).
//   sort_tile_prefixes_kernel: more than kLargeRun keys (long lists are
//     one CTA's work: 512 threads, two CTAs per SM walking the tile list),
//     prefixes of up to kLargeRun keys;
//   sort_mid_prefixes_kernel: kSortRun + 1 .. kLargeRun keys, one CTA of
//     kSortThreads per tile on the shared memory of the 2,048-key radix
//     sort (eight CTAs per SM), prefixes of up to kSortRun keys.
__global__ void __launch_bounds__(kLargeThreads, 2)
sort_tile_prefixes_kernel(const StepParams* __restrict__ P, const int* __restrict__ offset,
                          const int* __restrict__ order, int num_tiles,
                          const unsigned long long* __restrict__ keys, int* __restrict__ ids,
                          int* __restrict__ tile_line, int* __restrict__ tile_sorted)
{
    extern __shared__ __align__(16) unsigned char s_large[];
    LargeSmem& S = *reinterpret_cast<LargeSmem*>(s_large);
    const long long cap = P->capacity;
    for (int i = blockIdx.x; i < num_tiles; i += gridDim.x) {
        const int t = order[i];
        const long long start = min((long long)offset[t], cap);
        const long long end = min((long long)offset[t + 1], cap);
        const int n = (int)(end - start);
        if (n <= kLargeRun) continue;
        __syncthreads();  // the previous tile's last reads of S
        bool ok = false;
        const int m = select_nearest(keys + start, n, S);
        if (m == 1) {
            if (threadIdx.x == 0) ids[start] = S.val[0];
            ok = true;
        } else if (m > 1) {
            ok = radix_sort_tile<kLargeThreads, kLargeRun, true>(nullptr, m, S, ids + start);
        }
        if (threadIdx.x == 0) {
            if (ok) tile_sorted[t] = m;
            tile_line[t * kCountPitch + 1] = ok ? 0 : 1;
        }
    }
}

__global__ void __launch_bounds__(kSortThreads, MSP_SORT_MIN_BLOCKS)
sort_mid_prefixes_kernel(const StepParams* __restrict__ P, const int* __restrict__ offset,
                         const int* __restrict__ order, const unsigned long long* __restrict__ keys,
                         int* __restrict__ ids, int* __restrict__ tile_line,
                         int* __restrict__ tile_sorted)
{
    __shared__ RadixSmem S;
    const int t = order[blockIdx.x];
    const long long cap = P->capacity;
    const long long start = min((long long)offset[t], cap);
    const int n = (int)(min((long long)offset[t + 1], cap) - start);
    if (n <= kSortRun || n > kLargeRun) return;
    bool ok = false;
    const int m = select_nearest(keys + start, n, S);
    if (m == 1) {
        if (threadIdx.x == 0) ids[start] = S.val[0];
        ok = true;
    } else if (m > 1) {
        ok = radix_sort_tile<kSortThreads, kSortRun, true>(nullptr, m, S, ids + start);
    }
    if (threadIdx.x == 0) {
        if (ok) tile_sorted[t] = m;
        tile_line[t * kCountPitch + 1] = ok ? 0 : 1;
    }
}

__device__ void merge_sort_tile(unsigned long long* __restrict__ keys,
                                unsigned long long* __restrict__ keys_alt, int n,
                                unsigned long long* s, int* __restrict__ ids);

__global__ void __launch_bounds__(kSortThreads, MSP_SORT_MIN_BLOCKS)
sort_tiles_kernel(const StepParams* __restrict__ P, const int* __restrict__ offset,
                  const int* __restrict__ order, unsigned long long* __restrict__ keys,
                  unsigned long long* __restrict__ keys_alt, int* __restrict__ ids,
                  const int* __restrict__ tile_line, int mid_done, int huge_done)
{
    __shared__ union {
        unsigned long long bitonic[kSortRun + kSortRun / 16];
        RadixSmem radix;
    } sm;
    unsigned long long* s = sm.bitonic;
    const int t = order[blockIdx.x];
    const long long cap = P->capacity;
    const long long start = min((long long)offset[t], cap);
    const long long end = min((long long)offset[t + 1], cap);
    const int n = (int)(end - start);
    if (n <= 0) return;
    if (n <= kSortRun) {
        if (MSP_SORT_RADIX && n > kSortThreads) {
            if (radix_sort_tile(keys + start, n, sm.radix, ids + start)) return;
            __syncthreads();
        }
        sort_small(keys + start, n, s, nullptr, ids + start);
        return;
    }
    // n > kSortRun: already sorted (n <= kLargeRun: by sort_large_tiles_kernel
    // or, with prefix_sort, its prefix by sort_mid_prefixes_kernel; longer:
    // its prefix by sort_tile_prefixes_kernel) unless that kernel left the
    // tile here or was not launched (mid_done / huge_done = 0): then the
    // merge path sorts it whole
    if ((n <= kLargeRun ? mid_done : huge_done) && tile_line[t * kCountPitch + 1] == 0) return;
    merge_sort_tile(keys + start, keys_alt + start, n, s, ids + start);
}

// The whole list of a large tile: sorted runs of kSortRun (in place in
// `keys`), then pairwise merges along merge paths between `keys` and
// `keys_alt`; the ids in (depth, id) order to `ids`.  One CTA of
// kSortThreads threads.
__device__ void merge_sort_tile(unsigned long long* __restrict__ keys,
                                unsigned long long* __restrict__ keys_alt, int n,
                                unsigned long long* s, int* __restrict__ ids)
{
    unsigned long long* src = keys;
    unsigned long long* dst = keys_alt;
    for (int r0 = 0; r0 < n; r0 += kSortRun) {
        __syncthreads();
        sort_small(src + r0, min(kSortRun, n - r0), s, src + r0, nullptr);
    }
    __syncthreads();
    for (long long L = kSortRun; L < n; L <<= 1) {
        for (long long s0 = 0; s0 < n; s0 += 2 * L) {
            const unsigned long long* a = src + s0;
            const int la = (int)min(L, (long long)n - s0);
            const unsigned long long* b = a + la;
            const int lb = (int)max(0LL, min(L, (long long)n - s0 - la));
            const int total = la + lb;
            const int d0 = (int)((long long)total * threadIdx.x / kSortThreads);
            const int d1 = (int)((long long)total * (threadIdx.x + 1) / kSortThreads);
            int ia = merge_path(a, la, b, lb, d0);
            int ib = d0 - ia;
            unsigned long long* o = dst + s0 + d0;
            for (int q = d0; q < d1; q++) {
                bool take_a = ib >= lb || (ia < la && a[ia] < b[ib]);
                *o++ = take_a ? a[ia++] : b[ib++];
            }
        }
        __syncthreads();
        unsigned long long* tmp = src;
        src = dst;
        dst = tmp;
    }
    for (int i = threadIdx.x; i < n; i += kSortThreads)
        ids[i] = (int)(unsigned)(src[i] & 0xffffffffull);
}

// Tiles the forward raster flagged (a pixel ran past the selected prefix
// without terminating): their whole list, sorted.  Launched after every
// single-pass forward; exits at once when no tile was flagged.  Each CTA
// takes every gridDim.x-th tile of the tile list.
__global__ void __launch_bounds__(kSortThreads, MSP_SORT_MIN_BLOCKS)
sort_flagged_tiles_kernel(const StepParams* __restrict__ P, const int* __restrict__ offset,
                          const int* __restrict__ order, int num_tiles,
                          unsigned long long* __restrict__ keys,
                          unsigned long long* __restrict__ keys_alt, int* __restrict__ ids,
                          int* __restrict__ tile_sorted, const int* __restrict__ tile_flag)
{
    __shared__ unsigned long long s[kSortRun + kSortRun / 16];
    if (tile_flag[num_tiles] == 0) return;
    const long long cap = P->capacity;
    for (int i = blockIdx.x; i < num_tiles; i += gridDim.x) {
        const int t = order[i];
        if (!tile_flag[t]) continue;
        const long long start = min((long long)offset[t], cap);
        const int n = (int)(min((long long)offset[t + 1], cap) - start);
        __syncthreads();  // the previous tile's last reads of s
        merge_sort_tile(keys + start, keys_alt + start, n, s, ids + start);
        if (threadIdx.x == 0) tile_sorted[t] = n;
    }
}

// SM count of the current device (148, the B200's, if the query fails).
static int device_sms()
{
    static std::once_flag once[kMaxDeviceSlots];
    static int sms[kMaxDeviceSlots];
    int dev = 0;
    if (!once_per_device(once, [](int d) {
            int n = 0;
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
            sms[d] = n > 0 ? n : 148;
        }) || cudaGetDevice(&dev) != cudaSuccess)
        return 148;
    return sms[dev];
}

// The tiles of more than kSortRun keys first, then every other tile.
// Without prefix_sort: sort_large_tiles_kernel (2,049-8,192 keys), unless
// large_sort is false (the last view read back had no tile above kSortRun
// keys).  With prefix_sort: sort_tile_prefixes_kernel when huge_sort (the
// last view had a tile above kLargeRun keys), and sort_mid_prefixes_kernel.
// A tile of a range whose kernel was not launched takes the merge path.
int launch_sort_tiles(const StepParams* P, int num_tiles, bool prefix_sort, bool large_sort,
                      bool huge_sort, const Buffers& B, cudaStream_t s)
{
    if (num_tiles <= 0) return 0;
    static std::once_flag once[kMaxDeviceSlots];
    if (!once_per_device(once, [](int) {
            cudaFuncSetAttribute(sort_large_tiles_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(LargeSmem));
            cudaFuncSetAttribute(sort_tile_prefixes_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(LargeSmem));
        }))
        return 0;
    const int grid = std::min(num_tiles, 2 * device_sms());
    int launches = 1;
    const bool mid_done = prefix_sort || large_sort;
    const bool huge_done = prefix_sort && huge_sort;
    if (huge_done) {
        sort_tile_prefixes_kernel<<<grid, kLargeThreads, sizeof(LargeSmem), s>>>(
            P, B.tile_offset, B.tile_order, num_tiles, B.keys, B.sorted_ids, B.tile_count,
            B.tile_sorted);
        launches++;
    }
    if (prefix_sort)
        sort_mid_prefixes_kernel<<<num_tiles, kSortThreads, 0, s>>>(
            P, B.tile_offset, B.tile_order, B.keys, B.sorted_ids, B.tile_count, B.tile_sorted);
    else if (large_sort)
        sort_large_tiles_kernel<<<grid, kLargeThreads, sizeof(LargeSmem), s>>>(
            P, B.tile_offset, B.tile_order, num_tiles, B.keys, B.sorted_ids, B.tile_count);
    if (mid_done) launches++;
    sort_tiles_kernel<<<num_tiles, kSortThreads, 0, s>>>(P, B.tile_offset, B.tile_order, B.keys, B.keys_alt,
                                                        B.sorted_ids, B.tile_count, mid_done ? 1 : 0,
                                                        huge_done ? 1 : 0);
    return launches;
}

// ---------------------------------------------------------------------------
// Forward rasterizer: one CTA per 16x16 tile (or per (tile, depth chunk)),
// one thread per pixel, batches of 256 Gaussians staged in shared memory.
// Reference: nd_rasterize_forward_kernel (msplat_metal.metal:472-585) and
// rasterize_forward_chunked_kernel (:2633-2741).  The per-pixel loop is the
// reference's; the CTA leaves as soon as every pixel has terminated.  Each
// staged batch drops the Gaussians that cannot reach any pixel of the tile
// (tile_may_contribute), which changes no result: those never pass the
// per-pixel tests.
// Single pass, MODE: 0, every tile walks its whole list; 1, a tile walks
// its sorted prefix (tile_sorted, the whole list unless the large-tile sort
// selected the nearest keys), and when a pixel is still open at the end of
// a prefix shorter than the list, the tile is flagged (tile_flag); 2, the
// flagged tiles (by then sorted whole) only, their whole lists.
// ---------------------------------------------------------------------------
// Six resident CTAs per SM (40 registers): 0.377 ms at C1 against 0.385
// with 47 registers (5 CTAs) and 0.379 with 32 (8 CTAs, spilling).
template <bool CHUNKED, int MODE>
__global__ void __launch_bounds__(kTileThreads, MSP_FWD_MIN_BLOCKS)
raster_forward_kernel(const StepParams* __restrict__ P, const int* __restrict__ offset,
                      const int* __restrict__ order, const int* __restrict__ ids,
                      const float2* __restrict__ g_xy,
                      const float4* __restrict__ g_co, const float4* __restrict__ g_rgb,
                      float* __restrict__ out_img, float* __restrict__ final_T,
                      int* __restrict__ final_idx, float* __restrict__ chunk_T,
                      float* __restrict__ chunk_C, int* __restrict__ chunk_idx,
                      const int* __restrict__ tile_sorted, int* __restrict__ tile_flag,
                      int num_tiles)
{
    __shared__ float2 s_xy[kTileThreads];
    __shared__ float4 s_co[kTileThreads];
    __shared__ float4 s_rgb[kTileThreads];
    __shared__ int s_idx[kTileThreads];
    __shared__ int s_wcnt[kTileThreads / 32];
    if (!CHUNKED && MODE == 2 && tile_flag[num_tiles] == 0) return;  // nothing flagged
    const int tile = order[blockIdx.x];
    const int tx_n = P->tiles_x;
    const int W = P->img_w, H = P->img_h;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float tx0 = (float)((tile % tx_n) * kBlockX), ty0 = (float)((tile / tx_n) * kBlockY);
    const int px = (tile % tx_n) * kBlockX + (tid & 15);
    const int py = (tile / tx_n) * kBlockY + (tid >> 4);
    const bool inside = px < W && py < H;
    const long long cap = P->capacity;
    const int fbeg = (int)min((long long)offset[tile], cap);
    const int fend = (int)min((long long)offset[tile + 1], cap);
    int beg = fbeg, end = fend;
    int k = 0;
    if (CHUNKED) {
        k = blockIdx.y;
        beg = fbeg + k * kChunk;
        end = min(fbeg + (k + 1) * kChunk, fend);
        if (beg >= end) return;
    } else {
        if (MODE == 2 && tile_flag[tile] == 0) return;
        if (MODE == 1) end = min(fend, fbeg + tile_sorted[tile]);
    }
    const float fpx = (float)px, fpy = (float)py;
    float T = 1.f, c0 = 0.f, c1 = 0.f, c2 = 0.f;
    int last = beg - 1;
    bool done = !inside;
    for (int b0 = beg; b0 < end; b0 += kTileThreads) {
        if (__syncthreads_count(done) == kTileThreads) break;
        // Stage the batch, keeping (in list order) only the Gaussians that
        // can reach a pixel of this tile; s_idx keeps their list positions.
        const int idx = b0 + tid;
        bool keep = false;
        float2 xy = make_float2(0.f, 0.f);
        float4 co = make_float4(0.f, 0.f, 0.f, 0.f), rc = co;
        if (idx < end) {
            const int g = ids[idx];
            xy = g_xy[g];
            co = g_co[g];
            rc = g_rgb[g];
            keep = tile_may_contribute(xy, co, tx0, ty0, cull_limit(co));
        }
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        if (lane == 0) s_wcnt[warp] = __popc(bal);
        __syncthreads();
        int n = 0, woff = 0;
#pragma unroll
        for (int w = 0; w < kTileThreads / 32; w++) {
            const int cw = s_wcnt[w];
            woff += w < warp ? cw : 0;
            n += cw;
        }
        if (keep) {
            const int slot = woff + __popc(bal & ((1u << lane) - 1u));
            s_xy[slot] = xy;
            s_co[slot] = co;
            s_rgb[slot] = make_float4(fmaxf(rc.x + 0.5f, 0.f), fmaxf(rc.y + 0.5f, 0.f),
                                      fmaxf(rc.z + 0.5f, 0.f), 0.f);
            s_idx[slot] = idx;
        }
        __syncthreads();
        if (done) continue;
        for (int t = 0; t < n; t++) {
            const float4 co = s_co[t];
            const float2 xy = s_xy[t];
            const float dx = xy.x - fpx, dy = xy.y - fpy;
            const float sigma = fmaf(0.5f, fmaf(co.x, dx * dx, co.z * dy * dy), co.y * dx * dy);
            if (sigma < 0.f || sigma >= 5.55f) continue;
            const float alpha = fminf(0.999f, co.w * msp_expf_normal(-sigma));
            if (alpha < 1.f / 255.f) continue;
            const float next_T = T * (1.f - alpha);
            if (next_T <= 1e-4f) {
                last = s_idx[t] - 1;
                done = true;
                break;
            }
            const float vis = alpha * T;
            const float4 rgb = s_rgb[t];
            c0 = fmaf(rgb.x, vis, c0);
            c1 = fmaf(rgb.y, vis, c1);
            c2 = fmaf(rgb.z, vis, c2);
            T = next_T;
            last = s_idx[t];
        }
    }
    if (!CHUNKED && MODE == 1 && end < fend) {
        // a prefix: every pixel must have terminated inside it
        if (__syncthreads_count(!done) != 0 && tid == 0) {
            tile_flag[tile] = 1;
            atomicAdd(&tile_flag[num_tiles], 1);
        }
    }
    if (!inside) return;
    const size_t pix = (size_t)py * W + px;
    if (CHUNKED) {
        const size_t o = (size_t)k * ((size_t)W * H) + pix;
        chunk_T[o] = T;
        chunk_C[3 * o] = c0;
        chunk_C[3 * o + 1] = c1;
        chunk_C[3 * o + 2] = c2;
        chunk_idx[o] = last;
    } else {
        final_T[pix] = T;
        final_idx[pix] = last;
        out_img[3 * pix] = saturatef_ref(fmaf(P->bg[0], T, c0));
        out_img[3 * pix + 1] = saturatef_ref(fmaf(P->bg[1], T, c1));
        out_img[3 * pix + 2] = saturatef_ref(fmaf(P->bg[2], T, c2));
    }
}

// Merge of the depth chunks, rasterize_forward_merge_kernel
// (msplat_metal.metal:2746-2799).  Only chunks that hold Gaussians were
// written; the reference's loop stops at the first empty chunk, so those are
// the only ones it reads.
__global__ void __launch_bounds__(256)
merge_chunks_kernel(const StepParams* __restrict__ P, const int* __restrict__ offset,
                    const float* __restrict__ chunk_T, const float* __restrict__ chunk_C,
                    int* __restrict__ chunk_idx, float* __restrict__ out_img,
                    float* __restrict__ final_T, int* __restrict__ final_idx)
{
    const int W = P->img_w, H = P->img_h;
    const int px = blockIdx.x * 16 + (threadIdx.x & 15);
    const int py = blockIdx.y * 16 + (threadIdx.x >> 4);
    if (px >= W || py >= H) return;
    const size_t NP = (size_t)W * H;
    const size_t pix = (size_t)py * W + px;
    const int tile = (py / kBlockY) * P->tiles_x + (px / kBlockX);
    const long long cap = P->capacity;
    const int fbeg = (int)min((long long)offset[tile], cap);
    const int fend = (int)min((long long)offset[tile + 1], cap);
    const int K = P->k_max;
    const int kt = min(K, (fend - fbeg + kChunk - 1) / kChunk);
    float Tr = 1.f, r0 = 0.f, r1 = 0.f, r2 = 0.f;
    int last_idx = -1;
    int cutoff = kt;
    for (int k = 0; k < kt; k++) {
        const size_t o = (size_t)k * NP + pix;
        const int cf = chunk_idx[o];
        if (cf < 0 && k > 0) { cutoff = kt; break; }
        const float cT = chunk_T[o];
        r0 = fmaf(chunk_C[3 * o], Tr, r0);
        r1 = fmaf(chunk_C[3 * o + 1], Tr, r1);
        r2 = fmaf(chunk_C[3 * o + 2], Tr, r2);
        Tr *= cT;
        if (cf >= 0) last_idx = cf;
        if (Tr <= 1e-4f) { cutoff = k + 1; break; }
    }
    for (int k = cutoff; k < kt; k++) chunk_idx[(size_t)k * NP + pix] = -1;
    final_T[pix] = Tr;
    final_idx[pix] = last_idx;
    out_img[3 * pix] = saturatef_ref(fmaf(P->bg[0], Tr, r0));
    out_img[3 * pix + 1] = saturatef_ref(fmaf(P->bg[1], Tr, r1));
    out_img[3 * pix + 2] = saturatef_ref(fmaf(P->bg[2], Tr, r2));
}

// ---------------------------------------------------------------------------
// Work counts of the last single-pass forward, for the benchmark's
// instruction-per-evaluation and FP32 rooflines (not on the training path).
// Each pixel replays the reference's per-pixel loop over its tile's sorted
// list (nd_rasterize_forward_kernel, msplat_metal.metal:472-585) with the
// forward's arithmetic and counts, summed over the image:
//   out[0] list positions the loop visits (the terminating one included),
//   out[1] of those, pairs with 0 <= sigma < 5.55 (the exp is evaluated),
//   out[2] pairs blended into the pixel (alpha >= 1/255, not terminating):
//          E, the contributing pixel.Gaussian evaluations,
//   out[3] list positions the reference's backward walks for the pixel
//          (rasterize_backward_kernel, :898-1099: from the last contributor
//          back to the list start).
// One CTA per tile in plain tile order, list entries read from global memory.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kTileThreads)
count_raster_work_kernel(const StepParams* __restrict__ P, const int* __restrict__ offset,
                         const int* __restrict__ tile_sorted, const int* __restrict__ ids,
                         const float2* __restrict__ g_xy, const float4* __restrict__ g_co,
                         unsigned long long* __restrict__ out)
{
    const int tile = blockIdx.x;
    const int tx_n = P->tiles_x;
    const int px = (tile % tx_n) * kBlockX + (threadIdx.x & 15);
    const int py = (tile / tx_n) * kBlockY + (threadIdx.x >> 4);
    const long long cap = P->capacity;
    const int beg = (int)min((long long)offset[tile], cap);
    // the sorted prefix (when the forward sorted prefixes): every pixel
    // terminates inside it
    int end = (int)min((long long)offset[tile + 1], cap);
    if (tile_sorted) end = min(end, beg + tile_sorted[tile]);
    unsigned visited = 0, passed = 0, blended = 0, walk = 0;
    if (px < P->img_w && py < P->img_h) {
        const float fpx = (float)px, fpy = (float)py;
        float T = 1.f;
        int last = beg - 1;
        for (int i = beg; i < end; i++) {
            visited++;
            const int g = ids[i];
            const float4 co = g_co[g];
            const float2 xy = g_xy[g];
            const float dx = xy.x - fpx, dy = xy.y - fpy;
            const float sigma = fmaf(0.5f, fmaf(co.x, dx * dx, co.z * dy * dy), co.y * dx * dy);
            if (sigma < 0.f || sigma >= 5.55f) continue;
            passed++;
            const float alpha = fminf(0.999f, co.w * msp_expf_normal(-sigma));
            if (alpha < 1.f / 255.f) continue;
            const float next_T = T * (1.f - alpha);
            if (next_T <= 1e-4f) break;
            blended++;
            T = next_T;
            last = i;
        }
        walk = (unsigned)(last - beg + 1);
    }
    const unsigned v[4] = {visited, passed, blended, walk};
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const unsigned s = __reduce_add_sync(0xffffffffu, v[k]);
        if ((threadIdx.x & 31) == 0 && s) atomicAdd(&out[k], (unsigned long long)s);
    }
}

// tile_sorted for a forward without prefix_sort (which leaves it unwritten):
// every list sorted whole.  Introspection only (msplat_debug_buffer).
__global__ void whole_lists_kernel(const StepParams* __restrict__ P, int T,
                                   const int* __restrict__ offset, int* __restrict__ tile_sorted)
{
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    const long long cap = P->capacity;
    tile_sorted[t] = (int)(min((long long)offset[t + 1], cap) - min((long long)offset[t], cap));
}

void launch_whole_lists(const StepParams* P, int num_tiles, const Buffers& B, cudaStream_t s)
{
    if (num_tiles <= 0) return;
    whole_lists_kernel<<<(num_tiles + 255) / 256, 256, 0, s>>>(P, num_tiles, B.tile_offset,
                                                               B.tile_sorted);
}

void launch_count_raster_work(const StepParams* P, int num_tiles, bool prefix_sort, const Buffers& B,
                              unsigned long long* d_out, cudaStream_t s)
{
    if (num_tiles <= 0) return;
    count_raster_work_kernel<<<num_tiles, kTileThreads, 0, s>>>(P, B.tile_offset,
                                                               prefix_sort ? B.tile_sorted : nullptr,
                                                               B.sorted_ids,
                                                               B.proj.xy, B.proj.conic_op, d_out);
}

void launch_raster_forward(const StepParams* P, int num_tiles, int k_max, bool prefix_sort, int W, int H,
                           const Buffers& B, cudaStream_t s)
{
    if (num_tiles <= 0) return;
    if (k_max <= 1 && !prefix_sort) {
        raster_forward_kernel<false, 0><<<num_tiles, kTileThreads, 0, s>>>(
            P, B.tile_offset, B.tile_order, B.sorted_ids, B.proj.xy, B.proj.conic_op, B.proj.rgb, B.out_img,
            B.final_T, B.final_idx, nullptr, nullptr, nullptr, nullptr, nullptr, num_tiles);
    } else if (k_max <= 1) {
        // the prefixes, the whole sort of any flagged tile, the flagged tiles again
        raster_forward_kernel<false, 1><<<num_tiles, kTileThreads, 0, s>>>(
            P, B.tile_offset, B.tile_order, B.sorted_ids, B.proj.xy, B.proj.conic_op, B.proj.rgb, B.out_img,
            B.final_T, B.final_idx, nullptr, nullptr, nullptr, B.tile_sorted, B.tile_flag, num_tiles);
        sort_flagged_tiles_kernel<<<std::min(num_tiles, 2 * device_sms()), kSortThreads, 0, s>>>(
            P, B.tile_offset, B.tile_order, num_tiles, B.keys, B.keys_alt, B.sorted_ids,
            B.tile_sorted, B.tile_flag);
        raster_forward_kernel<false, 2><<<num_tiles, kTileThreads, 0, s>>>(
            P, B.tile_offset, B.tile_order, B.sorted_ids, B.proj.xy, B.proj.conic_op, B.proj.rgb, B.out_img,
            B.final_T, B.final_idx, nullptr, nullptr, nullptr, B.tile_sorted, B.tile_flag, num_tiles);
    } else {
        dim3 grid(num_tiles, k_max);
        raster_forward_kernel<true, 0><<<grid, kTileThreads, 0, s>>>(
            P, B.tile_offset, B.tile_order, B.sorted_ids, B.proj.xy, B.proj.conic_op, B.proj.rgb, nullptr,
            nullptr, nullptr, B.chunk_T, B.chunk_C, B.chunk_idx, nullptr, nullptr, num_tiles);
        dim3 mgrid((W + 15) / 16, (H + 15) / 16);
        merge_chunks_kernel<<<mgrid, 256, 0, s>>>(P, B.tile_offset, B.chunk_T, B.chunk_C,
                                                  B.chunk_idx, B.out_img, B.final_T,
                                                  B.final_idx);
    }
}

}  // namespace msp
