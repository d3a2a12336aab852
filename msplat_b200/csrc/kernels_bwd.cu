// kernels_bwd.cu -- backward half of the step: rasterizer VJP, projection
// VJP, and every Adam update.  Unlike the forward files this one is compiled
// with FMA contraction (its results are held to a tolerance, not to the
// bit); the few expressions that replay forward decisions (sigma, alpha) are
// written with explicit non-fused operations so they stay bit-identical.
#include <algorithm>

#include "engine.h"
#include "adam.cuh"
#include "msp_math.cuh"

namespace msp {

// ---------------------------------------------------------------------------
// Rasterizer backward.  Reference: rasterize_backward_kernel
// (msplat_metal.metal:898-1099) and, for depth chunks,
// compute_chunk_prefix_suffix_kernel (:2804-2840) plus
// rasterize_backward_chunked_kernel (:2844-3031).
// One CTA per 16x16 tile (per (tile, chunk)); each warp owns one 8x8
// quadrant and each thread replays two of its pixels, (x, y) and (x, y + 4),
// back to front.
// Each lane adds
// its pixels' contributions, the warp sums its lanes with
// a transposed butterfly (8 values in 9 shuffles, the opacity term in 5),
// then 9 lanes issue one RED each into the Gaussian's 9 contiguous
// accumulators: v_rgb[3] (gated by the clamp mask), v_conic[3], v_xy[2],
// v_opacity (w.r.t. the logit).  Staged batches drop the Gaussians that cannot
// reach any pixel of the tile, as the forward does, and each warp walks only
// those that can reach a pixel of its quadrant (quadrant_mask: the exact
// least sigma over each 8x8 rectangle of pixel centres, with the forward's
// conservative margins).
// ---------------------------------------------------------------------------

__device__ __forceinline__ float sel(bool c, float a, float b) { return c ? a : b; }

// Two pixels per thread halve the per-Gaussian overhead (shared-memory
// broadcasts, vote, warp reduction) per pixel; the 64-register cap (8 CTAs
// of 128 threads per SM) keeps enough warps resident.  Measured at C1: 0.99
// ms against 1.13 ms for one pixel per thread.
// Tuning constants; a variant build may override them (-DMSP_BWD_MIN_BLOCKS=...).
#ifndef MSP_BWD_MIN_BLOCKS
#define MSP_BWD_MIN_BLOCKS 8
#endif
#ifndef MSP_RAST_BATCH
#define MSP_RAST_BATCH 256
#endif
#ifndef MSP_PROJ_BWD_MIN_BLOCKS
#define MSP_PROJ_BWD_MIN_BLOCKS 5
#endif
constexpr int kBwdPPT = 2;
constexpr int kBwdMinBlocks = MSP_BWD_MIN_BLOCKS;
constexpr int kRastBatch = MSP_RAST_BATCH;

// Back-to-front state of one pixel.  Bs = sum_c (buffer_c + T_final*bg_c) *
// v_out_c, the colour "behind" the current Gaussian weighted by the pixel's
// output gradient: the reference's per-channel v_alpha terms (rgb_c*T -
// buffer_c*ra - T_final*bg_c*ra) * v_out_c summed over c need only this one
// scalar, updated as buffer_c += rgb_c * fac.
struct PixelBwd {
    float T, Bs;
    float vo0, vo1, vo2;
    int bin_final;
};

// One pixel's contribution to Gaussian (xy, co, rc) at list index idx,
// added into v[0..8]; rc holds the clamped colour max(rgb + 0.5, 0).
// sigma and alpha replay the forward bit for bit (its exact products, no
// contraction; this file is otherwise compiled with FMA contraction), so the
// skip decisions are the forward's (rasterize_backward_kernel :1023-1075).
// v[3..5] are summed without the factor 0.5 and v[8] without the factor
// -(1 - opacity); both are applied once after the warp reduction.
__device__ __forceinline__ bool backprop(PixelBwd& s, float fpx, float fpy, const float2 xy,
                                         const float4 co, const float4 rc, int idx, float v[9])
{
    if (idx > s.bin_final) return false;
    const float dx = xy.x - fpx, dy = xy.y - fpy;
    const float dxx = __fmul_rn(dx, dx);
    const float sigma = fmaf(0.5f, fmaf(co.x, dxx, __fmul_rn(__fmul_rn(co.z, dy), dy)),
                             __fmul_rn(__fmul_rn(co.y, dx), dy));
    if (sigma < 0.f || sigma >= 5.55f) return false;
    const float alpha = fminf(0.999f, __fmul_rn(co.w, msp_expf_normal(-sigma)));
    if (alpha < 1.f / 255.f || !(alpha < 0.999f)) return false;
    // 1 / (1 - alpha): the hardware reciprocal refined by one Newton step
    // (the product of these factors rebuilds T along the whole list, so a
    // last-ulp bias would compound; d lies in (0.001, 1], no special cases)
    const float d = 1.f - alpha;
    const float r0 = __fdividef(1.f, d);
    const float ra = fmaf(r0, fmaf(-d, r0, 1.f), r0);
    s.T *= ra;
    const float fac = alpha * s.T;
    const float rv = rc.x * s.vo0 + rc.y * s.vo1 + rc.z * s.vo2;
    const float v_alpha = s.T * rv - ra * s.Bs;
    s.Bs += fac * rv;
    v[0] += fac * s.vo0;
    v[1] += fac * s.vo1;
    v[2] += fac * s.vo2;
    const float v_sigma = -alpha * v_alpha;
    v[3] += v_sigma * dxx;
    v[4] += v_sigma * (dx * dy);
    v[5] += v_sigma * (dy * dy);
    v[6] += v_sigma * (co.x * dx + co.y * dy);
    v[7] += v_sigma * (co.y * dx + co.z * dy);
    v[8] += v_sigma;
    return true;
}

template <bool CHUNKED, int PPT>
__global__ void __launch_bounds__(256 / PPT, kBwdMinBlocks)
raster_backward_kernel(const StepParams* __restrict__ P, const int* __restrict__ offset,
                       const int* __restrict__ order, const int* __restrict__ ids,
                       const float2* __restrict__ g_xy,
                       const float4* __restrict__ g_co, const float4* __restrict__ g_rgb,
                       const float* __restrict__ final_T, const int* __restrict__ final_idx,
                       const float* __restrict__ v_rendered, const int* __restrict__ chunk_idx,
                       const float* __restrict__ prefix_T, const float* __restrict__ chunk_T,
                       const float* __restrict__ after_C, float* __restrict__ grad_acc)
{
    static_assert(PPT == 2, "a warp's 32 lanes x 2 pixels cover one 8x8 quadrant");
    constexpr int kThreads = 256 / PPT;
    __shared__ int s_id[kRastBatch];
    __shared__ float2 s_xy[kRastBatch];
    __shared__ float4 s_co[kRastBatch];
    __shared__ float4 s_rgb[kRastBatch];
    __shared__ int s_wmax[kThreads / 32];
    __shared__ int s_order[kRastBatch];
    __shared__ unsigned char s_quad[kRastBatch];
    __shared__ int s_wcnt[kRastBatch / 32];
    const int tile = order[blockIdx.x];
    const int tx_n = P->tiles_x;
    const int W = P->img_w, H = P->img_h;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tx0 = (tile % tx_n) * kBlockX, ty0 = (tile / tx_n) * kBlockY;
    // warp w owns the 8x8 quadrant (w & 1, w >> 1); lane: column lane & 7,
    // rows lane >> 3 and + 4
    const int px = tx0 + 8 * (warp & 1) + (lane & 7);
    const int by = ty0 + 8 * (warp >> 1);
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
    }
    const size_t NP = (size_t)W * H;
    PixelBwd st[PPT];
    int my_max = beg - 1;
#pragma unroll
    for (int h = 0; h < PPT; h++) {
        PixelBwd& s = st[h];
        const int py = by + (lane >> 3) + 4 * h;
        s = PixelBwd{0.f, 0.f, 0.f, 0.f, 0.f, beg - 1};
        if (px < W && py < H) {
            const size_t pix = (size_t)py * W + px;
            const float Tf = final_T[pix];
            s.vo0 = v_rendered[3 * pix];
            s.vo1 = v_rendered[3 * pix + 1];
            s.vo2 = v_rendered[3 * pix + 2];
            float b0 = 0.f, b1 = 0.f, b2 = 0.f;
            if (CHUNKED) {
                const size_t o = (size_t)k * NP + pix;
                const int bf = chunk_idx[o];
                if (bf >= beg) {
                    s.bin_final = bf;
                    s.T = prefix_T[o] * chunk_T[o];
                    b0 = after_C[3 * o];
                    b1 = after_C[3 * o + 1];
                    b2 = after_C[3 * o + 2];
                }
            } else {
                s.bin_final = final_idx[pix];
                s.T = Tf;
            }
            s.Bs = (b0 + Tf * P->bg[0]) * s.vo0 + (b1 + Tf * P->bg[1]) * s.vo1 +
                   (b2 + Tf * P->bg[2]) * s.vo2;
        }
        my_max = max(my_max, s.bin_final);
    }
    const float fpx = (float)px;
    const int warp_max = __reduce_max_sync(0xffffffffu, my_max);
    if (lane == 0) s_wmax[warp] = warp_max;
    __syncthreads();
    int tile_max = s_wmax[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; w++) tile_max = max(tile_max, s_wmax[w]);
    const int last = min(end - 1, tile_max);

    const float tx0f = (float)tx0, ty0f = (float)ty0;
    constexpr int kH = kRastBatch / kThreads;  // candidates staged per thread
    for (int bend = last; bend >= beg; bend -= kRastBatch) {
        const int n = min(kRastBatch, bend - beg + 1);
        __syncthreads();
        // Stage the batch (list positions bend, bend-1, ...) and list, in that
        // order, the slots of the Gaussians that can reach a pixel of this tile.
        unsigned keepbits = 0;
#pragma unroll
        for (int h = 0; h < kH; h++) {
            const int slot = tid + h * kThreads;
            bool keep = false;
            if (slot < n) {
                const int g = ids[bend - slot];
                const float2 xy = g_xy[g];
                const float4 co = g_co[g];
                const float4 raw = g_rgb[g];
                s_id[slot] = g;
                s_xy[slot] = xy;
                s_co[slot] = co;
                // clamped colour; .w holds the clamp mask (bit c: rgb_c + 0.5 >= 0)
                const int mask = (raw.x + 0.5f >= 0.f ? 1 : 0) | (raw.y + 0.5f >= 0.f ? 2 : 0) |
                                 (raw.z + 0.5f >= 0.f ? 4 : 0);
                s_rgb[slot] = make_float4(fmaxf(raw.x + 0.5f, 0.f), fmaxf(raw.y + 0.5f, 0.f),
                                          fmaxf(raw.z + 0.5f, 0.f), __int_as_float(mask));
                // the quadrants (one per warp) the Gaussian can reach; none:
                // it cannot reach the tile
                const unsigned qm = quadrant_mask(xy, co, tx0f, ty0f, cull_limit(co));
                keep = qm != 0u;
                s_quad[slot] = (unsigned char)qm;
            }
            const unsigned bal = __ballot_sync(0xffffffffu, keep);
            if (lane == 0) s_wcnt[h * (kThreads / 32) + warp] = __popc(bal);
            keepbits |= (keep ? 1u : 0u) << h;
        }
        __syncthreads();
        int m = 0;
        int woff[kH];
#pragma unroll
        for (int h = 0; h < kH; h++) woff[h] = 0;
#pragma unroll
        for (int c = 0; c < kRastBatch / 32; c++) {
            const int cw = s_wcnt[c];
#pragma unroll
            for (int h = 0; h < kH; h++) woff[h] += c < h * (kThreads / 32) + warp ? cw : 0;
            m += cw;
        }
#pragma unroll
        for (int h = 0; h < kH; h++) {
            const bool keep = (keepbits >> h) & 1u;
            const unsigned bal = __ballot_sync(0xffffffffu, keep);
            if (keep) s_order[woff[h] + __popc(bal & ((1u << lane) - 1u))] = tid + h * kThreads;
        }
        __syncthreads();
        // first listed Gaussian at or below this warp's last contributing index
        int t0 = 0, hi = m;
        while (t0 < hi) {
            const int mid = (t0 + hi) >> 1;
            if (bend - s_order[mid] > warp_max) t0 = mid + 1;
            else hi = mid;
        }
        // walk the listed Gaussians that can reach this warp's rows, in order
        for (int b = t0; b < m; b += 32) {
            const int oi = b + lane;
            const int my_slot = oi < m ? s_order[oi] : 0;
            unsigned bits = __ballot_sync(0xffffffffu, oi < m && ((s_quad[my_slot] >> warp) & 1u));
            while (bits) {
                const int t = __shfl_sync(0xffffffffu, my_slot, __ffs(bits) - 1);
                bits &= bits - 1u;
                const int idx = bend - t;
                const float2 xy = s_xy[t];
                const float4 co = s_co[t];
                const float4 rc = s_rgb[t];
                float v[9];
#pragma unroll
                for (int q = 0; q < 9; q++) v[q] = 0.f;
                bool on = false;
#pragma unroll
                for (int h = 0; h < PPT; h++)
                    on |= backprop(st[h], fpx, (float)(by + (lane >> 3) + 4 * h), xy, co, rc, idx, v);
                if (!__any_sync(0xffffffffu, on)) continue;
                // Transposed butterfly: afterwards lane L holds the warp sum of
                // value (L >> 2); the opacity term takes a plain butterfly.
                const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
                float u[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float send = sel(h16, v[q], v[q + 4]);
                    const float keep = sel(h16, v[q + 4], v[q]);
                    u[q] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                }
                float w2[2];
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    const float send = sel(h8, u[q], u[q + 2]);
                    const float keep = sel(h8, u[q + 2], u[q]);
                    w2[q] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                }
                float x;
                {
                    const float send = sel(h4, w2[0], w2[1]);
                    const float keep = sel(h4, w2[1], w2[0]);
                    x = keep + __shfl_xor_sync(0xffffffffu, send, 4);
                }
                x += __shfl_xor_sync(0xffffffffu, x, 2);
                x += __shfl_xor_sync(0xffffffffu, x, 1);
                float vop = v[8];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) vop += __shfl_xor_sync(0xffffffffu, vop, o);
                const int g = s_id[t];
                const int j = lane >> 2;
                if ((lane & 3) == 0) {
                    bool ok = x != 0.f;
                    if (j < 3) ok = ok && ((__float_as_int(rc.w) >> j) & 1);
                    if (j >= 3 && j < 6) x *= 0.5f;
                    if (ok) atomicAdd(grad_acc + (size_t)g * kGradStride + j, x);
                } else if (lane == 1) {
                    if (vop != 0.f) atomicAdd(grad_acc + (size_t)g * kGradStride + 8, -(1.f - co.w) * vop);
                }
            }
        }
    }
}

// compute_chunk_prefix_suffix_kernel (msplat_metal.metal:2804-2840), over
// the chunks that hold Gaussians (empty chunks have T = 1, C = 0 and change
// neither product nor sum).
__global__ void __launch_bounds__(256)
chunk_prefix_suffix_kernel(const StepParams* __restrict__ P, const int* __restrict__ offset,
                           const float* __restrict__ chunk_T, const float* __restrict__ chunk_C,
                           float* __restrict__ prefix_T, float* __restrict__ after_C)
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
    const int kt = min(P->k_max, (fend - fbeg + kChunk - 1) / kChunk);
    float pT = 1.f;
    for (int k = 0; k < kt; k++) {
        const size_t o = (size_t)k * NP + pix;
        prefix_T[o] = pT;
        pT *= chunk_T[o];
    }
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
    for (int k = kt - 1; k >= 0; k--) {
        const size_t o = (size_t)k * NP + pix;
        after_C[3 * o] = a0;
        after_C[3 * o + 1] = a1;
        after_C[3 * o + 2] = a2;
        const float pk = prefix_T[o];
        a0 += pk * chunk_C[3 * o];
        a1 += pk * chunk_C[3 * o + 1];
        a2 += pk * chunk_C[3 * o + 2];
    }
}

void launch_raster_backward(const StepParams* P, int num_tiles, int k_max, int W, int H,
                            const Buffers& B, cudaStream_t s)
{
    if (num_tiles <= 0) return;
    if (k_max <= 1) {
        raster_backward_kernel<false, kBwdPPT><<<num_tiles, 256 / kBwdPPT, 0, s>>>(
            P, B.tile_offset, B.tile_order, B.sorted_ids, B.proj.xy, B.proj.conic_op, B.proj.rgb, B.final_T,
            B.final_idx, B.v_rendered, nullptr, nullptr, nullptr, nullptr, B.grad_acc);
    } else {
        dim3 pgrid((W + 15) / 16, (H + 15) / 16);
        chunk_prefix_suffix_kernel<<<pgrid, 256, 0, s>>>(P, B.tile_offset, B.chunk_T, B.chunk_C,
                                                         B.prefix_T, B.after_C);
        dim3 grid(num_tiles, k_max);
        raster_backward_kernel<true, kBwdPPT><<<grid, 256 / kBwdPPT, 0, s>>>(
            P, B.tile_offset, B.tile_order, B.sorted_ids, B.proj.xy, B.proj.conic_op, B.proj.rgb, B.final_T,
            nullptr, B.v_rendered, B.chunk_idx, B.prefix_T, B.chunk_T, B.after_C, B.grad_acc);
    }
}

// ---------------------------------------------------------------------------
// Projection backward + every Adam update + densification statistics.
// Reference: project_and_sh_backward_kernel (msplat_metal.metal:1813-1986,
// VJPs :1216-1531), fused_adam_kernel (:1666-1689) launched for groups
// 0,1,2,5 over every element (msplat_metal.mm:1117-1139), and
// accumulate_grad_stats_kernel (:1643-1664).  One thread per Gaussian does
// the geometry VJP and the Adam steps of means/scales/quats/opacity/dc;
// each warp then updates its 32 Gaussians' SH-rest coefficients with
// coalesced loads (the element order of the update does not matter).
// ---------------------------------------------------------------------------
constexpr int kBwdThreads = 128;

struct M3 { float m[3][3]; };  // column-major m[col][row], as Metal's float3x3

__device__ __forceinline__ M3 mul3(const M3& A, const M3& B)
{
    M3 C;
#pragma unroll
    for (int c = 0; c < 3; c++)
#pragma unroll
        for (int r = 0; r < 3; r++)
            C.m[c][r] = (A.m[0][r] * B.m[c][0] + A.m[1][r] * B.m[c][1]) + A.m[2][r] * B.m[c][2];
    return C;
}
__device__ __forceinline__ M3 tr3(const M3& A)
{
    M3 T;
#pragma unroll
    for (int c = 0; c < 3; c++)
#pragma unroll
        for (int r = 0; r < 3; r++) T.m[c][r] = A.m[r][c];
    return T;
}
__device__ __forceinline__ M3 cols3(float a0, float a1, float a2, float b0, float b1, float b2,
                                   float c0, float c1, float c2)
{
    M3 M;
    M.m[0][0] = a0; M.m[0][1] = a1; M.m[0][2] = a2;
    M.m[1][0] = b0; M.m[1][1] = b1; M.m[1][2] = b2;
    M.m[2][0] = c0; M.m[2][1] = c1; M.m[2][2] = c2;
    return M;
}

__device__ __forceinline__ void adam_elem(float* __restrict__ p, float* __restrict__ ea,
                                          float* __restrict__ eas, float g, float step, float b1,
                                          float b2, float inv_bc2, float eps)
{
    float pp = *p, m = *ea, v = *eas;
    adam_math(pp, m, v, g, step, b1, b2, inv_bc2, eps);
    *p = pp;
    *ea = m;
    *eas = v;
}

// Adam over one warp's contiguous slab of a parameter group: `total`
// floats starting at element `e0`, `stride` floats per Gaussian.  grad_of
// returns the element's gradient, or false when the element is not updated
// (culled Gaussians for the SH groups).  Loads of kUnroll elements are issued
// before any update so the warp keeps several coalesced requests in flight.
template <int STRIDE, class G>
__device__ __forceinline__ void adam_slab(float* __restrict__ P, float* __restrict__ M,
                                          float* __restrict__ V, size_t e0, int total, int lane,
                                          float step, float b1, float b2, float inv_bc2, float eps,
                                          G grad_of)
{
    constexpr int kUnroll = 4;
    for (int base = lane; base < total; base += 32 * kUnroll) {
        float p[kUnroll], m[kUnroll], v[kUnroll], g[kUnroll];
        bool on[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            const int e = base + 32 * u;
            on[u] = e < total && grad_of(e / STRIDE, e % STRIDE, g[u]);
            if (on[u]) {
                p[u] = P[e0 + e];
                m[u] = M[e0 + e];
                v[u] = V[e0 + e];
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            if (!on[u]) continue;
            adam_math(p[u], m[u], v[u], g[u], step, b1, b2, inv_bc2, eps);
            const size_t e = e0 + base + 32 * u;
            P[e] = p[u];
            M[e] = m[u];
            V[e] = v[u];
        }
    }
}

// Per-Gaussian gradient slots in shared memory (phase 1 -> phase 2).
constexpr int kGradSlots = 12;  // v_mean[3], v_scale[3], v_quat[4], v_opacity, pad
constexpr int kBasisSlots = 19; // 15 SH-rest basis values + v_rgb[3] (odd stride: no bank conflicts)

// Adam for one warp's 32 Gaussians over the small groups -- means, scales,
// quats and opacity for every Gaussian, features_dc for the visible ones --
// with every parameter, first- and second-moment load of all five groups
// issued before the first update: 14 coalesced rounds of 32 elements, so a
// warp waits for memory once instead of once per group.  Same element
// updates as adam_slab group by group.
constexpr int kSmallRounds = 14;
// round -> group (means 3 rounds, scales 3, quats 4, opacity 1, dc 3), the
// round's 32-element step within its group, and the group's floats per
// Gaussian
__host__ __device__ constexpr int round_group(int r)
{
    return r < 3 ? 0 : r < 6 ? 1 : r < 10 ? 2 : r < 11 ? 5 : 3;
}
__host__ __device__ constexpr int round_u(int r)
{
    return r < 3 ? r : r < 6 ? r - 3 : r < 10 ? r - 6 : r < 11 ? 0 : r - 11;
}
__host__ __device__ constexpr int group_stride(int grp) { return grp == 2 ? 4 : grp == 5 ? 1 : 3; }

__device__ __forceinline__ void adam_small_groups(const AdamPtrs& A, const StepParams* __restrict__ P,
                                                  int g0, int cnt, int lane,
                                                  const float (*sg)[kGradSlots],
                                                  const float (*sb)[kBasisSlots],
                                                  const int* sv)
{
    float p[kSmallRounds], m[kSmallRounds], v[kSmallRounds], g[kSmallRounds];
    unsigned on = 0;
#pragma unroll
    for (int r = 0; r < kSmallRounds; r++) {
        const int grp = round_group(r), stride = group_stride(grp);
        const int e = lane + 32 * round_u(r);
        const int gl = e / stride, k = e - gl * stride;
        bool active = A.numel[grp] > 0 && e < cnt * stride;
        g[r] = 0.f;
        if (active) {
            if (grp == 0) g[r] = sg[gl][k];
            else if (grp == 1) g[r] = sg[gl][3 + k];
            else if (grp == 2) g[r] = sg[gl][6 + k];
            else if (grp == 5) g[r] = sg[gl][10];
            else {  // features_dc: visible Gaussians only
                active = sv[gl] != 0;
                g[r] = MSP_SH_C0 * sb[gl][15 + k];
            }
        }
        if (active) {
            const size_t idx = (size_t)g0 * stride + e;
            p[r] = A.param[grp][idx];
            m[r] = A.exp_avg[grp][idx];
            v[r] = A.exp_avg_sq[grp][idx];
            on |= 1u << r;
        }
    }
    const float b1 = P->beta1, b2 = P->beta2, eps = P->eps;
#pragma unroll
    for (int r = 0; r < kSmallRounds; r++) {
        if (!((on >> r) & 1u)) continue;
        const int grp = round_group(r), stride = group_stride(grp);
        adam_math(p[r], m[r], v[r], g[r], P->adam_step[grp], b1, b2, 1.0f / P->adam_bc2[grp], eps);
        const size_t idx = (size_t)g0 * stride + lane + 32 * round_u(r);
        A.param[grp][idx] = p[r];
        A.exp_avg[grp][idx] = m[r];
        A.exp_avg_sq[grp][idx] = v[r];
    }
}

// Writes one warp's contiguous slab of a gradient group (same walk as
// adam_slab); elements that grad_of declines are written as 0.
template <int STRIDE, class G>
__device__ __forceinline__ void grad_slab(float* __restrict__ out, size_t e0, int total, int lane,
                                          G grad_of)
{
    for (int e = lane; e < total; e += 32) {
        float g = 0.f;
        if (!grad_of(e / STRIDE, e % STRIDE, g)) g = 0.f;
        out[e0 + e] = g;
    }
}

// The accumulating form of grad_slab: adds each visible Gaussian's
// gradients (sv[gl] != 0) to the slab and leaves the rest untouched; four
// elements per lane per round, loads issued before the adds.
template <int STRIDE, class G>
__device__ __forceinline__ void grad_slab_add(float* __restrict__ out, size_t e0, int total, int lane,
                                              const int* sv, G grad_of)
{
    constexpr int kU = 4;
    for (int eb = lane; eb < total; eb += 32 * kU) {
        float g[kU], o[kU];
        bool on[kU];
#pragma unroll
        for (int u = 0; u < kU; u++) {
            const int e = eb + 32 * u;
            on[u] = e < total && sv[e / STRIDE] != 0 && grad_of(e / STRIDE, e % STRIDE, g[u]);
            if (on[u]) o[u] = out[e0 + e];
        }
#pragma unroll
        for (int u = 0; u < kU; u++)
            if (on[u]) out[e0 + eb + 32 * u] = o[u] + g[u];
    }
}



// Geometry and colour VJP of one visible Gaussian (project_and_sh_backward_kernel,
// msplat_metal.metal:1813-1986; VJPs :1216-1531): from its 9 raster
// gradients `ga` fills gr[] (v_mean, v_scale, v_quat, v_opacity) and the
// row bs[] (15 SH-rest basis values of the view direction, then v_rgb).
__device__ __forceinline__ void gaussian_vjp(const StepParams* __restrict__ P,
                                             const float* __restrict__ ga, const float4 co,
                                             const float p[3], float ls0, float ls1, float ls2,
                                             float q0, float q1, float q2, float q3,
                                             float gr[kGradSlots], float* bs, bool with_basis)
{
    const float vr0 = ga[0], vr1 = ga[1], vr2 = ga[2];
    const float vc0 = ga[3], vc1 = ga[4], vc2 = ga[5];
    const float vx = ga[6], vy = ga[7];
    const float vop = ga[8];
    const float fx = P->fx, fy = P->fy;
    const float* vm = P->viewmat;
    const float* pm = P->projmat;
    float vmean[3];
    // project_pix_vjp (:1216-1234); v_depth is always 0 (:1860-1864)
    const float h3 = ((pm[12] * p[0] + pm[13] * p[1]) + pm[14] * p[2]) + pm[15];
    const float rw = 1.f / (h3 + 1e-6f);
    const float vnx = (0.5f * (float)P->img_w) * vx, vny = (0.5f * (float)P->img_h) * vy;
    const float vp0 = vnx * rw, vp1 = vny * rw, vp2 = 0.f;
    vmean[0] = ((pm[0] * vp0 + pm[4] * vp1) + pm[8] * vp2) + vm[8] * 0.f;
    vmean[1] = ((pm[1] * vp0 + pm[5] * vp1) + pm[9] * vp2) + vm[9] * 0.f;
    vmean[2] = ((pm[2] * vp0 + pm[6] * vp1) + pm[10] * vp2) + vm[10] * 0.f;
    // cov2d_to_conic_vjp (:1253-1264): ((-X) G) X
    const float X00 = -co.x, X01 = -co.y, X10 = -co.y, X11 = -co.z;
    const float XG00 = X00 * vc0 + X10 * vc1, XG01 = X01 * vc0 + X11 * vc1;
    const float XG10 = X00 * vc1 + X10 * vc2, XG11 = X01 * vc1 + X11 * vc2;
    const float VS00 = XG00 * co.x + XG10 * co.y, VS01 = XG01 * co.x + XG11 * co.y;
    const float VS10 = XG00 * co.y + XG10 * co.z, VS11 = XG01 * co.y + XG11 * co.z;
    const float vcv0 = VS00, vcv1 = VS10 + VS01, vcv2 = VS11;
    // recompute cov3d (:1875-1878)
    const float es[3] = {msp_expf(ls0), msp_expf(ls1), msp_expf(ls2)};
    const float qs = rsqrt_ieee(((q3 * q3 + q0 * q0) + q1 * q1) + q2 * q2);
    const float w = q0 * qs, x = q1 * qs, y = q2 * qs, z = q3 * qs;
    const M3 R = cols3(1.f - 2.f * (y * y + z * z), 2.f * (x * y + w * z), 2.f * (x * z - w * y),
                       2.f * (x * y - w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z + w * x),
                       2.f * (x * z + w * y), 2.f * (y * z - w * x), 1.f - 2.f * (x * x + y * y));
    const float gs = P->glob_scale;
    const float sc[3] = {gs * es[0], gs * es[1], gs * es[2]};
    M3 Mm;
#pragma unroll
    for (int c = 0; c < 3; c++)
#pragma unroll
        for (int r = 0; r < 3; r++) Mm.m[c][r] = R.m[c][r] * sc[c];
    const M3 tmp = mul3(Mm, tr3(Mm));
    const float cv[6] = {tmp.m[0][0], tmp.m[0][1], tmp.m[0][2], tmp.m[1][1], tmp.m[1][2], tmp.m[2][2]};
    // project_cov3d_ewa_vjp (:1339-1407)
    float pv0 = ((vm[0] * p[0] + vm[1] * p[1]) + vm[2] * p[2]) + vm[3];
    float pv1 = ((vm[4] * p[0] + vm[5] * p[1]) + vm[6] * p[2]) + vm[7];
    const float pv2 = ((vm[8] * p[0] + vm[9] * p[1]) + vm[10] * p[2]) + vm[11];
    const float lim_x = 1.3f * P->tan_fovx, lim_y = 1.3f * P->tan_fovy;
    pv0 = pv2 * fminf(lim_x, fmaxf(-lim_x, pv0 / pv2));
    pv1 = pv2 * fminf(lim_y, fmaxf(-lim_y, pv1 / pv2));
    const float rz = 1.f / pv2, rz2 = rz * rz;
    const M3 Wm = cols3(vm[0], vm[4], vm[8], vm[1], vm[5], vm[9], vm[2], vm[6], vm[10]);
    const M3 J = cols3(fx * rz, 0.f, 0.f, 0.f, fy * rz, 0.f, (-fx * pv0) * rz2,
                       (-fy * pv1) * rz2, 0.f);
    const M3 V = cols3(cv[0], cv[1], cv[2], cv[1], cv[3], cv[4], cv[2], cv[4], cv[5]);
    const M3 vcov = cols3(vcv0, 0.5f * vcv1, 0.f, 0.5f * vcv1, vcv2, 0.f, 0.f, 0.f, 0.f);
    const M3 T = mul3(J, Wm);
    const M3 vV = mul3(mul3(tr3(T), vcov), T);
    const M3 vT1 = mul3(mul3(vcov, T), tr3(V));
    const M3 vT2 = mul3(mul3(tr3(vcov), T), V);
    M3 vT;
#pragma unroll
    for (int c = 0; c < 3; c++)
#pragma unroll
        for (int r = 0; r < 3; r++) vT.m[c][r] = vT1.m[c][r] + vT2.m[c][r];
    const float vcov3d[6] = {vV.m[0][0], vV.m[0][1] + vV.m[1][0], vV.m[0][2] + vV.m[2][0],
                             vV.m[1][1], vV.m[1][2] + vV.m[2][1], vV.m[2][2]};
    const M3 vJ = mul3(vT, tr3(Wm));
    const float fx_rz2 = fx * rz2, fy_rz2 = fy * rz2, rz3 = rz2 * rz;
    const float vt0 = -fx_rz2 * vJ.m[2][0];
    const float vt1 = -fy_rz2 * vJ.m[2][1];
    const float vt2 = ((-fx_rz2 * vJ.m[0][0] + 2.f * fx * pv0 * rz3 * vJ.m[2][0]) -
                       fy_rz2 * vJ.m[1][1]) + 2.f * fy * pv1 * rz3 * vJ.m[2][1];
#pragma unroll
    for (int c = 0; c < 3; c++)
        vmean[c] += (vt0 * Wm.m[c][0] + vt1 * Wm.m[c][1]) + vt2 * Wm.m[c][2];
    // scale_rot_to_cov3d_vjp (:1498-1531)
    const M3 vVs = cols3(vcov3d[0], 0.5f * vcov3d[1], 0.5f * vcov3d[2], 0.5f * vcov3d[1],
                         vcov3d[3], 0.5f * vcov3d[4], 0.5f * vcov3d[2], 0.5f * vcov3d[4],
                         vcov3d[5]);
    const M3 Sm = cols3(sc[0], 0.f, 0.f, 0.f, sc[1], 0.f, 0.f, 0.f, sc[2]);
    const M3 M2 = mul3(R, Sm);
    M3 vVs2;
#pragma unroll
    for (int c = 0; c < 3; c++)
#pragma unroll
        for (int r = 0; r < 3; r++) vVs2.m[c][r] = 2.f * vVs.m[c][r];
    const M3 vM = mul3(vVs2, M2);
#pragma unroll
    for (int c = 0; c < 3; c++)
        gr[3 + c] = ((R.m[c][0] * vM.m[c][0] + R.m[c][1] * vM.m[c][1]) + R.m[c][2] * vM.m[c][2]) * es[c];
    const M3 vR = mul3(vM, Sm);
    const float (*v)[3] = vR.m;
    gr[6] = 2.f * ((x * (v[1][2] - v[2][1]) + y * (v[2][0] - v[0][2])) + z * (v[0][1] - v[1][0]));
    gr[7] = 2.f * (((-2.f * x * (v[1][1] + v[2][2]) + y * (v[0][1] + v[1][0])) +
                    z * (v[0][2] + v[2][0])) + w * (v[1][2] - v[2][1]));
    gr[8] = 2.f * (((x * (v[0][1] + v[1][0]) - 2.f * y * (v[0][0] + v[2][2])) +
                    z * (v[1][2] + v[2][1])) + w * (v[2][0] - v[0][2]));
    gr[9] = 2.f * (((x * (v[0][2] + v[2][0]) + y * (v[1][2] + v[2][1])) -
                    2.f * z * (v[0][0] + v[1][1])) + w * (v[0][1] - v[1][0]));
    gr[0] = vmean[0];
    gr[1] = vmean[1];
    gr[2] = vmean[2];
    gr[10] = vop;
    // SH basis of the view direction for the dc/rest Adam (:1915-1985)
    if (with_basis) sh_rest_basis(P->cam_pos, p, bs);
    bs[15] = vr0;
    bs[16] = vr1;
    bs[17] = vr2;
}

// GRAD_OUT = false: the single-GPU step, Adam applied in place.
// GRAD_OUT = true: the data-parallel step, gradients written to G (the
// same values Adam would have consumed) and no parameter touched.
template <bool GRAD_OUT>
__global__ void __launch_bounds__(kBwdThreads, MSP_PROJ_BWD_MIN_BLOCKS)
project_backward_adam_kernel(const StepParams* __restrict__ P, int N,
                             const int* __restrict__ radii, const float4* __restrict__ g_co,
                             const float* __restrict__ grad_acc, AdamPtrs A, StatPtrs St,
                             GradOut G, int nb_rest)
{
    __shared__ float s_grad[kBwdThreads][kGradSlots];
    __shared__ float s_basis[kBwdThreads][kBasisSlots];
    __shared__ int s_vis[kBwdThreads];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int base = blockIdx.x * kBwdThreads;
    const int i = base + tid;
    const float b1 = P->beta1, b2 = P->beta2, eps = P->eps;
    bool vis = false;
    float gr[kGradSlots];
#pragma unroll
    for (int k = 0; k < kGradSlots; k++) gr[k] = 0.f;
    if (i < N) {
        const int rad = radii[i];
        vis = rad > 0;
        if (vis) {
            const float* __restrict__ means = A.param[0];
            const float* __restrict__ scales = A.param[1];
            const float* __restrict__ quats = A.param[2];
            const float* ga = grad_acc + (size_t)i * kGradStride;
            const float p[3] = {means[3 * (size_t)i], means[3 * (size_t)i + 1], means[3 * (size_t)i + 2]};
            const float ls0 = scales[3 * (size_t)i], ls1 = scales[3 * (size_t)i + 1],
                        ls2 = scales[3 * (size_t)i + 2];
            const float q0 = quats[4 * (size_t)i], q1 = quats[4 * (size_t)i + 1],
                        q2 = quats[4 * (size_t)i + 2], q3 = quats[4 * (size_t)i + 3];
            // densification statistics (accumulate_grad_stats_kernel), read
            // before the VJP so their loads overlap it
            const float st_vis = St.vis_counts[i], st_norm = St.grad_norm[i], st_max = St.max_2d[i];
            // the SH-rest basis only when this kernel forms the rest gradient
            const bool with_basis =
                GRAD_OUT ? !(G.compact || G.rest_done) : (A.numel[4] > 0 && nb_rest > 0);
            gaussian_vjp(P, ga, g_co[i], p, ls0, ls1, ls2, q0, q1, q2, q3, gr, s_basis[tid],
                         with_basis);
            const float vx = ga[6], vy = ga[7];
            St.vis_counts[i] = st_vis + 1.0f;
            St.grad_norm[i] = st_norm + sqrtf(vx * vx + vy * vy);
            St.max_2d[i] = fmaxf(st_max, (float)rad * P->inv_max_dim);
        }
    }
#pragma unroll
    for (int k = 0; k < kGradSlots; k++) s_grad[tid][k] = gr[k];
    s_vis[tid] = vis;
    __syncthreads();
    // Phase 2: Adam over this warp's 32 Gaussians, group by group.
    const int wbase = warp * 32;
    const int g0 = base + wbase;
    if (g0 >= N) return;
    const int cnt = min(32, N - g0);
    const float(*sg)[kGradSlots] = s_grad + wbase;
    const float(*sb)[kBasisSlots] = s_basis + wbase;
    const int* sv = s_vis + wbase;
    if constexpr (GRAD_OUT) {
        const size_t gb = (size_t)g0;
        if (G.accumulate) {
            // another view of the same step: add the visible Gaussians'
            // gradients to the buffer, count the view in vis
            if (!__any_sync(0xffffffffu, lane < cnt && sv[lane])) return;
            grad_slab_add<3>(G.g[0], gb * 3, cnt * 3, lane, sv,
                             [&](int gl, int k, float& g) { g = sg[gl][k]; return true; });
            grad_slab_add<3>(G.g[1], gb * 3, cnt * 3, lane, sv,
                             [&](int gl, int k, float& g) { g = sg[gl][3 + k]; return true; });
            grad_slab_add<4>(G.g[2], gb * 4, cnt * 4, lane, sv,
                             [&](int gl, int k, float& g) { g = sg[gl][6 + k]; return true; });
            grad_slab_add<1>(G.g[5], gb, cnt, lane, sv,
                             [&](int gl, int, float& g) { g = sg[gl][10]; return true; });
            grad_slab_add<3>(G.g[3], gb * 3, cnt * 3, lane, sv, [&](int gl, int k, float& g) {
                g = MSP_SH_C0 * sb[gl][15 + k];
                return true;
            });
            if (G.rest_done) {
                if (lane < cnt && sv[lane]) G.vis[g0 + lane] += 1.f;
                return;
            }
            const int stride = P->rest_stride;
            const int used = nb_rest * 3;
            auto rest_add = [&](int gl, int kk, float& g) {
                if (kk >= used) return false;
                const int b = kk / 3, c = kk - 3 * b;
                g = sb[gl][b] * sb[gl][15 + c];
                return true;
            };
            if (stride == 45) grad_slab_add<45>(G.g[4], gb * 45, cnt * 45, lane, sv, rest_add);
            else if (stride == 24) grad_slab_add<24>(G.g[4], gb * 24, cnt * 24, lane, sv, rest_add);
            else if (stride == 9) grad_slab_add<9>(G.g[4], gb * 9, cnt * 9, lane, sv, rest_add);
            else if (stride == 72) grad_slab_add<72>(G.g[4], gb * 72, cnt * 72, lane, sv, rest_add);
            if (lane < cnt && sv[lane]) G.vis[g0 + lane] += 1.f;
            return;
        }
        grad_slab<3>(G.g[0], gb * 3, cnt * 3, lane,
                     [&](int gl, int k, float& g) { g = sg[gl][k]; return true; });
        grad_slab<3>(G.g[1], gb * 3, cnt * 3, lane,
                     [&](int gl, int k, float& g) { g = sg[gl][3 + k]; return true; });
        grad_slab<4>(G.g[2], gb * 4, cnt * 4, lane,
                     [&](int gl, int k, float& g) { g = sg[gl][6 + k]; return true; });
        grad_slab<1>(G.g[5], gb, cnt, lane,
                     [&](int gl, int, float& g) { g = sg[gl][10]; return true; });
        if (G.compact) {
            // v_rgb of the visible Gaussians (0 for the others) and the camera
            grad_slab<3>(G.g[3], gb * 3, cnt * 3, lane, [&](int gl, int k, float& g) {
                g = sb[gl][15 + k];
                return sv[gl] != 0;
            });
            if (lane < cnt) G.vis[g0 + lane] = sv[lane] ? 1.f : 0.f;
            if (g0 == 0 && lane < 3) G.cam[lane] = P->cam_pos[lane];
            return;
        }
        grad_slab<3>(G.g[3], gb * 3, cnt * 3, lane, [&](int gl, int k, float& g) {
            g = MSP_SH_C0 * sb[gl][15 + k];
            return sv[gl] != 0;
        });
        if (G.rest_done) {
            if (lane < cnt) G.vis[g0 + lane] = sv[lane] ? 1.f : 0.f;
            return;
        }
        const int stride = P->rest_stride;
        const int used = nb_rest * 3;
        auto rest_grad = [&](int gl, int kk, float& g) {
            if (kk >= used || !sv[gl]) return false;
            const int b = kk / 3, c = kk - 3 * b;
            g = sb[gl][b] * sb[gl][15 + c];
            return true;
        };
        if (stride == 45) grad_slab<45>(G.g[4], gb * 45, cnt * 45, lane, rest_grad);
        else if (stride == 24) grad_slab<24>(G.g[4], gb * 24, cnt * 24, lane, rest_grad);
        else if (stride == 9) grad_slab<9>(G.g[4], gb * 9, cnt * 9, lane, rest_grad);
        else if (stride == 72) grad_slab<72>(G.g[4], gb * 72, cnt * 72, lane, rest_grad);
        if (lane < cnt) G.vis[g0 + lane] = sv[lane] ? 1.f : 0.f;
        return;
    }
    // means, scales, quats, opacity (every Gaussian: zero gradient when
    // culled) and features_dc (visible only)
    adam_small_groups(A, P, g0, cnt, lane, sg, sb, sv);
    if (A.numel[4] > 0 && nb_rest > 0) {  // features_rest, visible only, degrees in use
        const int stride = P->rest_stride;
        const int used = nb_rest * 3;
        auto rest_grad = [&](int gl, int kk, float& g) {
            if (kk >= used || !sv[gl]) return false;
            const int b = kk / 3, c = kk - 3 * b;
            g = sb[gl][b] * sb[gl][15 + c];
            return true;
        };
        if (stride == 45)
            adam_slab<45>(A.param[4], A.exp_avg[4], A.exp_avg_sq[4], (size_t)g0 * 45, cnt * 45,
                          lane, P->adam_step[4], b1, b2, 1.0f / P->adam_bc2[4], eps, rest_grad);
        else if (stride == 24)
            adam_slab<24>(A.param[4], A.exp_avg[4], A.exp_avg_sq[4], (size_t)g0 * 24, cnt * 24,
                          lane, P->adam_step[4], b1, b2, 1.0f / P->adam_bc2[4], eps, rest_grad);
        else if (stride == 9)
            adam_slab<9>(A.param[4], A.exp_avg[4], A.exp_avg_sq[4], (size_t)g0 * 9, cnt * 9,
                         lane, P->adam_step[4], b1, b2, 1.0f / P->adam_bc2[4], eps, rest_grad);
        else if (stride == 72)
            adam_slab<72>(A.param[4], A.exp_avg[4], A.exp_avg_sq[4], (size_t)g0 * 72, cnt * 72,
                          lane, P->adam_step[4], b1, b2, 1.0f / P->adam_bc2[4], eps, rest_grad);
    }
}

// SH-rest bases updated: degrees_to_use 0 -> 0, 1 -> 3, 2 -> 8, >= 3 -> 15
// (the reference stops at degree 3 here, msplat_metal.metal:1931-1985).
int rest_bases_updated(int degrees_to_use, int rest_stride)
{
    int nb = degrees_to_use < 1 ? 0 : degrees_to_use == 1 ? 3 : degrees_to_use == 2 ? 8 : 15;
    if (nb * 3 > rest_stride) nb = rest_stride / 3;
    return nb;
}

// ---------------------------------------------------------------------------
// SH-rest Adam (the fused SH update of project_and_sh_backward_kernel,
// msplat_metal.metal:1931-1985, for features_rest only), as its own
// streaming kernel: 75% of the optimiser's bytes, and it needs nothing from
// the geometry VJP -- only the view direction (from the forward's copy of
// the mean, so the VJP may update the means meanwhile), v_rgb and
// visibility.  It runs on the engine's side stream, concurrently with
// project_backward_adam_kernel: this kernel streams at the bandwidth bound
// while the other waits on its VJP's latency.  Each lane
// first builds its Gaussian's 15 basis values in shared memory; then each
// warp streams its 32 Gaussians' contiguous rest slab, kU independent
// elements per lane per round so every lane keeps 3*kU loads in flight.
// Culled Gaussians are neither read nor written.
// ---------------------------------------------------------------------------
constexpr int kRestThreads = 256;

template <int RS>
__global__ void __launch_bounds__(kRestThreads)
rest_adam_kernel(const StepParams* __restrict__ P, int N, const int* __restrict__ radii,
                 const float* __restrict__ grad_acc, const float* __restrict__ sh_mean,
                 float* __restrict__ rest, float* __restrict__ rest_m, float* __restrict__ rest_v,
                 int used)
{
    __shared__ float s_b[kRestThreads][17];  // 15 basis values + pad (odd stride)
    __shared__ float s_c[kRestThreads][3];   // v_rgb
    __shared__ int s_vis[kRestThreads];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int base = blockIdx.x * kRestThreads;
    const int i = base + tid;
    bool vis = false;
    if (i < N && radii[i] > 0) {
        vis = true;
        const float p[3] = {sh_mean[3 * (size_t)i], sh_mean[3 * (size_t)i + 1],
                            sh_mean[3 * (size_t)i + 2]};
        sh_rest_basis(P->cam_pos, p, s_b[tid]);
        const float* ga = grad_acc + (size_t)i * kGradStride;
        s_c[tid][0] = ga[0];
        s_c[tid][1] = ga[1];
        s_c[tid][2] = ga[2];
    }
    s_vis[tid] = vis;
    __syncthreads();
    const int wbase = warp * 32;
    const int g0 = base + wbase;
    if (g0 >= N) return;
    const int cnt = min(32, N - g0);
    if (!__any_sync(0xffffffffu, s_vis[wbase + (lane < cnt ? lane : 0)])) return;
    const float step = P->adam_step[4], inv_bc2 = 1.0f / P->adam_bc2[4];
    const float b1 = P->beta1, b2 = P->beta2, eps = P->eps;
    const size_t e0 = (size_t)g0 * RS;
    const int total = cnt * RS;
    constexpr int kU = 8;
    for (int eb = lane; eb < total; eb += 32 * kU) {
        float g[kU], pv[kU], mv[kU], vv[kU];
        bool on[kU];
#pragma unroll
        for (int u = 0; u < kU; u++) {
            const int e = eb + 32 * u;
            const int gl = e / RS, kk = e - gl * RS;
            on[u] = e < total && kk < used && s_vis[wbase + gl];
            if (on[u]) {
                const int b = kk / 3, c = kk - 3 * b;
                g[u] = s_b[wbase + gl][b] * s_c[wbase + gl][c];
                pv[u] = rest[e0 + e];
                mv[u] = rest_m[e0 + e];
                vv[u] = rest_v[e0 + e];
            }
        }
#pragma unroll
        for (int u = 0; u < kU; u++) {
            if (!on[u]) continue;
            adam_math(pv[u], mv[u], vv[u], g[u], step, b1, b2, inv_bc2, eps);
            const size_t e = e0 + eb + 32 * u;
            rest[e] = pv[u];
            rest_m[e] = mv[u];
            rest_v[e] = vv[u];
        }
    }
}

// SH-rest gradients of the data-parallel step in the full layout: the
// gradient half's counterpart of rest_adam_kernel (75% of the gradient
// bytes), streamed on the side stream beside the projection VJP.  Element
// (i, b, c) is basis_b(view direction of the forward's mean) * v_rgb_c, the
// product project_backward_adam_kernel<true> forms.  Overwrite: every
// element is written (0 for culled Gaussians and for degrees not in use).
// Accumulate: the visible Gaussians' used elements are added; nothing else
// is touched.
template <int RS>
__global__ void __launch_bounds__(kRestThreads)
rest_grads_kernel(const StepParams* __restrict__ P, int N, const int* __restrict__ radii,
                  const float* __restrict__ grad_acc, const float* __restrict__ sh_mean,
                  float* __restrict__ out, int used, int accumulate)
{
    __shared__ float s_b[kRestThreads][17];  // 15 basis values + pad (odd stride)
    __shared__ float s_c[kRestThreads][3];   // v_rgb
    __shared__ int s_vis[kRestThreads];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int base = blockIdx.x * kRestThreads;
    const int i = base + tid;
    bool vis = false;
    if (i < N && radii[i] > 0) {
        vis = true;
        const float p[3] = {sh_mean[3 * (size_t)i], sh_mean[3 * (size_t)i + 1],
                            sh_mean[3 * (size_t)i + 2]};
        sh_rest_basis(P->cam_pos, p, s_b[tid]);
        const float* ga = grad_acc + (size_t)i * kGradStride;
        s_c[tid][0] = ga[0];
        s_c[tid][1] = ga[1];
        s_c[tid][2] = ga[2];
    }
    s_vis[tid] = vis;
    __syncthreads();
    const int wbase = warp * 32;
    const int g0 = base + wbase;
    if (g0 >= N) return;
    const int cnt = min(32, N - g0);
    if (accumulate && !__any_sync(0xffffffffu, s_vis[wbase + (lane < cnt ? lane : 0)])) return;
    const size_t e0 = (size_t)g0 * RS;
    const int total = cnt * RS;
    constexpr int kU = 8;
    for (int eb = lane; eb < total; eb += 32 * kU) {
        float g[kU], o[kU];
        bool on[kU];
#pragma unroll
        for (int u = 0; u < kU; u++) {
            const int e = eb + 32 * u;
            const int gl = e / RS, kk = e - gl * RS;
            const bool real = e < total && kk < used && s_vis[wbase + gl];
            g[u] = 0.f;
            if (real) {
                const int b = kk / 3, c = kk - 3 * b;
                g[u] = s_b[wbase + gl][b] * s_c[wbase + gl][c];
            }
            on[u] = accumulate ? real : e < total;
            if (accumulate && on[u]) o[u] = out[e0 + e];
        }
#pragma unroll
        for (int u = 0; u < kU; u++)
            if (on[u]) out[e0 + eb + 32 * u] = accumulate ? o[u] + g[u] : g[u];
    }
}

int launch_project_backward_adam(const StepParams* P, int N, int degrees_to_use_host,
                                 int rest_stride_host, const Buffers& B, const AdamPtrs& A,
                                 const StatPtrs& St, cudaStream_t s)
{
    if (N <= 0) return 0;
    const int nb = rest_bases_updated(degrees_to_use_host, rest_stride_host);
    AdamPtrs A2 = A;
    int launches = 1;
    bool joined = false;
    const SideStream& side = engine_side();
    if (A.numel[4] > 0 && nb > 0) {
        const int grid = (N + kRestThreads - 1) / kRestThreads;
        const int used = nb * 3;
        // fork: the side stream starts after everything queued so far
        const bool forked = cudaEventRecord(side.fork, s) == cudaSuccess &&
                            cudaStreamWaitEvent(side.stream, side.fork, 0) == cudaSuccess;
        const cudaStream_t rs = forked ? side.stream : s;
#define MSP_REST(RS)                                                                            \
    rest_adam_kernel<RS><<<grid, kRestThreads, 0, rs>>>(P, N, B.proj.radii, B.grad_acc,       \
                                                        B.proj.sh_mean, A.param[4], A.exp_avg[4], \
                                                        A.exp_avg_sq[4], used)
        bool done = true;
        switch (rest_stride_host) {
            case 45: MSP_REST(45); break;
            case 24: MSP_REST(24); break;
            case 9: MSP_REST(9); break;
            case 72: MSP_REST(72); break;
            default: done = false; break;
        }
#undef MSP_REST
        if (done) {
            A2.numel[4] = 0;  // the rest group is done
            launches++;
        }
        // join: what the engine stream queues after this stage waits for it
        if (forked) {
            if (cudaEventRecord(side.join, side.stream) == cudaSuccess) joined = true;
            else cudaStreamSynchronize(side.stream);
        }
    }
    const int grid = (N + kBwdThreads - 1) / kBwdThreads;
    project_backward_adam_kernel<false><<<grid, kBwdThreads, 0, s>>>(
        P, N, B.proj.radii, B.proj.conic_op, B.grad_acc, A2, St, GradOut{}, nb);
    if (joined) cudaStreamWaitEvent(s, side.join, 0);
    return launches;
}

int launch_project_backward_grads(const StepParams* P, int N, int degrees_to_use_host,
                                  int rest_stride_host, const Buffers& B, const AdamPtrs& A,
                                  const StatPtrs& St, const GradOut& G, cudaStream_t s)
{
    if (N <= 0) return 0;
    const int nb = rest_bases_updated(degrees_to_use_host, rest_stride_host);
    GradOut G2 = G;
    int launches = 1;
    bool joined = false;
    const bool full = !G.compact && rest_stride_host > 0;
    const SideStream& side = engine_side();
    if (full && (rest_stride_host == 45 || rest_stride_host == 24 || rest_stride_host == 9 ||
                 rest_stride_host == 72)) {
        const int grid = (N + kRestThreads - 1) / kRestThreads;
        const int used = nb * 3;
        const bool forked = cudaEventRecord(side.fork, s) == cudaSuccess &&
                            cudaStreamWaitEvent(side.stream, side.fork, 0) == cudaSuccess;
        const cudaStream_t rs = forked ? side.stream : s;
#define MSP_REST(RS)                                                                         \
    rest_grads_kernel<RS><<<grid, kRestThreads, 0, rs>>>(P, N, B.proj.radii, B.grad_acc,    \
                                                         B.proj.sh_mean, G.g[4], used,      \
                                                         G.accumulate)
        switch (rest_stride_host) {
            case 45: MSP_REST(45); break;
            case 24: MSP_REST(24); break;
            case 9: MSP_REST(9); break;
            case 72: MSP_REST(72); break;
        }
#undef MSP_REST
        G2.rest_done = 1;
        launches++;
        if (forked) {
            if (cudaEventRecord(side.join, side.stream) == cudaSuccess) joined = true;
            else cudaStreamSynchronize(side.stream);
        }
    }
    const int grid = (N + kBwdThreads - 1) / kBwdThreads;
    project_backward_adam_kernel<true><<<grid, kBwdThreads, 0, s>>>(
        P, N, B.proj.radii, B.proj.conic_op, B.grad_acc, A, St, G2, nb);
    if (joined) cudaStreamWaitEvent(s, side.join, 0);
    return launches;
}

// ---------------------------------------------------------------------------
// Adam from a gradient buffer (the data-parallel step, after the gradients of
// all views were summed).  Same update and the same visible-only rule for
// the SH groups as project_backward_adam_kernel: groups 3 and 4 skip
// Gaussians no view saw, and group 4 only updates the degrees in use.
// One block row per group (blockIdx.y); 32-bit element indices (the host
// checks N * stride < 2^31).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
adam_apply_kernel(ApplyArgs a)
{
    const int gi = blockIdx.y;
    float* __restrict__ P = a.param[gi];
    if (!P) return;
    float* __restrict__ M = a.exp_avg[gi];
    float* __restrict__ V = a.exp_avg_sq[gi];
    const float* __restrict__ Gd = a.grad[gi];
    const int S = a.stride[gi];
    const int e_end = a.end * S;
    const float step = a.step[gi], inv_bc2 = 1.0f / a.bc2[gi];
    const bool sh = gi == 3 || gi == 4;
    for (int e = a.begin * S + blockIdx.x * blockDim.x + threadIdx.x; e < e_end;
         e += gridDim.x * blockDim.x) {
        if (sh) {
            const int i = e / S;
            if (!(a.vis[i] > 0.f)) continue;
            if (gi == 4 && e - i * S >= a.used_rest) continue;
        }
        adam_elem(P + e, M + e, V + e, Gd[e] * a.scale, step, a.beta1, a.beta2, inv_bc2, a.eps);
    }
}

void launch_adam_apply(const ApplyArgs& a, cudaStream_t s)
{
    if (a.end <= a.begin) return;
    long long widest = 0;
    for (int gi = 0; gi < kGroups; gi++)
        if (a.param[gi]) widest = std::max(widest, (long long)(a.end - a.begin) * a.stride[gi]);
    if (widest <= 0) return;
    const long long blocks = std::min((widest + 255) / 256, 148LL * 16);
    adam_apply_kernel<<<dim3((unsigned)blocks, kGroups), 256, 0, s>>>(a);
}

}  // namespace msp
