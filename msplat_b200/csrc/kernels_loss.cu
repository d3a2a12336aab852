// kernels_loss.cu -- L1 + SSIM loss and its gradient w.r.t. the rendered
// image.  Three passes over 16x16 pixel tiles, each summing in the
// reference's order (compiled with --fmad=false) so v_rendered is
// bit-identical to the CPU oracle.
//   pass 1  ssim_h_fwd_kernel             (msplat_metal.metal:3053-3115)
//   pass 2  ssim_fused_v_fwd_h_bwd_kernel (msplat_metal.metal:3226-3313)
//   pass 3  ssim_v_bwd_kernel             (msplat_metal.metal:3396-3464)
// x = gt, y = rendered.  The loss sum here is the intended one
// (sum over pixels of w*(1 - mean_c ssim) + (1-w)*mean_c |x-y|); the
// reference's threadgroup accounting differs on partial edge tiles and its
// value is never read back synchronously.
#include "engine.h"
#include "msp_math.cuh"

namespace msp {

constexpr int kS = 16;          // tile edge
constexpr int kHalo = 5;        // half window
constexpr int kWide = kS + 2 * kHalo;  // 26

__global__ void __launch_bounds__(256)
ssim_h_fwd_kernel(const StepParams* __restrict__ P, const float* __restrict__ rd,
                  const float* __restrict__ gt, float* __restrict__ hbuf)
{
    __shared__ float s_gt[3][kS][kWide];
    __shared__ float s_rd[3][kS][kWide];
    const int W = P->img_w, H = P->img_h;
    const int tid = threadIdx.x, lx = tid & 15, ly = tid >> 4;
    const int bx = blockIdx.x * kS - kHalo, by = blockIdx.y * kS;
    for (int i = tid; i < kS * kWide; i += 256) {
        const int sy = i / kWide, sx = i % kWide;
        const int gy = by + sy, gx = bx + sx;
        float g3[3] = {0.f, 0.f, 0.f}, r3[3] = {0.f, 0.f, 0.f};
        if (gx >= 0 && gx < W && gy >= 0 && gy < H) {
            const size_t q = ((size_t)gy * W + gx) * 3;
#pragma unroll
            for (int c = 0; c < 3; c++) {
                g3[c] = gt[q + c];
                r3[c] = rd[q + c];
            }
        }
#pragma unroll
        for (int c = 0; c < 3; c++) {
            s_gt[c][sy][sx] = g3[c];
            s_rd[c][sy][sx] = r3[c];
        }
    }
    __syncthreads();
    const int px = blockIdx.x * kS + lx, py = by + ly;
    if (px >= W || py >= H) return;
    float* o = hbuf + ((size_t)py * W + px) * 15;
#pragma unroll
    for (int c = 0; c < 3; c++) {
        float mx = 0.f, my = 0.f, sx = 0.f, sy = 0.f, cxy = 0.f;
#pragma unroll
        for (int d = 0; d < 11; d++) {
            const float w = kGauss1D[d];
            const float gv = s_gt[c][ly][lx + d], rv = s_rd[c][ly][lx + d];
            mx += w * gv;
            my += w * rv;
            sx += w * gv * gv;
            sy += w * rv * rv;
            cxy += w * gv * rv;
        }
        o[c * 5 + 0] = mx;
        o[c * 5 + 1] = my;
        o[c * 5 + 2] = sx;
        o[c * 5 + 3] = sy;
        o[c * 5 + 4] = cxy;
    }
}

__global__ void __launch_bounds__(256)
ssim_fused_kernel(const StepParams* __restrict__ P, const float* __restrict__ rd,
                  const float* __restrict__ gt, const float* __restrict__ hbuf,
                  float* __restrict__ dbuf, float* __restrict__ loss_sum)
{
    __shared__ float s_hp[kWide][kWide][5];
    __shared__ float s_f[3][kS][kWide];
    __shared__ float s_red[8];
    const int W = P->img_w, H = P->img_h;
    const float wssim = P->ssim_weight;
    const int tid = threadIdx.x, lx = tid & 15, ly = tid >> 4;
    const int bx = blockIdx.x * kS - kHalo, by = blockIdx.y * kS - kHalo;
    const int px = blockIdx.x * kS + lx, py = blockIdx.y * kS + ly;
    const bool inside = px < W && py < H;
    float loss = 0.f;
    for (int c = 0; c < 3; c++) {
        for (int i = tid; i < kWide * kWide; i += 256) {
            const int sy = i / kWide, sx = i % kWide;
            const int gy = by + sy, gx = bx + sx;
            float v[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
            if (gx >= 0 && gx < W && gy >= 0 && gy < H) {
                const float* hp = hbuf + ((size_t)gy * W + gx) * 15 + c * 5;
#pragma unroll
                for (int f = 0; f < 5; f++) v[f] = hp[f];
            }
#pragma unroll
            for (int f = 0; f < 5; f++) s_hp[sy][sx][f] = v[f];
        }
        __syncthreads();
        for (int i = tid; i < kS * kWide; i += 256) {
            const int dy = i / kWide, dx = i % kWide;
            float mx = 0.f, my = 0.f, sx = 0.f, sy = 0.f, cxy = 0.f;
#pragma unroll
            for (int k = 0; k < 11; k++) {
                const float w = kGauss1D[k];
                mx += w * s_hp[dy + k][dx][0];
                my += w * s_hp[dy + k][dx][1];
                sx += w * s_hp[dy + k][dx][2];
                sy += w * s_hp[dy + k][dx][3];
                cxy += w * s_hp[dy + k][dx][4];
            }
            const float sxs = sx - mx * mx, sys = sy - my * my, sxy = cxy - mx * my;
            const float A = 2.0f * mx * my + kSsimC1, B = 2.0f * sxy + kSsimC2;
            const float Cd = mx * mx + my * my + kSsimC1, D = sxs + sys + kSsimC2;
            const float iCD = 1.0f / (Cd * D);
            const float dmu = 2.0f * B * (mx * Cd - A * my) / (Cd * Cd * D);
            const float dsyq = -A * B * iCD / D, dsxy = 2.0f * A * iCD;
            s_f[0][dy][dx] = dmu - 2.0f * my * dsyq - mx * dsxy;
            s_f[1][dy][dx] = 2.0f * dsyq;
            s_f[2][dy][dx] = dsxy;
            if (dx >= kHalo && dx < kHalo + kS) {
                const int gpx = bx + dx, gpy = by + dy + kHalo;
                if (gpx >= 0 && gpx < W && gpy >= 0 && gpy < H) {
                    const float ssim = (A * B) / (Cd * D);
                    const size_t q = ((size_t)gpy * W + gpx) * 3 + c;
                    const float l1 = fabsf(gt[q] - rd[q]);
                    loss += wssim * (1.0f - ssim) + (1.0f - wssim) * l1;
                }
            }
        }
        __syncthreads();
        if (inside) {
            float h1 = 0.f, h2 = 0.f, h3 = 0.f;
#pragma unroll
            for (int d = 0; d < 11; d++) {
                const float w = kGauss1D[10 - d];
                h1 += w * s_f[0][ly][lx + d];
                h2 += w * s_f[1][ly][lx + d];
                h3 += w * s_f[2][ly][lx + d];
            }
            float* o = dbuf + ((size_t)py * W + px) * 9 + c * 3;
            o[0] = h1;
            o[1] = h2;
            o[2] = h3;
        }
        __syncthreads();
    }
    // CTA sum of the loss terms, one atomic per CTA.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) loss += __shfl_xor_sync(0xffffffffu, loss, o);
    if ((tid & 31) == 0) s_red[tid >> 5] = loss;
    __syncthreads();
    if (tid == 0) {
        float s = 0.f;
        for (int w = 0; w < 8; w++) s += s_red[w];
        atomicAdd(loss_sum, s);
    }
}

__global__ void __launch_bounds__(256)
ssim_v_bwd_kernel(const StepParams* __restrict__ P, const float* __restrict__ rd,
                  const float* __restrict__ gt, const float* __restrict__ dbuf,
                  float* __restrict__ v_rendered)
{
    __shared__ float s_d[kWide][kS][9];
    const int W = P->img_w, H = P->img_h;
    const int tid = threadIdx.x, lx = tid & 15, ly = tid >> 4;
    const int bx = blockIdx.x * kS, by = blockIdx.y * kS - kHalo;
    for (int i = tid; i < kWide * kS; i += 256) {
        const int sy = i / kS, sx = i % kS;
        const int gy = by + sy, gx = bx + sx;
        float v[9] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (gx >= 0 && gx < W && gy >= 0 && gy < H) {
            const float* d = dbuf + ((size_t)gy * W + gx) * 9;
#pragma unroll
            for (int f = 0; f < 9; f++) v[f] = d[f];
        }
#pragma unroll
        for (int f = 0; f < 9; f++) s_d[sy][sx][f] = v[f];
    }
    __syncthreads();
    const int px = bx + lx, py = blockIdx.y * kS + ly;
    if (px >= W || py >= H) return;
    const float wssim = P->ssim_weight, inv_n = P->loss_inv_n;
#pragma unroll
    for (int c = 0; c < 3; c++) {
        float c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
        for (int d = 0; d < 11; d++) {
            const float w = kGauss1D[10 - d];
            c1 += w * s_d[ly + d][lx][c * 3 + 0];
            c2 += w * s_d[ly + d][lx][c * 3 + 1];
            c3 += w * s_d[ly + d][lx][c * 3 + 2];
        }
        const size_t q = ((size_t)py * W + px) * 3 + c;
        const float rv = rd[q], gv = gt[q];
        const float v_ssim = c1 + rv * c2 + gv * c3;
        const float v_l1 = (gv > rv) ? -1.0f : ((gv < rv) ? 1.0f : 0.0f);
        v_rendered[q] = inv_n * (-wssim * v_ssim + (1.0f - wssim) * v_l1);
    }
}

void launch_ssim(const StepParams* P, int W, int H, const float* gt, const Buffers& B,
                 cudaStream_t s)
{
    dim3 grid((W + kS - 1) / kS, (H + kS - 1) / kS);
    ssim_h_fwd_kernel<<<grid, 256, 0, s>>>(P, B.out_img, gt, B.ssim_h);
    ssim_fused_kernel<<<grid, 256, 0, s>>>(P, B.out_img, gt, B.ssim_h, B.ssim_d, B.loss_sum);
    ssim_v_bwd_kernel<<<grid, 256, 0, s>>>(P, B.out_img, gt, B.ssim_d, B.v_rendered);
}

}  // namespace msp
