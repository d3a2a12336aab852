// kernels_loss.cu -- L1 + SSIM loss and its gradient w.r.t. the rendered
// image, in one kernel per 16x16 pixel tile.  It evaluates the reference's
// three separable passes, each summing in the reference's order (compiled
// with --fmad=false) so v_rendered is bit-identical to the CPU oracle:
//   pass 1  ssim_h_fwd_kernel             (msplat_metal.metal:3053-3115)
//   pass 2  ssim_fused_v_fwd_h_bwd_kernel (msplat_metal.metal:3226-3313),
//           including its derivative fields on the 5 columns outside the
//           image, computed from zero-padded statistics
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

// ---------------------------------------------------------------------------
// The tile's gradient
// needs derivative fields on rows/columns +-5 around it, which need the
// statistics on those rows +-5, which need the images on +-10.  Every sum is
// evaluated in the reference's order, so the result is identical to its
// three passes; the 15- and 9-float-per-pixel
// intermediates never reach memory.
// ---------------------------------------------------------------------------
constexpr int kIn = kS + 4 * kHalo;   // 36: input rows/cols
constexpr int kInP = kIn + 1;         // padded row pitch

__global__ void __launch_bounds__(256)
ssim_loss_fused_kernel(const StepParams* __restrict__ P, const float* __restrict__ rd,
                       const float* __restrict__ gt, float* __restrict__ v_rendered,
                       float* __restrict__ loss_sum)
{
    __shared__ float s_x[kIn][kInP];           // gt
    __shared__ float s_y[kIn][kInP];           // rendered
    __shared__ float s_h[5][kIn][kWide];       // horizontal sums: rows +-10, cols +-5
    __shared__ float s_f[3][kWide][kWide + 1]; // derivative fields: rows +-5, cols +-5
    __shared__ float s_dh[3][kWide][kS];       // horizontal backward: rows +-5, tile cols
    __shared__ float s_red[8];
    const int W = P->img_w, H = P->img_h;
    const float wssim = P->ssim_weight, inv_n = P->loss_inv_n;
    const int tid = threadIdx.x, lx = tid & 15, ly = tid >> 4;
    const int R0 = blockIdx.y * kS, C0 = blockIdx.x * kS;
    const int px = C0 + lx, py = R0 + ly;
    float loss = 0.f;
    for (int c = 0; c < 3; c++) {
        __syncthreads();
        for (int i = tid; i < kIn * kIn; i += 256) {
            const int r = i / kIn, cc = i % kIn;
            const int gy = R0 - 2 * kHalo + r, gx = C0 - 2 * kHalo + cc;
            float xv = 0.f, yv = 0.f;
            if (gx >= 0 && gx < W && gy >= 0 && gy < H) {
                const size_t q = ((size_t)gy * W + gx) * 3 + c;
                xv = gt[q];
                yv = rd[q];
            }
            s_x[r][cc] = xv;
            s_y[r][cc] = yv;
        }
        __syncthreads();
        // pass 1: horizontal sums at image (R0-10+r, C0-5+cc); zero off the image
        for (int i = tid; i < kIn * kWide; i += 256) {
            const int r = i / kWide, cc = i % kWide;
            const int gy = R0 - 2 * kHalo + r, gx = C0 - kHalo + cc;
            float mx = 0.f, my = 0.f, sx = 0.f, sy = 0.f, cxy = 0.f;
            if (gx >= 0 && gx < W && gy >= 0 && gy < H) {
#pragma unroll
                for (int d = 0; d < 11; d++) {
                    const float w = kGauss1D[d];
                    const float gv = s_x[r][cc + d], rv = s_y[r][cc + d];
                    mx += w * gv;
                    my += w * rv;
                    sx += w * gv * gv;
                    sy += w * rv * rv;
                    cxy += w * gv * rv;
                }
            }
            s_h[0][r][cc] = mx;
            s_h[1][r][cc] = my;
            s_h[2][r][cc] = sx;
            s_h[3][r][cc] = sy;
            s_h[4][r][cc] = cxy;
        }
        __syncthreads();
        // pass 2: vertical sums -> SSIM and derivative fields at image
        // (R0-5+fr, C0-5+fc), including the columns off the image
        for (int i = tid; i < kWide * kWide; i += 256) {
            const int fr = i / kWide, fc = i % kWide;
            float mx = 0.f, my = 0.f, sx = 0.f, sy = 0.f, cxy = 0.f;
#pragma unroll
            for (int k = 0; k < 11; k++) {
                const float w = kGauss1D[k];
                mx += w * s_h[0][fr + k][fc];
                my += w * s_h[1][fr + k][fc];
                sx += w * s_h[2][fr + k][fc];
                sy += w * s_h[3][fr + k][fc];
                cxy += w * s_h[4][fr + k][fc];
            }
            const float sxs = sx - mx * mx, sys = sy - my * my, sxy = cxy - mx * my;
            const float A = 2.0f * mx * my + kSsimC1, B = 2.0f * sxy + kSsimC2;
            const float Cd = mx * mx + my * my + kSsimC1, D = sxs + sys + kSsimC2;
            const float iCD = 1.0f / (Cd * D);
            const float dmu = 2.0f * B * (mx * Cd - A * my) / (Cd * Cd * D);
            const float dsyq = -A * B * iCD / D, dsxy = 2.0f * A * iCD;
            s_f[0][fr][fc] = dmu - 2.0f * my * dsyq - mx * dsxy;
            s_f[1][fr][fc] = 2.0f * dsyq;
            s_f[2][fr][fc] = dsxy;
            if (fr >= kHalo && fr < kHalo + kS && fc >= kHalo && fc < kHalo + kS) {
                const int gy = R0 - kHalo + fr, gx = C0 - kHalo + fc;
                if (gx < W && gy < H) {
                    const float ssim = (A * B) / (Cd * D);
                    const size_t q = ((size_t)gy * W + gx) * 3 + c;
                    const float l1 = fabsf(gt[q] - rd[q]);
                    loss += wssim * (1.0f - ssim) + (1.0f - wssim) * l1;
                }
            }
        }
        __syncthreads();
        // pass 2b: horizontal backward at image (R0-5+dr, C0+dc); zero off the image
        for (int i = tid; i < kWide * kS; i += 256) {
            const int dr = i / kS, dc = i % kS;
            const int gy = R0 - kHalo + dr, gx = C0 + dc;
            float h1 = 0.f, h2 = 0.f, h3 = 0.f;
            if (gx < W && gy >= 0 && gy < H) {
#pragma unroll
                for (int d = 0; d < 11; d++) {
                    const float w = kGauss1D[10 - d];
                    h1 += w * s_f[0][dr][dc + d];
                    h2 += w * s_f[1][dr][dc + d];
                    h3 += w * s_f[2][dr][dc + d];
                }
            }
            s_dh[0][dr][dc] = h1;
            s_dh[1][dr][dc] = h2;
            s_dh[2][dr][dc] = h3;
        }
        __syncthreads();
        // pass 3: vertical backward + L1 sign for the tile's own pixel
        if (px < W && py < H) {
            float c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
            for (int d = 0; d < 11; d++) {
                const float w = kGauss1D[10 - d];
                c1 += w * s_dh[0][ly + d][lx];
                c2 += w * s_dh[1][ly + d][lx];
                c3 += w * s_dh[2][ly + d][lx];
            }
            const float rv = s_y[ly + 2 * kHalo][lx + 2 * kHalo];
            const float gv = s_x[ly + 2 * kHalo][lx + 2 * kHalo];
            const float v_ssim = c1 + rv * c2 + gv * c3;
            const float v_l1 = (gv > rv) ? -1.0f : ((gv < rv) ? 1.0f : 0.0f);
            v_rendered[((size_t)py * W + px) * 3 + c] = inv_n * (-wssim * v_ssim + (1.0f - wssim) * v_l1);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) loss += __shfl_xor_sync(0xffffffffu, loss, o);
    if ((tid & 31) == 0) s_red[tid >> 5] = loss;
    __syncthreads();
    if (tid == 0) {
        float sum = 0.f;
        for (int w = 0; w < 8; w++) sum += s_red[w];
        atomicAdd(loss_sum, sum);
    }
}

void launch_ssim(const StepParams* P, int W, int H, const float* gt, const Buffers& B,
                 cudaStream_t s)
{
    dim3 grid((W + kS - 1) / kS, (H + kS - 1) / kS);
    ssim_loss_fused_kernel<<<grid, 256, 0, s>>>(P, B.out_img, gt, B.v_rendered, B.loss_sum);
}

}  // namespace msp
