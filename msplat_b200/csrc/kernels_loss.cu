// kernels_loss.cu -- L1 + SSIM loss and its gradient w.r.t. the rendered
// image, in one kernel per 32x32 pixel tile.  It evaluates the reference's
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

// ---------------------------------------------------------------------------
// One CTA per 32x32 tile of pixels, one colour channel at a time.  The
// tile's gradient needs derivative fields on rows/columns +-5 around it,
// which need the statistics on those rows +-5, which need the images on
// +-10.  Each pass gives every thread a short run of adjacent outputs and
// streams the run's inputs once, in ascending order; since output o of a
// run receives its taps in that same ascending order, every sum is evaluated
// in the reference's order (bit-identical results) while each input is read
// from shared memory once per run instead of once per tap.
// ---------------------------------------------------------------------------
constexpr int kT = 32;                  // tile edge
constexpr int kHalo = 5;                // half window
constexpr int kIn = kT + 4 * kHalo;     // 52: input rows/cols (+-10)
constexpr int kInP = kIn + 1;           // input row pitch
constexpr int kHc = kT + 2 * kHalo;     // 42: statistic / field columns (+-5)
constexpr int kFr = kT + 2 * kHalo;     // 42: field rows (+-5)
constexpr int kFP = kHc + 1;            // field row pitch
constexpr int kSsimThreads = 256;
// run lengths per pass (outputs per thread)
constexpr int kR1 = 3;   // pass 1: 52 rows x 14 runs of 3 columns = 728 runs
constexpr int kR2 = 7;   // pass 2: 42 columns x 6 runs of 7 rows = 252 runs
constexpr int kR3 = 2;   // pass 2b: 42 rows x 16 runs of 2 columns = 672 runs
constexpr int kR4 = 4;   // pass 3: 32 columns x 8 runs of 4 rows = 256 runs

struct SsimSmem {
    float x[kIn][kInP];          // gt
    float y[kIn][kInP];          // rendered
    float h[5][kIn][kHc];        // horizontal sums: rows +-10, cols +-5 (reused for dh)
    float f[3][kFr][kFP];        // derivative fields: rows +-5, cols +-5
    float red[kSsimThreads / 32];
};
static_assert(sizeof(float) * 3 * kFr * kT <= sizeof(float) * 5 * kIn * kHc,
              "horizontal backward sums must fit in the statistics buffer");

__global__ void __launch_bounds__(kSsimThreads, 2)
ssim_loss_fused_kernel(const StepParams* __restrict__ P, const float* __restrict__ rd,
                       const float* __restrict__ gt, float* __restrict__ v_rendered,
                       float* __restrict__ loss_sum)
{
    extern __shared__ __align__(16) unsigned char ssim_raw[];
    SsimSmem& S = *reinterpret_cast<SsimSmem*>(ssim_raw);
    float (*dh)[kFr][kT] = reinterpret_cast<float (*)[kFr][kT]>(&S.h[0][0][0]);
    const int W = P->img_w, H = P->img_h;
    const float wssim = P->ssim_weight, inv_n = P->loss_inv_n;
    const int tid = threadIdx.x;
    const int R0 = blockIdx.y * kT, C0 = blockIdx.x * kT;
    float loss = 0.f;
    for (int c = 0; c < 3; c++) {
        __syncthreads();
        for (int i = tid; i < kIn * kIn; i += kSsimThreads) {
            const int r = i / kIn, cc = i - r * kIn;
            const int gy = R0 - 2 * kHalo + r, gx = C0 - 2 * kHalo + cc;
            float xv = 0.f, yv = 0.f;
            if (gx >= 0 && gx < W && gy >= 0 && gy < H) {
                const size_t q = ((size_t)gy * W + gx) * 3 + c;
                xv = gt[q];
                yv = rd[q];
            }
            S.x[r][cc] = xv;
            S.y[r][cc] = yv;
        }
        __syncthreads();
        // pass 1 (ssim_h_fwd): horizontal sums at image (R0-10+r, C0-5+cc);
        // zero off the image
        for (int run = tid; run < kIn * (kHc / kR1); run += kSsimThreads) {
            const int r = run / (kHc / kR1), cc0 = (run - r * (kHc / kR1)) * kR1;
            const int gy = R0 - 2 * kHalo + r;
            float a[kR1][5];
#pragma unroll
            for (int o = 0; o < kR1; o++)
#pragma unroll
                for (int q = 0; q < 5; q++) a[o][q] = 0.f;
#pragma unroll
            for (int q = 0; q < kR1 + 10; q++) {
                const float gv = S.x[r][cc0 + q], rv = S.y[r][cc0 + q];
#pragma unroll
                for (int o = 0; o < kR1; o++) {
                    const int d = q - o;
                    if (d < 0 || d > 10) continue;
                    const float w = kGauss1D[d];
                    a[o][0] += w * gv;
                    a[o][1] += w * rv;
                    a[o][2] += w * gv * gv;
                    a[o][3] += w * rv * rv;
                    a[o][4] += w * gv * rv;
                }
            }
#pragma unroll
            for (int o = 0; o < kR1; o++) {
                const int gx = C0 - kHalo + cc0 + o;
                const bool in = gx >= 0 && gx < W && gy >= 0 && gy < H;
#pragma unroll
                for (int q = 0; q < 5; q++) S.h[q][r][cc0 + o] = in ? a[o][q] : 0.f;
            }
        }
        __syncthreads();
        // pass 2 (ssim_fused_v_fwd_h_bwd): vertical sums -> SSIM and the
        // derivative fields at image (R0-5+fr, C0-5+fc), columns off the
        // image included
        for (int run = tid; run < kHc * (kFr / kR2); run += kSsimThreads) {
            const int grp = run / kHc, fc = run - grp * kHc;
            const int fr0 = grp * kR2;
            float a[kR2][5];
#pragma unroll
            for (int o = 0; o < kR2; o++)
#pragma unroll
                for (int q = 0; q < 5; q++) a[o][q] = 0.f;
#pragma unroll
            for (int q = 0; q < kR2 + 10; q++) {
                float hv[5];
#pragma unroll
                for (int t = 0; t < 5; t++) hv[t] = S.h[t][fr0 + q][fc];
#pragma unroll
                for (int o = 0; o < kR2; o++) {
                    const int k = q - o;
                    if (k < 0 || k > 10) continue;
                    const float w = kGauss1D[k];
#pragma unroll
                    for (int t = 0; t < 5; t++) a[o][t] += w * hv[t];
                }
            }
#pragma unroll
            for (int o = 0; o < kR2; o++) {
                const int fr = fr0 + o;
                const float mx = a[o][0], my = a[o][1], sx = a[o][2], sy = a[o][3], cxy = a[o][4];
                const float sxs = sx - mx * mx, sys = sy - my * my, sxy = cxy - mx * my;
                const float A = 2.0f * mx * my + kSsimC1, B = 2.0f * sxy + kSsimC2;
                const float Cd = mx * mx + my * my + kSsimC1, D = sxs + sys + kSsimC2;
                const float iCD = 1.0f / (Cd * D);
                const float dmu = 2.0f * B * (mx * Cd - A * my) / (Cd * Cd * D);
                const float dsyq = -A * B * iCD / D, dsxy = 2.0f * A * iCD;
                S.f[0][fr][fc] = dmu - 2.0f * my * dsyq - mx * dsxy;
                S.f[1][fr][fc] = 2.0f * dsyq;
                S.f[2][fr][fc] = dsxy;
                if (fr >= kHalo && fr < kHalo + kT && fc >= kHalo && fc < kHalo + kT) {
                    const int gy = R0 - kHalo + fr, gx = C0 - kHalo + fc;
                    if (gx < W && gy < H) {
                        const float ssim = (A * B) / (Cd * D);
                        const float l1 = fabsf(S.x[fr + kHalo][fc + kHalo] - S.y[fr + kHalo][fc + kHalo]);
                        loss += wssim * (1.0f - ssim) + (1.0f - wssim) * l1;
                    }
                }
            }
        }
        __syncthreads();
        // pass 2b: horizontal backward at image (R0-5+dr, C0+dc); zero off the image
        for (int run = tid; run < kFr * (kT / kR3); run += kSsimThreads) {
            const int dr = run / (kT / kR3), dc0 = (run - dr * (kT / kR3)) * kR3;
            const int gy = R0 - kHalo + dr;
            float a[kR3][3];
#pragma unroll
            for (int o = 0; o < kR3; o++) a[o][0] = a[o][1] = a[o][2] = 0.f;
#pragma unroll
            for (int q = 0; q < kR3 + 10; q++) {
                const float f0 = S.f[0][dr][dc0 + q], f1 = S.f[1][dr][dc0 + q],
                            f2 = S.f[2][dr][dc0 + q];
#pragma unroll
                for (int o = 0; o < kR3; o++) {
                    const int d = q - o;
                    if (d < 0 || d > 10) continue;
                    const float w = kGauss1D[10 - d];
                    a[o][0] += w * f0;
                    a[o][1] += w * f1;
                    a[o][2] += w * f2;
                }
            }
#pragma unroll
            for (int o = 0; o < kR3; o++) {
                const int gx = C0 + dc0 + o;
                const bool in = gx < W && gy >= 0 && gy < H;
                dh[0][dr][dc0 + o] = in ? a[o][0] : 0.f;
                dh[1][dr][dc0 + o] = in ? a[o][1] : 0.f;
                dh[2][dr][dc0 + o] = in ? a[o][2] : 0.f;
            }
        }
        __syncthreads();
        // pass 3 (ssim_v_bwd): vertical backward + L1 sign for the tile's pixels
        {
            const int grp = tid / kT, lx = tid - grp * kT;
            const int ly0 = grp * kR4;
            const int px = C0 + lx;
            float a[kR4][3];
#pragma unroll
            for (int o = 0; o < kR4; o++) a[o][0] = a[o][1] = a[o][2] = 0.f;
#pragma unroll
            for (int q = 0; q < kR4 + 10; q++) {
                const float d0 = dh[0][ly0 + q][lx], d1 = dh[1][ly0 + q][lx],
                            d2 = dh[2][ly0 + q][lx];
#pragma unroll
                for (int o = 0; o < kR4; o++) {
                    const int d = q - o;
                    if (d < 0 || d > 10) continue;
                    const float w = kGauss1D[10 - d];
                    a[o][0] += w * d0;
                    a[o][1] += w * d1;
                    a[o][2] += w * d2;
                }
            }
#pragma unroll
            for (int o = 0; o < kR4; o++) {
                const int ly = ly0 + o, py = R0 + ly;
                if (px < W && py < H) {
                    const float rv = S.y[ly + 2 * kHalo][lx + 2 * kHalo];
                    const float gv = S.x[ly + 2 * kHalo][lx + 2 * kHalo];
                    const float v_ssim = a[o][0] + rv * a[o][1] + gv * a[o][2];
                    const float v_l1 = (gv > rv) ? -1.0f : ((gv < rv) ? 1.0f : 0.0f);
                    v_rendered[((size_t)py * W + px) * 3 + c] =
                        inv_n * (-wssim * v_ssim + (1.0f - wssim) * v_l1);
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) loss += __shfl_xor_sync(0xffffffffu, loss, o);
    if ((tid & 31) == 0) S.red[tid >> 5] = loss;
    __syncthreads();
    if (tid == 0) {
        float sum = 0.f;
        for (int w = 0; w < kSsimThreads / 32; w++) sum += S.red[w];
        atomicAdd(loss_sum, sum);
    }
}

void launch_ssim(const StepParams* P, int W, int H, const float* gt, const Buffers& B,
                 cudaStream_t s)
{
    static std::once_flag once[kMaxDeviceSlots];
    const int smem = (int)sizeof(SsimSmem);
    once_per_device(once, [smem](int) {
        cudaFuncSetAttribute(ssim_loss_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem);
    });
    dim3 grid((W + kT - 1) / kT, (H + kT - 1) / kT);
    ssim_loss_fused_kernel<<<grid, kSsimThreads, smem, s>>>(P, B.out_img, gt, B.v_rendered,
                                                             B.loss_sum);
}

}  // namespace msp
