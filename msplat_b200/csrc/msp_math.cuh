// msp_math.cuh -- scalar maths shared by the engine's kernels.
//
// The deterministic part of the step (projection, binning keys, the forward
// raster, the loss) is compiled with --fmad=false so that a*b+c is never
// contracted; explicit fmaf() is used exactly where the reference kernels
// call fma() (core/metal/msplat_metal.metal).  exp() is msp_expf(), the
// method below; sqrt and division are IEEE round-to-nearest (no fast math),
// and rsqrt(x) is 1.0f/sqrtf(x).  The CPU oracle evaluates the same
// sequences, which makes tile membership, per-tile order and the forward
// image bit-identical between the two.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace msp {

constexpr int kBlockX = 16;
constexpr int kBlockY = 16;
constexpr int kTileThreads = kBlockX * kBlockY;  // one thread per pixel of a tile
constexpr int kChunk = 512;                      // depth chunk of the chunked raster

__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

// exp(x): Cody & Waite (1980) argument reduction x = k*ln2 + r with ln2
// split into a high part with 15 significant bits (k*ln2_hi is exact) and a
// low part.  k = x/ln2 rounded to nearest comes from one fma against
// 1.5*2^23: the sum t carries k in its low mantissa bits, so k needs no
// rounding or conversion instruction.  e^r = 1 + r + r^2 q(r) with q the
// degree-4 minimax fit of the relative error on |r| <= ln2/2 (3.1e-9;
// coefficients from oracle/derive_exp_coefficients.py), in Horner form.
// Over every float input the result is within 0.90 ulp of exp().
constexpr float kExpRound = 12582912.0f;  // 1.5 * 2^23
constexpr int kExpRoundBits = 0x4B400000;
__device__ __forceinline__ float expf_poly(float x, float* tout)
{
    const float log2e = 1.44269502162933349609375f;
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.428606765330187045e-06f;
    const float t = fmaf(x, log2e, kExpRound);
    const float k = __fsub_rn(t, kExpRound);
    float r = fmaf(-k, ln2_hi, x);
    r = fmaf(-k, ln2_lo, r);
    float p = 0.0013814594130963087f;
    p = fmaf(p, r, 0.0083687193691730499f);
    p = fmaf(p, r, 0.041668388992547989f);
    p = fmaf(p, r, 0.1666652113199234f);
    p = fmaf(p, r, 0.49999994039535522f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    *tout = t;
    return p;
}

// The scale by 2^k takes two exact steps so that the subnormal range rounds
// once.
__device__ __forceinline__ float msp_expf(float x)
{
    if (x != x) return x + x;
    if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
    if (x < -103.97208404541015625f) return 0.0f;
    float t;
    const float p = expf_poly(x, &t);
    const int ki = __float_as_int(t) - kExpRoundBits;
    const int e1 = ki / 2;
    const int e2 = ki - e1;
    return __fmul_rn(__fmul_rn(p, pow2i(e1)), pow2i(e2));
}

// Same value as msp_expf for x in [-80, 80], where p*2^k is normal: the
// scale is then an exact add of k to p's exponent field (t << 23 leaves
// k << 23, the bits of 1.5*2^23 shifting out).
__device__ __forceinline__ float msp_expf_normal(float x)
{
    float t;
    const float p = expf_poly(x, &t);
    return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

__device__ __forceinline__ float rsqrt_ieee(float x) { return __fdiv_rn(1.0f, __fsqrt_rn(x)); }

// Truncating float->int; saturates and maps NaN to 0.
__device__ __forceinline__ int f2i(float x) { return __float2int_rz(x); }

__device__ __forceinline__ float sigmoid_ref(float x) { return __fdiv_rn(1.f, 1.f + msp_expf(-x)); }

__device__ __forceinline__ float saturatef_ref(float x) { return fminf(fmaxf(x, 0.f), 1.f); }

// Culling of staged Gaussians in the rasterizers.  A pixel only takes a
// Gaussian when sigma lies in [0, 5.55) and alpha = min(0.999, opacity *
// exp(-sigma)) >= 1/255, i.e. sigma <= min(5.55, ln(255 opacity)).  The
// tests below only drop a Gaussian for pixels it provably cannot reach:
// the cut-off gets margins far above float rounding (1e-3 absolute and
// relative, and 1e-5 of the terms' magnitude on sigma), and conics that are
// not positive definite, or NaNs, are always kept.

// Cut-off with margins, or +inf when the Gaussian must be kept.
__device__ __forceinline__ float cull_limit(float4 co)
{
    const float a = co.x, b = co.y, c = co.z;
    if (!(a > 0.f && c > 0.f && a * c - b * b > 0.f)) return 3.0e38f;
    const float cut = fminf(5.55f, __logf(255.f * co.w));
    if (!(cut == cut)) return 3.0e38f;
    return cut + fabsf(cut) * 1e-3f + 1e-3f;
}

// Whether the Gaussian (centre xy, conic co) can reach any pixel centre of
// the w x h rectangle whose first pixel centre is (x0, y0): the least sigma
// over the rectangle of pixel centres (0 if the centre lies inside, else the
// least of the four edge minima, exact for a convex quadratic) against lim.
__device__ __forceinline__ bool rect_may_contribute(float2 xy, float4 co, float x0, float y0,
                                                    float w1, float h1, float lim)
{
    if (lim >= 1.0e38f) return true;
    const float a = co.x, b = co.y, c = co.z;
    const float dxl = xy.x - (x0 + w1), dxh = xy.x - x0;
    const float dyl = xy.y - (y0 + h1), dyh = xy.y - y0;
    if (dxl <= 0.f && dxh >= 0.f && dyl <= 0.f && dyh >= 0.f) return lim >= 0.f;
    const float ia = 1.f / a, ic = 1.f / c;
    float qmin = 3.0e38f;
    auto edge = [&](float dx, float dy) {
        const float t0 = 0.5f * a * dx * dx, t1 = 0.5f * c * dy * dy, t2 = b * dx * dy;
        qmin = fminf(qmin, (t0 + t1 + t2) - 1e-5f * (t0 + t1 + fabsf(t2)));
    };
    edge(dxl, fminf(fmaxf(-b * dxl * ic, dyl), dyh));
    edge(dxh, fminf(fmaxf(-b * dxh * ic, dyl), dyh));
    edge(fminf(fmaxf(-b * dyl * ia, dxl), dxh), dyl);
    edge(fminf(fmaxf(-b * dyh * ia, dxl), dxh), dyh);
    return qmin <= lim;
}

// The 16x16 tile whose first pixel centre is (x0, y0).
__device__ __forceinline__ bool tile_may_contribute(float2 xy, float4 co, float x0, float y0,
                                                    float lim)
{
    return rect_may_contribute(xy, co, x0, y0, 15.f, 15.f, lim);
}

// The 8x8 quadrants of the tile (bit 2*qy + qx) that the Gaussian can reach;
// zero exactly when tile_may_contribute is false.
__device__ __forceinline__ unsigned quadrant_mask(float2 xy, float4 co, float x0, float y0,
                                                  float lim)
{
    if (lim >= 1.0e38f) return 0xfu;
    unsigned m = 0u;
#pragma unroll
    for (int q = 0; q < 4; q++)
        if (rect_may_contribute(xy, co, x0 + 8.f * (q & 1), y0 + 8.f * (q >> 1), 7.f, 7.f, lim))
            m |= 1u << q;
    return m;
}

__device__ __forceinline__ int num_sh_bases(int degree)
{
    return degree == 0 ? 1 : degree == 1 ? 4 : degree == 2 ? 9 : degree == 3 ? 16 : 25;
}

// Reference SH constants (msplat_metal.metal:14-39).
#define MSP_SH_C0 0.28209479177387814f
#define MSP_SH_C1 0.4886025119029199f
__device__ __constant__ static const float kSH_C2[5] = {
    1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
    -1.0925484305920792f, 0.5462742152960396f};
__device__ __constant__ static const float kSH_C3[7] = {
    -0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
    0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
    -0.5900435899266435f};
__device__ __constant__ static const float kSH_C4[9] = {
    2.5033429417967046f, (float)-1.7701307697799304, 0.9461746957575601f,
    -0.6690465435572892f, 0.10578554691520431f, -0.6690465435572892f,
    0.47308734787878004f, -1.7701307697799304f, 0.6258357354491761f};

// SH-rest basis values (degrees 1-3, 15 of them) of the unit direction from
// the camera to mean p: the factors of the rest gradient, g[b][c] =
// basis[b] * v_rgb[c] (msplat_metal.metal:1915-1985).
__device__ __forceinline__ void sh_rest_basis(const float cam[3], const float p[3], float* bs)
{
    const float d0 = p[0] - cam[0], d1 = p[1] - cam[1], d2 = p[2] - cam[2];
    const float dn = rsqrt_ieee((d0 * d0 + d1 * d1) + d2 * d2);
    const float ux = d0 * dn, uy = d1 * dn, uz = d2 * dn;
    const float xx = ux * ux, xy = ux * uy, xz = ux * uz, yy = uy * uy, yz = uy * uz, zz = uz * uz;
    bs[0] = -MSP_SH_C1 * uy;
    bs[1] = MSP_SH_C1 * uz;
    bs[2] = -MSP_SH_C1 * ux;
    bs[3] = kSH_C2[0] * xy;
    bs[4] = kSH_C2[1] * yz;
    bs[5] = kSH_C2[2] * ((2.f * zz - xx) - yy);
    bs[6] = kSH_C2[3] * xz;
    bs[7] = kSH_C2[4] * (xx - yy);
    bs[8] = kSH_C3[0] * uy * (3.f * xx - yy);
    bs[9] = kSH_C3[1] * xy * uz;
    bs[10] = kSH_C3[2] * uy * ((4.f * zz - xx) - yy);
    bs[11] = kSH_C3[3] * uz * ((2.f * zz - 3.f * xx) - 3.f * yy);
    bs[12] = kSH_C3[4] * ux * ((4.f * zz - xx) - yy);
    bs[13] = kSH_C3[5] * uz * (xx - yy);
    bs[14] = kSH_C3[6] * ux * (xx - 3.f * yy);
}

// 1D SSIM window (msplat_metal.metal:3041-3045).
__device__ __constant__ static const float kGauss1D[11] = {
    0.0010283801f, 0.0075987581f, 0.0360007721f, 0.1093606895f, 0.2130055377f,
    0.2660117249f,
    0.2130055377f, 0.1093606895f, 0.0360007721f, 0.0075987581f, 0.0010283801f};
constexpr float kSsimC1 = 0.0001f;
constexpr float kSsimC2 = 0.0009f;

}  // namespace msp
