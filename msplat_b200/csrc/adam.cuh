// adam.cuh -- the Adam update shared by every kernel that applies it.
#pragma once
#include <cuda_runtime.h>

namespace msp {

__device__ __forceinline__ float sqrt_approx(float x)
{
    float r;
    asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// One Adam update (fused_adam_kernel, msplat_metal.metal:1666-1689):
//   m = b1 m + (1 - b1) g;  v = b2 v + (1 - b2) g^2;
//   p -= step * m / (sqrt(v) / bc2 + eps)
// with the square root and the division done by the hardware's approximate
// instructions (a few ulp, as the reference's fast-math Metal build does;
// the parameters' bar is 1e-4 relative).  inv_bc2 = 1 / bc2.
__device__ __forceinline__ void adam_math(float& p, float& m, float& v, float g, float step,
                                          float b1, float b2, float inv_bc2, float eps)
{
    m = fmaf(b1, m, (1.0f - b1) * g);
    v = fmaf(b2, v, (1.0f - b2) * g * g);
    p = p - __fdividef(step * m, fmaf(sqrt_approx(v), inv_bc2, eps));
}

}  // namespace msp
