/*
 * msplat_oracle.c -- CPU restatement of msplat's training step (TEST
 * INFRASTRUCTURE ONLY; see msplat_oracle.h for who may use it).
 *
 * Each function below restates one reference kernel or host routine and
 * cites it as <file>:<lines> within Plinth-it/msplat v1.1.3.  Per-pixel and
 * per-Gaussian loops replace the GPU grid; the SIMD-group reductions and
 * atomics of the backward become sequential sums in double precision.  The
 * warp/threadgroup skipping in rasterize_backward_kernel only skips work that
 * contributes nothing, so it is not restated.
 *
 * Build: gcc -O2 -ffp-contract=off -fopenmp -shared -fPIC (see Makefile).
 */
#include "msplat_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define BLOCK_X 16
#define BLOCK_Y 16
#define CHUNK_SIZE 512

/* ------------------------------------------------------------------------ */
/* Shared scalar maths                                                       */
/* ------------------------------------------------------------------------ */

static float bits_to_float(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t float_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* 2^e for e in [-126, 127], built in the exponent field. */
static float pow2i(int e) { return bits_to_float((uint32_t)(e + 127) << 23); }

/*
 * exp(x): Cody & Waite (1980) argument reduction x = k*ln2 + r with ln2
 * split into a high part with 15 significant bits (k*ln2_hi is exact) and a
 * low part; k = x/ln2 rounded to nearest is read from the low mantissa bits
 * of t = fma(x, log2e, 1.5*2^23).  e^r = 1 + r + r^2 q(r), q the degree-4
 * minimax fit of the relative error on |r| <= ln2/2 (3.1e-9; coefficients
 * from derive_exp_coefficients.py), in Horner form with fmaf; the result is
 * scaled by 2^k in two exact steps so the subnormal range rounds once.
 * Within 0.90 ulp of exp() over every float input.  The CUDA engine
 * evaluates the identical sequence, so both sides produce the same bits.
 */
float msp_expf(float x)
{
    if (x != x) return x + x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541015625f) return 0.0f;
    const float log2e = 1.44269502162933349609375f;   /* nearest float to 1/ln2 */
    const float ln2_hi = 0.693145751953125f;          /* ln2 rounded to 15 bits */
    const float ln2_lo = 1.428606765330187045e-06f;   /* ln2 - ln2_hi */
    const float round_const = 12582912.0f;            /* 1.5 * 2^23 */
    const float t = fmaf(x, log2e, round_const);
    const float k = t - round_const;
    float r = fmaf(-k, ln2_hi, x);
    r = fmaf(-k, ln2_lo, r);
    float p = 0.0013814594130963087f;
    p = fmaf(p, r, 0.0083687193691730499f);
    p = fmaf(p, r, 0.041668388992547989f);
    p = fmaf(p, r, 0.1666652113199234f);
    p = fmaf(p, r, 0.49999994039535522f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    uint32_t tb;
    memcpy(&tb, &t, sizeof tb);
    const int ki = (int)(tb - 0x4B400000u);
    const int e1 = ki / 2;
    const int e2 = ki - e1;
    return (p * pow2i(e1)) * pow2i(e2);
}

static float rsqrt_ieee(float x) { return 1.0f / sqrtf(x); }

/* Truncating float->int with saturation; NaN -> 0. */
static int f2i(float x)
{
    if (x != x) return 0;
    if (x >= 2147483648.0f) return 2147483647;
    if (x <= -2147483648.0f) return (-2147483647 - 1);
    return (int)x;
}

static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

/* Reference SH constants, core/metal/msplat_metal.metal:14-39. */
static const float SH_C0 = 0.28209479177387814f;
static const float SH_C1 = 0.4886025119029199f;
static const float SH_C2[5] = {1.0925484305920792f, -1.0925484305920792f,
                               0.31539156525252005f, -1.0925484305920792f,
                               0.5462742152960396f};
static const float SH_C3[7] = {-0.5900435899266435f, 2.890611442640554f,
                               -0.4570457994644658f, 0.3731763325901154f,
                               -0.4570457994644658f, 1.445305721320277f,
                               -0.5900435899266435f};
static const float SH_C4[9] = {2.5033429417967046f, (float)-1.7701307697799304,
                               0.9461746957575601f, -0.6690465435572892f,
                               0.10578554691520431f, -0.6690465435572892f,
                               0.47308734787878004f, -1.7701307697799304f,
                               0.6258357354491761f};

/* 1D SSIM window, msplat_metal.metal:3041-3045. */
static const float GAUSS_1D[11] = {
    0.0010283801f, 0.0075987581f, 0.0360007721f, 0.1093606895f, 0.2130055377f,
    0.2660117249f,
    0.2130055377f, 0.1093606895f, 0.0360007721f, 0.0075987581f, 0.0010283801f};
#define SSIM_C1 0.0001f
#define SSIM_C2 0.0009f

static int num_sh_bases(int degree)  /* msplat_metal.metal:41-51 */
{
    if (degree == 0) return 1;
    if (degree == 1) return 4;
    if (degree == 2) return 9;
    if (degree == 3) return 16;
    return 25;
}

static float sigmoidf_ref(float x) { return 1.f / (1.f + msp_expf(-x)); }

/* Column-major 3x3: m[c][r], as Metal's float3x3. */
typedef struct { float m[3][3]; } mat3;

static mat3 mat3_mul(mat3 A, mat3 B)
{
    mat3 C;
    for (int c = 0; c < 3; c++)
        for (int r = 0; r < 3; r++)
            C.m[c][r] = (A.m[0][r] * B.m[c][0] + A.m[1][r] * B.m[c][1]) +
                        A.m[2][r] * B.m[c][2];
    return C;
}
static mat3 mat3_t(mat3 A)
{
    mat3 T;
    for (int c = 0; c < 3; c++)
        for (int r = 0; r < 3; r++) T.m[c][r] = A.m[r][c];
    return T;
}
static mat3 mat3_add(mat3 A, mat3 B)
{
    mat3 C;
    for (int c = 0; c < 3; c++)
        for (int r = 0; r < 3; r++) C.m[c][r] = A.m[c][r] + B.m[c][r];
    return C;
}
static mat3 mat3_scale(float s, mat3 A)
{
    mat3 C;
    for (int c = 0; c < 3; c++)
        for (int r = 0; r < 3; r++) C.m[c][r] = s * A.m[c][r];
    return C;
}
static mat3 mat3_cols(float a0, float a1, float a2, float b0, float b1,
                      float b2, float c0, float c1, float c2)
{
    mat3 M;
    M.m[0][0] = a0; M.m[0][1] = a1; M.m[0][2] = a2;
    M.m[1][0] = b0; M.m[1][1] = b1; M.m[1][2] = b2;
    M.m[2][0] = c0; M.m[2][1] = c1; M.m[2][2] = c2;
    return M;
}
static float dot3(const float a[3], const float b[3])
{
    return (a[0] * b[0] + a[1] * b[1]) + a[2] * b[2];
}

/* quat_to_rotmat, msplat_metal.metal:111-131 (memory order w,x,y,z read as
 * float4 fields x,y,z,w). */
static mat3 quat_to_rotmat(const float q[4])
{
    float s = rsqrt_ieee(((q[3] * q[3] + q[0] * q[0]) + q[1] * q[1]) + q[2] * q[2]);
    float w = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
    return mat3_cols(1.f - 2.f * (y * y + z * z), 2.f * (x * y + w * z),
                     2.f * (x * z - w * y), 2.f * (x * y - w * z),
                     1.f - 2.f * (x * x + z * z), 2.f * (y * z + w * x),
                     2.f * (x * z + w * y), 2.f * (y * z - w * x),
                     1.f - 2.f * (x * x + y * y));
}

/* scale_rot_to_cov3d, msplat_metal.metal:147-188.  M = R*S is formed
 * column by column (S diagonal), tmp = M * M^T. */
static void scale_rot_to_cov3d(const float s[3], float glob, const float q[4],
                               float cov[6])
{
    mat3 R = quat_to_rotmat(q);
    mat3 M;
    for (int c = 0; c < 3; c++) {
        float sc = glob * s[c];
        for (int r = 0; r < 3; r++) M.m[c][r] = R.m[c][r] * sc;
    }
    mat3 tmp = mat3_mul(M, mat3_t(M));
    cov[0] = tmp.m[0][0]; cov[1] = tmp.m[0][1]; cov[2] = tmp.m[0][2];
    cov[3] = tmp.m[1][1]; cov[4] = tmp.m[1][2]; cov[5] = tmp.m[2][2];
}

/* transform_4x3 / transform_4x4, msplat_metal.metal:90-108. */
static void transform_4x3(const float *m, const float p[3], float o[3])
{
    o[0] = ((m[0] * p[0] + m[1] * p[1]) + m[2] * p[2]) + m[3];
    o[1] = ((m[4] * p[0] + m[5] * p[1]) + m[6] * p[2]) + m[7];
    o[2] = ((m[8] * p[0] + m[9] * p[1]) + m[10] * p[2]) + m[11];
}
static void transform_4x4(const float *m, const float p[3], float o[4])
{
    transform_4x3(m, p, o);
    o[3] = ((m[12] * p[0] + m[13] * p[1]) + m[14] * p[2]) + m[15];
}

/* project_cov3d_ewa, msplat_metal.metal:192-281. */
static void project_cov3d_ewa(const float cov[6], const float *vm, float fx,
                              float fy, float tan_fovx, float tan_fovy,
                              const float pv_in[3], float out[3])
{
    float pv[3] = {pv_in[0], pv_in[1], pv_in[2]};
    float lim_x = 1.3f * tan_fovx, lim_y = 1.3f * tan_fovy;
    pv[0] = pv[2] * fminf(lim_x, fmaxf(-lim_x, pv[0] / pv[2]));
    pv[1] = pv[2] * fminf(lim_y, fmaxf(-lim_y, pv[1] / pv[2]));
    float rz = 1.f / pv[2];
    float rz2 = rz * rz;
    float j00 = fx * rz, j11 = fy * rz;
    float j20 = (-fx * pv[0]) * rz2, j21 = (-fy * pv[1]) * rz2;
    float t0[3], t1[3];
    for (int k = 0; k < 3; k++) {
        t0[k] = j00 * vm[k] + j20 * vm[8 + k];
        t1[k] = j11 * vm[4 + k] + j21 * vm[8 + k];
    }
    float v00 = cov[0], v01 = cov[1], v02 = cov[2];
    float v11 = cov[3], v12 = cov[4], v22 = cov[5];
    float tv0[3] = {(t0[0] * v00 + t0[1] * v01) + t0[2] * v02,
                    (t0[0] * v01 + t0[1] * v11) + t0[2] * v12,
                    (t0[0] * v02 + t0[1] * v12) + t0[2] * v22};
    float tv1[3] = {(t1[0] * v00 + t1[1] * v01) + t1[2] * v02,
                    (t1[0] * v01 + t1[1] * v11) + t1[2] * v12,
                    (t1[0] * v02 + t1[1] * v12) + t1[2] * v22};
    out[0] = dot3(tv0, t0) + 0.3f;
    out[1] = dot3(tv0, t1);
    out[2] = dot3(tv1, t1) + 0.3f;
}

/* get_bbox / get_tile_bbox, msplat_metal.metal:57-87. */
static void get_tile_bbox(float cx, float cy, float dx, float dy, int tiles_x,
                          int tiles_y, int bmin[2], int bmax[2])
{
    float tcx = cx / (float)BLOCK_X, tcy = cy / (float)BLOCK_Y;
    float trx = dx / (float)BLOCK_X, try_ = dy / (float)BLOCK_Y;
    bmin[0] = imin(imax(0, f2i(tcx - trx)), tiles_x);
    bmax[0] = imin(imax(0, f2i((tcx + trx) + 1)), tiles_x);
    bmin[1] = imin(imax(0, f2i(tcy - try_)), tiles_y);
    bmax[1] = imin(imax(0, f2i((tcy + try_) + 1)), tiles_y);
}

/* sh_coeffs_to_color, msplat_metal.metal:587-654. */
static void sh_to_color(int degree, const float vd[3], const float *dc,
                        const float *rest, float col[3])
{
    for (int c = 0; c < 3; c++) col[c] = SH_C0 * dc[c];
    if (degree < 1) return;
    float x = vd[0], y = vd[1], z = vd[2];
    float xx = x * x, xy = x * y, xz = x * z, yy = y * y, yz = y * z, zz = z * z;
    for (int c = 0; c < 3; c++) {
        const float *r = rest;
        col[c] += SH_C1 * ((-y * r[0 * 3 + c] + z * r[1 * 3 + c]) - x * r[2 * 3 + c]);
        if (degree < 2) continue;
        col[c] += ((((SH_C2[0] * xy * r[3 * 3 + c] + SH_C2[1] * yz * r[4 * 3 + c]) +
                     SH_C2[2] * ((2.f * zz - xx) - yy) * r[5 * 3 + c]) +
                    SH_C2[3] * xz * r[6 * 3 + c]) +
                   SH_C2[4] * (xx - yy) * r[7 * 3 + c]);
        if (degree < 3) continue;
        col[c] += ((((((SH_C3[0] * y * (3.f * xx - yy) * r[8 * 3 + c] +
                        SH_C3[1] * xy * z * r[9 * 3 + c]) +
                       SH_C3[2] * y * ((4.f * zz - xx) - yy) * r[10 * 3 + c]) +
                      SH_C3[3] * z * ((2.f * zz - 3.f * xx) - 3.f * yy) * r[11 * 3 + c]) +
                     SH_C3[4] * x * ((4.f * zz - xx) - yy) * r[12 * 3 + c]) +
                    SH_C3[5] * z * (xx - yy) * r[13 * 3 + c]) +
                   SH_C3[6] * x * (xx - 3.f * yy) * r[14 * 3 + c]);
        if (degree < 4) continue;
        col[c] += ((((((((SH_C4[0] * xy * (xx - yy) * r[15 * 3 + c] +
                          SH_C4[1] * yz * (3.f * xx - yy) * r[16 * 3 + c]) +
                         SH_C4[2] * xy * (7.f * zz - 1.f) * r[17 * 3 + c]) +
                        SH_C4[3] * yz * (7.f * zz - 3.f) * r[18 * 3 + c]) +
                       SH_C4[4] * (zz * (35.f * zz - 30.f) + 3.f) * r[19 * 3 + c]) +
                      SH_C4[5] * xz * (7.f * zz - 3.f) * r[20 * 3 + c]) +
                     SH_C4[6] * (xx - yy) * (7.f * zz - 1.f) * r[21 * 3 + c]) +
                    SH_C4[7] * xz * (xx - 3.f * yy) * r[22 * 3 + c]) +
                   SH_C4[8] * (xx * (xx - 3.f * yy) - yy * (3.f * xx - yy)) * r[23 * 3 + c]);
    }
}

static void normalize3(const float v[3], float o[3])
{
    float s = rsqrt_ieee(dot3(v, v));
    o[0] = v[0] * s; o[1] = v[1] * s; o[2] = v[2] * s;
}

/* ------------------------------------------------------------------------ */

void orc_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* K_max rule, msplat_metal.mm:873-889 (capacity = 16 * num_points, :809). */
int32_t orc_chunk_k_max(int32_t num_points, int32_t num_tiles)
{
    if (num_tiles >= 400) return 1;
    int64_t capacity = (int64_t)num_points * 16;
    uint32_t avg = (uint32_t)(capacity / (num_tiles > 1 ? num_tiles : 1));
    uint32_t cons = avg * 6;
    uint32_t k = (cons + CHUNK_SIZE - 1) / CHUNK_SIZE;
    if (k < 2) k = 2;
    uint32_t abs_max = (uint32_t)((capacity + CHUNK_SIZE - 1) / CHUNK_SIZE);
    if (k > abs_max) k = abs_max;
    return (int32_t)k;
}

/* project_and_sh_forward_kernel, msplat_metal.metal:1695-1787. */
void orc_project_sh_forward(const orc_params *P, const float *means,
                            const float *scales, const float *quats,
                            const float *features_dc, const float *features_rest,
                            orc_state *S)
{
    const int N = P->num_points;
    const int rest_stride = (num_sh_bases(P->degree) - 1) * 3;
#pragma omp parallel for schedule(static)
    for (int i = 0; i < N; i++) {
        S->radii[i] = 0;
        S->num_tiles_hit[i] = 0;
        const float *p = means + 3 * (int64_t)i;
        float pv[3];
        transform_4x3(P->viewmat, p, pv);
        if (pv[2] <= P->clip_thresh) continue;                  /* :134-145 */
        float s[3] = {msp_expf(scales[3 * (int64_t)i]), msp_expf(scales[3 * (int64_t)i + 1]),
                      msp_expf(scales[3 * (int64_t)i + 2])};
        float cov3d[6];
        scale_rot_to_cov3d(s, P->glob_scale, quats + 4 * (int64_t)i, cov3d);
        float tan_fovx = 0.5f * (float)P->img_w / P->fx;
        float tan_fovy = 0.5f * (float)P->img_h / P->fy;
        float cov2d[3];
        project_cov3d_ewa(cov3d, P->viewmat, P->fx, P->fy, tan_fovx, tan_fovy, pv, cov2d);
        /* compute_cov2d_bounds, :283-305 */
        float det = cov2d[0] * cov2d[2] - cov2d[1] * cov2d[1];
        if (det == 0.f) continue;
        float inv_det = 1.f / det;
        float conic[3] = {cov2d[2] * inv_det, -cov2d[1] * inv_det, cov2d[0] * inv_det};
        float b = 0.5f * (cov2d[0] + cov2d[2]);
        float disc = sqrtf(fmaxf(0.1f, b * b - det));
        float radius = ceilf(3.f * sqrtf(b + disc));
        memcpy(S->conics + 3 * (int64_t)i, conic, sizeof(conic));
        /* project_pix, :308-317 */
        float ph[4];
        transform_4x4(P->projmat, p, ph);
        float rw = 1.f / (ph[3] + 1e-6f);
        float ndx = ph[0] * rw, ndy = ph[1] * rw;
        float cx = ((0.5f * (float)P->img_w) * ndx + P->cx) - 0.5f;
        float cy = ((0.5f * (float)P->img_h) * ndy + P->cy) - 0.5f;
        float ax = ceilf(3.0f * sqrtf(cov2d[0]));
        float ay = ceilf(3.0f * sqrtf(cov2d[2]));
        int bmin[2], bmax[2];
        get_tile_bbox(cx, cy, ax, ay, P->tiles_x, P->tiles_y, bmin, bmax);
        int area = (bmax[0] - bmin[0]) * (bmax[1] - bmin[1]);
        if (area <= 0) continue;
        S->num_tiles_hit[i] = area;
        S->depths[i] = pv[2];
        S->radii[i] = f2i(radius);
        S->xys[2 * (int64_t)i] = cx;
        S->xys[2 * (int64_t)i + 1] = cy;
        S->aabb[2 * (int64_t)i] = ax;
        S->aabb[2 * (int64_t)i + 1] = ay;
        float d[3] = {p[0] - P->cam_pos[0], p[1] - P->cam_pos[1], p[2] - P->cam_pos[2]};
        float vd[3];
        normalize3(d, vd);
        sh_to_color(P->degrees_to_use, vd, features_dc + 3 * (int64_t)i,
                    features_rest + (int64_t)rest_stride * i, S->colors + 3 * (int64_t)i);
    }
}

static int cmp_u64(const void *a, const void *b)
{
    uint64_t x = *(const uint64_t *)a, y = *(const uint64_t *)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

/*
 * Tile binning and per-tile sort with the cap removed:
 * scatter_to_prealloc_bins_kernel (msplat_metal.metal:2025-2059), the
 * inclusive prefix_sum_kernel (:2312-2364) and bitonic_sort_per_tile_kernel
 * (:2064-2138).  Key = (float bits of depth << 32) | id, ascending, so ties
 * in depth order by id.  Tile ranges are [start, end).
 */
int orc_bin_and_sort(const orc_params *P, orc_state *S)
{
    const int N = P->num_points;
    const int T = P->tiles_x * P->tiles_y;
    int64_t *count = (int64_t *)calloc((size_t)T + 1, sizeof(int64_t));
    for (int i = 0; i < N; i++) {
        if (S->radii[i] <= 0) continue;
        int bmin[2], bmax[2];
        get_tile_bbox(S->xys[2 * (int64_t)i], S->xys[2 * (int64_t)i + 1], S->aabb[2 * (int64_t)i],
                      S->aabb[2 * (int64_t)i + 1], P->tiles_x, P->tiles_y, bmin, bmax);
        for (int ty = bmin[1]; ty < bmax[1]; ty++)
            for (int tx = bmin[0]; tx < bmax[0]; tx++) count[ty * P->tiles_x + tx]++;
    }
    int64_t total = 0;
    int32_t maxc = 0;
    int64_t *start = (int64_t *)malloc(((size_t)T + 1) * sizeof(int64_t));
    for (int t = 0; t < T; t++) {
        start[t] = total;
        total += count[t];
        if (count[t] > maxc) maxc = (int32_t)count[t];
    }
    start[T] = total;
    S->num_isects = total;
    S->max_tile_count = maxc;
    if (total > S->isect_capacity) {
        free(count); free(start);
        return -1;
    }
    uint64_t *keys = (uint64_t *)malloc((size_t)(total > 0 ? total : 1) * sizeof(uint64_t));
    int64_t *fill = (int64_t *)calloc((size_t)T + 1, sizeof(int64_t));
    for (int i = 0; i < N; i++) {
        if (S->radii[i] <= 0) continue;
        int bmin[2], bmax[2];
        get_tile_bbox(S->xys[2 * (int64_t)i], S->xys[2 * (int64_t)i + 1], S->aabb[2 * (int64_t)i],
                      S->aabb[2 * (int64_t)i + 1], P->tiles_x, P->tiles_y, bmin, bmax);
        uint64_t key = ((uint64_t)float_to_bits(S->depths[i]) << 32) | (uint64_t)(uint32_t)i;
        for (int ty = bmin[1]; ty < bmax[1]; ty++)
            for (int tx = bmin[0]; tx < bmax[0]; tx++) {
                int t = ty * P->tiles_x + tx;
                keys[start[t] + fill[t]++] = key;
            }
    }
#pragma omp parallel for schedule(dynamic, 16)
    for (int t = 0; t < T; t++) {
        qsort(keys + start[t], (size_t)count[t], sizeof(uint64_t), cmp_u64);
    }
    for (int t = 0; t < T; t++) {
        S->tile_bins[2 * t] = (int32_t)start[t];
        S->tile_bins[2 * t + 1] = (int32_t)start[t + 1];
    }
    for (int64_t k = 0; k < total; k++) S->gaussian_ids[k] = (int32_t)(keys[k] & 0xFFFFFFFFu);
    free(keys); free(fill); free(count); free(start);
    return 0;
}

/*
 * One pixel's front-to-back compositing over sorted intersections
 * [beg, end): nd_rasterize_forward_kernel :538-572 and the per-chunk loop of
 * rasterize_forward_chunked_kernel :2711-2731 (identical maths).
 */
static void composite_pixel(const orc_state *S, const float *sig_opac, int beg,
                            int end, float px, float py, float *T_out,
                            float C[3], int *last_out)
{
    float T = 1.f;
    float c0 = 0.f, c1 = 0.f, c2 = 0.f;
    int last = beg - 1;
    for (int idx = beg; idx < end; idx++) {
        int g = S->gaussian_ids[idx];
        const float *cn = S->conics + 3 * (int64_t)g;
        float dx = S->xys[2 * (int64_t)g] - px, dy = S->xys[2 * (int64_t)g + 1] - py;
        float sigma = fmaf(0.5f, fmaf(cn[0], dx * dx, cn[2] * dy * dy), cn[1] * dx * dy);
        if (sigma < 0.f || sigma >= 5.55f) continue;
        float alpha = fminf(0.999f, sig_opac[g] * msp_expf(-sigma));
        if (alpha < 1.f / 255.f) continue;
        float next_T = T * (1.f - alpha);
        if (next_T <= 1e-4f) { last = idx - 1; break; }
        float vis = alpha * T;
        const float *rc = S->colors + 3 * (int64_t)g;
        c0 = fmaf(fmaxf(rc[0] + 0.5f, 0.f), vis, c0);
        c1 = fmaf(fmaxf(rc[1] + 0.5f, 0.f), vis, c1);
        c2 = fmaf(fmaxf(rc[2] + 0.5f, 0.f), vis, c2);
        T = next_T;
        last = idx;
    }
    *T_out = T; C[0] = c0; C[1] = c1; C[2] = c2; *last_out = last;
}

static float saturatef(float x) { return fminf(fmaxf(x, 0.f), 1.f); }

/* Chunk buffers shared by the chunked forward and backward. */
typedef struct {
    int K;
    float *cT, *cC, *pT, *aC;
    int32_t *cidx;
} chunk_bufs;
static chunk_bufs g_chunks;

static void chunks_ensure(int K, int64_t P)
{
    free(g_chunks.cT); free(g_chunks.cC); free(g_chunks.pT); free(g_chunks.aC);
    free(g_chunks.cidx);
    g_chunks.K = K;
    g_chunks.cT = (float *)malloc((size_t)(K * P) * sizeof(float));
    g_chunks.cC = (float *)malloc((size_t)(K * P * 3) * sizeof(float));
    g_chunks.pT = (float *)malloc((size_t)(K * P) * sizeof(float));
    g_chunks.aC = (float *)malloc((size_t)(K * P * 3) * sizeof(float));
    g_chunks.cidx = (int32_t *)malloc((size_t)(K * P) * sizeof(int32_t));
}

static float *sigmoid_all(const orc_params *P, const float *opac)
{
    float *s = (float *)malloc((size_t)(P->num_points > 0 ? P->num_points : 1) * sizeof(float));
#pragma omp parallel for schedule(static)
    for (int i = 0; i < P->num_points; i++) s[i] = sigmoidf_ref(opac[i]);
    return s;
}

/*
 * Forward raster.  k_max == 1: nd_rasterize_forward_kernel (:472-585).
 * k_max > 1: rasterize_forward_chunked_kernel (:2633-2741) followed by
 * rasterize_forward_merge_kernel (:2746-2799), including the merge's
 * absolute 1e-4 cutoff that invalidates later chunks for the backward.
 */
void orc_rasterize_forward(const orc_params *P, const float *opacities, orc_state *S)
{
    const int W = P->img_w, H = P->img_h;
    const int64_t NP = (int64_t)W * H;
    float *so = sigmoid_all(P, opacities);
    const float bg0 = P->background[0], bg1 = P->background[1], bg2 = P->background[2];
    if (P->k_max <= 1) {
#pragma omp parallel for schedule(dynamic, 4)
        for (int i = 0; i < H; i++) {
            for (int j = 0; j < W; j++) {
                int tile = (i / BLOCK_Y) * P->tiles_x + (j / BLOCK_X);
                int beg = S->tile_bins[2 * tile], end = S->tile_bins[2 * tile + 1];
                float T, C[3];
                int last;
                composite_pixel(S, so, beg, end, (float)j, (float)i, &T, C, &last);
                int64_t pix = (int64_t)i * W + j;
                S->final_T[pix] = T;
                S->final_idx[pix] = last;
                S->out_img[3 * pix + 0] = saturatef(fmaf(bg0, T, C[0]));
                S->out_img[3 * pix + 1] = saturatef(fmaf(bg1, T, C[1]));
                S->out_img[3 * pix + 2] = saturatef(fmaf(bg2, T, C[2]));
            }
        }
        free(so);
        return;
    }
    const int K = P->k_max;
    chunks_ensure(K, NP);
#pragma omp parallel for schedule(dynamic, 4)
    for (int i = 0; i < H; i++) {
        for (int j = 0; j < W; j++) {
            int tile = (i / BLOCK_Y) * P->tiles_x + (j / BLOCK_X);
            int fbeg = S->tile_bins[2 * tile], fend = S->tile_bins[2 * tile + 1];
            int64_t pix = (int64_t)i * W + j;
            for (int k = 0; k < K; k++) {
                int cs = fbeg + k * CHUNK_SIZE;
                int ce = imin(fbeg + (k + 1) * CHUNK_SIZE, fend);
                int64_t o = (int64_t)k * NP + pix;
                if (cs >= ce) {
                    g_chunks.cT[o] = 1.f;
                    g_chunks.cC[3 * o] = g_chunks.cC[3 * o + 1] = g_chunks.cC[3 * o + 2] = 0.f;
                    g_chunks.cidx[o] = -1;
                    continue;
                }
                float T, C[3];
                int last;
                composite_pixel(S, so, cs, ce, (float)j, (float)i, &T, C, &last);
                g_chunks.cT[o] = T;
                g_chunks.cC[3 * o] = C[0]; g_chunks.cC[3 * o + 1] = C[1]; g_chunks.cC[3 * o + 2] = C[2];
                g_chunks.cidx[o] = last;
            }
            /* merge, :2764-2798 */
            float Tr = 1.f, R0 = 0.f, R1 = 0.f, R2 = 0.f;
            int last_idx = -1, cutoff = K;
            for (int k = 0; k < K; k++) {
                int64_t o = (int64_t)k * NP + pix;
                int cf = g_chunks.cidx[o];
                if (cf < 0 && k > 0) break;
                float cT = g_chunks.cT[o];
                R0 = fmaf(g_chunks.cC[3 * o], Tr, R0);
                R1 = fmaf(g_chunks.cC[3 * o + 1], Tr, R1);
                R2 = fmaf(g_chunks.cC[3 * o + 2], Tr, R2);
                Tr *= cT;
                if (cf >= 0) last_idx = cf;
                if (Tr <= 1e-4f) { cutoff = k + 1; break; }
            }
            for (int k = cutoff; k < K; k++) g_chunks.cidx[(int64_t)k * NP + pix] = -1;
            S->final_T[pix] = Tr;
            S->final_idx[pix] = last_idx;
            S->out_img[3 * pix + 0] = saturatef(fmaf(bg0, Tr, R0));
            S->out_img[3 * pix + 1] = saturatef(fmaf(bg1, Tr, R1));
            S->out_img[3 * pix + 2] = saturatef(fmaf(bg2, Tr, R2));
        }
    }
    free(so);
}

/*
 * L1 + SSIM loss and its gradient: ssim_h_fwd_kernel (:3053-3115),
 * ssim_fused_v_fwd_h_bwd_kernel (:3226-3313) and ssim_v_bwd_kernel
 * (:3396-3464).  x = gt, y = rendered.  The fused kernel evaluates the
 * derivative fields on the 5 columns either side of every 16-wide
 * threadgroup, including columns outside the image, from zero-padded
 * statistics; those fields are kept here, so pixels within 5 px of the
 * left/right border receive the same extra term as in the reference.
 * The loss is the per-pixel mean of w*(1 - mean_c ssim) + (1-w)*mean_c |x-y|.
 */
void orc_ssim_loss(const orc_params *P, const float *gt, orc_state *S)
{
    const int W = P->img_w, H = P->img_h;
    const float *rd = S->out_img;
    const float w_ssim = P->ssim_weight;
    float *hbuf = (float *)malloc((size_t)W * H * 15 * sizeof(float));
    /* pass 1: horizontal sums */
#pragma omp parallel for schedule(static)
    for (int py = 0; py < H; py++)
        for (int px = 0; px < W; px++)
            for (int c = 0; c < 3; c++) {
                float mx = 0, my = 0, sx = 0, sy = 0, cxy = 0;
                for (int dx = 0; dx < 11; dx++) {
                    float w = GAUSS_1D[dx];
                    int gx = px - 5 + dx;
                    float gv = 0.f, rv = 0.f;
                    if (gx >= 0 && gx < W) {
                        gv = gt[((int64_t)py * W + gx) * 3 + c];
                        rv = rd[((int64_t)py * W + gx) * 3 + c];
                    }
                    mx += w * gv; my += w * rv;
                    sx += w * gv * gv; sy += w * rv * rv; cxy += w * gv * rv;
                }
                float *o = hbuf + ((int64_t)py * W + px) * 15 + c * 5;
                o[0] = mx; o[1] = my; o[2] = sx; o[3] = sy; o[4] = cxy;
            }
    /* pass 2: vertical sums -> fields f1,f2,f3 on columns [-5, W+5) -> horizontal conv */
    const int FW = W + 10;
    float *f = (float *)malloc((size_t)FW * H * 9 * sizeof(float));
    float *dh = (float *)malloc((size_t)W * H * 9 * sizeof(float));
    float *smap = (float *)malloc((size_t)W * H * 3 * sizeof(float));
#pragma omp parallel for schedule(static)
    for (int r = 0; r < H; r++) {
        for (int fc = 0; fc < FW; fc++) {
            int col = fc - 5;
            for (int c = 0; c < 3; c++) {
                float mx = 0, my = 0, sx = 0, sy = 0, cxy = 0;
                for (int k = 0; k < 11; k++) {
                    float w = GAUSS_1D[k];
                    int gy = r - 5 + k;
                    float h0 = 0, h1 = 0, h2 = 0, h3 = 0, h4 = 0;
                    if (col >= 0 && col < W && gy >= 0 && gy < H) {
                        const float *hp = hbuf + ((int64_t)gy * W + col) * 15 + c * 5;
                        h0 = hp[0]; h1 = hp[1]; h2 = hp[2]; h3 = hp[3]; h4 = hp[4];
                    }
                    mx += w * h0; my += w * h1; sx += w * h2; sy += w * h3; cxy += w * h4;
                }
                float sxs = sx - mx * mx, sys = sy - my * my, sxy = cxy - mx * my;
                float A = 2.0f * mx * my + SSIM_C1, B = 2.0f * sxy + SSIM_C2;
                float Cd = (mx * mx + my * my) + SSIM_C1, D = (sxs + sys) + SSIM_C2;
                float iCD = 1.0f / (Cd * D);
                float dmu = 2.0f * B * (mx * Cd - A * my) / (Cd * Cd * D);
                float dsyq = -A * B * iCD / D, dsxy = 2.0f * A * iCD;
                float *fo = f + ((int64_t)r * FW + fc) * 9 + c * 3;
                fo[0] = (dmu - 2.0f * my * dsyq) - mx * dsxy;
                fo[1] = 2.0f * dsyq;
                fo[2] = dsxy;
                if (col >= 0 && col < W) smap[((int64_t)r * W + col) * 3 + c] = (A * B) / (Cd * D);
            }
        }
    }
    double loss_total = 0.0;
    for (int r = 0; r < H; r++)
        for (int col = 0; col < W; col++) {
            double ss = 0.0, ll = 0.0;
            for (int c = 0; c < 3; c++) {
                int64_t q = ((int64_t)r * W + col) * 3 + c;
                ss += (double)smap[q];
                ll += fabs((double)gt[q] - (double)rd[q]);
            }
            loss_total += (double)w_ssim * (1.0 - ss / 3.0) + (1.0 - (double)w_ssim) * ll / 3.0;
        }
    free(smap);
    S->loss = loss_total / ((double)W * H);
    /* horizontal backward conv with reversed taps */
#pragma omp parallel for schedule(static)
    for (int r = 0; r < H; r++)
        for (int px = 0; px < W; px++)
            for (int c = 0; c < 3; c++) {
                float a1 = 0, a2 = 0, a3 = 0;
                for (int dx = 0; dx < 11; dx++) {
                    float w = GAUSS_1D[10 - dx];
                    const float *fo = f + ((int64_t)r * FW + (px + dx)) * 9 + c * 3;
                    a1 += w * fo[0]; a2 += w * fo[1]; a3 += w * fo[2];
                }
                float *o = dh + ((int64_t)r * W + px) * 9 + c * 3;
                o[0] = a1; o[1] = a2; o[2] = a3;
            }
    /* pass 3: vertical backward conv, combine with L1 sign */
    const float inv_n = P->loss_inv_n;
#pragma omp parallel for schedule(static)
    for (int py = 0; py < H; py++)
        for (int px = 0; px < W; px++)
            for (int c = 0; c < 3; c++) {
                float c1 = 0, c2 = 0, c3 = 0;
                for (int dy = 0; dy < 11; dy++) {
                    float w = GAUSS_1D[10 - dy];
                    int gy = py - 5 + dy;
                    float v1 = 0, v2 = 0, v3 = 0;
                    if (gy >= 0 && gy < H) {
                        const float *o = dh + ((int64_t)gy * W + px) * 9 + c * 3;
                        v1 = o[0]; v2 = o[1]; v3 = o[2];
                    }
                    c1 += w * v1; c2 += w * v2; c3 += w * v3;
                }
                int64_t q = ((int64_t)py * W + px) * 3 + c;
                float rv = rd[q], gv = gt[q];
                float v_ssim = (c1 + rv * c2) + gv * c3;
                float v_l1 = (gv > rv) ? -1.0f : ((gv < rv) ? 1.0f : 0.0f);
                S->v_rendered[q] = inv_n * (-w_ssim * v_ssim + (1.0f - w_ssim) * v_l1);
            }
    free(hbuf); free(f); free(dh);
}

/* Double-precision accumulation target of the backward. */
static void atomic_addd(double *p, double v)
{
#pragma omp atomic
    *p += v;
}

/*
 * One pixel's back-to-front replay over [beg, bin_final]:
 * rasterize_backward_kernel :975-1098 (monolithic, T0 = final T, buffer 0)
 * and rasterize_backward_chunked_kernel :2934-3030 (chunked, T0 and buffer
 * from the prefix/suffix pass).  Only alpha < 0.999 contributes (:1049).
 */
static void backprop_pixel(const orc_state *S, const float *so, int beg,
                           int bin_final, float px, float py, float T,
                           float b0, float b1, float b2, const float Tfb[3],
                           const float vo[3], double *acc)
{
    for (int idx = bin_final; idx >= beg; idx--) {
        int g = S->gaussian_ids[idx];
        const float *cn = S->conics + 3 * (int64_t)g;
        float op = so[g];
        float dx = S->xys[2 * (int64_t)g] - px, dy = S->xys[2 * (int64_t)g + 1] - py;
        float sigma = fmaf(0.5f, fmaf(cn[0], dx * dx, cn[2] * dy * dy), cn[1] * dx * dy);
        if (sigma < 0.f || sigma >= 5.55f) continue;
        float vis = msp_expf(-sigma);
        float alpha = fminf(0.999f, op * vis);
        if (alpha < 1.f / 255.f) continue;
        if (!(alpha < 0.999f)) continue;
        float ra = 1.f / (1.f - alpha);
        T *= ra;
        float fac = alpha * T;
        const float *raw = S->colors + 3 * (int64_t)g;
        float rgb0 = fmaxf(raw[0] + 0.5f, 0.f), rgb1 = fmaxf(raw[1] + 0.5f, 0.f),
              rgb2 = fmaxf(raw[2] + 0.5f, 0.f);
        float nra = -ra;
        float e0 = fmaf(rgb0, T, fmaf(-b0, ra, nra * Tfb[0]));
        float e1 = fmaf(rgb1, T, fmaf(-b1, ra, nra * Tfb[1]));
        float e2 = fmaf(rgb2, T, fmaf(-b2, ra, nra * Tfb[2]));
        float v_alpha = (e0 * vo[0] + e1 * vo[1]) + e2 * vo[2];
        b0 = fmaf(rgb0, fac, b0); b1 = fmaf(rgb1, fac, b1); b2 = fmaf(rgb2, fac, b2);
        float v_sigma = -alpha * v_alpha;
        double *a = acc + 9 * (int64_t)g;
        if (raw[0] + 0.5f >= 0.f) atomic_addd(&a[0], (double)(fac * vo[0]));
        if (raw[1] + 0.5f >= 0.f) atomic_addd(&a[1], (double)(fac * vo[1]));
        if (raw[2] + 0.5f >= 0.f) atomic_addd(&a[2], (double)(fac * vo[2]));
        float hv = 0.5f * v_sigma;
        atomic_addd(&a[3], (double)(hv * (dx * dx)));
        atomic_addd(&a[4], (double)(hv * (dx * dy)));
        atomic_addd(&a[5], (double)(hv * (dy * dy)));
        atomic_addd(&a[6], (double)(v_sigma * fmaf(cn[0], dx, cn[1] * dy)));
        atomic_addd(&a[7], (double)(v_sigma * fmaf(cn[1], dx, cn[2] * dy)));
        atomic_addd(&a[8], (double)(-v_sigma * (1.f - op)));
    }
}

/*
 * Backward raster.  k_max == 1: rasterize_backward_kernel (:898-1099).
 * k_max > 1: compute_chunk_prefix_suffix_kernel (:2804-2840) then
 * rasterize_backward_chunked_kernel (:2844-3031).
 */
void orc_rasterize_backward(const orc_params *P, const float *opacities, orc_state *S)
{
    const int W = P->img_w, H = P->img_h, N = P->num_points;
    const int64_t NP = (int64_t)W * H;
    float *so = sigmoid_all(P, opacities);
    double *acc = (double *)calloc((size_t)(N > 0 ? N : 1) * 9, sizeof(double));
    const float *bg = P->background;
    if (P->k_max <= 1) {
#pragma omp parallel for schedule(dynamic, 4)
        for (int i = 0; i < H; i++)
            for (int j = 0; j < W; j++) {
                int tile = (i / BLOCK_Y) * P->tiles_x + (j / BLOCK_X);
                int beg = S->tile_bins[2 * tile];
                int64_t pix = (int64_t)i * W + j;
                float Tf = S->final_T[pix];
                float Tfb[3] = {Tf * bg[0], Tf * bg[1], Tf * bg[2]};
                const float *vo = S->v_rendered + 3 * pix;
                backprop_pixel(S, so, beg, S->final_idx[pix], (float)j, (float)i, Tf,
                               0.f, 0.f, 0.f, Tfb, vo, acc);
            }
    } else {
        const int K = P->k_max;
#pragma omp parallel for schedule(static)
        for (int64_t pix = 0; pix < NP; pix++) {
            float pTv = 1.f;
            for (int k = 0; k < K; k++) {
                int64_t o = (int64_t)k * NP + pix;
                g_chunks.pT[o] = pTv;
                pTv *= g_chunks.cT[o];
            }
            float a0 = 0.f, a1 = 0.f, a2 = 0.f;
            for (int k = K - 1; k >= 0; k--) {
                int64_t o = (int64_t)k * NP + pix;
                g_chunks.aC[3 * o] = a0; g_chunks.aC[3 * o + 1] = a1; g_chunks.aC[3 * o + 2] = a2;
                float pk = g_chunks.pT[o];
                a0 += pk * g_chunks.cC[3 * o];
                a1 += pk * g_chunks.cC[3 * o + 1];
                a2 += pk * g_chunks.cC[3 * o + 2];
            }
        }
#pragma omp parallel for schedule(dynamic, 4)
        for (int i = 0; i < H; i++)
            for (int j = 0; j < W; j++) {
                int tile = (i / BLOCK_Y) * P->tiles_x + (j / BLOCK_X);
                int fbeg = S->tile_bins[2 * tile], fend = S->tile_bins[2 * tile + 1];
                int64_t pix = (int64_t)i * W + j;
                float Tf = S->final_T[pix];
                float Tfb[3] = {Tf * bg[0], Tf * bg[1], Tf * bg[2]};
                const float *vo = S->v_rendered + 3 * pix;
                for (int k = 0; k < K; k++) {
                    int cs = fbeg + k * CHUNK_SIZE;
                    int ce = imin(fbeg + (k + 1) * CHUNK_SIZE, fend);
                    int64_t o = (int64_t)k * NP + pix;
                    int bf = g_chunks.cidx[o];
                    if (cs >= ce || bf < cs) continue;
                    float T0 = g_chunks.pT[o] * g_chunks.cT[o];
                    backprop_pixel(S, so, cs, bf, (float)j, (float)i, T0, g_chunks.aC[3 * o],
                                   g_chunks.aC[3 * o + 1], g_chunks.aC[3 * o + 2], Tfb, vo, acc);
                }
            }
    }
    for (int g = 0; g < N; g++) {
        const double *a = acc + 9 * (int64_t)g;
        S->v_rgb[3 * (int64_t)g + 0] = (float)a[0];
        S->v_rgb[3 * (int64_t)g + 1] = (float)a[1];
        S->v_rgb[3 * (int64_t)g + 2] = (float)a[2];
        S->v_conic[3 * (int64_t)g + 0] = (float)a[3];
        S->v_conic[3 * (int64_t)g + 1] = (float)a[4];
        S->v_conic[3 * (int64_t)g + 2] = (float)a[5];
        S->v_xy[2 * (int64_t)g + 0] = (float)a[6];
        S->v_xy[2 * (int64_t)g + 1] = (float)a[7];
        S->v_opacity[g] = (float)a[8];
    }
    free(acc);
    free(so);
}

/* quat_to_rotmat_vjp, msplat_metal.metal:1409-1452 (v_R column-major). */
static void quat_to_rotmat_vjp(const float q[4], mat3 vR, float vq[4])
{
    float s = rsqrt_ieee(((q[3] * q[3] + q[0] * q[0]) + q[1] * q[1]) + q[2] * q[2]);
    float w = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
    float (*v)[3] = vR.m;
    vq[0] = 2.f * ((x * (v[1][2] - v[2][1]) + y * (v[2][0] - v[0][2])) + z * (v[0][1] - v[1][0]));
    vq[1] = 2.f * (((-2.f * x * (v[1][1] + v[2][2]) + y * (v[0][1] + v[1][0])) +
                    z * (v[0][2] + v[2][0])) + w * (v[1][2] - v[2][1]));
    vq[2] = 2.f * (((x * (v[0][1] + v[1][0]) - 2.f * y * (v[0][0] + v[2][2])) +
                    z * (v[1][2] + v[2][1])) + w * (v[2][0] - v[0][2]));
    vq[3] = 2.f * (((x * (v[0][2] + v[2][0]) + y * (v[1][2] + v[2][1])) -
                    2.f * z * (v[0][0] + v[1][1])) + w * (v[0][1] - v[1][0]));
}

/* adam_update_element, msplat_metal.metal:1791-1800 (also fused_adam_kernel :1666-1689). */
static void adam_elem(float *p, float *ea, float *eas, float g, float step,
                      float b1, float b2, float bc2, float eps)
{
    float m = fmaf(b1, *ea, (1.0f - b1) * g);
    float v = fmaf(b2, *eas, (1.0f - b2) * g * g);
    *p -= step * m / (sqrtf(v) / bc2 + eps);
    *ea = m;
    *eas = v;
}

/*
 * project_and_sh_backward_kernel, msplat_metal.metal:1813-1986, with the
 * VJPs project_pix_vjp (:1216-1234), cov2d_to_conic_vjp (:1253-1264),
 * project_cov3d_ewa_vjp (:1339-1407), scale_rot_to_cov3d_vjp (:1498-1531)
 * and the in-place SH Adam for visible Gaussians.
 */
void orc_project_sh_backward_adam(const orc_params *P, const float *means,
                                  const float *scales, const float *quats,
                                  float *features_dc, float *features_rest,
                                  float *dc_ea, float *dc_eas, float *rest_ea,
                                  float *rest_eas, orc_state *S)
{
    const int N = P->num_points;
    const int rest_stride = (num_sh_bases(P->degree) - 1) * 3;
    const float *vm = P->viewmat, *pm = P->projmat;
    memset(S->v_mean3d, 0, sizeof(float) * 3 * (size_t)N);
    memset(S->v_scale, 0, sizeof(float) * 3 * (size_t)N);
    memset(S->v_quat, 0, sizeof(float) * 4 * (size_t)N);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < N; i++) {
        if (S->radii[i] <= 0) continue;
        const float *p = means + 3 * (int64_t)i;
        float fx = P->fx, fy = P->fy;
        /* project_pix_vjp */
        float ph[4];
        transform_4x4(pm, p, ph);
        float rw = 1.f / (ph[3] + 1e-6f);
        float vxy0 = S->v_xy[2 * (int64_t)i], vxy1 = S->v_xy[2 * (int64_t)i + 1];
        float vnx = (0.5f * (float)P->img_w) * vxy0, vny = (0.5f * (float)P->img_h) * vxy1;
        float vp0 = vnx * rw, vp1 = vny * rw, vp2 = 0.f;
        float vmean[3];
        vmean[0] = (pm[0] * vp0 + pm[4] * vp1) + pm[8] * vp2;
        vmean[1] = (pm[1] * vp0 + pm[5] * vp1) + pm[9] * vp2;
        vmean[2] = (pm[2] * vp0 + pm[6] * vp1) + pm[10] * vp2;
        /* v_depth is never written (always 0), :1860-1864 */
        vmean[0] = vmean[0] + vm[8] * 0.f;
        vmean[1] = vmean[1] + vm[9] * 0.f;
        vmean[2] = vmean[2] + vm[10] * 0.f;
        /* cov2d_to_conic_vjp: v_Sigma = ((-1*X)*G)*X */
        const float *cn = S->conics + 3 * (int64_t)i;
        const float *vc = S->v_conic + 3 * (int64_t)i;
        float X[2][2] = {{-cn[0], -cn[1]}, {-cn[1], -cn[2]}};
        float G[2][2] = {{vc[0], vc[1]}, {vc[1], vc[2]}};
        float XG[2][2], VS[2][2];
        for (int c = 0; c < 2; c++)
            for (int r = 0; r < 2; r++) XG[c][r] = X[0][r] * G[c][0] + X[1][r] * G[c][1];
        float Xp[2][2] = {{cn[0], cn[1]}, {cn[1], cn[2]}};
        for (int c = 0; c < 2; c++)
            for (int r = 0; r < 2; r++) VS[c][r] = XG[0][r] * Xp[c][0] + XG[1][r] * Xp[c][1];
        float vcov2d[3] = {VS[0][0], VS[1][0] + VS[0][1], VS[1][1]};
        /* recompute cov3d */
        float es[3] = {msp_expf(scales[3 * (int64_t)i]), msp_expf(scales[3 * (int64_t)i + 1]),
                       msp_expf(scales[3 * (int64_t)i + 2])};
        const float *q = quats + 4 * (int64_t)i;
        float cov3d[6];
        scale_rot_to_cov3d(es, P->glob_scale, q, cov3d);
        float tan_fovx = 0.5f * (float)P->img_w / fx, tan_fovy = 0.5f * (float)P->img_h / fy;
        float pv[3];
        transform_4x3(vm, p, pv);
        /* project_cov3d_ewa_vjp */
        float lim_x = 1.3f * tan_fovx, lim_y = 1.3f * tan_fovy;
        pv[0] = pv[2] * fminf(lim_x, fmaxf(-lim_x, pv[0] / pv[2]));
        pv[1] = pv[2] * fminf(lim_y, fmaxf(-lim_y, pv[1] / pv[2]));
        float rz = 1.f / pv[2], rz2 = rz * rz;
        mat3 Wm = mat3_cols(vm[0], vm[4], vm[8], vm[1], vm[5], vm[9], vm[2], vm[6], vm[10]);
        mat3 J = mat3_cols(fx * rz, 0.f, 0.f, 0.f, fy * rz, 0.f, (-fx * pv[0]) * rz2,
                           (-fy * pv[1]) * rz2, 0.f);
        mat3 V = mat3_cols(cov3d[0], cov3d[1], cov3d[2], cov3d[1], cov3d[3], cov3d[4],
                           cov3d[2], cov3d[4], cov3d[5]);
        mat3 vcov = mat3_cols(vcov2d[0], 0.5f * vcov2d[1], 0.f, 0.5f * vcov2d[1], vcov2d[2],
                              0.f, 0.f, 0.f, 0.f);
        mat3 T = mat3_mul(J, Wm);
        mat3 Tt = mat3_t(T), Vt = mat3_t(V);
        mat3 vV = mat3_mul(mat3_mul(Tt, vcov), T);
        mat3 vT = mat3_add(mat3_mul(mat3_mul(vcov, T), Vt),
                           mat3_mul(mat3_mul(mat3_t(vcov), T), V));
        float vcov3d[6] = {vV.m[0][0], vV.m[0][1] + vV.m[1][0], vV.m[0][2] + vV.m[2][0],
                           vV.m[1][1], vV.m[1][2] + vV.m[2][1], vV.m[2][2]};
        mat3 vJ = mat3_mul(vT, mat3_t(Wm));
        float fx_rz2 = fx * rz2, fy_rz2 = fy * rz2, rz3 = rz2 * rz;
        float vt[3];
        vt[0] = -fx_rz2 * vJ.m[2][0];
        vt[1] = -fy_rz2 * vJ.m[2][1];
        vt[2] = ((-fx_rz2 * vJ.m[0][0] + 2.f * fx * pv[0] * rz3 * vJ.m[2][0]) -
                 fy_rz2 * vJ.m[1][1]) + 2.f * fy * pv[1] * rz3 * vJ.m[2][1];
        for (int k = 0; k < 3; k++) vmean[k] += dot3(vt, Wm.m[k]);
        /* scale_rot_to_cov3d_vjp */
        mat3 vVs = mat3_cols(vcov3d[0], 0.5f * vcov3d[1], 0.5f * vcov3d[2], 0.5f * vcov3d[1],
                             vcov3d[3], 0.5f * vcov3d[4], 0.5f * vcov3d[2], 0.5f * vcov3d[4],
                             vcov3d[5]);
        mat3 R = quat_to_rotmat(q);
        mat3 Sm = mat3_cols(P->glob_scale * es[0], 0.f, 0.f, 0.f, P->glob_scale * es[1], 0.f,
                            0.f, 0.f, P->glob_scale * es[2]);
        mat3 M = mat3_mul(R, Sm);
        mat3 vM = mat3_mul(mat3_scale(2.f, vVs), M);
        float vs[3];
        for (int k = 0; k < 3; k++) vs[k] = dot3(R.m[k], vM.m[k]);
        mat3 vR = mat3_mul(vM, Sm);
        float vq[4];
        quat_to_rotmat_vjp(q, vR, vq);
        for (int k = 0; k < 3; k++) {
            S->v_mean3d[3 * (int64_t)i + k] = vmean[k];
            S->v_scale[3 * (int64_t)i + k] = vs[k] * es[k];
        }
        for (int k = 0; k < 4; k++) S->v_quat[4 * (int64_t)i + k] = vq[k];

        /* fused SH backward + Adam (groups 3 and 4) */
        float d[3] = {p[0] - P->cam_pos[0], p[1] - P->cam_pos[1], p[2] - P->cam_pos[2]};
        float vd[3];
        normalize3(d, vd);
        const float *vcol = S->v_rgb + 3 * (int64_t)i;
        const float b1 = P->beta1, b2 = P->beta2, eps = P->eps;
        for (int c = 0; c < 3; c++) {
            int64_t e = 3 * (int64_t)i + c;
            adam_elem(&features_dc[e], &dc_ea[e], &dc_eas[e], SH_C0 * vcol[c],
                      P->adam_step_size[3], b1, b2, P->adam_bc2_sqrt[3], eps);
        }
        if (P->degrees_to_use < 1) continue;
        float x = vd[0], y = vd[1], z = vd[2];
        float xx = x * x, xy = x * y, xz = x * z, yy = y * y, yz = y * z, zz = z * z;
        float basis[15];
        basis[0] = -SH_C1 * y; basis[1] = SH_C1 * z; basis[2] = -SH_C1 * x;
        basis[3] = SH_C2[0] * xy; basis[4] = SH_C2[1] * yz;
        basis[5] = SH_C2[2] * ((2.f * zz - xx) - yy);
        basis[6] = SH_C2[3] * xz; basis[7] = SH_C2[4] * (xx - yy);
        basis[8] = SH_C3[0] * y * (3.f * xx - yy);
        basis[9] = SH_C3[1] * xy * z;
        basis[10] = SH_C3[2] * y * ((4.f * zz - xx) - yy);
        basis[11] = SH_C3[3] * z * ((2.f * zz - 3.f * xx) - 3.f * yy);
        basis[12] = SH_C3[4] * x * ((4.f * zz - xx) - yy);
        basis[13] = SH_C3[5] * z * (xx - yy);
        basis[14] = SH_C3[6] * x * (xx - 3.f * yy);
        int nb = P->degrees_to_use >= 3 ? 15 : (P->degrees_to_use == 2 ? 8 : 3);
        for (int bb = 0; bb < nb; bb++)
            for (int c = 0; c < 3; c++) {
                int64_t e = (int64_t)rest_stride * i + bb * 3 + c;
                adam_elem(&features_rest[e], &rest_ea[e], &rest_eas[e], basis[bb] * vcol[c],
                          P->adam_step_size[4], b1, b2, P->adam_bc2_sqrt[4], eps);
            }
    }
}

/* fused_adam_kernel, msplat_metal.metal:1666-1689. */
void orc_fused_adam(float *params, const float *grads, float *exp_avg,
                    float *exp_avg_sq, float step_size, float beta1,
                    float beta2, float bc2_sqrt, float eps, int64_t n)
{
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < n; t++)
        adam_elem(&params[t], &exp_avg[t], &exp_avg_sq[t], grads[t], step_size, beta1,
                  beta2, bc2_sqrt, eps);
}

/* accumulate_grad_stats_kernel, msplat_metal.metal:1643-1664. */
void orc_grad_stats(const orc_params *P, const orc_state *S, float *vis_counts,
                    float *xys_grad_norm, float *max_2d_size)
{
#pragma omp parallel for schedule(static)
    for (int i = 0; i < P->num_points; i++) {
        if (S->radii[i] <= 0) continue;
        vis_counts[i] += 1.0f;
        float gx = S->v_xy[2 * (int64_t)i], gy = S->v_xy[2 * (int64_t)i + 1];
        xys_grad_norm[i] += sqrtf(gx * gx + gy * gy);
        float r = (float)S->radii[i] * P->inv_max_dim;
        max_2d_size[i] = fmaxf(max_2d_size[i], r);
    }
}

/*
 * msplat_train_step, msplat_metal.mm:771-1330: forward, fused loss,
 * backward raster, projection backward with SH Adam, Adam for groups
 * 0,1,2,5 over every element, then the densification statistics.
 */
int orc_train_step(const orc_params *P, orc_state *S, float *params[6],
                   float *exp_avg[6], float *exp_avg_sq[6], const float *gt,
                   float *vis_counts, float *xys_grad_norm, float *max_2d_size)
{
    const int N = P->num_points;
    orc_project_sh_forward(P, params[0], params[1], params[2], params[3], params[4], S);
    if (orc_bin_and_sort(P, S) != 0) return -1;
    orc_rasterize_forward(P, params[5], S);
    orc_ssim_loss(P, gt, S);
    orc_rasterize_backward(P, params[5], S);
    orc_project_sh_backward_adam(P, params[0], params[1], params[2], params[3], params[4],
                                 exp_avg[3], exp_avg_sq[3], exp_avg[4], exp_avg_sq[4], S);
    const float *grads[6] = {S->v_mean3d, S->v_scale, S->v_quat, NULL, NULL, S->v_opacity};
    const int64_t sizes[6] = {3 * (int64_t)N, 3 * (int64_t)N, 4 * (int64_t)N, 0, 0, (int64_t)N};
    for (int g = 0; g < 6; g++) {
        if (g == 3 || g == 4) continue;
        orc_fused_adam(params[g], grads[g], exp_avg[g], exp_avg_sq[g], P->adam_step_size[g],
                       P->beta1, P->beta2, P->adam_bc2_sqrt[g], P->eps, sizes[g]);
    }
    orc_grad_stats(P, S, vis_counts, xys_grad_norm, max_2d_size);
    return 0;
}

/* msplat_render / forward_pipeline(compute_loss=false), msplat_metal.mm:752-769. */
int orc_render(const orc_params *P, orc_state *S, const float *params[6])
{
    orc_project_sh_forward(P, params[0], params[1], params[2], params[3], params[4], S);
    if (orc_bin_and_sort(P, S) != 0) return -1;
    orc_rasterize_forward(P, params[5], S);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Densification                                                             */
/* ------------------------------------------------------------------------ */

/*
 * msplat_densify (core/metal/msplat_metal.mm:1337-1592) with its kernels
 * restated in stage order: densify_classify_kernel (msplat_metal.metal:
 * 3475-3509), inclusive prefix sums of the split and duplicate flags
 * (block_reduce_kernel / block_scan_propagate_kernel :2368-2439),
 * densify_append_split_kernel (:3514-3600), densify_append_dup_kernel
 * (:3604-3651), densify_cull_classify_kernel (:3656-3694) over 3N slots, the
 * keep prefix sum and the stable compaction of the 18 buffers
 * (compact_scatter_kernel / compact_copy_back_kernel :3698-3729).
 * bufs / exp_avg / exp_avg_sq: group order means, scales, quats,
 * features_dc, features_rest (fr_stride floats per Gaussian), opacities, each
 * with room for 3N rows.  random_samples: [2N, 3] standard normals, child k
 * of the split with ordinal o takes row 2o + k.  The flag dumps may be NULL.
 * Returns the new count, or -1 when 3N exceeds buf_capacity.
 */
int orc_densify(int N, int buf_capacity, float grad_thresh, float size_thresh,
                float screen_thresh, int check_screen, float cull_alpha_thresh,
                float cull_scale_thresh, float cull_screen_size, int check_huge,
                const float *xys_grad_norm, const float *vis_counts, const float *max_2d_size,
                float half_max_dim, float *bufs[6], int fr_stride, float *exp_avg[6],
                float *exp_avg_sq[6], const float *random_samples, int *split_flag_out,
                int *dup_flag_out, int *keep_flag_out)
{
    const int worst = 3 * N;
    if (worst > buf_capacity) return -1;
    const int strides[6] = {3, 3, 4, 3, fr_stride, 1};
    const float log_size_fac = logf(1.6f);
    int *split = (int *)calloc((size_t)(N > 0 ? N : 1), sizeof(int));
    int *dup = (int *)calloc((size_t)(N > 0 ? N : 1), sizeof(int));
    int *keep = (int *)calloc((size_t)(worst > 0 ? worst : 1), sizeof(int));
    /* classify (:3475-3509) */
    for (int i = 0; i < N; i++) {
        const float vc = vis_counts[i];
        if (vc <= 0.0f) continue;
        const float avg_grad = (xys_grad_norm[i] / vc) * half_max_dim;
        const int high_grad = avg_grad > grad_thresh;
        const float *s = bufs[1] + 3 * (size_t)i;
        const float max_scale = fmaxf(fmaxf(msp_expf(s[0]), msp_expf(s[1])), msp_expf(s[2]));
        const int is_large = max_scale > size_thresh;
        int do_split = is_large;
        if (check_screen && max_2d_size[i] > screen_thresh) do_split = 1;
        split[i] = do_split && high_grad;
        dup[i] = !is_large && high_grad;
    }
    int n_split = 0, n_dup = 0;
    int *split_ord = (int *)calloc((size_t)(N > 0 ? N : 1), sizeof(int));
    int *dup_ord = (int *)calloc((size_t)(N > 0 ? N : 1), sizeof(int));
    for (int i = 0; i < N; i++) {
        split_ord[i] = n_split;
        n_split += split[i];
        dup_ord[i] = n_dup;
        n_dup += dup[i];
    }
    /* split children (:3514-3600): child k at N + 2*ord + k */
    for (int i = 0; i < N; i++) {
        if (!split[i]) continue;
        const int ord = split_ord[i];
        float *q = bufs[2] + 4 * (size_t)i;
        float qw = q[0], qx = q[1], qy = q[2], qz = q[3];
        const float qlen = sqrtf(((qw * qw + qx * qx) + qy * qy) + qz * qz);
        qw /= qlen; qx /= qlen; qy /= qlen; qz /= qlen;
        float *sp = bufs[1] + 3 * (size_t)i;
        const float sx = msp_expf(sp[0]), sy = msp_expf(sp[1]), sz = msp_expf(sp[2]);
        for (int k = 0; k < 2; k++) {
            const size_t child = (size_t)N + 2 * (size_t)ord + k;
            const float *rs = random_samples + 3 * (size_t)(ord * 2 + k);
            const float r0 = rs[0] * sx, r1 = rs[1] * sy, r2 = rs[2] * sz;
            const float v0 = ((1.f - 2.f * (qy * qy + qz * qz)) * r0 + 2.f * (qx * qy - qw * qz) * r1) +
                             2.f * (qx * qz + qw * qy) * r2;
            const float v1 = (2.f * (qx * qy + qw * qz) * r0 + (1.f - 2.f * (qx * qx + qz * qz)) * r1) +
                             2.f * (qy * qz - qw * qx) * r2;
            const float v2 = (2.f * (qx * qz - qw * qy) * r0 + 2.f * (qy * qz + qw * qx) * r1) +
                             (1.f - 2.f * (qx * qx + qy * qy)) * r2;
            float *pm = bufs[0];
            pm[child * 3] = pm[(size_t)i * 3] + v0;
            pm[child * 3 + 1] = pm[(size_t)i * 3 + 1] + v1;
            pm[child * 3 + 2] = pm[(size_t)i * 3 + 2] + v2;
            for (int j = 0; j < 3; j++) bufs[1][child * 3 + j] = sp[j] - log_size_fac;
            for (int j = 0; j < 4; j++) bufs[2][child * 4 + j] = q[j];
            for (int j = 0; j < 3; j++) bufs[3][child * 3 + j] = bufs[3][(size_t)i * 3 + j];
            for (int j = 0; j < fr_stride; j++)
                bufs[4][child * fr_stride + j] = bufs[4][(size_t)i * fr_stride + j];
            bufs[5][child] = bufs[5][i];
            for (int g = 0; g < 6; g++)
                for (int j = 0; j < strides[g]; j++) {
                    exp_avg[g][child * strides[g] + j] = 0.f;
                    exp_avg_sq[g][child * strides[g] + j] = 0.f;
                }
        }
        for (int j = 0; j < 3; j++) sp[j] -= log_size_fac;
    }
    /* duplicates (:3604-3651): at N + 2*nSplits + ord, copied after the split
     * stage (a parent that also splits is copied with its shrunk scale) */
    for (int i = 0; i < N; i++) {
        if (!dup[i]) continue;
        const size_t dst = (size_t)N + 2 * (size_t)n_split + dup_ord[i];
        for (int g = 0; g < 6; g++)
            for (int j = 0; j < strides[g]; j++) {
                bufs[g][dst * strides[g] + j] = bufs[g][(size_t)i * strides[g] + j];
                exp_avg[g][dst * strides[g] + j] = 0.f;
                exp_avg_sq[g][dst * strides[g] + j] = 0.f;
            }
    }
    /* cull classification over the grown population (:3656-3694) */
    const int n_new = N + 2 * n_split + n_dup;
    for (int i = 0; i < n_new; i++) {
        const float op = sigmoidf_ref(bufs[5][i]);
        int cull = op < cull_alpha_thresh;
        if (i < N && split[i]) cull = 1;
        if (check_huge) {
            const float *s = bufs[1] + 3 * (size_t)i;
            const float max_s = fmaxf(fmaxf(msp_expf(s[0]), msp_expf(s[1])), msp_expf(s[2]));
            if (max_s > cull_scale_thresh) cull = 1;
            if (check_screen && i < N && max_2d_size[i] > cull_screen_size) cull = 1;
        }
        keep[i] = !cull;
    }
    /* stable compaction of the 18 buffers (:3698-3729) */
    int n_keep = 0;
    for (int i = 0; i < n_new; i++) {
        if (!keep[i]) continue;
        if (n_keep != i)
            for (int g = 0; g < 6; g++) {
                const int S = strides[g];
                memmove(bufs[g] + (size_t)n_keep * S, bufs[g] + (size_t)i * S, sizeof(float) * S);
                memmove(exp_avg[g] + (size_t)n_keep * S, exp_avg[g] + (size_t)i * S, sizeof(float) * S);
                memmove(exp_avg_sq[g] + (size_t)n_keep * S, exp_avg_sq[g] + (size_t)i * S,
                        sizeof(float) * S);
            }
        n_keep++;
    }
    if (split_flag_out) memcpy(split_flag_out, split, sizeof(int) * (size_t)N);
    if (dup_flag_out) memcpy(dup_flag_out, dup, sizeof(int) * (size_t)N);
    if (keep_flag_out) memcpy(keep_flag_out, keep, sizeof(int) * (size_t)worst);
    free(split); free(dup); free(keep); free(split_ord); free(dup_ord);
    return n_keep;
}

/*
 * The opacity reset of Model::afterTrain (core/src/model.cpp:280-290):
 * logits above logit(0.2) are lowered to it, and the opacity moments are
 * zeroed.
 */
void orc_reset_opacity(float *opacities, float *exp_avg5, float *exp_avg_sq5, int n)
{
    const float reset_logit = -1.3862943611198906f;
    for (int i = 0; i < n; i++) {
        if (opacities[i] > reset_logit) opacities[i] = reset_logit;
        exp_avg5[i] = 0.f;
        exp_avg_sq5[i] = 0.f;
    }
}

/*
 * Mean distance to the k-1 nearest other points (PointsTensor::scales,
 * core/include/kdtree_tensor.hpp:27-41, a nanoflann v1.5.5 k-d tree, which
 * is exact): squared distances formed as nanoflann's L2_Simple_Adaptor
 * forms them (result += diff * diff over x, y, z), the k smallest kept
 * (the point itself is the first), then the mean of their square roots.
 * Exhaustive search; test infrastructure for msplat_knn_mean_distance.
 */
void orc_knn_mean_distance(const float *xyz, int64_t n, int k, float *out)
{
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t i = 0; i < n; i++) {
        float best[8];
        for (int j = 0; j < k; j++) best[j] = 3.402823466e38f;
        const float *q = xyz + 3 * i;
        for (int64_t j = 0; j < n; j++) {
            float d = 0.0f;
            for (int a = 0; a < 3; a++) {
                const float diff = q[a] - xyz[3 * j + a];
                d += diff * diff;
            }
            if (d < best[k - 1]) {
                int m = k - 1;
                while (m > 0 && best[m - 1] > d) {
                    best[m] = best[m - 1];
                    m--;
                }
                best[m] = d;
            }
        }
        float sum = 0.0f;
        for (int j = 1; j < k; j++) sum += sqrtf(best[j]);
        out[i] = sum / (float)(k - 1);
    }
}
