/*
 * msplat_oracle.h -- CPU restatement of msplat's per-iteration training step.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA engine in msplat_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  The product never links it.
 *
 * Reference: Plinth-it/msplat v1.1.3.  Kernel maths follows
 * core/metal/msplat_metal.metal; the dispatch order and the chunk rule follow
 * core/metal/msplat_metal.mm (msplat_train_step :771-1330, forward_pipeline
 * :462-750).  Every function in msplat_oracle.c cites the lines it restates.
 *
 * Arithmetic contract shared with the CUDA engine (so that tile membership,
 * per-tile sort order and the forward image are bit-exact):
 *   - no FMA contraction (compiled with -ffp-contract=off); fma() of the
 *     reference is fmaf();
 *   - exp() is msp_expf(): Cody & Waite argument reduction plus a degree-6
 *     minimax polynomial (see msplat_oracle.c);
 *   - sqrt, division are IEEE round-to-nearest; rsqrt(x) is 1.0f/sqrtf(x);
 *   - float->int conversion truncates, saturates and maps NaN to 0.
 */
#ifndef MSPLAT_ORACLE_H
#define MSPLAT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_N_GROUPS 6

typedef struct {
    int32_t num_points;
    int32_t img_w, img_h;
    int32_t tiles_x, tiles_y;
    int32_t degree;          /* SH degree of the stored coefficients */
    int32_t degrees_to_use;  /* SH degree evaluated this step */
    int32_t k_max;           /* depth chunks: 1 = monolithic raster */
    float viewmat[16];       /* row-major world->camera */
    float projmat[16];       /* row-major proj * view */
    float fx, fy, cx, cy;
    float glob_scale, clip_thresh;
    float cam_pos[3];
    float background[3];
    float ssim_weight, loss_inv_n, inv_max_dim;
    float adam_step_size[ORC_N_GROUPS]; /* lr / (1 - beta1^t) */
    float adam_bc2_sqrt[ORC_N_GROUPS];  /* sqrt(1 - beta2^t) */
    float beta1, beta2, eps;
} orc_params;

/* Caller-owned buffers for intermediates (any pointer may be NULL when the
 * caller does not want that dump, except where a stage needs it). */
typedef struct {
    /* projection, per Gaussian */
    float *xys;            /* N*2 */
    float *depths;         /* N   */
    int32_t *radii;        /* N   */
    float *conics;         /* N*3 */
    int32_t *num_tiles_hit;/* N   */
    float *colors;         /* N*3 (raw SH output) */
    float *aabb;           /* N*2 */
    /* binning */
    int32_t *tile_bins;    /* T*2 [start, end) */
    int32_t *gaussian_ids; /* isect_capacity */
    int64_t isect_capacity;
    int64_t num_isects;    /* out */
    /* raster forward */
    float *out_img;        /* H*W*3 */
    float *final_T;        /* H*W   */
    int32_t *final_idx;    /* H*W   */
    /* loss */
    float *v_rendered;     /* H*W*3 */
    double loss;           /* mean per-pixel loss (out) */
    /* raster backward (accumulated in double, stored as float) */
    float *v_xy;           /* N*2 */
    float *v_conic;        /* N*3 */
    float *v_rgb;          /* N*3 */
    float *v_opacity;      /* N   */
    /* projection backward */
    float *v_mean3d;       /* N*3 */
    float *v_scale;        /* N*3 */
    float *v_quat;         /* N*4 */
    /* diagnostics (out) */
    int32_t max_tile_count;
} orc_state;

float msp_expf(float x);

void orc_set_threads(int n);

/* k_max from the reference's chunk rule (msplat_metal.mm:873-889). */
int32_t orc_chunk_k_max(int32_t num_points, int32_t num_tiles);

/* Stages. */
void orc_project_sh_forward(const orc_params *P, const float *means,
                            const float *scales, const float *quats,
                            const float *features_dc, const float *features_rest,
                            orc_state *S);
int orc_bin_and_sort(const orc_params *P, orc_state *S);
void orc_rasterize_forward(const orc_params *P, const float *opacities,
                           orc_state *S);
void orc_ssim_loss(const orc_params *P, const float *gt, orc_state *S);
void orc_rasterize_backward(const orc_params *P, const float *opacities,
                            orc_state *S);
void orc_project_sh_backward_adam(const orc_params *P, const float *means,
                                  const float *scales, const float *quats,
                                  float *features_dc, float *features_rest,
                                  float *dc_exp_avg, float *dc_exp_avg_sq,
                                  float *rest_exp_avg, float *rest_exp_avg_sq,
                                  orc_state *S);
void orc_fused_adam(float *params, const float *grads, float *exp_avg,
                    float *exp_avg_sq, float step_size, float beta1,
                    float beta2, float bc2_sqrt, float eps, int64_t n);
void orc_grad_stats(const orc_params *P, const orc_state *S, float *vis_counts,
                    float *xys_grad_norm, float *max_2d_size);

/* Whole step: params[g] / exp_avg[g] / exp_avg_sq[g] are updated in place,
 * groups ordered means, scales, quats, features_dc, features_rest, opacities.
 * Returns 0, or -1 when isect_capacity is too small. */
int orc_train_step(const orc_params *P, orc_state *S, float *params[6],
                   float *exp_avg[6], float *exp_avg_sq[6], const float *gt,
                   float *vis_counts, float *xys_grad_norm, float *max_2d_size);

/* Densification, msplat_densify (bindings.h:69-84): see msplat_oracle.c. */
int orc_densify(int N, int buf_capacity, float grad_thresh, float size_thresh,
                float screen_thresh, int check_screen, float cull_alpha_thresh,
                float cull_scale_thresh, float cull_screen_size, int check_huge,
                const float *xys_grad_norm, const float *vis_counts, const float *max_2d_size,
                float half_max_dim, float *bufs[6], int fr_stride, float *exp_avg[6],
                float *exp_avg_sq[6], const float *random_samples, int *split_flag_out,
                int *dup_flag_out, int *keep_flag_out);
void orc_reset_opacity(float *opacities, float *exp_avg5, float *exp_avg_sq5, int n);

/* Initial-scale k-NN (kdtree_tensor.hpp:27-41): see msplat_oracle.c. */
void orc_knn_mean_distance(const float *xyz, int64_t n, int k, float *out);

/* Forward only (msplat_render): fills S->out_img / final_T / final_idx. */
int orc_render(const orc_params *P, orc_state *S, const float *params[6]);

#ifdef __cplusplus
}
#endif
#endif
