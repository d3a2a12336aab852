// ref_driver.cpp -- replays msplat's host dispatch sequence over the
// reference's own kernels compiled through the MSL shim.  TEST
// INFRASTRUCTURE ONLY: the oracle is checked against this library.
//
// Follows core/metal/msplat_metal.mm: forward_pipeline (:462-750) for
// ref_render, msplat_train_step (:771-1330) for ref_train_step -- buffer
// zeroing (:1158-1174), dispatch order and grids (:1295-1326), the depth
// chunk rule (:873-889), the SH Adam hyper-parameter block (:1078-1092) and
// fused_adam over groups 0, 1, 2, 5 (:1117-1139).  The only departure is
// that threadgroups at the right/bottom image edge of the 16x16
// dispatchThreads grids (SSIM passes) get all 256 threads (the kernels'
// cooperative tile loads stride by 256 and would otherwise leave part of
// the tile unwritten; every access is bounds-checked); see msl_runtime.hpp.
#include <omp.h>

#include <cmath>
#include <cstring>
#include <vector>

#include "msl_runtime.hpp"
#include "msplat_metal_ref.inc"

extern "C" {
#include "msplat_oracle.h"
}

using namespace msl;

namespace {

struct RefBuffers {
    std::vector<float> xys, depths, conics, colors, aabb;
    std::vector<int> radii, num_tiles_hit;
    std::vector<uint> counters;      // tile_scatter_counters (atomic_uint)
    std::vector<uint64_t> bins;      // prealloc_bins [T * MAX_TILE_ELEMS]
    std::vector<int> tile_offsets, tile_bins, gaussian_ids;
    std::vector<float> packed_xy_opac, packed_conic, packed_rgb;
    std::vector<float> out_img, final_Ts;
    std::vector<int> final_idx;
    std::vector<float> chunk_T, chunk_C, prefix_T, after_C;
    std::vector<int> chunk_idx;
    std::vector<float> ssim_h, loss_inter, v_rendered;
    std::vector<float> v_xy, v_conic, v_rgb, v_opacity, v_depth, v_mean3d, v_scale, v_quat;
    float loss_sum = 0.f;
    uint overflow = 0;
};

RefBuffers g;

template <class T>
void zero(std::vector<T>& v, size_t n)
{
    v.assign(n, T{});
}

atomic_float* AF(std::vector<float>& v) { return reinterpret_cast<atomic_float*>(v.data()); }
atomic_uint* AU(std::vector<uint>& v) { return reinterpret_cast<atomic_uint*>(v.data()); }

uint kmax_rule(int N, int num_tiles)
{
    // msplat_metal.mm:873-889
    if (num_tiles >= 400) return 1;
    const long long capacity = (long long)N * 16;
    const uint avg = (uint)(capacity / std::max(1, num_tiles));
    const uint cons = avg * 6;
    uint k = (cons + 512 - 1) / 512;
    if (k < 2) k = 2;
    const uint abs_max = (uint)((capacity + 512 - 1) / 512);
    if (k > abs_max) k = abs_max;
    return k;
}

int forward(const orc_params* P, const float* means, const float* scales, const float* quats,
            const float* dc, const float* rest, const float* opac, uint& K_max)
{
    const int N = P->num_points;
    const uint W = (uint)P->img_w, H = (uint)P->img_h;
    const uint tx = (uint)P->tiles_x, ty = (uint)P->tiles_y, T = tx * ty;
    const size_t NP = (size_t)W * H;
    const long long capacity = (long long)N * 16;
    zero(g.xys, 2 * (size_t)N); zero(g.depths, N); zero(g.conics, 3 * (size_t)N);
    zero(g.colors, 3 * (size_t)N); zero(g.aabb, 2 * (size_t)N);
    zero(g.radii, N); zero(g.num_tiles_hit, N);
    zero(g.counters, T);
    g.bins.resize((size_t)T * MAX_TILE_ELEMS);
    zero(g.tile_offsets, T); zero(g.tile_bins, 2 * (size_t)T);
    g.overflow = 0;
    g.loss_sum = 0.f;
    zero(g.out_img, 3 * NP); zero(g.final_Ts, NP); zero(g.final_idx, NP);

    const int num_points = N;
    const uint num_points_u = (uint)N;
    const float4 intrins(P->fx, P->fy, P->cx, P->cy);
    const uint2 img_size2(W, H);
    const uint3 img_size3(W, H, 1);
    const uint3 tile_bounds(tx, ty, 1);
    const float3 cam_pos(P->cam_pos[0], P->cam_pos[1], P->cam_pos[2]);
    const float glob_scale = P->glob_scale, clip = P->clip_thresh;
    const uint degree = (uint)P->degree, dtu = (uint)P->degrees_to_use;
    const uint channels = 3;

    dispatch_threads_1d(num_points_u, [&](uint i) {
        project_and_sh_forward_kernel(num_points, means, scales, glob_scale, quats, P->viewmat,
                                      P->projmat, intrins, img_size2, tile_bounds, clip,
                                      g.xys.data(), g.depths.data(), g.radii.data(),
                                      g.conics.data(), g.num_tiles_hit.data(), degree, dtu,
                                      cam_pos, dc, rest, g.colors.data(), g.aabb.data(),
                                      uint3(i, 0, 0));
    });
    atomic_uint* ov = reinterpret_cast<atomic_uint*>(&g.overflow);
    dispatch_threads_1d(num_points_u, [&](uint i) {
        scatter_to_prealloc_bins_kernel(num_points_u, g.xys.data(), g.depths.data(),
                                        g.radii.data(), g.aabb.data(), tile_bounds, AU(g.counters),
                                        g.bins.data(), ov, i);
    });
    const uint Tu = T;
    dispatch_threadgroups(uint3(1, 1, 1), uint3(1024, 1, 1), [&](const ThreadIds& t) {
        prefix_sum_kernel(Tu, reinterpret_cast<const int*>(g.counters.data()),
                          g.tile_offsets.data(), t.tr, 1024u, t.sgid, t.lane, 32u);
    });
    const long long total = T ? g.tile_offsets[T - 1] : 0;
    const long long cap = std::max(capacity, total);
    zero(g.gaussian_ids, cap); zero(g.packed_xy_opac, 3 * cap); zero(g.packed_conic, 3 * cap);
    zero(g.packed_rgb, 3 * cap);
    dispatch_threadgroups(uint3(T, 1, 1), uint3(256, 1, 1), [&](const ThreadIds& t) {
        bitonic_sort_per_tile_kernel(g.tile_offsets.data(),
                                     reinterpret_cast<const int*>(g.counters.data()),
                                     g.bins.data(), g.gaussian_ids.data(), Tu, g.xys.data(),
                                     g.conics.data(), g.colors.data(), opac,
                                     g.packed_xy_opac.data(), g.packed_conic.data(),
                                     g.packed_rgb.data(), g.tile_bins.data(), t.tgid.x, t.tr);
    });
    K_max = kmax_rule(N, (int)T);
    const uint2 blockDim(8, 8);
    const float* bg = P->background;
    const uint rx = (W + 7) / 8, ry = (H + 7) / 8;
    if (K_max <= 1) {
        dispatch_threadgroups(uint3(rx, ry, 1), uint3(8, 8, 1), [&](const ThreadIds& t) {
            nd_rasterize_forward_kernel(tile_bounds, img_size3, channels, g.tile_bins.data(),
                                        g.packed_xy_opac.data(), g.packed_conic.data(),
                                        g.packed_rgb.data(), g.final_Ts.data(), g.final_idx.data(),
                                        g.out_img.data(), bg, blockDim, uint2(t.tgid.x, t.tgid.y),
                                        uint2(t.lid.x, t.lid.y), t.tr);
        });
    } else {
        const size_t KP = (size_t)K_max * NP;
        zero(g.chunk_T, KP); zero(g.chunk_C, 3 * KP); zero(g.chunk_idx, KP);
        const uint chunk = 512, Ku = K_max;
        dispatch_threadgroups(uint3(rx, ry, K_max), uint3(8, 8, 1), [&](const ThreadIds& t) {
            rasterize_forward_chunked_kernel(tile_bounds, img_size3, channels, g.tile_bins.data(),
                                             g.packed_xy_opac.data(), g.packed_conic.data(),
                                             g.packed_rgb.data(), g.chunk_T.data(),
                                             g.chunk_C.data(), g.chunk_idx.data(), chunk, Ku,
                                             blockDim, t.tgid, t.tr);
        });
        const uint npix = (uint)NP;
        dispatch_threads_2d(W, H, [&](uint2 gp) {
            rasterize_forward_merge_kernel(npix, Ku, g.chunk_T.data(), g.chunk_C.data(),
                                           g.chunk_idx.data(), g.final_Ts.data(),
                                           g.final_idx.data(), g.out_img.data(), bg, img_size2, gp);
        });
    }
    return g.overflow ? 1 : 0;
}

void fill_forward_outputs(const orc_params* P, orc_state* S)
{
    const int N = P->num_points;
    const int T = P->tiles_x * P->tiles_y;
    const size_t NP = (size_t)P->img_w * P->img_h;
    std::memcpy(S->xys, g.xys.data(), sizeof(float) * 2 * N);
    std::memcpy(S->depths, g.depths.data(), sizeof(float) * N);
    std::memcpy(S->radii, g.radii.data(), sizeof(int) * N);
    std::memcpy(S->conics, g.conics.data(), sizeof(float) * 3 * N);
    std::memcpy(S->num_tiles_hit, g.num_tiles_hit.data(), sizeof(int) * N);
    std::memcpy(S->colors, g.colors.data(), sizeof(float) * 3 * N);
    std::memcpy(S->aabb, g.aabb.data(), sizeof(float) * 2 * N);
    std::memcpy(S->tile_bins, g.tile_bins.data(), sizeof(int) * 2 * T);
    const long long total = T ? g.tile_offsets[T - 1] : 0;
    S->num_isects = total;
    int maxc = 0;
    for (int t = 0; t < T; t++) maxc = std::max(maxc, (int)g.counters[t]);
    S->max_tile_count = maxc;
    if (total <= S->isect_capacity)
        std::memcpy(S->gaussian_ids, g.gaussian_ids.data(), sizeof(int) * total);
    std::memcpy(S->out_img, g.out_img.data(), sizeof(float) * 3 * NP);
    std::memcpy(S->final_T, g.final_Ts.data(), sizeof(float) * NP);
    std::memcpy(S->final_idx, g.final_idx.data(), sizeof(int) * NP);
}

}  // namespace

extern "C" {

void ref_set_threads(int n)
{
    if (n > 0) omp_set_num_threads(n);
}

int ref_tile_cap(void) { return MAX_TILE_ELEMS; }

// msplat_render (msplat_metal.mm:752-769).  Returns 0, or 1 when a tile
// exceeded the per-tile cap (the reference then drops Gaussians).
int ref_render(const orc_params* P, orc_state* S, const float* params[6])
{
    uint K_max = 1;
    const int rc = forward(P, params[0], params[1], params[2], params[3], params[4], params[5], K_max);
    fill_forward_outputs(P, S);
    return rc;
}

// msplat_train_step (msplat_metal.mm:771-1330).
int ref_train_step(const orc_params* P, orc_state* S, float* params[6], float* exp_avg[6],
                   float* exp_avg_sq[6], const float* gt, float* vis_counts, float* xys_grad_norm,
                   float* max_2d_size)
{
    const int N = P->num_points;
    const uint W = (uint)P->img_w, H = (uint)P->img_h;
    const size_t NP = (size_t)W * H;
    uint K_max = 1;
    const int rc = forward(P, params[0], params[1], params[2], params[3], params[4], params[5], K_max);
    // blit-zero of the accumulators (msplat_metal.mm:1158-1174)
    zero(g.v_xy, 2 * (size_t)N); zero(g.v_conic, 3 * (size_t)N); zero(g.v_rgb, 3 * (size_t)N);
    zero(g.v_opacity, N); zero(g.v_depth, N); zero(g.v_mean3d, 3 * (size_t)N);
    zero(g.v_scale, 3 * (size_t)N); zero(g.v_quat, 4 * (size_t)N);
    zero(g.ssim_h, 15 * NP); zero(g.loss_inter, 15 * NP); zero(g.v_rendered, 3 * NP);
    const uint2 isz(W, H);
    const float ssim_w = P->ssim_weight, inv_n = P->loss_inv_n;
    atomic_float* loss = reinterpret_cast<atomic_float*>(&g.loss_sum);
    const uint3 sgrid((W + 15) / 16, (H + 15) / 16, 1), stg(16, 16, 1);
    dispatch_threadgroups(sgrid, stg, [&](const ThreadIds& t) {
        ssim_h_fwd_kernel(g.out_img.data(), gt, isz, g.ssim_h.data(), uint2(t.gp.x, t.gp.y),
                          uint2(t.lid.x, t.lid.y), t.tr, uint2(t.tgid.x, t.tgid.y));
    });
    dispatch_threadgroups(sgrid, stg, [&](const ThreadIds& t) {
        ssim_fused_v_fwd_h_bwd_kernel(g.out_img.data(), gt, g.ssim_h.data(), isz, ssim_w, inv_n,
                                      g.loss_inter.data(), loss, uint2(t.gp.x, t.gp.y),
                                      uint2(t.lid.x, t.lid.y), t.tr, uint2(t.tgid.x, t.tgid.y),
                                      uint2(16, 16));
    });
    dispatch_threadgroups(sgrid, stg, [&](const ThreadIds& t) {
        ssim_v_bwd_kernel(g.out_img.data(), gt, g.loss_inter.data(), isz, ssim_w, inv_n,
                          g.v_rendered.data(), uint2(t.gp.x, t.gp.y), uint2(t.lid.x, t.lid.y),
                          t.tr, uint2(t.tgid.x, t.tgid.y));
    });
    const uint3 rast_tb((W + 15) / 16, (H + 15) / 16, 1);
    const uint rx = (W + 7) / 8, ry = (H + 7) / 8;
    const float* bg = P->background;
    if (K_max <= 1) {
        dispatch_threadgroups(uint3(rx, ry, 1), uint3(8, 8, 1), [&](const ThreadIds& t) {
            rasterize_backward_kernel(rast_tb, isz, g.gaussian_ids.data(), g.tile_bins.data(),
                                      g.packed_xy_opac.data(), g.packed_conic.data(),
                                      g.packed_rgb.data(), bg, g.final_Ts.data(),
                                      g.final_idx.data(), g.v_rendered.data(), AF(g.v_xy),
                                      AF(g.v_conic), AF(g.v_rgb), AF(g.v_opacity), t.gp, t.tgid,
                                      t.tr, 32u, t.lane);
        });
    } else {
        const size_t KP = (size_t)K_max * NP;
        zero(g.prefix_T, KP); zero(g.after_C, 3 * KP);
        const uint npix = (uint)NP, Ku = K_max, chunk = 512;
        dispatch_threads_2d(W, H, [&](uint2 gp) {
            compute_chunk_prefix_suffix_kernel(npix, Ku, g.chunk_T.data(), g.chunk_C.data(),
                                               g.chunk_idx.data(), g.prefix_T.data(),
                                               g.after_C.data(), isz, gp);
        });
        dispatch_threadgroups(uint3(rx, ry, K_max), uint3(8, 8, 1), [&](const ThreadIds& t) {
            rasterize_backward_chunked_kernel(
                rast_tb, isz, g.gaussian_ids.data(), g.tile_bins.data(), g.packed_xy_opac.data(),
                g.packed_conic.data(), g.packed_rgb.data(), bg, g.final_Ts.data(),
                g.chunk_idx.data(), g.prefix_T.data(), g.chunk_T.data(), g.after_C.data(),
                g.v_rendered.data(), AF(g.v_xy), AF(g.v_conic), AF(g.v_rgb), AF(g.v_opacity),
                chunk, Ku, t.gp, t.tgid, t.tr, 32u, t.lane);
        });
    }
    SHAdamParams hp;
    hp.dc_step_size = P->adam_step_size[3];
    hp.dc_bc2_sqrt = P->adam_bc2_sqrt[3];
    hp.rest_step_size = P->adam_step_size[4];
    hp.rest_bc2_sqrt = P->adam_bc2_sqrt[4];
    hp.beta1 = P->beta1;
    hp.beta2 = P->beta2;
    hp.eps = P->eps;
    const float4 intrins(P->fx, P->fy, P->cx, P->cy);
    const float3 cam_pos(P->cam_pos[0], P->cam_pos[1], P->cam_pos[2]);
    const uint degree = (uint)P->degree, dtu = (uint)P->degrees_to_use;
    const int num_points = N;
    const float glob_scale = P->glob_scale;
    dispatch_threads_1d((uint)N, [&](uint i) {
        project_and_sh_backward_kernel(num_points, params[0], params[1], glob_scale, params[2],
                                       P->viewmat, P->projmat, intrins, isz, g.radii.data(),
                                       g.conics.data(), g.v_xy.data(), g.v_depth.data(),
                                       g.v_conic.data(), g.v_mean3d.data(), g.v_scale.data(),
                                       g.v_quat.data(), degree, dtu, cam_pos, g.v_rgb.data(),
                                       params[3], params[4], exp_avg[3], exp_avg_sq[3],
                                       exp_avg[4], exp_avg_sq[4], hp, i);
    });
    const float* grads[6] = {g.v_mean3d.data(), g.v_scale.data(), g.v_quat.data(), nullptr,
                             nullptr, g.v_opacity.data()};
    const uint numel[6] = {3u * N, 3u * N, 4u * N, 0, 0, (uint)N};
    for (int gi = 0; gi < 6; gi++) {
        if (gi == 3 || gi == 4) continue;
        const uint n = numel[gi];
        const float step = P->adam_step_size[gi], b1 = P->beta1, b2 = P->beta2;
        const float bc2 = P->adam_bc2_sqrt[gi], eps = P->eps;
        dispatch_threads_1d(n, [&](uint tid) {
            fused_adam_kernel(params[gi], grads[gi], exp_avg[gi], exp_avg_sq[gi], step, b1, b2,
                              bc2, eps, n, tid);
        });
    }
    const float inv_max_dim = P->inv_max_dim;
    dispatch_threads_1d((uint)N, [&](uint i) {
        accumulate_grad_stats_kernel(num_points, g.radii.data(), g.v_xy.data(), vis_counts,
                                     xys_grad_norm, max_2d_size, inv_max_dim, i);
    });
    fill_forward_outputs(P, S);
    std::memcpy(S->v_rendered, g.v_rendered.data(), sizeof(float) * 3 * NP);
    S->loss = (double)g.loss_sum / ((double)W * H);
    std::memcpy(S->v_xy, g.v_xy.data(), sizeof(float) * 2 * N);
    std::memcpy(S->v_conic, g.v_conic.data(), sizeof(float) * 3 * N);
    std::memcpy(S->v_rgb, g.v_rgb.data(), sizeof(float) * 3 * N);
    std::memcpy(S->v_opacity, g.v_opacity.data(), sizeof(float) * N);
    std::memcpy(S->v_mean3d, g.v_mean3d.data(), sizeof(float) * 3 * N);
    std::memcpy(S->v_scale, g.v_scale.data(), sizeof(float) * 3 * N);
    std::memcpy(S->v_quat, g.v_quat.data(), sizeof(float) * 4 * N);
    return rc;
}

// msplat_densify (msplat_metal.mm:1337-1592): the nine stages in order,
// with the scan kernels on 1024-thread threadgroups and the compaction of
// the 18 buffers through the scratch buffer.  Same arguments as
// orc_densify; returns the new count, or -1 when 3N exceeds the capacity.
int ref_densify(int N, int buf_capacity, float grad_thresh, float size_thresh,
                float screen_thresh, int check_screen, float cull_alpha_thresh,
                float cull_scale_thresh, float cull_screen_size, int check_huge,
                const float* xys_grad_norm, const float* vis_counts, const float* max_2d_size,
                float half_max_dim, float* bufs[6], int fr_stride, float* exp_avg[6],
                float* exp_avg_sq[6], const float* random_samples, int* split_flag_out,
                int* dup_flag_out, int* keep_flag_out)
{
    const int worst = 3 * N;
    if (worst > buf_capacity) return -1;
    const int cap = std::max(buf_capacity, 1);
    std::vector<int> split_flag(cap), dup_flag(cap), split_prefix(cap), dup_prefix(cap),
        keep_flag(cap), keep_prefix(cap), block_totals((cap + 1023) / 1024 + 1);
    std::vector<float> scratch((size_t)cap * std::max(fr_stride, 4));
    const float log_size_fac = std::log(1.6f);
    const uint N_u = (uint)N;
    const uint K = (uint)((N + 1023) / 1024);
    const int strides[6] = {3, 3, 4, 3, fr_stride, 1};
    auto scan = [&](uint n, const int* in, int* out) {
        const uint blocks = (n + 1023) / 1024;
        dispatch_threadgroups(uint3(blocks, 1, 1), uint3(1024, 1, 1), [&](const ThreadIds& t) {
            block_reduce_kernel(n, in, block_totals.data(), t.tgid.x, t.tr, t.sgid, t.lane);
        });
        dispatch_threadgroups(uint3(blocks, 1, 1), uint3(1024, 1, 1), [&](const ThreadIds& t) {
            block_scan_propagate_kernel(n, in, out, block_totals.data(), t.tgid.x, t.tr, t.sgid,
                                        t.lane, 32u);
        });
    };
    dispatch_threads_1d(N_u, [&](uint i) {
        densify_classify_kernel(N, xys_grad_norm, vis_counts, bufs[1], max_2d_size, half_max_dim,
                                grad_thresh, size_thresh, screen_thresh, check_screen,
                                split_flag.data(), dup_flag.data(), i);
    });
    (void)K;
    scan(N_u, split_flag.data(), split_prefix.data());
    scan(N_u, dup_flag.data(), dup_prefix.data());
    dispatch_threads_1d(N_u, [&](uint i) {
        densify_append_split_kernel(N, split_flag.data(), split_prefix.data(), random_samples,
                                    log_size_fac, bufs[0], bufs[1], bufs[2], bufs[3], bufs[4],
                                    bufs[5], fr_stride, exp_avg[0], exp_avg[1], exp_avg[2],
                                    exp_avg[3], exp_avg[4], exp_avg[5], exp_avg_sq[0],
                                    exp_avg_sq[1], exp_avg_sq[2], exp_avg_sq[3], exp_avg_sq[4],
                                    exp_avg_sq[5], i);
    });
    dispatch_threads_1d(N_u, [&](uint i) {
        densify_append_dup_kernel(N, dup_flag.data(), dup_prefix.data(), split_prefix.data(),
                                  bufs[0], bufs[1], bufs[2], bufs[3], bufs[4], bufs[5], fr_stride,
                                  exp_avg[0], exp_avg[1], exp_avg[2], exp_avg[3], exp_avg[4],
                                  exp_avg[5], exp_avg_sq[0], exp_avg_sq[1], exp_avg_sq[2],
                                  exp_avg_sq[3], exp_avg_sq[4], exp_avg_sq[5], i);
    });
    const uint wc = (uint)worst;
    dispatch_threads_1d(wc, [&](uint i) {
        densify_cull_classify_kernel(N, split_prefix.data(), dup_prefix.data(), split_flag.data(),
                                     bufs[5], bufs[1], max_2d_size, cull_alpha_thresh,
                                     cull_scale_thresh, cull_screen_size, check_huge,
                                     check_screen, keep_flag.data(), i);
    });
    scan(wc, keep_flag.data(), keep_prefix.data());
    for (int b = 0; b < 18; b++) {
        float* buf = b < 6 ? bufs[b] : b < 12 ? exp_avg[b - 6] : exp_avg_sq[b - 12];
        const uint stride = (uint)strides[b % 6];
        const uint total = wc * stride;
        dispatch_threads_1d(total, [&](uint t) {
            compact_scatter_kernel(buf, scratch.data(), keep_prefix.data(), keep_flag.data(), wc,
                                   stride, t);
        });
        const uint last = wc ? wc - 1 : 0;
        dispatch_threads_1d(total, [&](uint t) {
            compact_copy_back_kernel(scratch.data(), buf, keep_prefix.data(), last, stride, t);
        });
    }
    if (split_flag_out) std::memcpy(split_flag_out, split_flag.data(), sizeof(int) * N);
    if (dup_flag_out) std::memcpy(dup_flag_out, dup_flag.data(), sizeof(int) * N);
    if (keep_flag_out) std::memcpy(keep_flag_out, keep_flag.data(), sizeof(int) * worst);
    return worst ? keep_prefix[worst - 1] : 0;
}

}  // extern "C"
