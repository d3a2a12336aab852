"""Shared set-up for parity tests: one scene, one camera, the engine (through
the C-ABI) and the CPU oracle on identical float32 inputs."""
from __future__ import annotations

import numpy as np

from msplat_b200 import camera, engine, synthetic
from oracle import oracle

BG = engine.DEFAULT_BG


def setup_cam(cam, step=10**9, sh_degree=3, interval=1000, rest_bases=15):
    return camera.prepare_camera(cam, step=step, sh_degree=sh_degree, sh_degree_interval=interval,
                                 rest_bases=rest_bases)


# Tiles of more than SORT_RUN keys may sort only the front of their list
# when the raster is single-pass (the engine's nearest-key selection, on
# after a view with such a tile); the positions past that prefix are never
# read.
SORT_RUN = 2048


def tile_ids_engine(cs, n_isect):
    T = cs.tile_bounds[0] * cs.tile_bounds[1]
    off = engine.debug_buffer("tile_offset", T + 1, np.int32)
    ids = engine.debug_buffer("sorted_ids", int(off[-1]), np.int32)
    srt = engine.debug_buffer("tile_sorted", T, np.int32)
    return off, ids, srt


def sorted_prefix_mask(off, srt):
    """True at the list positions inside each tile's sorted prefix."""
    counts = np.diff(off)
    tile = np.repeat(np.arange(counts.size), counts)
    return (np.arange(int(off[-1])) - off[:-1][tile]) < np.minimum(srt, counts)[tile]


def oracle_ranges(run, cs):
    T = cs.tile_bounds[0] * cs.tile_bounds[1]
    tb = run.tile_bins.reshape(T, 2)
    return tb, run.gaussian_ids[: run.num_isects]


def engine_forward_dump(n, cs):
    xy = engine.debug_buffer("xy", 2 * n, np.float32)
    depth = engine.debug_buffer("depth", n, np.float32)
    radii = engine.debug_buffer("radii", n, np.int32)
    co = engine.debug_buffer("conic_op", 4 * n, np.float32).reshape(n, 4)
    rgb = engine.debug_buffer("rgb", 4 * n, np.float32).reshape(n, 4)
    P = cs.width * cs.height
    img = engine.debug_buffer("out_img", 3 * P, np.float32)
    fT = engine.debug_buffer("final_T", P, np.float32)
    fi = engine.debug_buffer("final_idx", P, np.int32)
    return dict(xy=xy, depth=depth, radii=radii, conic=co[:, :3], opac=co[:, 3], rgb=rgb[:, :3],
                img=img, final_T=fT, final_idx=fi)


def assert_forward_bitexact(run, eng, cs):
    n = eng["radii"].shape[0]
    np.testing.assert_array_equal(eng["radii"], run.radii)
    vis = run.radii > 0
    np.testing.assert_array_equal(eng["xy"].reshape(n, 2)[vis], run.xys.reshape(n, 2)[vis])
    np.testing.assert_array_equal(eng["depth"][vis], run.depths[vis])
    np.testing.assert_array_equal(eng["conic"][vis], run.conics.reshape(n, 3)[vis])
    np.testing.assert_array_equal(eng["rgb"][vis], run.colors.reshape(n, 3)[vis])
    off, ids, srt = tile_ids_engine(cs, run.num_isects)
    tb, oids = oracle_ranges(run, cs)
    np.testing.assert_array_equal(off[:-1], tb[:, 0])
    np.testing.assert_array_equal(off[1:], tb[:, 1])
    counts = np.diff(off)
    whole = (counts <= SORT_RUN) | (run.P.k_max > 1)
    np.testing.assert_array_equal(srt[whole], counts[whole])
    assert ((srt >= 1) & (srt <= counts))[counts > 0].all()
    mask = sorted_prefix_mask(off, srt)
    np.testing.assert_array_equal(ids[mask], oids[mask])
    np.testing.assert_array_equal(eng["final_idx"], run.final_idx)
    np.testing.assert_array_equal(eng["final_T"], run.final_T)
    np.testing.assert_array_equal(eng["img"], run.out_img)


def close(a, b, rtol, atol_frac):
    """|a-b| <= rtol*max(|a|,|b|) + atol_frac*max|b| (the combined tolerance
    for float-atomic reductions)."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    scale = max(float(np.abs(b).max()) if b.size else 0.0, 1e-30)
    tol = rtol * np.maximum(np.abs(a), np.abs(b)) + atol_frac * scale
    bad = np.abs(a - b) > tol
    return int(bad.sum()), float((np.abs(a - b) / scale).max()) if a.size else 0.0


# Gradient bar (north star: 1e-4 relative), with an absolute floor for the
# float-atomic sums: |a-b| <= GRAD_RTOL*max(|a|,|b|) + GRAD_ATOL_FRAC*max|ref|.
# No outliers are allowed on gradients.
GRAD_RTOL = 1e-4
GRAD_ATOL_FRAC = 2e-6


def engine_geometry_grads(groups, cs, gt_dev, ssim_weight=0.2):
    """The engine's pre-Adam gradients of one step from `groups` (a fresh
    model, so the fused step's in-place update does not interfere), through
    msplat_train_step_grads: the same forward, backward and projection VJP
    as msplat_train_step, with the Adam phase replaced by a gradient write.
    Returns v_mean3d [N,3], v_scale [N,3] (log-space), v_quat [N,4] and
    v_opacity [N,1] (logit), zero for culled Gaussians."""
    import torch

    from msplat_b200 import multigpu
    model = engine.GaussianModel(groups)
    buf = torch.zeros(multigpu.grad_floats(model.n, model.rest_bases), dtype=torch.float32,
                      device="cuda")
    multigpu.EngineOps().grads(model, cs, gt_dev, buf, ssim_weight, BG, 1.0, 0.01)
    torch.cuda.synchronize()
    views, _ = multigpu.grad_views(buf, model.n, model.rest_bases)
    out = {"v_mean3d": views[0], "v_scale": views[1], "v_quat": views[2], "v_opacity": views[5]}
    return {k: v.cpu().numpy() for k, v in out.items()}


def assert_geometry_grads(eng, run, label=""):
    """Geometry gradients against the oracle's at the gradient bar, every
    entry (no outlier allowance)."""
    n = eng["v_mean3d"].shape[0]
    ref = {"v_mean3d": run.v_mean3d.reshape(n, 3), "v_scale": run.v_scale.reshape(n, 3),
           "v_quat": run.v_quat.reshape(n, 4), "v_opacity": run.v_opacity.reshape(n, 1)}
    for key, want in ref.items():
        bad, worst = close(eng[key], want, GRAD_RTOL, GRAD_ATOL_FRAC)
        print(f"  {label}{key}: out-of-tolerance={bad} worst|diff|/max={worst:.3g}")
        assert bad == 0, f"{label}{key}: {bad} entries out of tolerance (worst {worst:.3g} of max)"
