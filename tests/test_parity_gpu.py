"""Parity of the CUDA engine (called through its C-ABI) against the CPU
oracle on identical seeded inputs.

Bars (north star): per-tile intersection counts and per-tile sorted id lists
bit-exact; the forward (image, final T, last index) bit-exact, which is
stricter than the 1e-5 absolute image bar; v_rendered bit-exact; raster
gradients and Adam-updated parameters within 1e-4 relative plus a small
absolute floor (the backward sums with float atomics in a different order
than the oracle's double-precision sums).

Parameters and moments may have a few outliers (PARAM_OUTLIER_FRAC of the
tensor, at least 3, none beyond 1e-4 of the tensor's max): Adam's update
lr * g / (|g| + eps) amplifies ulp-level differences of a gradient that is
within a few eps of zero without bound, so no two implementations that
round differently agree there to 1e-4.  The gradients themselves have no
such allowance.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from msplat_b200 import _lib, camera, engine, synthetic
from oracle import oracle
from tests import harness

pytestmark = pytest.mark.gpu

GRAD_RTOL = harness.GRAD_RTOL            # 1e-4
GRAD_ATOL_FRAC = harness.GRAD_ATOL_FRAC  # absolute floor, as a fraction of the tensor's max |value|
PARAM_RTOL = 1e-4
PARAM_OUTLIER_FRAC, PARAM_OUTLIER_CAP = 2e-6, 1e-4


@pytest.fixture(scope="module", autouse=True)
def gpu():
    import torch
    assert torch.cuda.is_available(), "GPU parity tests need a CUDA device"
    engine.bind_stream()
    yield
    from msplat_b200 import _lib
    _lib.load().cleanup_msplat_cuda()


def _warm(model, cam_setup, warm):
    """warm: one render whose read-back (the view's largest tile) the next
    call sees, so tiles of more than 2,048 keys sort their nearest keys
    only.  Otherwise the engine is cleaned up first: no earlier view, every
    list sorted whole."""
    import torch
    if warm:
        engine.render(model, cam_setup)
        torch.cuda.synchronize()
    else:
        _lib.load().cleanup_msplat_cuda()


def _render_pair(g, cam_setup, warm=False):
    model = engine.GaussianModel(g.groups())
    _warm(model, cam_setup, warm)
    engine.render(model, cam_setup)
    eng = harness.engine_forward_dump(g.n, cam_setup)
    # room for scenes of many intersections per Gaussian (the oracle does
    # not grow its buffer)
    run = oracle.Run(cam_setup, g.n, isect_capacity=64 * max(g.n, 1))
    run.render(g.groups())
    return run, eng


def _scene(n, w, h, seed=0, mean_range=1.0, log_mu=math.log(0.02), log_sigma=0.3, distance=3.0,
           clusters=0):
    g = synthetic.gaussians(n, seed, mean_range=mean_range, log_scale_mu=log_mu,
                            log_scale_sigma=log_sigma, clusters=clusters)
    cam = synthetic.front_camera(w, h, distance)
    return g, harness.setup_cam(cam)


def test_render_c0_chunked_bitexact():
    g, cams = synthetic.scene("C0")
    cs = harness.setup_cam(cams[0])
    run, eng = _render_pair(g, cs)
    assert run.P.k_max > 1  # 256 tiles < 400: the chunked path
    assert run.S.max_tile_count > 2048  # C0 exceeds the reference's per-tile cap
    harness.assert_forward_bitexact(run, eng, cs)


def test_render_monolithic_bitexact():
    g, cs = _scene(40_000, 640, 480, seed=3)
    run, eng = _render_pair(g, cs)
    assert run.P.k_max == 1
    harness.assert_forward_bitexact(run, eng, cs)


def test_render_ragged_image_bitexact():
    g, cs = _scene(6_000, 100, 75, seed=4)
    run, eng = _render_pair(g, cs)
    harness.assert_forward_bitexact(run, eng, cs)


def test_render_sphere_camera_bitexact():
    g = synthetic.gaussians(60_000, 5, mean_range=2.0, log_scale_mu=math.log(0.01),
                            log_scale_sigma=0.4)
    cams = synthetic.fibonacci_cameras(16, 4.0, 648, 420)
    for cam in cams[:3]:
        cs = harness.setup_cam(cam)
        run, eng = _render_pair(g, cs)
        harness.assert_forward_bitexact(run, eng, cs)


def test_big_tiles_merge_sort_bitexact():
    # Everything piles into a few tiles: lists longer than the 4096-key
    # shared-memory sort take the merge path.
    g, cs = _scene(30_000, 320, 240, seed=6, clusters=2, log_mu=math.log(0.03), log_sigma=0.5)
    run, eng = _render_pair(g, cs)
    assert run.S.max_tile_count > 4096
    harness.assert_forward_bitexact(run, eng, cs)


@pytest.mark.parametrize("levels", [1, 3])
def test_tied_depths_sort_bitexact(levels):
    # Every mean on one of `levels` planes facing the camera: most tiles hold
    # long runs of keys with the same depth, whose order is the ids' (the
    # radix sort of depths reports runs longer than it orders itself and
    # those tiles take the bitonic sort of the full (depth, id) keys).  One
    # level: every key of a tile ties.
    g, cs = _scene(20_000, 640, 480, seed=9, log_mu=math.log(0.03))
    planes = np.linspace(-0.2, 0.2, levels).astype(np.float32)
    g.means[:, 2] = planes[np.arange(g.n) % levels]
    run, eng = _render_pair(g, cs)
    counts = np.diff(run.tile_bins.reshape(-1, 2), axis=1)[:, 0]
    assert run.P.k_max == 1 and (counts > 128).sum() > 100
    harness.assert_forward_bitexact(run, eng, cs)
    depths = run.depths[run.radii > 0]
    assert len(np.unique(depths)) == levels


def test_distinct_depths_radix_sizes_bitexact():
    # Tiles from a few keys up to the 2,048 the shared-memory sorts hold
    # (radix above 128 keys, bitonic at or below), distinct depths.
    g, cs = _scene(60_000, 640, 480, seed=10, log_mu=math.log(0.025), log_sigma=0.5)
    run, eng = _render_pair(g, cs)
    counts = np.diff(run.tile_bins.reshape(-1, 2), axis=1)[:, 0]
    assert 1024 < run.S.max_tile_count <= 2048
    assert ((counts > 0) & (counts <= 128)).sum() > 100 and (counts > 1024).sum() > 100
    harness.assert_forward_bitexact(run, eng, cs)


@pytest.mark.parametrize("warm", [False, True])
@pytest.mark.parametrize("levels", [0, 20_000, 60])
def test_sort_sizes_and_depth_ties_bitexact(levels, warm):
    # Tiles of 129-2,048 keys (128-thread radix sort) and 2,049-6,400 keys
    # (512-thread radix sort).  levels = 0: distinct means, yet most large
    # tiles hold a few equal depths (a tile of 4,000 float depths usually
    # does); 20,000 depth planes: runs of up to ~6 equal depths, put in id
    # order inside the radix sorts; 60 planes: runs of ~100, longer than the
    # radix sorts order, so those tiles fall back to the bitonic (small) and
    # merge (large) sorts of the full (depth, id) keys.  warm: the tiles of
    # more than 2,048 keys sort their nearest keys instead (prefixes with the
    # same ties), falling back to whole sorts where the ties refuse them.
    g, cs = _scene(250_000, 640, 480, seed=12, log_mu=math.log(0.03), log_sigma=0.5)
    if levels:
        planes = np.linspace(-0.5, 0.5, levels).astype(np.float32)
        g.means[:, 2] = planes[np.arange(g.n) % levels]
    run, eng = _render_pair(g, cs, warm=warm)
    counts = np.diff(run.tile_bins.reshape(-1, 2), axis=1)[:, 0]
    assert run.P.k_max == 1
    assert ((counts > 128) & (counts <= 2048)).sum() > 100
    assert ((counts > 2048) & (counts <= 8192)).sum() > 100
    harness.assert_forward_bitexact(run, eng, cs)


def _clustered_scene():
    return _scene(150_000, 640, 480, seed=12, log_mu=math.log(0.03), log_sigma=0.5, clusters=2)


@pytest.mark.parametrize("prefix", [False, True])
def test_sort_tiles_beyond_large_radix_bitexact(prefix):
    # Two dense clusters: tiles of more than 8,192 keys beside tiles the two
    # radix sorts take, single-pass raster.  With no earlier view (the
    # engine just cleaned up) the long lists are sorted whole (merge path);
    # after a view that had such tiles they sort only their nearest keys,
    # and every pixel terminates inside those.
    g, cs = _clustered_scene()
    run, eng = _render_pair(g, cs, warm=prefix)
    counts = np.diff(run.tile_bins.reshape(-1, 2), axis=1)[:, 0]
    assert run.P.k_max == 1 and (counts > 8192).sum() > 10
    assert ((counts > 2048) & (counts <= 8192)).sum() > 10
    harness.assert_forward_bitexact(run, eng, cs)
    srt = engine.debug_buffer("tile_sorted", counts.size, np.int32)
    assert bool(_lib.load().msplat_last_binning() & 1) == prefix
    if prefix:
        assert (srt < counts).sum() > 10  # prefixes in use
    else:
        np.testing.assert_array_equal(srt, counts)


def test_long_tiles_after_a_light_view_bitexact():
    # A view whose tiles all hold at most 2,048 keys, then the two-cluster
    # scene: the engine launches neither the 512-thread radix sort nor the
    # nearest-key sort for it, so every tile of more than 2,048 keys takes
    # the merge path whole.
    import torch
    _lib.load().cleanup_msplat_cuda()
    lg, lcs = _scene(6_000, 100, 75, seed=4)
    engine.render(engine.GaussianModel(lg.groups()), lcs)
    torch.cuda.synchronize()
    g, cs = _clustered_scene()
    model = engine.GaussianModel(g.groups())
    engine.render(model, cs)
    assert _lib.load().msplat_last_binning() == 0
    eng = harness.engine_forward_dump(g.n, cs)
    run = oracle.Run(cs, g.n, isect_capacity=64 * g.n)
    run.render(g.groups())
    counts = np.diff(run.tile_bins.reshape(-1, 2), axis=1)[:, 0]
    assert ((counts > 2048) & (counts <= 8192)).sum() > 10 and (counts > 8192).sum() > 10
    harness.assert_forward_bitexact(run, eng, cs)


def test_long_tiles_after_a_mid_view_bitexact():
    # A view whose largest tile holds 2,049-8,192 keys, then the two-cluster
    # scene: the mid-size tiles sort their nearest keys, but the kernel for
    # tiles above 8,192 keys is not launched, so those take the merge path
    # whole.
    import torch
    _lib.load().cleanup_msplat_cuda()
    mg, mcs = _scene(250_000, 640, 480, seed=12, log_mu=math.log(0.03), log_sigma=0.5)
    engine.render(engine.GaussianModel(mg.groups()), mcs)
    torch.cuda.synchronize()
    g, cs = _clustered_scene()
    model = engine.GaussianModel(g.groups())
    engine.render(model, cs)
    assert _lib.load().msplat_last_binning() & 1
    eng = harness.engine_forward_dump(g.n, cs)
    run = oracle.Run(cs, g.n, isect_capacity=64 * g.n)
    run.render(g.groups())
    harness.assert_forward_bitexact(run, eng, cs)
    counts = np.diff(run.tile_bins.reshape(-1, 2), axis=1)[:, 0]
    srt = engine.debug_buffer("tile_sorted", counts.size, np.int32)
    huge = counts > 8192
    assert huge.sum() > 10
    np.testing.assert_array_equal(srt[huge], counts[huge])
    mid = (counts > 2048) & (counts <= 8192)
    # prefixes in use (a mid tile whose pixels walk past ~1,024 keys is
    # flagged by the raster and sorted whole)
    assert (srt[mid] < counts[mid]).sum() > 0


def test_prefix_overrun_sorts_whole_tiles_bitexact():
    # The same clusters, nearly transparent (alpha about 0.0045 at a
    # Gaussian's centre): no pixel reaches T = 1e-4, every pixel of a long
    # list runs past its sorted prefix, so the forward flags those tiles,
    # sorts them whole and rasterizes them again.
    g, cs = _clustered_scene()
    g.opacities[:] = np.float32(math.log(0.0045 / (1 - 0.0045)))
    run, eng = _render_pair(g, cs, warm=True)
    counts = np.diff(run.tile_bins.reshape(-1, 2), axis=1)[:, 0]
    assert (counts > 8192).sum() > 10
    harness.assert_forward_bitexact(run, eng, cs)
    srt = engine.debug_buffer("tile_sorted", counts.size, np.int32)
    np.testing.assert_array_equal(srt, counts)  # every tile sorted whole in the end


@pytest.mark.parametrize("mean_range", [1.0, 2.0])
def test_dense_binning_bitexact(mean_range):
    # Large Gaussians, 34-41 intersections each (rects of up to ~100 tiles):
    # after a warm view the projection counts the large rects by the corners
    # of a 2D difference array, which the scan sums back into counts.
    # mean_range 2: rects reach the image's last tile row and column, whose
    # outer corners are dropped.  Tile ranges, sorted lists and image
    # bit-exact.
    log_mu = math.log(0.06) if mean_range == 1.0 else math.log(0.08)
    g, cs = _scene(40_000, 640, 480, seed=3, mean_range=mean_range, log_mu=log_mu, log_sigma=0.5)
    run, eng = _render_pair(g, cs, warm=True)
    assert run.num_isects > 16 * g.n
    assert _lib.load().msplat_last_binning() & 2
    harness.assert_forward_bitexact(run, eng, cs)


def test_render_all_culled():
    g, cs = _scene(1_000, 64, 64, seed=7, distance=-3.0)  # everything behind the camera
    run, eng = _render_pair(g, cs)
    assert (run.radii == 0).all()
    harness.assert_forward_bitexact(run, eng, cs)
    img = eng["img"].reshape(64, 64, 3)
    np.testing.assert_allclose(img, np.broadcast_to(np.float32(engine.DEFAULT_BG), img.shape))


def test_render_single_gaussian():
    g, cs = _scene(1, 48, 48, seed=8, mean_range=0.01)
    run, eng = _render_pair(g, cs)
    harness.assert_forward_bitexact(run, eng, cs)


# ---------------------------------------------------------------------------
# Training steps
# ---------------------------------------------------------------------------

def _train_pair(g, cs, gt, steps=1, dtu=None, ssim_weight=0.2, warm=False):
    import torch
    if dtu is not None:
        cs.degrees_to_use = dtu
    model = engine.GaussianModel(g.groups())
    _warm(model, cs, warm)
    gt_dev = torch.as_tensor(gt).cuda().contiguous()
    params = [x.copy() for x in g.groups()]
    m = [np.zeros_like(x) for x in params]
    v = [np.zeros_like(x) for x in params]
    st = [np.zeros(g.n, np.float32) for _ in range(3)]
    for _ in range(steps):
        engine.train_step(model, cs, gt_dev, ssim_weight=ssim_weight)
        steps_sz, bc2 = model.adam_scalars()
        run = oracle.Run(cs, g.n, ssim_weight=ssim_weight, adam_steps=steps_sz, adam_bc2=bc2,
                         isect_capacity=64 * max(g.n, 1))
        run.train_step(params, m, v, gt, *st)
    torch.cuda.synchronize()
    return model, run, params, m, v, st


def _report(label, bad, worst):
    print(f"  {label}: out-of-tolerance={bad} worst|diff|/max={worst:.3g}")


def _check_train(model, run, params, m, v, st, cs, check_grads=True, exact_forward=True):
    n = model.n
    P = cs.width * cs.height
    v_rend = engine.debug_buffer("v_rendered", 3 * P, np.float32)
    if exact_forward:
        # one step from identical inputs: the loss gradient is bit-exact
        np.testing.assert_array_equal(v_rend, run.v_rendered)
    else:
        bad, worst = harness.close(v_rend, run.v_rendered, 1e-3, 1e-4)
        _report("v_rendered", bad, worst)
        assert bad <= max(1, P // 2000)
    vis = run.radii > 0
    if check_grads:
        ga = engine.debug_buffer("grad_acc", 9 * n, np.float32).reshape(n, 9)
        for name, eng_cols, ref in (("v_rgb", ga[:, 0:3], run.v_rgb.reshape(n, 3)),
                                    ("v_conic", ga[:, 3:6], run.v_conic.reshape(n, 3)),
                                    ("v_xy", ga[:, 6:8], run.v_xy.reshape(n, 2)),
                                    ("v_opacity", ga[:, 8:9], run.v_opacity.reshape(n, 1))):
            bad, worst = harness.close(eng_cols[vis], ref[vis], GRAD_RTOL, GRAD_ATOL_FRAC)
            _report(name, bad, worst)
            assert bad == 0, f"{name}: {bad} entries out of tolerance (worst {worst:.3g} of max)"
    names = ("means", "scales", "quats", "features_dc", "features_rest", "opacities")
    for gi, name in enumerate(names):
        e_p = model.params[gi].cpu().numpy()
        e_m = model.exp_avg[gi].cpu().numpy()
        e_v = model.exp_avg_sq[gi].cpu().numpy()
        for label, a, b in (("param", e_p, params[gi]), ("exp_avg", e_m, m[gi]),
                            ("exp_avg_sq", e_v, v[gi])):
            bad, worst = harness.close(a, b, PARAM_RTOL, 1e-6)
            _report(f"{name}.{label}", bad, worst)
            allowed = max(3, int(PARAM_OUTLIER_FRAC * a.size))
            assert bad <= allowed and worst <= PARAM_OUTLIER_CAP, (
                f"{name}.{label}: {bad} out of tolerance (allowed {allowed}), worst {worst:.3g}")
    for label, a, b in (("vis_counts", model.vis_counts, st[0]), ("grad_norm", model.xys_grad_norm, st[1]),
                        ("max_2d", model.max_2d_size, st[2])):
        bad, worst = harness.close(a.cpu().numpy(), b, GRAD_RTOL, GRAD_ATOL_FRAC)
        assert bad == 0, f"{label}: {bad} out of tolerance (worst {worst:.3g})"


def _check_geometry_grads(g, cs, gt, run, ssim_weight=0.2):
    """The projection VJP's outputs (v_mean3d, v_scale, v_quat) and the
    opacity gradient before Adam, from msplat_train_step_grads on the same
    inputs, against the oracle's first step at the gradient bar, every entry."""
    import torch
    eng = harness.engine_geometry_grads(g.groups(), cs, torch.as_tensor(gt).cuda().contiguous(),
                                        ssim_weight)
    harness.assert_geometry_grads(eng, run)


def test_train_step_c0():
    g, cams = synthetic.scene("C0")
    cs = harness.setup_cam(cams[0])
    gt = synthetic.target_image(cs.width, cs.height, 1)
    out = _train_pair(g, cs, gt)
    _check_train(*out, cs)
    run = out[1]
    assert abs(_lib.load().msplat_last_loss(1) - run.loss) <= 1e-4 * abs(run.loss)
    _check_geometry_grads(g, cs, gt, run)


def test_train_step_monolithic():
    g, cs = _scene(40_000, 640, 480, seed=9)
    gt = synthetic.target_image(cs.width, cs.height, 2)
    out = _train_pair(g, cs, gt)
    _check_train(*out, cs)
    _check_geometry_grads(g, cs, gt, out[1])


@pytest.mark.parametrize("dtu", [0, 1, 2])
def test_train_step_partial_sh(dtu):
    g, cs = _scene(8_000, 160, 120, seed=10 + dtu)
    gt = synthetic.target_image(cs.width, cs.height, 3)
    out = _train_pair(g, cs, gt, dtu=dtu)
    _check_train(*out, cs)
    _check_geometry_grads(g, cs, gt, out[1])


def test_train_three_steps():
    g, cs = _scene(20_000, 480, 320, seed=12)
    gt = synthetic.target_image(cs.width, cs.height, 4)
    _check_train(*_train_pair(g, cs, gt, steps=3), cs, check_grads=False, exact_forward=False)


def test_train_step_prefix_sorted_tiles():
    # Long lists that sort only their nearest keys: the backward walks the
    # same prefixes.
    g, cs = _clustered_scene()
    gt = synthetic.target_image(cs.width, cs.height, 6)
    out = _train_pair(g, cs, gt, warm=True)
    counts = np.diff(out[1].tile_bins.reshape(-1, 2), axis=1)[:, 0]
    srt = engine.debug_buffer("tile_sorted", counts.size, np.int32)
    assert (srt < counts).sum() > 10
    _check_train(*out, cs)
    _check_geometry_grads(g, cs, gt, out[1])


def test_train_step_dense_binning():
    # ~24 intersections per Gaussian, rects reaching the image borders
    g, cs = _scene(20_000, 480, 320, seed=5, mean_range=2.0, log_mu=math.log(0.1), log_sigma=0.4)
    gt = synthetic.target_image(cs.width, cs.height, 7)
    out = _train_pair(g, cs, gt, warm=True)
    assert _lib.load().msplat_last_binning() & 2
    _check_train(*out, cs)
    _check_geometry_grads(g, cs, gt, out[1])


def test_train_step_l1_only():
    g, cs = _scene(8_000, 128, 96, seed=13)
    gt = synthetic.target_image(cs.width, cs.height, 5)
    out = _train_pair(g, cs, gt, ssim_weight=0.0)
    _check_train(*out, cs)
    _check_geometry_grads(g, cs, gt, out[1], ssim_weight=0.0)
