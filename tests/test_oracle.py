"""CPU tests of the oracle itself: its exp against float64, the reference's
chunk rule, determinism, thread-count independence and a closed-form
single-Gaussian case."""
from __future__ import annotations

import math

import numpy as np
import pytest

from msplat_b200 import camera, synthetic
from oracle import oracle
from tests import harness


def _ulp_err(got: float, want: float) -> float:
    g = np.float32(got)
    spacing = float(np.spacing(np.float32(want)))
    return abs(float(g) - want) / spacing if spacing > 0 else 0.0


def test_expf_accuracy():
    xs = np.concatenate([np.linspace(-87.0, 88.0, 20001), np.linspace(-6.0, 0.0, 20001),
                         np.array([0.0, -0.0, 1e-8, -1e-8, 0.5, -0.5])]).astype(np.float32)
    worst = max(_ulp_err(oracle.expf(float(x)), math.exp(float(x))) for x in xs)
    assert worst <= 1.0, worst


def test_expf_special_values():
    assert oracle.expf(0.0) == 1.0
    assert oracle.expf(100.0) == math.inf
    assert oracle.expf(-200.0) == 0.0
    assert math.isnan(oracle.expf(float("nan")))
    # subnormal range rounds once
    assert _ulp_err(oracle.expf(-100.0), math.exp(-100.0)) <= 2.0


def test_chunk_rule():
    # msplat_metal.mm:873-889
    assert oracle.chunk_k_max(65_536, 256) == 48
    assert oracle.chunk_k_max(1_000_000, 4346) == 1
    assert oracle.chunk_k_max(100, 399) == 2
    assert oracle.chunk_k_max(10, 4) == 1  # raised to 2, then clamped to ceil(16N/512) = 1
    assert oracle.chunk_k_max(100_000, 100) == 188


def _c0_small():
    g = synthetic.gaussians(4_000, 21, mean_range=1.0, log_scale_mu=math.log(0.03))
    cs = harness.setup_cam(synthetic.front_camera(96, 64, 3.0))
    return g, cs


def test_render_deterministic_and_thread_independent():
    g, cs = _c0_small()
    out = []
    for threads in (1, 4):
        oracle.set_threads(threads)
        run = oracle.Run(cs, g.n)
        run.render(g.groups())
        out.append((run.out_img.copy(), run.final_idx.copy(), run.gaussian_ids[: run.num_isects].copy()))
    oracle.set_threads(0)
    for a, b in zip(out[0], out[1]):
        np.testing.assert_array_equal(a, b)


def test_sorted_order_and_ranges():
    g, cs = _c0_small()
    run = oracle.Run(cs, g.n)
    run.render(g.groups())
    T = cs.tile_bounds[0] * cs.tile_bounds[1]
    tb = run.tile_bins.reshape(T, 2)
    assert tb[0, 0] == 0 and tb[-1, 1] == run.num_isects
    assert (tb[1:, 0] == tb[:-1, 1]).all()
    ids = run.gaussian_ids
    depth_bits = run.depths.view(np.uint32)
    for t in range(T):
        seg = ids[tb[t, 0]:tb[t, 1]]
        keys = (depth_bits[seg].astype(np.uint64) << np.uint64(32)) | seg.astype(np.uint64)
        assert (np.diff(keys.astype(np.float64)) > 0).all() or len(seg) < 2
    # every intersection is a visible Gaussian whose tile rect covers the tile
    assert (run.radii[ids[: run.num_isects]] > 0).all()
    assert run.num_isects == int(run.num_tiles_hit.sum())


def test_single_gaussian_closed_form():
    # One isotropic Gaussian at the origin, camera at distance 3 on +z.
    n = 1
    s = 0.05
    g = synthetic.Gaussians(np.zeros((1, 3), np.float32), np.full((1, 3), math.log(s), np.float32),
                            np.array([[1, 0, 0, 0]], np.float32), np.zeros((1, 3), np.float32),
                            np.zeros((1, 15, 3), np.float32), np.array([[2.0]], np.float32))
    cs = harness.setup_cam(synthetic.front_camera(64, 64, 3.0))
    run = oracle.Run(cs, n)
    run.render(g.groups())
    f = cs.fx
    var = (f * s / 3.0) ** 2 + 0.3
    np.testing.assert_allclose(run.conics, [1 / var, 0.0, 1 / var], rtol=1e-5, atol=1e-7)
    assert run.radii[0] == math.ceil(3 * math.sqrt(var + math.sqrt(max(0.1, 0.0))))
    np.testing.assert_allclose(run.xys, [31.5, 31.5], atol=1e-4)
    # pixel nearest the centre: alpha = sigmoid(2) * exp(-0.5 * d^2 / var)
    img = run.out_img.reshape(64, 64, 3)
    a = 1 / (1 + math.exp(-2.0)) * math.exp(-0.5 * (0.5 ** 2 + 0.5 ** 2) / var)
    bg = np.array(harness.BG)
    want = (0.5 * a + bg * (1 - a))  # dc = 0 -> colour max(0 + 0.5, 0) = 0.5
    np.testing.assert_allclose(img[31, 31], want, rtol=1e-5)
