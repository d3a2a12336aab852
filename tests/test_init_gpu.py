"""Initialisation from a point cloud on the device: the grid k-NN
(msplat_knn_mean_distance) against an exhaustive search with nanoflann's
distance arithmetic (oracle orc_knn_mean_distance), bit-exact, on clouds
that stress the grid -- clusters, a uniform background, far outliers,
duplicate points, flat and collinear sets; then msplat_init_gaussians'
arrays against their definitions."""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import pytest

from msplat_b200 import _lib
from oracle import oracle

pytestmark = pytest.mark.gpu


def _clouds():
    rng = np.random.default_rng(3)
    yield "clusters+uniform+outliers", np.concatenate([
        rng.normal(0, 0.02, (6000, 3)) + rng.uniform(-1, 1, (6000, 3)).round(0),
        rng.uniform(-2, 2, (4000, 3)),
        rng.uniform(-1, 1, (20, 3)) * 500.0,
    ])
    base = rng.uniform(-1, 1, (3000, 3))
    yield "duplicates", np.concatenate([base, base[:500], base[:50]])
    flat = rng.uniform(-1, 1, (5000, 3))
    flat[:, 2] = 0.25
    yield "flat", flat
    line = np.zeros((2000, 3))
    line[:, 0] = rng.uniform(-3, 3, 2000)
    yield "collinear", line
    yield "tiny", rng.uniform(-1, 1, (5, 3))


@pytest.mark.parametrize("name,xyz", list(_clouds()), ids=[c[0] for c in _clouds()])
def test_knn_matches_exhaustive_search(name, xyz):
    import torch
    assert torch.cuda.is_available()
    xyz = np.ascontiguousarray(xyz, np.float32)
    n = xyz.shape[0]
    got = np.zeros(n, np.float32)
    _lib.check(_lib.load().msplat_knn_mean_distance(xyz.ctypes.data, n, 4, got.ctypes.data), "knn")
    want = np.zeros(n, np.float32)
    oracle.load().orc_knn_mean_distance(oracle._fp(xyz), C.c_int64(n), 4, oracle._fp(want))
    assert got.tobytes() == want.tobytes(), (name, np.flatnonzero(got != want)[:5])


def test_init_gaussians_definition():
    import torch
    rng = np.random.default_rng(9)
    n = 3000
    xyz = np.ascontiguousarray(rng.uniform(-1, 1, (n, 3)), np.float32)
    rgb = np.ascontiguousarray(rng.integers(0, 256, (n, 3)), np.uint8)
    out = [torch.zeros(s, device="cuda") for s in ((n, 3), (n, 3), (n, 4), (n, 3), (n, 15, 3), (n, 1))]
    _lib.check(_lib.load().msplat_init_gaussians(
        xyz.ctypes.data, rgb.ctypes.data, n, 3, *[C.c_void_p(t.data_ptr()) for t in out]), "init")
    means, scales, quats, dc, rest, op = (t.cpu().numpy() for t in out)
    assert means.tobytes() == xyz.tobytes()
    dist = np.zeros(n, np.float32)
    oracle.load().orc_knn_mean_distance(oracle._fp(xyz), C.c_int64(n), 4, oracle._fp(dist))
    want_scale = np.array([math.log(float(d)) for d in dist], np.float32)  # logf of a float
    assert np.abs(scales[:, 0] - want_scale).max() <= 1e-6 * np.abs(want_scale).max()
    assert (scales[:, 0] == scales[:, 1]).all() and (scales[:, 1] == scales[:, 2]).all()
    np.testing.assert_allclose(np.linalg.norm(quats, axis=1), 1.0, atol=1e-5)
    want_dc = ((rgb / 255.0 - 0.5) / 0.28209479177387814).astype(np.float32)
    assert dc.tobytes() == want_dc.tobytes()
    assert not rest.any()
    # logit(0.1) = std::log(0.1f / 0.9f), one value for every Gaussian
    assert (op == op[0, 0]).all() and abs(float(op[0, 0]) - math.log(0.1 / 0.9)) < 1e-6
