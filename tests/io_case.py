"""Seeded Gaussian sets for the model-file tests (checkpoint, PLY, .splat):
values spread past every clamp the .splat writer applies (colours, quaternion
components and opacities out of range) so the byte conversions are all
exercised."""
from __future__ import annotations

import numpy as np

from oracle import files

# name: (gaussians, SH-rest bases, seed, keep_crs, crs scale, crs translation)
CASES = {
    "deg3": (37, 15, 21, False, 1.0, (0.0, 0.0, 0.0)),
    "deg2_crs": (29, 8, 22, True, 0.37, (12.5, -3.25, 101.0)),
    "deg0": (11, 0, 23, False, 1.0, (0.0, 0.0, 0.0)),
}


def gaussians(n: int, rest_bases: int, seed: int):
    rng = np.random.default_rng(seed)
    shapes = files.group_shapes(n, rest_bases)
    means = rng.normal(0, 2.0, shapes[0])
    scales = rng.normal(np.log(0.05), 1.0, shapes[1])
    quats = rng.normal(0, 0.8, shapes[2])          # components beyond +-1 hit the u8 clamp
    dc = rng.normal(0, 2.5, shapes[3])              # colours beyond [0, 1] hit the clamp
    rest = rng.normal(0, 0.3, shapes[4])
    op = rng.normal(0, 4.0, shapes[5])
    return [np.ascontiguousarray(a, np.float32) for a in (means, scales, quats, dc, rest, op)]


def moments(params, seed: int):
    rng = np.random.default_rng(seed + 1000)
    m = [rng.normal(0, 1e-3, a.shape).astype(np.float32) for a in params]
    v = [np.abs(rng.normal(0, 1e-6, a.shape)).astype(np.float32) for a in params]
    return m, v
