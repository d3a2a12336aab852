"""A seeded densification input shared by the CPU and GPU densify tests:
Gaussians with their Adam state in buffers of 3N rows, densification
statistics that put some Gaussians above the gradient threshold, and the
standard-normal samples for split children."""
from __future__ import annotations

import math

import numpy as np

from msplat_b200 import synthetic


def make(n: int, seed: int, rest_bases: int = 15):
    g = synthetic.gaussians(n, seed, mean_range=1.0, log_scale_mu=math.log(0.02),
                            log_scale_sigma=0.8)
    rng = np.random.default_rng(seed + 100)
    groups = [np.asarray(a, np.float32).reshape(n, -1) for a in g.groups()]
    groups[4] = groups[4][:, :3 * rest_bases]
    cap = 3 * n
    bufs, ea, es = [], [], []
    for a in groups:
        b = np.zeros((cap,) + a.shape[1:], np.float32)
        b[:n] = a
        bufs.append(b)
        m = np.zeros_like(b)
        m[:n] = rng.normal(0, 0.01, a.shape).astype(np.float32)
        v = np.zeros_like(b)
        v[:n] = np.abs(rng.normal(0, 0.01, a.shape)).astype(np.float32)
        ea.append(m)
        es.append(v)
    # opacity logits spread across the 0.1 cull threshold
    bufs[5][:n, 0] = rng.normal(-1.0, 1.5, n).astype(np.float32)
    vis = rng.integers(0, 6, n).astype(np.float32)
    gnorm = (rng.gamma(1.0, 0.15, n) * vis).astype(np.float32)
    max2d = rng.uniform(0.0, 0.3, n).astype(np.float32)
    samples = rng.standard_normal((2 * n, 3)).astype(np.float32)
    return bufs, ea, es, gnorm, vis, max2d, samples
