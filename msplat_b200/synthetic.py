"""Seeded synthetic scenes and cameras for the benchmark configurations.

The reference benchmarks on mip-NeRF 360 "garden" (1297x840 is its 4x
downscale); that dataset is not available here, so seeded synthetic inputs
with the shapes and distributions of BASELINE.json's configs stand in:

  C0  65,536 G, means U[-1,1]^3, log-scales N(log 0.02, 0.3), 256x256,
      one camera at (0,0,3) looking at the origin, 60 deg horizontal FoV.
  C1  1,000,000 G, means U[-2,2]^3, log-scales N(log 0.01, 0.4), 1297x840,
      16 cameras on a radius-4 Fibonacci sphere looking inward (up = +Y).
  C2  3,000,000 G, 70% from 10 clusters (centres U[-1,1]^3, sigma 0.05),
      30% U[-2,2]^3, log-scales N(log 0.03, 0.5), 1920x1080, distance 3.
  C4  6,000,000 G drawn as C1, 8 cameras at 1920x1080 on the radius-4 sphere.

Common: quats N(0,1)^4 normalised (stored w, x, y, z), opacity logits
N(0,1), SH degree 3 with DC N(0,0.3) and rest N(0,0.05), target U[0,1].
RNG: numpy.random.default_rng(seed), drawn in the order listed in
`gaussians()`.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from .camera import Camera, look_at_c2w, pinhole


@dataclass
class Gaussians:
    means: np.ndarray        # (N,3)
    scales: np.ndarray       # (N,3) log
    quats: np.ndarray        # (N,4) w x y z
    features_dc: np.ndarray  # (N,3)
    features_rest: np.ndarray  # (N,15,3)
    opacities: np.ndarray    # (N,1) logit

    @property
    def n(self) -> int:
        return int(self.means.shape[0])

    def groups(self) -> list:
        return [self.means, self.scales, self.quats, self.features_dc, self.features_rest,
                self.opacities]

    def copy(self) -> "Gaussians":
        return Gaussians(*[g.copy() for g in self.groups()])


def gaussians(n: int, seed: int, mean_range: float = 1.0, log_scale_mu: float = math.log(0.02),
              log_scale_sigma: float = 0.3, sh_degree: int = 3, clusters: int = 0,
              cluster_frac: float = 0.7, cluster_sigma: float = 0.05) -> Gaussians:
    rng = np.random.default_rng(seed)
    f = np.float32
    if clusters > 0:
        centres = rng.uniform(-1.0, 1.0, size=(clusters, 3))
        n_cl = int(round(n * cluster_frac))
        which = rng.integers(0, clusters, size=n_cl)
        m_cl = centres[which] + rng.normal(0.0, cluster_sigma, size=(n_cl, 3))
        m_un = rng.uniform(-2.0, 2.0, size=(n - n_cl, 3))
        means = np.concatenate([m_cl, m_un], axis=0)
        means = means[rng.permutation(n)]
    else:
        means = rng.uniform(-mean_range, mean_range, size=(n, 3))
    scales = rng.normal(log_scale_mu, log_scale_sigma, size=(n, 3))
    q = rng.normal(0.0, 1.0, size=(n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    opac = rng.normal(0.0, 1.0, size=(n, 1))
    dc = rng.normal(0.0, 0.3, size=(n, 3))
    nb = (sh_degree + 1) ** 2 - 1
    rest = rng.normal(0.0, 0.05, size=(n, nb, 3))
    return Gaussians(means.astype(f), scales.astype(f), q.astype(f), dc.astype(f),
                     rest.astype(f), opac.astype(f))


def fibonacci_cameras(count: int, radius: float, width: int, height: int,
                      fov_x_deg: float = 60.0) -> list:
    fx, fy, cx, cy = pinhole(width, height, fov_x_deg)
    cams = []
    golden = math.pi * (3.0 - math.sqrt(5.0))
    for i in range(count):
        y = 1.0 - 2.0 * (i + 0.5) / count
        r = math.sqrt(max(0.0, 1.0 - y * y))
        th = golden * i
        pos = (radius * r * math.cos(th), radius * y, radius * r * math.sin(th))
        cams.append(Camera(width, height, fx, fy, cx, cy, look_at_c2w(pos)))
    return cams


def front_camera(width: int, height: int, distance: float, fov_x_deg: float = 60.0) -> Camera:
    """Camera at (0, 0, distance) looking at the origin: the OpenGL
    camera-to-world rotation is the identity."""
    fx, fy, cx, cy = pinhole(width, height, fov_x_deg)
    c2w = np.eye(4, dtype=np.float32)
    c2w[2, 3] = distance
    return Camera(width, height, fx, fy, cx, cy, c2w)


def target_image(width: int, height: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).uniform(0.0, 1.0, size=(height, width, 3)).astype(np.float32)


CONFIGS = {
    "C0": dict(n=65_536, width=256, height=256, seed=0, mean_range=1.0,
               log_scale_mu=math.log(0.02), log_scale_sigma=0.3, camera="front", distance=3.0),
    "C1": dict(n=1_000_000, width=1297, height=840, seed=0, mean_range=2.0,
               log_scale_mu=math.log(0.01), log_scale_sigma=0.4, camera="sphere", cameras=16,
               radius=4.0),
    "C2": dict(n=3_000_000, width=1920, height=1080, seed=0, mean_range=2.0,
               log_scale_mu=math.log(0.03), log_scale_sigma=0.5, camera="front", distance=3.0,
               clusters=10),
    "C4": dict(n=6_000_000, width=1920, height=1080, seed=0, mean_range=2.0,
               log_scale_mu=math.log(0.01), log_scale_sigma=0.4, camera="sphere", cameras=8,
               radius=4.0),
    # C4 at a quarter of the Gaussians and a quarter of the pixels, with
    # twice the scales (the same radii in pixels at half the focal length):
    # the same intersections per tile (~4,000) on a quarter of the tiles --
    # a case small enough for detailed profiler captures of C4's per-tile
    # kernels
    "C4q": dict(n=1_500_000, width=960, height=540, seed=0, mean_range=2.0,
                log_scale_mu=math.log(0.02), log_scale_sigma=0.4, camera="sphere", cameras=8,
                radius=4.0),
}


def scene(name: str, n: int | None = None, width: int | None = None,
          height: int | None = None, seed: int | None = None):
    """(gaussians, cameras) for a named config, optionally resized."""
    c = dict(CONFIGS[name])
    n = c["n"] if n is None else n
    w = c["width"] if width is None else width
    h = c["height"] if height is None else height
    s = c["seed"] if seed is None else seed
    g = gaussians(n, s, mean_range=c["mean_range"], log_scale_mu=c["log_scale_mu"],
                  log_scale_sigma=c["log_scale_sigma"], clusters=c.get("clusters", 0))
    if c["camera"] == "front":
        cams = [front_camera(w, h, c["distance"])]
    else:
        cams = fibonacci_cameras(c["cameras"], c["radius"], w, h)
    return g, cams
