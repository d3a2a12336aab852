"""Camera set-up of the training step, in float32 like the reference host.

`prepare_camera` restates Model::prepareCam (core/src/model.cpp:490-534):
view matrix from a camera-to-world pose with the OpenGL->OpenCV column flip
(:502-509), projection * view with near 0.001 and far 1000 (:510-513),
degrees_to_use = min(step // sh_degree_interval, sh_degree) (:523) and the
16x16 tile bounds (:525-527).  Every operation is float32, in the
reference's order, so the matrices match a C++ build of the same routine.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

f32 = np.float32


@dataclass
class Camera:
    """Pinhole camera: intrinsics in pixels and a 4x4 row-major OpenGL
    camera-to-world pose (the layout of Camera::camToWorld)."""
    width: int
    height: int
    fx: float
    fy: float
    cx: float
    cy: float
    cam_to_world: np.ndarray = field(default_factory=lambda: np.eye(4, dtype=np.float32))


@dataclass
class CamSetup:
    """Model::CamSetup plus the matrices kept in Camera's cache."""
    fx: float
    fy: float
    cx: float
    cy: float
    height: int
    width: int
    degree: int
    degrees_to_use: int
    tile_bounds: tuple
    cam_pos: np.ndarray
    viewmat: np.ndarray   # (16,) float32 row-major
    projmat: np.ndarray   # (16,) float32 row-major proj * view


def _atanf(x) -> np.float32:
    return f32(math.atan(float(f32(x))))


def _tanf(x) -> np.float32:
    return f32(math.tan(float(f32(x))))


def view_and_proj(cam_to_world: np.ndarray, width: int, height: int, fx: float, fy: float):
    """View and projection*view matrices (model.cpp:496-514)."""
    d = np.asarray(cam_to_world, dtype=np.float32).reshape(16)
    fovx = f32(f32(2.0) * _atanf(f32(width) / (f32(2.0) * f32(fx))))
    fovy = f32(f32(2.0) * _atanf(f32(height) / (f32(2.0) * f32(fy))))
    R = np.zeros((3, 3), np.float32)
    T = np.zeros(3, np.float32)
    for i in range(3):
        R[i, 0] = d[i * 4 + 0]
        R[i, 1] = -d[i * 4 + 1]
        R[i, 2] = -d[i * 4 + 2]
        T[i] = d[i * 4 + 3]
    Rinv = R.T.copy()
    Tinv = np.zeros(3, np.float32)
    for i in range(3):
        acc = f32(f32(Rinv[i, 0] * T[0]) + f32(Rinv[i, 1] * T[1]))
        acc = f32(acc + f32(Rinv[i, 2] * T[2]))
        Tinv[i] = -acc
    vm = np.array([Rinv[0, 0], Rinv[0, 1], Rinv[0, 2], Tinv[0],
                   Rinv[1, 0], Rinv[1, 1], Rinv[1, 2], Tinv[1],
                   Rinv[2, 0], Rinv[2, 1], Rinv[2, 2], Tinv[2],
                   0, 0, 0, 1], dtype=np.float32)
    t_p = f32(f32(0.001) * _tanf(f32(0.5) * fovy))
    r_p = f32(f32(0.001) * _tanf(f32(0.5) * fovx))
    n, fz = f32(0.001), f32(1000.0)
    pm = np.array([f32(n / r_p), 0, 0, 0,
                   0, f32(n / t_p), 0, 0,
                   0, 0, f32(f32(fz + n) / f32(fz - n)), f32(-f32(fz * n) / f32(fz - n)),
                   0, 0, 1, 0], dtype=np.float32)
    pvm = np.zeros(16, np.float32)
    for i in range(4):
        for j in range(4):
            acc = f32(0.0)
            for k in range(4):
                acc = f32(acc + f32(pm[i * 4 + k] * vm[k * 4 + j]))
            pvm[i * 4 + j] = acc
    return vm, pvm, T.copy()


def num_sh_bases(degree: int) -> int:
    return {0: 1, 1: 4, 2: 9, 3: 16}.get(degree, 25)


def degree_from_rest_bases(rest_bases: int) -> int:
    """Model::prepareCam: degree from features_rest.size(-2) (model.cpp:524-525)."""
    b = rest_bases + 1
    return 0 if b <= 1 else 1 if b <= 4 else 2 if b <= 9 else 3 if b <= 16 else 4


def prepare_camera(cam: Camera, step: int, sh_degree: int, sh_degree_interval: int,
                   rest_bases: int, downscale: float = 1.0) -> CamSetup:
    sf = f32(downscale)
    fx, fy = f32(f32(cam.fx) / sf), f32(f32(cam.fy) / sf)
    cx, cy = f32(f32(cam.cx) / sf), f32(f32(cam.cy) / sf)
    height = int(f32(cam.height) / sf)
    width = int(f32(cam.width) / sf)
    vm, pvm, pos = view_and_proj(cam.cam_to_world, width, height, fx, fy)
    dtu = min(step // sh_degree_interval, sh_degree)
    return CamSetup(fx=float(fx), fy=float(fy), cx=float(cx), cy=float(cy), height=height,
                    width=width, degree=degree_from_rest_bases(rest_bases), degrees_to_use=dtu,
                    tile_bounds=((width + 15) // 16, (height + 15) // 16, 1), cam_pos=pos,
                    viewmat=vm, projmat=pvm)


def look_at_c2w(position, target=(0.0, 0.0, 0.0), up=(0.0, 1.0, 0.0)) -> np.ndarray:
    """OpenGL camera-to-world pose at `position` looking at `target`
    (camera looks along its -Z axis, +Y up)."""
    p = np.asarray(position, np.float64)
    z = p - np.asarray(target, np.float64)
    z /= np.linalg.norm(z)
    u = np.asarray(up, np.float64)
    if abs(float(np.dot(u, z))) > 0.999:
        u = np.array([0.0, 0.0, 1.0]) if abs(z[2]) < 0.9 else np.array([1.0, 0.0, 0.0])
    x = np.cross(u, z)
    x /= np.linalg.norm(x)
    y = np.cross(z, x)
    m = np.eye(4)
    m[:3, 0], m[:3, 1], m[:3, 2], m[:3, 3] = x, y, z, p
    return m.astype(np.float32)


def pinhole(width: int, height: int, fov_x_deg: float = 60.0) -> tuple:
    """fx = fy from a horizontal field of view; principal point at the centre."""
    fx = width / (2.0 * math.tan(math.radians(fov_x_deg) / 2.0))
    return float(fx), float(fx), width / 2.0, height / 2.0
