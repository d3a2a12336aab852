"""Camera set-up (Model::prepareCam restatement) and synthetic generators."""
from __future__ import annotations

import math

import numpy as np

from msplat_b200 import camera, synthetic


def test_front_camera_view_matrix():
    cam = synthetic.front_camera(256, 256, 3.0)
    cs = camera.prepare_camera(cam, step=0, sh_degree=3, sh_degree_interval=1000, rest_bases=15)
    vm = cs.viewmat.reshape(4, 4)
    np.testing.assert_array_equal(vm[:3, :3], np.diag([1, -1, -1]).astype(np.float32))
    np.testing.assert_array_equal(vm[:3, 3], [0, 0, 3])
    assert cs.degrees_to_use == 0 and cs.degree == 3
    assert cs.tile_bounds == (16, 16, 1)
    assert abs(cs.fx - 256 / (2 * math.tan(math.radians(30)))) < 1e-3
    # the origin projects to the principal point minus the half-pixel offset
    p = cs.projmat.reshape(4, 4) @ np.array([0, 0, 0, 1], np.float32)
    assert abs(p[3] - 3.0) < 1e-6


def test_degrees_to_use_schedule():
    cam = synthetic.front_camera(64, 48, 3.0)
    for step, want in ((0, 0), (999, 0), (1000, 1), (2500, 2), (10**6, 3)):
        cs = camera.prepare_camera(cam, step=step, sh_degree=3, sh_degree_interval=1000, rest_bases=15)
        assert cs.degrees_to_use == want


def test_sphere_cameras_look_inward():
    cams = synthetic.fibonacci_cameras(16, 4.0, 64, 48)
    for c in cams:
        cs = camera.prepare_camera(c, step=0, sh_degree=3, sh_degree_interval=1000, rest_bases=15)
        vm = cs.viewmat.reshape(4, 4)
        o = vm @ np.array([0, 0, 0, 1], np.float32)
        assert abs(o[2] - 4.0) < 1e-4 and abs(o[0]) < 1e-4 and abs(o[1]) < 1e-4
        assert abs(np.linalg.norm(cs.cam_pos) - 4.0) < 1e-4


def test_generator_deterministic():
    a = synthetic.gaussians(1000, 0)
    b = synthetic.gaussians(1000, 0)
    for x, y in zip(a.groups(), b.groups()):
        np.testing.assert_array_equal(x, y)
    np.testing.assert_allclose(np.linalg.norm(a.quats, axis=1), 1.0, rtol=1e-6)
    assert a.features_rest.shape == (1000, 15, 3)
    c = synthetic.gaussians(1000, 0, clusters=10)
    assert c.means.shape == (1000, 3)
