"""The reference's own Model, Trainer and C API (core/src/model.cpp,
msplat_api.mm, the loaders), compiled unmodified from its sources over the
CUDA engine through the backend seam msplat_b200/seam/ (bindings.h on the
engine, MTensor on CUDA shared memory: libmsplat_model_cuda.so), against the
same sources over the reference's own kernels on the CPU
(oracle/_ref/libmsplat_ref_trainer.so).  Both are driven through the same C
API on the same seeded COLMAP dataset, as tests/test_trainer_gpu.py drives
the engine's native trainer: bit-exact before training (initial Gaussians,
renders, RGBA, PLY / .splat / checkpoint bytes), then step by step through
every schedule and a densification, with parameters within the
float-atomic tolerance of the parity tests."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

from msplat_b200 import _lib
from msplat_b200.seam import build_seam
from oracle import files
from oracle import trainer as ref_trainer
from tests import dataset_case, harness

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_trainer.available(),
                                 reason="oracle/_ref/libmsplat_ref_trainer.so not built"),
              pytest.mark.skipif(not os.path.exists(build_seam.LIB),
                                 reason="msplat_b200/seam/_build/libmsplat_model_cuda.so not built")]


@pytest.fixture(scope="module")
def libs():
    import torch
    assert torch.cuda.is_available()
    engine = _lib.load()
    return ref_trainer.bind(C.CDLL(build_seam.LIB)), ref_trainer.reference(), engine


@pytest.fixture
def colmap(tmp_path):
    dataset_case.write_colmap(str(tmp_path / "scene"), n_points=400)
    return str(tmp_path / "scene")


def _pair(libs, path, **cfg):
    seam, ref, _ = libs
    c = ref_trainer.default_config(**cfg)
    return ref_trainer.Session(seam, path, c), ref_trainer.Session(ref, path, c)


def _ckpt(session, path):
    session.lib.msplat_trainer_save_checkpoint(session.t, str(path).encode())
    return open(path, "rb").read()


def test_initial_state_bit_exact(libs, colmap, tmp_path):
    engine = libs[2]
    engine.msplat_kernel_launches(1)
    a, b = _pair(libs, colmap, numDownscales=0)
    try:
        assert _ckpt(a, tmp_path / "a.msplat") == _ckpt(b, tmp_path / "b.msplat")
        for i in (0, 3):
            assert a.render(i).tobytes() == b.render(i).tobytes()
        pose = np.eye(4, dtype=np.float32)
        pose[:3, 3] = (0.1, -0.2, 1.5)
        assert a.render_pose(pose, 2).tobytes() == b.render_pose(pose, 2).tobytes()
        assert a.render_rgba(pose, 2).tobytes() == b.render_rgba(pose, 2).tobytes()
        for ext, fn in ((".ply", "msplat_trainer_export_ply"), (".splat", "msplat_trainer_export_splat")):
            getattr(a.lib, fn)(a.t, str(tmp_path / f"a{ext}").encode())
            getattr(b.lib, fn)(b.t, str(tmp_path / f"b{ext}").encode())
            assert (tmp_path / f"a{ext}").read_bytes() == (tmp_path / f"b{ext}").read_bytes()
    finally:
        a.close()
        b.close()
    # the renders ran on the B200 engine (same library instance as this process's)
    assert engine.msplat_kernel_launches(0) > 0


def test_training_follows_reference(libs, colmap, tmp_path):
    """13 steps with every schedule active: resolution pyramid (2x until step
    3), SH degree growth every 2 steps, opacity reset at step 3 (the
    reference's host loop over the shared opacities) and a densification at
    step 12 (the engine's densify on the Model's buffers)."""
    cfg = dict(iterations=100, numDownscales=1, resolutionSchedule=3, shDegreeInterval=2,
               refineEvery=3, warmupLength=1, resetAlphaEvery=5, densifyGradThresh=1e-6)
    a, b = _pair(libs, colmap, **cfg)
    try:
        for _ in range(13):
            sa, sb = a.step(), b.step()
            assert sa[0] == sb[0]
            assert sa[1] == sb[1], (sa, sb)
        assert sa[1] != 400   # densified
        pa = files.read_checkpoint(_ckpt(a, tmp_path / "a.msplat"))
        pb = files.read_checkpoint(_ckpt(b, tmp_path / "b.msplat"))
        for k in ("step", "num_active", "adam_step_count", "adam_lr", "means_lr_init"):
            assert pa[k] == pb[k], k
        for g in range(6):
            bad, worst = harness.close(pa["params"][g], pb["params"][g], 1e-3, 1e-4)
            assert bad <= max(3, pa["params"][g].size // 500_000), (g, bad, worst)
    finally:
        a.close()
        b.close()


def test_evaluate_and_resume(libs, colmap, tmp_path):
    seam, ref, _ = libs
    c = ref_trainer.default_config(numDownscales=0, iterations=8)
    a = ref_trainer.Session(seam, colmap, c, eval_mode=True, test_every=3)
    b = ref_trainer.Session(ref, colmap, c, eval_mode=True, test_every=3)
    try:
        assert seam.msplat_dataset_num_test(a.ds) == ref.msplat_dataset_num_test(b.ds) == 3
        for _ in range(4):
            a.step()
            b.step()
        ea, eb = a.evaluate(), b.evaluate()
        assert ea[3:] == eb[3:]
        for x, y in zip(ea[:3], eb[:3]):
            assert abs(x - y) <= 1e-3 * max(1.0, abs(y)), (ea, eb)
        # a checkpoint of the reference's CPU build resumes on the seam build
        blob = _ckpt(b, tmp_path / "ref.msplat")
        fresh = ref_trainer.Session(seam, colmap, c, eval_mode=True, test_every=3)
        try:
            assert seam.msplat_trainer_load_checkpoint(fresh.t, str(tmp_path / "ref.msplat").encode()) == 4
            assert seam.msplat_trainer_iteration(fresh.t) == 4
            assert _ckpt(fresh, tmp_path / "again.msplat") == blob
            assert fresh.step()[0] == 5
        finally:
            fresh.close()
    finally:
        a.close()
        b.close()
