"""The native trainer (include/msplat_c_api.h on the CUDA engine) against
the reference's own trainer: core/src/msplat_api.mm and model.cpp compiled
from the reference's sources and run on the CPU over the reference's
kernels (oracle/_ref/libmsplat_ref_trainer.so), both driven through the same
C API on the same seeded COLMAP dataset.

Bit-exact before training (initial Gaussians from the point cloud, renders,
RGBA conversion, PLY / .splat / checkpoint bytes); through training the
camera order, learning-rate, SH and resolution schedules, opacity reset and
densification follow the reference step for step, with parameters within
the float-atomic tolerance of the parity tests.  Then the reference's own
Python-level tests (tests/test_msplat.py) on the native GaussianTrainer.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

from msplat_b200 import _lib
from oracle import files
from oracle import trainer as ref_trainer
from tests import dataset_case, harness

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_trainer.available(),
                                 reason="oracle/_ref/libmsplat_ref_trainer.so not built")]


@pytest.fixture(scope="module")
def libs():
    import torch
    assert torch.cuda.is_available()
    _lib.load()
    return ref_trainer.bind(C.CDLL(_lib.LIB_PATH)), ref_trainer.reference()


@pytest.fixture
def colmap(tmp_path):
    dataset_case.write_colmap(str(tmp_path / "scene"), n_points=400)
    return str(tmp_path / "scene")


def _pair(libs, path, **cfg):
    ours, ref = libs
    c = ref_trainer.default_config(**cfg)
    return ref_trainer.Session(ours, path, c), ref_trainer.Session(ref, path, c)


def _ckpt(session, path):
    session.lib.msplat_trainer_save_checkpoint(session.t, str(path).encode())
    return open(path, "rb").read()


def test_initial_state_bit_exact(libs, colmap, tmp_path):
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


def test_training_follows_reference(libs, colmap, tmp_path):
    """13 steps with every schedule active: resolution pyramid (2x until step
    3), SH degree growth every 2 steps, opacity reset at step 3 and a
    densification at step 12."""
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
    ours, ref = libs
    c = ref_trainer.default_config(numDownscales=0, iterations=8)
    a = ref_trainer.Session(ours, colmap, c, eval_mode=True, test_every=3)
    b = ref_trainer.Session(ref, colmap, c, eval_mode=True, test_every=3)
    try:
        assert ours.msplat_dataset_num_test(a.ds) == ref.msplat_dataset_num_test(b.ds) == 3
        for _ in range(4):
            a.step()
            b.step()
        ea, eb = a.evaluate(), b.evaluate()
        assert ea[3:] == eb[3:]
        for x, y in zip(ea[:3], eb[:3]):
            assert abs(x - y) <= 1e-3 * max(1.0, abs(y)), (ea, eb)
        # a reference checkpoint resumes on the engine, and the engine writes it back unchanged
        blob = _ckpt(b, tmp_path / "ref.msplat")
        fresh = ref_trainer.Session(ours, colmap, c, eval_mode=True, test_every=3)
        try:
            assert ours.msplat_trainer_load_checkpoint(fresh.t, str(tmp_path / "ref.msplat").encode()) == 4
            assert ours.msplat_trainer_iteration(fresh.t) == 4
            assert _ckpt(fresh, tmp_path / "again.msplat") == blob
            assert fresh.step()[0] == 5
        finally:
            fresh.close()
    finally:
        a.close()
        b.close()


# ---- the reference's tests/test_msplat.py, on the native Python API -----------------

def test_python_api(colmap, tmp_path):
    from msplat_b200 import Dataset, GaussianTrainer, TrainingConfig, load_dataset, sync
    ds = load_dataset(colmap)
    assert ds.num_train == 8 and ds.num_test == 0
    cfg = TrainingConfig(iterations=10, num_downscales=0)
    assert cfg.sh_degree == 3 and cfg.refine_every == 100
    trainer = GaussianTrainer(ds, cfg)
    for _ in range(5):
        stats = trainer.step()
    assert stats.iteration == 5 and stats.splat_count > 0 and stats.ms_per_step > 0
    img = trainer.render(0)
    sync()
    assert img.ndim == 3 and img.shape[2] == 3 and img.dtype == np.float32
    pose = ds.camera_pose(1)
    assert trainer.render_from_pose(pose, 1).shape == trainer.render(1).shape
    trainer.train(lambda s: None, callback_every=5)
    assert trainer.iteration == 10
    trainer.export_ply(tmp_path / "s.ply")
    trainer.export_splat(tmp_path / "s.splat")
    assert os.path.getsize(tmp_path / "s.ply") > 1000 and os.path.getsize(tmp_path / "s.splat") > 1000
    trainer.save_checkpoint(tmp_path / "c.msplat")
    count = trainer.splat_count
    t2 = GaussianTrainer(Dataset(colmap), TrainingConfig(iterations=20, num_downscales=0))
    t2.load_checkpoint(tmp_path / "c.msplat")
    assert t2.iteration == 10 and t2.splat_count == count
    for _ in range(10):
        s = t2.step()
    assert t2.iteration == 20 and s.splat_count > 0
    with pytest.raises(RuntimeError, match="No test cameras"):
        t2.evaluate()
    ev = GaussianTrainer(Dataset(colmap, eval_mode=True, test_every=4),
                         TrainingConfig(iterations=6, num_downscales=0))
    ev.train(lambda s: None, callback_every=0)
    m = ev.evaluate()
    assert set(m) == {"psnr", "ssim", "l1", "num_test", "num_gaussians"}
    assert m["num_test"] == 2 and 0 < m["ssim"] < 1 and m["l1"] > 0
    with pytest.raises(ValueError):
        TrainingConfig(bg_color=[1, 2])
