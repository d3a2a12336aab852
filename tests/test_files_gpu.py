"""Model files from and to device buffers: a checkpoint of a training model
reloads bit-exact (parameters, Adam moments, step count, learning rates)
and training resumes from it (the reference's test_checkpoint_save_load /
test_checkpoint_resume_training); PLY and .splat exports of device
parameters match the reference's writers on the same values; a PLY loads
back onto the device."""
from __future__ import annotations

import os

import numpy as np
import pytest

from msplat_b200 import engine, synthetic
from oracle import files
from tests import harness, io_case
from tests.test_files import eng_load_ply

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "io")


@pytest.fixture(scope="module", autouse=True)
def gpu():
    import torch
    assert torch.cuda.is_available(), "model-file GPU tests need a CUDA device"
    engine.bind_stream()
    yield


def _trained(steps=4):
    import torch
    g, cams = synthetic.scene("C0", n=6000)
    cs = harness.setup_cam(cams[0])
    gt = torch.as_tensor(synthetic.target_image(cs.width, cs.height, 1), device="cuda")
    model = engine.GaussianModel(g.groups())
    for step in range(1, steps + 1):
        model.schedule_means_lr(step, 1000)
        engine.train_step(model, cs, gt)
    return model, cs, gt


def _host(ts):
    return [t.detach().cpu().numpy() for t in ts]


def test_checkpoint_save_load_resume(tmp_path):
    import torch
    model, cs, gt = _trained(4)
    path = tmp_path / "m.msplat"
    model.save_checkpoint(path, 4)
    p, m, v = _host(model.params), _host(model.exp_avg), _host(model.exp_avg_sq)
    assert path.read_bytes() == files.checkpoint_bytes(
        4, model.n, model.sh_degree, model.step_count, model.lr, model.means_lr_init,
        model.means_lr_final, p, m, v)
    loaded, step = engine.GaussianModel.load_checkpoint(path)
    assert step == 4 and loaded.n == model.n and loaded.capacity == 4 * model.n
    assert loaded.step_count == model.step_count and loaded.sh_degree == model.sh_degree
    assert loaded.lr == [float(np.float32(x)) for x in model.lr]
    for got, want in zip((loaded.params, loaded.exp_avg, loaded.exp_avg_sq), (p, m, v)):
        for a, b in zip(_host(got), want):
            assert a.tobytes() == b.tobytes()
    # resume: one more step on each gives the same loss (the forward is
    # deterministic) and parameters within the float-atomic tolerance
    l0 = engine.train_step(model, cs, gt)
    l1 = engine.train_step(loaded, cs, gt)
    torch.cuda.synchronize()
    assert l0 == l1
    for a, b in zip(_host(loaded.params), _host(model.params)):
        bad, _ = harness.close(a, b, 1e-5, 1e-6)
        assert bad <= 3


def test_exports_match_reference(tmp_path):
    import torch
    model, *_ = _trained(3)
    model.keep_crs, model.crs_scale, model.crs_translation = True, 0.42, (3.5, -7.0, 11.25)
    model.save(tmp_path / "d.ply", 3)
    model.save(tmp_path / "d.splat", 3)
    torch.cuda.synchronize()
    host = _host(model.params)
    if files.RefIO.available():
        ref = files.RefIO()
        ref.save_ply(tmp_path / "r.ply", 3, host, True, 0.42, (3.5, -7.0, 11.25))
        ref.save_splat(tmp_path / "r.splat", host, True, 0.42, (3.5, -7.0, 11.25))
        assert (tmp_path / "d.ply").read_bytes() == (tmp_path / "r.ply").read_bytes()
        assert (tmp_path / "d.splat").read_bytes() == (tmp_path / "r.splat").read_bytes()
    model.keep_crs = False
    model.save_ply(tmp_path / "p.ply", 3)
    assert (tmp_path / "p.ply").read_bytes() == files.ply_bytes(3, host)
    assert os.path.getsize(tmp_path / "d.splat") == 32 * model.n


@pytest.mark.parametrize("name", sorted(io_case.CASES))
def test_load_ply_onto_device(name):
    n, rb, seed, keep, scale, trans = io_case.CASES[name]
    model, step = engine.GaussianModel.load_ply(os.path.join(GOLDEN, f"{name}.ply"), "cuda", keep,
                                                scale, trans)
    assert step == 0 and model.n == n and model.rest_bases == rb and model.capacity == 4 * n
    if files.RefIO.available():
        want, _ = files.RefIO().load_ply(os.path.join(GOLDEN, f"{name}.ply"), n, rb, keep, scale,
                                         trans)
    elif keep:   # the host-memory path of the same reader (pinned on the CPU)
        want, _, _ = eng_load_ply(os.path.join(GOLDEN, f"{name}.ply"), n, rb, keep, scale, trans)
    else:
        want = io_case.gaussians(n, rb, seed)
    for a, b in zip(_host(model.params), want):
        assert a.tobytes() == b.tobytes()
    assert not any(t.any() for t in model.exp_avg + model.exp_avg_sq)
