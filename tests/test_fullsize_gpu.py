"""Parity at the benchmark configurations' full sizes: C1 (1M Gaussians,
1297x840, a sphere camera) and C2 (3M Gaussians, 70% in ten tight clusters,
1920x1080: tiles with several thousand Gaussians, sorted by the merge path).
Forward: radii, centres, depths, conics, colours, tile ranges, per-tile
sorted id lists, image, final T and final index bit-exact with the CPU
oracle.  Training step: the bars of tests/test_parity_gpu.py (v_rendered
bit-exact, gradients within 1e-4 relative, Adam-updated parameters and
moments within 1e-4 relative)."""
from __future__ import annotations

import numpy as np
import pytest

from msplat_b200 import _lib, engine, synthetic
from oracle import oracle
from tests import harness

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def gpu():
    import torch
    assert torch.cuda.is_available()
    engine.bind_stream()
    yield


@pytest.mark.parametrize("config", ["C1", "C2"])
def test_forward_full_size_bitexact(config):
    g, cams = synthetic.scene(config)
    cs = harness.setup_cam(cams[0])
    model = engine.GaussianModel(g.groups(), capacity=g.n)
    lib = _lib.load()
    engine.render(model, cs)
    if lib.msplat_device_errors() & 1:
        # the intersection buffer (sized at 16 per Gaussian) overflowed:
        # the engine grows it from the count it read back, as a training
        # loop's next step would; render again
        engine.render(model, cs)
    assert lib.msplat_device_errors() == 0
    eng = harness.engine_forward_dump(g.n, cs)
    n_isect = int(lib.msplat_num_intersections())
    run = oracle.Run(cs, g.n, isect_capacity=n_isect + 1)
    run.render(g.groups())
    harness.assert_forward_bitexact(run, eng, cs)
    if config == "C2":
        tb, _ = harness.oracle_ranges(run, cs)
        assert int((tb[:, 1] - tb[:, 0]).max()) > 2048   # the merge path ran


def _target(config, cs):
    """The bench's target: a render of an independent seed-1 scene of the
    same configuration (bit-exact with the oracle's render of it)."""
    import torch
    tg, _ = synthetic.scene(config, seed=1)
    tmodel = engine.GaussianModel(tg.groups(), capacity=tg.n)
    lib = _lib.load()
    ptr = engine.render(tmodel, cs)
    if lib.msplat_device_errors() & 1:
        ptr = engine.render(tmodel, cs)
    assert lib.msplat_device_errors() == 0
    gt = engine.download(ptr, cs.height * cs.width * 3, np.float32).reshape(cs.height, cs.width, 3)
    del tmodel
    torch.cuda.synchronize()
    return gt


@pytest.mark.parametrize("config", ["C1", "C2"])
def test_train_step_full_size(config):
    """One training step at the benchmark configurations' full sizes against
    the oracle: v_rendered bit-exact, raster gradients (v_rgb, v_conic, v_xy,
    v_opacity) and the densification statistics within the gradient bar,
    Adam-updated parameters and both moments of all six groups within the
    parameter bar; then the projection VJP's geometry gradients (from
    msplat_train_step_grads on the same inputs) within the gradient bar with
    no outlier.  C1: 1M Gaussians at 1297x840, tiles up to ~1,400 keys,
    single-pass raster.  C2: 3M clustered Gaussians at 1920x1080, tiles of
    several thousand keys (merge-path sort, long backward walks)."""
    import torch

    from tests import test_parity_gpu as tp
    g, cams = synthetic.scene(config)
    cs = harness.setup_cam(cams[0])
    gt = _target(config, cs)
    gt_dev = torch.as_tensor(gt).cuda().contiguous()
    lib = _lib.load()
    # size the engine's intersection buffer for this view first (a render
    # that overflows grows it for the next call), so the step runs whole
    model = engine.GaussianModel(g.groups(), capacity=g.n)
    engine.render(model, cs)
    if lib.msplat_device_errors() & 1:
        engine.render(model, cs)
    n_isect = int(lib.msplat_num_intersections())
    engine.train_step(model, cs, gt_dev)
    torch.cuda.synchronize()
    assert lib.msplat_device_errors() == 0
    steps, bc2 = model.adam_scalars()
    params = [x.copy() for x in g.groups()]
    m = [np.zeros_like(x) for x in params]
    v = [np.zeros_like(x) for x in params]
    st = [np.zeros(g.n, np.float32) for _ in range(3)]
    run = oracle.Run(cs, g.n, adam_steps=steps, adam_bc2=bc2, isect_capacity=n_isect + 1)
    run.train_step(params, m, v, gt, *st)
    assert run.num_isects == n_isect
    tp._check_train(model, run, params, m, v, st, cs)
    if config == "C2":
        tb, _ = harness.oracle_ranges(run, cs)
        assert int((tb[:, 1] - tb[:, 0]).max()) > 2048
    del model
    geo = harness.engine_geometry_grads(g.groups(), cs, gt_dev)
    harness.assert_geometry_grads(geo, run, f"{config} ")
