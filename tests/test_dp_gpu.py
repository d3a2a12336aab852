"""The data-parallel halves on the GPU.

1. One rank: msplat_train_step_grads + msplat_adam_apply(scale 1) must give
   msplat_train_step's parameters, moments and statistics -- on the chunked
   and the single-pass raster path and with only part of the SH degrees in
   use.  The gradient code and the Adam arithmetic are the same, but the
   raster backward sums with float atomics whose order varies run to run,
   so the bar is 1e-4 relative plus 5e-6 of the tensor's largest magnitude
   for parameters and moments: the parity suite's one-step gradient floor
   (2e-6) grown for three steps of moment accumulation, where near-zero
   entries carry the absolute error of the atomics-ordered sums.
2. Two NCCL ranks (tests/dp_worker.py under torchrun, when the box has two
   GPUs): the replicas must be bit-identical to each other (every rank
   applies the same summed buffer), and within the same bar of a one-GPU
   emulation that sums the two views' gradients and applies scale 1/2.
"""
from __future__ import annotations

import math
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

from msplat_b200 import engine, multigpu, synthetic
from tests import harness

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PARAM_RTOL, PARAM_ATOL_FRAC = 1e-4, 5e-6
STAT_RTOL, STAT_ATOL_FRAC = 1e-4, 2e-6


# Two runs of the step differ only in the order of the raster backward's
# float atomics.  Where a Gaussian's gradient is a near-cancelling sum, that
# order moves the result by a few ulp of the gross sum, far above any floor
# relative to the tensor's maximum, and Adam carries it into the moments.
# So a handful of entries (at most 2 per million, never fewer than 3) may
# exceed the bar, and none may exceed 1e-4 of the tensor's maximum.
MAX_OUTLIER_FRAC, OUTLIER_CAP = 2e-6, 1e-4


def _assert_close(a, b, rtol, atol_frac, what):
    bad, worst = harness.close(a, b, rtol, atol_frac)
    allowed = max(3, int(MAX_OUTLIER_FRAC * np.asarray(a).size))
    assert bad <= allowed and worst <= OUTLIER_CAP, (
        f"{what}: {bad} entries out of tolerance (allowed {allowed}), worst {worst:.3g} of max")


@pytest.fixture(scope="module", autouse=True)
def gpu():
    import torch
    assert torch.cuda.is_available(), "data-parallel GPU tests need a CUDA device"
    engine.bind_stream()
    yield


def _scene(n, w, h, seed=0):
    g = synthetic.gaussians(n, seed, mean_range=1.0, log_scale_mu=math.log(0.02),
                            log_scale_sigma=0.3)
    cams = [synthetic.front_camera(w, h, 3.0 + 0.3 * k) for k in range(3)]
    return g, cams


def _gt(cs, seed):
    import torch
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return torch.rand(cs.height, cs.width, 3, device="cuda", generator=gen)


def _state(model):
    out = {}
    for i in range(6):
        out[f"p{i}"] = model.params[i].cpu().numpy()
        out[f"m{i}"] = model.exp_avg[i].cpu().numpy()
        out[f"v{i}"] = model.exp_avg_sq[i].cpu().numpy()
    out["vis"] = model.vis_counts.cpu().numpy()
    out["gn"] = model.xys_grad_norm.cpu().numpy()
    out["m2d"] = model.max_2d_size.cpu().numpy()
    return out


@pytest.mark.parametrize("case", ["chunked", "mono", "sh_partial"])
def test_split_step_equals_fused_step(case):
    import torch
    n, w, h = (20_000, 256, 192) if case == "chunked" else (30_000, 640, 480)
    g, cams = _scene(n, w, h)
    fused = engine.GaussianModel(g.groups())
    split = engine.GaussianModel(g.groups())
    ops = multigpu.EngineOps()
    grad = ops.alloc(multigpu.grad_floats(n, split.rest_bases))
    for step in range(3):
        # sh_partial: degrees in use 0, 1, 2 over the three steps
        cs = harness.setup_cam(cams[step % len(cams)],
                               step=step if case == "sh_partial" else 10**9, interval=1)
        gt = _gt(cs, step)
        engine.train_step(fused, cs, gt)
        split.step_count += 1
        ops.grads(split, cs, gt, grad, 0.2, engine.DEFAULT_BG, 1.0, 0.01)
        ops.adam_apply(split, cs, grad, 1.0)
    torch.cuda.synchronize()
    a, b = _state(fused), _state(split)
    for k in a:
        if k in ("vis", "gn", "m2d"):
            _assert_close(b[k], a[k], STAT_RTOL, STAT_ATOL_FRAC, f"{case}: {k}")
        else:
            _assert_close(b[k], a[k], PARAM_RTOL, PARAM_ATOL_FRAC, f"{case}: {k}")
    # the visible-only rule: Gaussians never seen keep their SH moments at 0
    never = a["vis"] == 0
    assert not b["m3"][never].any() and not b["m4"][never].any()


def test_two_rank_nccl_matches_summed_views():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    n, w, h = 20_000, 320, 240
    g, cams = _scene(n, w, h, seed=5)
    # single-GPU emulation: rank r trains view (step * 2 + r) % 3
    model = engine.GaussianModel(g.groups())
    ops = multigpu.EngineOps()
    total = ops.alloc(multigpu.grad_floats(n, model.rest_bases))
    part = torch.empty_like(total)
    for step in range(3):
        model.step_count += 1
        total.zero_()
        for r in range(2):
            v = (step * 2 + r) % 3
            cs = harness.setup_cam(cams[v])
            ops.grads(model, cs, _gt(cs, v), part, 0.2, engine.DEFAULT_BG, 1.0, 0.01)
            total += part
        ops.adam_apply(model, harness.setup_cam(cams[0]), total, 0.5)
    torch.cuda.synchronize()
    want = {f"p{i}": model.params[i].cpu().numpy() for i in range(6)}
    with tempfile.TemporaryDirectory() as d:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
               "--master-addr", "127.0.0.1", "--master-port", "29561",
               os.path.join(ROOT, "tests", "dp_worker.py"), d, str(n), str(w), str(h), "5"]
        env = dict(os.environ, PYTHONPATH=ROOT)
        res = subprocess.run(["timeout", "-k", "30", "300"] + cmd, cwd=ROOT, env=env,
                             capture_output=True, text=True)
        assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
        got = [dict(np.load(os.path.join(d, f"rank{r}.npz"))) for r in range(2)]
    for k, v in want.items():
        np.testing.assert_array_equal(got[0][k], got[1][k], err_msg=f"replicas differ: {k}")
        _assert_close(got[0][k], v, PARAM_RTOL, PARAM_ATOL_FRAC, f"vs emulation: {k}")
