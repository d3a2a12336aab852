"""Densification on the GPU (msplat_densify through the C-ABI) against the
CPU oracle: bit-exact new count, flags and all 18 compacted buffers (the
classification, the split children's positions and the cull decisions use
the shared arithmetic contract); the opacity reset likewise; and the
densification branch of the refinement schedule on a model that trains."""
from __future__ import annotations

import numpy as np
import pytest

from msplat_b200 import engine, synthetic
from oracle import oracle
from tests import densify_case, harness

pytestmark = pytest.mark.gpu

THRESH = {"grad": 60.0, "size": 0.04}
SETTINGS = [dict(check_screen=True, check_huge=True), dict(check_screen=False, check_huge=False)]


@pytest.fixture(scope="module", autouse=True)
def gpu():
    import torch
    assert torch.cuda.is_available(), "densify GPU tests need a CUDA device"
    engine.bind_stream()
    yield


def _gpu_model(bufs, ea, es, n, gnorm, vis, max2d):
    import torch
    groups = [b[:n] for b in bufs]
    model = engine.GaussianModel(groups, capacity=bufs[0].shape[0])
    for g in range(6):
        model._m[g].copy_(torch.as_tensor(ea[g]))
        model._v[g].copy_(torch.as_tensor(es[g]))
    for dst, src in zip(model._stats, (vis, gnorm, max2d)):
        dst[:n].copy_(torch.as_tensor(src))
    return model


@pytest.mark.parametrize("setting", range(len(SETTINGS)))
def test_densify_matches_oracle(setting):
    import torch
    kw = SETTINGS[setting]
    n = 20_000
    bufs, ea, es, gnorm, vis, max2d, samples = densify_case.make(n, 11 + setting)
    model = _gpu_model(bufs, ea, es, n, gnorm, vis, max2d)
    count = model.densify(7, THRESH["grad"], THRESH["size"], 0.05, kw["check_screen"],
                          kw["check_huge"], half_max_dim=648.5,
                          random_samples=torch.as_tensor(samples, device="cuda"))
    torch.cuda.synchronize()
    want, split, dup, keep = oracle.densify(bufs, ea, es, n, gnorm, vis, max2d, samples,
                                            half_max_dim=648.5, grad_thresh=THRESH["grad"],
                                            size_thresh=THRESH["size"], **kw)
    assert split.sum() > 100 and dup.sum() > 100
    assert count == want
    for g in range(6):
        np.testing.assert_array_equal(model.params[g].cpu().numpy(), bufs[g][:want],
                                      err_msg=f"params {g}")
        np.testing.assert_array_equal(model.exp_avg[g].cpu().numpy(), ea[g][:want],
                                      err_msg=f"exp_avg {g}")
        np.testing.assert_array_equal(model.exp_avg_sq[g].cpu().numpy(), es[g][:want],
                                      err_msg=f"exp_avg_sq {g}")


def test_reset_opacity_matches_oracle():
    import torch
    n = 5000
    bufs, ea, es, gnorm, vis, max2d, _ = densify_case.make(n, 21)
    model = _gpu_model(bufs, ea, es, n, gnorm, vis, max2d)
    model.reset_opacity()
    torch.cuda.synchronize()
    op, m5, v5 = bufs[5][:n].copy(), ea[5][:n].copy(), es[5][:n].copy()
    oracle.load().orc_reset_opacity(oracle._fp(op), oracle._fp(m5), oracle._fp(v5), n)
    np.testing.assert_array_equal(model.params[5].cpu().numpy(), op)
    assert not model.exp_avg[5].any() and not model.exp_avg_sq[5].any()


def test_schedule_densifies_a_training_model():
    """Train a few steps, then the schedule's densification step: the count
    changes, the buffers grow as needed, and training goes on."""
    import torch
    g, cams = synthetic.scene("C0", n=8000)
    cs = harness.setup_cam(cams[0])
    gt = torch.as_tensor(synthetic.target_image(cs.width, cs.height, 1), device="cuda")
    model = engine.GaussianModel(g.groups(), capacity=8000)
    sched = engine.Schedule(max_steps=10_000, num_cameras=1, refine_every=2, warmup_length=1,
                            reset_alpha_every=100, densify_grad_thresh=1e-6)
    done = None
    for step in range(1, 5):
        engine.train_step(model, cs, gt)
        out = sched.after_train(model, step, cs.width, cs.height)
        if out["densified"]:
            done = out["densified"]
    assert done is not None and done[1] != done[0]
    assert model.capacity >= 3 * done[0]
    assert int(model.vis_counts.sum().item()) == 0   # statistics reset
    engine.train_step(model, cs, gt)
    torch.cuda.synchronize()
    assert torch.isfinite(model.params[0]).all()
