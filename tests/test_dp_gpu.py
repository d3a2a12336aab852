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
2. Two ranks (tests/dp_worker.py under torchrun, when the box has two
   GPUs), through NCCL and through the peer-memory kernel: the replicas must
   be bit-identical to each other, and within the same bar of a one-GPU
   emulation that sums the two views' gradients and applies scale 1/2.
   Batched steps (two views per rank, gradients accumulated with
   msplat_train_step_grads_accumulate): within the bar of one GPU training
   the same four-view batches (multigpu.train_batch), and on one GPU the
   accumulated buffer within the one-step bar of the mean of its views.
3. The peer-memory optimiser: at world 1 bit-identical to msplat_adam_apply
   on the same gradients; its compact exchange (v_rgb instead of the SH
   gradients) within the bar of the full one; and its cross-GPU waits give
   up and report when a peer never signals (a second rank that does not
   exist), leaving the GPU usable.
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


@pytest.mark.parametrize("case", ["chunked", "mono"])
def test_accumulated_views_equal_mean_of_views(case):
    """A batch of two views through msplat_train_step_grads_accumulate
    (multigpu.accumulate_views: the first view writes, the second adds, each
    loss normalised by 2) equals the mean of the two views' own gradients
    within the one-step gradient bar (the runs differ only in the order of
    the raster backward's atomics); the visibility entries are exact counts."""
    import torch
    n, w, h = (20_000, 256, 192) if case == "chunked" else (30_000, 640, 480)
    g, cams = _scene(n, w, h)
    model = engine.GaussianModel(g.groups())
    ops = multigpu.EngineOps()
    nf = multigpu.grad_floats(n, model.rest_bases)
    ga, gb, acc = (ops.alloc(nf) for _ in range(3))
    css = [harness.setup_cam(cams[k]) for k in range(2)]
    gts = [_gt(cs, 10 + k) for k, cs in enumerate(css)]
    ops.grads(model, css[0], gts[0], ga, 0.2, engine.DEFAULT_BG, 1.0, 0.01)
    ops.grads(model, css[1], gts[1], gb, 0.2, engine.DEFAULT_BG, 1.0, 0.01)
    acc.fill_(float("nan"))  # every entry must be written by the first view
    multigpu.accumulate_views(ops, model, css, gts, acc)
    torch.cuda.synchronize()
    (sa, va), (sb, vb), (sc, vc) = (multigpu.grad_views(t, n, model.rest_bases)
                                    for t in (ga, gb, acc))
    np.testing.assert_array_equal(vc.cpu().numpy(), (va + vb).cpu().numpy())
    assert ((va > 0) != (vb > 0)).any(), "the two views should see different Gaussians"
    for gi in range(6):
        want = (0.5 * (sa[gi] + sb[gi])).cpu().numpy()
        got = sc[gi].cpu().numpy()
        assert np.isfinite(got).all(), f"group {gi}: unwritten entries"
        _assert_close(got, want, STAT_RTOL, STAT_ATOL_FRAC, f"{case}: group {gi}")


def _single_rank_group():
    import socket
    import torch
    import torch.distributed as dist
    if dist.is_initialized():
        return
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            device_id=torch.device("cuda", torch.cuda.current_device()))


def test_peer_apply_equals_adam_apply_one_rank():
    """The peer-memory optimiser at world 1 and msplat_adam_apply, given the
    same gradient buffer, produce the same bits (same sum, scale 1, same
    update)."""
    import torch
    import torch.distributed as dist
    n, w, h = 30_000, 640, 480
    g, cams = _scene(n, w, h, seed=3)
    ref = engine.GaussianModel(g.groups())
    peer_model = engine.GaussianModel(g.groups())
    ops = multigpu.EngineOps()
    grad = ops.alloc(multigpu.grad_floats(n, ref.rest_bases))
    _single_rank_group()
    dp = multigpu.DataParallel(peer_model, 0, 1, mode="peer", compact=False)
    try:
        for step in range(3):
            cs = harness.setup_cam(cams[step % len(cams)], step=step, interval=1)
            ref.step_count += 1
            ops.grads(ref, cs, _gt(cs, step), grad, 0.2, engine.DEFAULT_BG, 1.0, 0.01)
            ops.adam_apply(ref, cs, grad, 1.0)
            peer_model.step_count += 1
            dp.grad.copy_(grad)
            dp.apply(cs)
            # the next gradients are taken at the reference's parameters
            for a, b in zip(peer_model.params, ref.params):
                assert torch.equal(a, b), "parameters differ"
        torch.cuda.synchronize()
        assert dp.peer_errors() == 0
        for i in range(6):
            assert torch.equal(peer_model.exp_avg[i], ref.exp_avg[i]), f"exp_avg {i}"
            assert torch.equal(peer_model.exp_avg_sq[i], ref.exp_avg_sq[i]), f"exp_avg_sq {i}"
    finally:
        dp.shutdown()
        dist.destroy_process_group()


def test_peer_compact_equals_full_one_rank():
    """Exchanging v_rgb and rebuilding the SH gradients from the camera gives
    the parameters of the full gradient exchange (within the bar: the two
    runs take their gradients with differently ordered float atomics)."""
    import torch
    import torch.distributed as dist
    n, w, h = 30_000, 640, 480
    g, cams = _scene(n, w, h, seed=6)
    models = [engine.GaussianModel(g.groups()) for _ in range(2)]
    _single_rank_group()
    dps = [multigpu.DataParallel(m, 0, 1, mode="peer", compact=c)
           for m, c in zip(models, (False, True))]
    try:
        for step in range(3):
            cs = harness.setup_cam(cams[step % len(cams)], step=step + 1, interval=1)
            gt = _gt(cs, step)
            for dp in dps:
                dp.train_step(cs, gt)
        torch.cuda.synchronize()
        assert all(dp.peer_errors() == 0 for dp in dps)
        a, b = _state(models[0]), _state(models[1])
        for k in a:
            if k in ("vis", "gn", "m2d"):
                _assert_close(b[k], a[k], STAT_RTOL, STAT_ATOL_FRAC, f"compact: {k}")
            else:
                _assert_close(b[k], a[k], PARAM_RTOL, PARAM_ATOL_FRAC, f"compact: {k}")
    finally:
        for dp in dps:
            dp.shutdown()
        dist.destroy_process_group()


def test_peer_wait_times_out_and_reports():
    """A world-2 step whose second rank never signals: both cross-GPU waits
    give up after their limit, the error bits are set, and the GPU stays
    usable."""
    import ctypes as C
    import time
    import torch
    from msplat_b200 import _lib
    lib = _lib.load()
    n = 4096
    g, cams = _scene(n, 320, 240, seed=4)
    model = engine.GaussianModel(g.groups())
    grad = torch.zeros(multigpu.grad_floats(n, model.rest_bases), device="cuda")
    flags = [torch.zeros(4, dtype=torch.int32, device="cuda") for _ in range(2)]
    lib.msplat_dp_errors(1)
    P = C.c_void_p
    grads_arr = (P * 2)(grad.data_ptr(), grad.data_ptr())
    params_arr = (P * 12)(*([p.data_ptr() for p in model.params] * 2))
    flags_arr = (P * 2)(flags[0].data_ptr(), flags[1].data_ptr())
    steps, bc2s = engine.adam_scalars(1, engine.LR_INIT)
    t0 = time.perf_counter()
    rc = lib.msplat_dp_reduce_adam(0, 2, n, model.rest_bases, 3, 3, grads_arr, params_arr,
                                   engine._ptr_array(model.exp_avg),
                                   engine._ptr_array(model.exp_avg_sq), flags_arr, 1,
                                   _lib.farr(steps), _lib.farr(bc2s), 0.9, 0.999, 1e-8, 0, 0.2)
    assert rc == 0
    errs = lib.msplat_dp_errors(1)
    elapsed = time.perf_counter() - t0
    assert errs == 3, f"error bits {errs}"
    assert elapsed < 5.0
    assert flags[0][0].item() == 1 and flags[1][0].item() == 1   # rank 0 signalled phase 0
    # the context still works
    cs = harness.setup_cam(cams[0])
    engine.render(model, cs)
    torch.cuda.synchronize()
    assert lib.msplat_dp_errors(0) == 0


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
    for mode, port in (("nccl", 29561), ("peer", 29562)):
        with tempfile.TemporaryDirectory() as d:
            cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                   "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(port),
                   os.path.join(ROOT, "tests", "dp_worker.py"), d, str(n), str(w), str(h), "5",
                   mode]
            env = dict(os.environ, PYTHONPATH=ROOT)
            res = subprocess.run(["timeout", "-k", "30", "300"] + cmd, cwd=ROOT, env=env,
                                 capture_output=True, text=True)
            assert res.returncode == 0, mode + res.stdout[-3000:] + res.stderr[-3000:]
            got = [dict(np.load(os.path.join(d, f"rank{r}.npz"))) for r in range(2)]
        for k, v in want.items():
            np.testing.assert_array_equal(got[0][k], got[1][k], err_msg=f"{mode}: replicas differ: {k}")
            _assert_close(got[0][k], v, PARAM_RTOL, PARAM_ATOL_FRAC, f"{mode} vs emulation: {k}")


def test_two_rank_batched_views_match_single_gpu_batch():
    """Two ranks, two views each per step (a batch of four; full-layout
    exchange with accumulated gradients) through the peer kernel and NCCL:
    replicas bit-identical, and within the bar of one GPU training the same
    batches with multigpu.train_batch."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    n, w, h = 20_000, 320, 240
    g, cams = _scene(n, w, h, seed=6)
    model = engine.GaussianModel(g.groups())
    buf = multigpu.EngineOps().alloc(multigpu.grad_floats(n, model.rest_bases))
    for step in range(3):
        css = [harness.setup_cam(cams[(step * 4 + b) % 3]) for b in range(4)]
        gts = [_gt(cs, (step * 4 + b) % 3) for b, cs in enumerate(css)]
        multigpu.train_batch(model, css, gts, buf)
    torch.cuda.synchronize()
    want = {f"p{i}": model.params[i].cpu().numpy() for i in range(6)}
    for mode, port in (("nccl", 29563), ("peer", 29564)):
        with tempfile.TemporaryDirectory() as d:
            cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                   "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(port),
                   os.path.join(ROOT, "tests", "dp_worker.py"), d, str(n), str(w), str(h), "6",
                   mode, "2"]
            env = dict(os.environ, PYTHONPATH=ROOT)
            res = subprocess.run(["timeout", "-k", "30", "300"] + cmd, cwd=ROOT, env=env,
                                 capture_output=True, text=True)
            assert res.returncode == 0, mode + res.stdout[-3000:] + res.stderr[-3000:]
            got = [dict(np.load(os.path.join(d, f"rank{r}.npz"))) for r in range(2)]
        for k, v in want.items():
            np.testing.assert_array_equal(got[0][k], got[1][k], err_msg=f"{mode}: replicas differ: {k}")
            _assert_close(got[0][k], v, PARAM_RTOL, PARAM_ATOL_FRAC, f"{mode} vs one GPU: {k}")
