"""The data-parallel protocol of msplat_b200.multigpu on two gloo ranks (CPU).

The engine's two halves are replaced by a stand-in (`FakeOps`) with the same
buffer layout and the same optimiser rules, so the test checks the host
logic: each rank fills its gradient buffer for its own view, the buffers are
summed across ranks, every rank applies Adam with grad_scale = 1/world, and
the replicas stay identical and equal to a single-process run that sums the
two views' gradients itself.  Also covered: sync_stats, max_over_ranks,
barrier and shutdown.
"""
from __future__ import annotations

import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from msplat_b200 import engine, multigpu, synthetic

N = 96
REST_BASES = 15
STEPS = 3


class FakeCam:
    def __init__(self, view: int, degree: int = 3, degrees_to_use: int = 2):
        self.view, self.degree, self.degrees_to_use = view, degree, degrees_to_use


def fake_grads(model, view: int, out) -> None:
    """Deterministic per-view gradient in the engine's buffer layout: SH
    groups zero where the Gaussian is not visible, SH-rest zero beyond the
    degrees in use (2 -> 8 bases)."""
    groups, vis = multigpu.grad_views(out, model.n, model.rest_bases)
    seen = (torch.arange(model.n) % (view + 2) != 0).float()
    vis.copy_(seen)
    for gi, g in enumerate(groups):
        g.copy_(torch.sin(model.params[gi].reshape(model.n, -1) * (view + 1) + gi))
    groups[3].mul_(seen[:, None])
    groups[4].mul_(seen[:, None])
    groups[4][:, 8 * 3:] = 0.0


def fake_adam(model, cam, grad, scale) -> None:
    """The optimiser rules of msplat_adam_apply, in torch on the CPU."""
    groups, vis = multigpu.grad_views(grad, model.n, model.rest_bases)
    steps, bc2s = model.adam_scalars()
    b1, b2, eps = model.beta1, model.beta2, model.eps
    used = {0: 0, 1: 3, 2: 8}.get(min(cam.degrees_to_use, cam.degree), 15) * 3
    for gi in range(6):
        p = model.params[gi].view(model.n, -1)
        m = model.exp_avg[gi].view(model.n, -1)
        v = model.exp_avg_sq[gi].view(model.n, -1)
        g = groups[gi] * scale
        mask = torch.ones_like(p, dtype=torch.bool)
        if gi in (3, 4):
            mask &= (vis > 0)[:, None]
        if gi == 4:
            mask[:, used:] = False
        mm = b1 * m + (1 - b1) * g
        vv = b2 * v + (1 - b2) * g * g
        pp = p - steps[gi] * mm / (torch.sqrt(vv) / bc2s[gi] + eps)
        p.copy_(torch.where(mask, pp, p))
        m.copy_(torch.where(mask, mm, m))
        v.copy_(torch.where(mask, vv, v))


class FakeOps:
    def alloc(self, count):
        return torch.empty(count, dtype=torch.float32)

    def grads(self, model, cam, gt, out, *args, accumulate=False, batch=1):
        # the engine's contract: gradients of the loss normalised by the
        # rank's view count; `accumulate` adds them (and the visibility) to out
        tmp = torch.empty_like(out) if accumulate else out
        fake_grads(model, cam.view, tmp)
        tmp[:-model.n] /= batch
        if accumulate:
            out += tmp
        model.vis_counts += 1.0
        model.xys_grad_norm += float(cam.view)
        model.max_2d_size.copy_(torch.maximum(model.max_2d_size,
                                              torch.full_like(model.max_2d_size, cam.view * 0.1)))
        return float(cam.view)

    def adam_apply(self, model, cam, grad, scale):
        fake_adam(model, cam, grad, scale)


def _model():
    g = synthetic.gaussians(N, 3, sh_degree=3)
    return engine.GaussianModel(g.groups(), device="cpu")


def _worker(rank, world, port, out_dir, vpr=1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    model = _model()
    dp = multigpu.DataParallel(model, rank, world, ops=FakeOps(), backend="gloo", timeout_s=60,
                               views_per_rank=vpr)
    losses = []
    for s in range(STEPS):
        if vpr == 1:
            losses.append(dp.train_step(FakeCam(s * world + rank), None))
        else:
            # rank r takes views r, r + world, ... of the step's batch
            cams = [FakeCam(s * world * vpr + k * world + rank) for k in range(vpr)]
            losses.append(dp.train_views(cams, [None] * vpr))
    dp.barrier()
    mx = dp.max_over_ranks(float(rank) + 0.5)
    dp.sync_stats()
    dp.shutdown()
    arrs = {f"p{i}": t.numpy() for i, t in enumerate(model.params)}
    arrs.update({f"m{i}": t.numpy() for i, t in enumerate(model.exp_avg)})
    arrs.update({f"v{i}": t.numpy() for i, t in enumerate(model.exp_avg_sq)})
    arrs.update(vis=model.vis_counts.numpy(), gn=model.xys_grad_norm.numpy(),
                m2d=model.max_2d_size.numpy(), losses=np.array(losses), mx=np.array([mx]))
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **arrs)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def two_ranks():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), d), nprocs=2, join=True,
                           start_method="spawn")
        yield [dict(np.load(os.path.join(d, f"rank{r}.npz"))) for r in range(2)]


@pytest.fixture(scope="module")
def two_ranks_batched():
    """Two ranks, two views each per step (a batch of four)."""
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), d, 2), nprocs=2, join=True,
                           start_method="spawn")
        yield [dict(np.load(os.path.join(d, f"rank{r}.npz"))) for r in range(2)]


def test_batched_views_match_single_device_batch(two_ranks_batched):
    """world 2 x 2 views per rank == one device training the same batches of
    four views (multigpu.train_batch), and the replicas stay identical."""
    r0, r1 = two_ranks_batched
    for k in r0:
        if k.startswith(("p", "m", "v")) and k[1:].isdigit():
            np.testing.assert_array_equal(r0[k], r1[k], err_msg=k)
    model = _model()
    buf = torch.empty(multigpu.grad_floats(N, REST_BASES))
    batch = 4
    for s in range(STEPS):
        cams = [FakeCam(s * batch + v) for v in range(batch)]
        multigpu.train_batch(model, cams, [None] * batch, buf, ops=FakeOps())
    for i in range(6):
        np.testing.assert_allclose(r0[f"p{i}"], model.params[i].numpy(), rtol=1e-6, atol=1e-7,
                                   err_msg=f"group {i}")
    # every view of every step counted once across the ranks
    np.testing.assert_array_equal(r0["vis"], np.full(N, batch * STEPS, np.float32))


def test_batched_views_reject_wrong_count_and_compact():
    with pytest.raises(ValueError):
        multigpu.accumulate_views(FakeOps(), _model(), [FakeCam(0), FakeCam(1)], [None, None],
                                  torch.empty(multigpu.grad_floats(N, REST_BASES)), compact=True)


def test_replicas_identical(two_ranks):
    r0, r1 = two_ranks
    for k in r0:
        if k.startswith(("p", "m", "v")) and k[1:].isdigit():
            np.testing.assert_array_equal(r0[k], r1[k], err_msg=k)


def test_matches_single_process_sum_of_views(two_ranks):
    world = 2
    model = _model()
    buf = torch.empty(multigpu.grad_floats(N, REST_BASES))
    tmp = torch.empty_like(buf)
    for s in range(STEPS):
        model.step_count += 1
        buf.zero_()
        for r in range(world):
            fake_grads(model, s * world + r, tmp)
            buf += tmp
        fake_adam(model, FakeCam(0), buf, 1.0 / world)
    for i in range(6):
        np.testing.assert_allclose(two_ranks[0][f"p{i}"], model.params[i].numpy(), rtol=1e-6,
                                   atol=1e-7, err_msg=f"group {i}")


def test_views_differ_per_rank_and_stats_combine(two_ranks):
    r0, r1 = two_ranks
    assert list(r0["losses"]) == [0.0, 2.0, 4.0] and list(r1["losses"]) == [1.0, 3.0, 5.0]
    np.testing.assert_array_equal(r0["vis"], np.full(N, 2.0 * STEPS, np.float32))
    np.testing.assert_array_equal(r0["gn"], np.full(N, 15.0, np.float32))
    np.testing.assert_allclose(r0["m2d"], np.full(N, 0.5, np.float32), rtol=1e-6)
    assert r0["mx"][0] == 1.5 and r1["mx"][0] == 1.5


def test_grad_buffer_layout():
    bufs, vis = multigpu.grad_views(torch.arange(multigpu.grad_floats(4, 15), dtype=torch.float32),
                                    4, 15)
    assert [tuple(b.shape) for b in bufs] == [(4, 3), (4, 3), (4, 4), (4, 3), (4, 45), (4, 1)]
    assert vis.shape == (4,) and vis[0].item() == 59 * 4


# ---- a rank that leaves or stalls between steps ---------------------------------

def _failure_worker(rank, world, port, out_dir, how):
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    model = _model()
    dp = multigpu.DataParallel(model, rank, world, ops=FakeOps(), backend="gloo", timeout_s=3)
    dp.train_step(FakeCam(rank), None)      # one complete step on both ranks
    if rank == 1:
        if how == "stall":
            time.sleep(8)                   # between steps, nothing in flight
        os._exit(0)                         # leaves without shutting down
    after_one = [t.clone() for t in model.params + model.exp_avg + model.exp_avg_sq]
    t0 = time.monotonic()
    err = ""
    try:
        dp.train_step(FakeCam(world + rank), None)
    except multigpu.PeerLostError as e:
        err = str(e)
    elapsed = time.monotonic() - t0
    now = model.params + model.exp_avg + model.exp_avg_sq
    unchanged = all(torch.equal(a, b) for a, b in zip(after_one, now))
    np.savez(os.path.join(out_dir, "rank0.npz"), elapsed=np.array([elapsed]),
             unchanged=np.array([unchanged]), step=np.array([model.step_count]),
             err=np.array([err]))
    os._exit(0)                             # the group is broken: skip its teardown


@pytest.mark.parametrize("how", ["exit", "stall"])
def test_survivor_reports_a_lost_peer(how):
    """Rank 1 completes a step, then exits (or stalls for 8 s) between
    steps.  Rank 0's next step fails on the host within the process group's
    3 s timeout (or as soon as the connection closes) with PeerLostError, and
    its replica and step count are those of the last complete step."""
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_failure_worker, args=(2, _free_port(), d, how), nprocs=2,
                           join=True, start_method="spawn")
        r = np.load(os.path.join(d, "rank0.npz"))
        assert "no parameter was updated" in str(r["err"][0]), r["err"]
        assert bool(r["unchanged"][0])
        assert int(r["step"][0]) == 1
        assert float(r["elapsed"][0]) < 15.0
