"""msplat_stage_input: per-step host inputs copied on the copy stream into
two alternating device buffers, ordered against the engine stream (a
buffer is rewritten only after the step that read it two stagings ago), and
a training step fed through it gives the same loss as one fed from a
device tensor."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from msplat_b200 import _lib, engine, synthetic
from tests import harness

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def gpu():
    import torch
    assert torch.cuda.is_available()
    engine.bind_stream()
    yield


def _stage(arr):
    out = C.c_void_p()
    _lib.check(_lib.load().msplat_stage_input(C.c_void_p(arr.data_ptr()), arr.numel() * 4,
                                              C.byref(out)), "stage")
    return out.value


def test_alternating_buffers_and_growth():
    import torch
    hosts = [torch.full((1000 * (1 + i % 3),), float(i), dtype=torch.float32).pin_memory()
             for i in range(6)]
    ptrs = []
    for h in hosts:
        p = _stage(h)
        ptrs.append(p)
        torch.cuda.current_stream().synchronize()
        got = engine.download(p, h.numel(), np.float32)
        assert (got == h.numpy()).all()
    assert ptrs[0] != ptrs[1]
    # the same two slots alternate (grown in place when a larger input comes)
    assert len(set(ptrs[4:6])) == 2


def test_step_through_staged_input_matches_device_input():
    import torch
    g, cams = synthetic.scene("C0", n=5000)
    cs = harness.setup_cam(cams[0])
    gt = torch.as_tensor(synthetic.target_image(cs.width, cs.height, 3))
    a = engine.GaussianModel(g.groups())
    b = engine.GaussianModel(g.groups())
    la = engine.train_step(a, cs, gt.cuda())
    lib = _lib.load()
    lib.msplat_last_loss(1)
    la = lib.msplat_last_loss(1)
    host = gt.contiguous().pin_memory()
    engine.train_step(b, cs, engine.DevicePtr(_stage(host)))
    lb = lib.msplat_last_loss(1)
    # the loss is a float-atomic sum over blocks: equal to a few ulp
    assert abs(la - lb) <= 1e-6 * abs(la)
    for x, y in zip(a.params, b.params):
        bad, _ = harness.close(x.cpu().numpy(), y.cpu().numpy(), 1e-5, 1e-6)
        assert bad <= 3
