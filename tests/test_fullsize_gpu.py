"""Forward parity at the benchmark configurations' full sizes: C1 (1M
Gaussians, 1297x840, a sphere camera) and C2 (3M Gaussians, 70% in ten
tight clusters, 1920x1080: tiles with several thousand Gaussians, sorted by
the merge path).  Radii, centres, depths, conics, colours, tile ranges,
per-tile sorted id lists, image, final T and final index bit-exact with the
CPU oracle."""
from __future__ import annotations

import pytest

from msplat_b200 import engine, synthetic
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
    engine.render(model, cs)
    eng = harness.engine_forward_dump(g.n, cs)
    run = oracle.Run(cs, g.n)
    run.render(g.groups())
    harness.assert_forward_bitexact(run, eng, cs)
    if config == "C2":
        tb, _ = harness.oracle_ranges(run, cs)
        assert int((tb[:, 1] - tb[:, 0]).max()) > 2048   # the merge path ran
