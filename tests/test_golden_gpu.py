"""The CUDA engine (through its C-ABI) against golden fixtures produced by
the reference's own kernels (tests/golden/make_golden.py)."""
from __future__ import annotations

import numpy as np
import pytest

from msplat_b200 import engine
from tests import harness
from tests.golden import make_golden as mg
from tests.test_golden import check_against_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def gpu():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    engine.bind_stream()


@pytest.mark.parametrize("name", sorted(mg.CASES))
def test_engine_matches_reference_golden(name):
    import torch
    g, cs, gt = mg.case_inputs(name)
    model = engine.GaussianModel(g.groups())
    engine.train_step(model, cs, torch.as_tensor(gt).cuda().contiguous())
    torch.cuda.synchronize()
    n = g.n
    T = cs.tile_bounds[0] * cs.tile_bounds[1]
    P = cs.width * cs.height
    fwd = harness.engine_forward_dump(n, cs)
    off = engine.debug_buffer("tile_offset", T + 1, np.int32)
    ga = engine.debug_buffer("grad_acc", 9 * n, np.float32).reshape(n, 9)
    vis = fwd["radii"] > 0
    zero_culled = lambda a: np.where(vis[:, None], a, 0).astype(np.float32)
    out = {
        "radii": fwd["radii"], "xys": fwd["xy"], "conics": fwd["conic"].reshape(-1),
        "colors": fwd["rgb"].reshape(-1),
        "tile_bins": np.stack([off[:-1], off[1:]], 1).astype(np.int32).reshape(-1),
        "gaussian_ids": engine.debug_buffer("sorted_ids", int(off[-1]), np.int32),
        "out_img": fwd["img"], "final_T": fwd["final_T"], "final_idx": fwd["final_idx"],
        "v_rendered": engine.debug_buffer("v_rendered", 3 * P, np.float32),
        "v_rgb": zero_culled(ga[:, 0:3]).reshape(-1), "v_conic": zero_culled(ga[:, 3:6]).reshape(-1),
        "v_xy": zero_culled(ga[:, 6:8]).reshape(-1), "v_opacity": zero_culled(ga[:, 8:9]).reshape(-1),
    }
    # the fused step applies Adam to the projection VJP's outputs in place;
    # the same VJP's gradients come from msplat_train_step_grads on a fresh
    # model with the same inputs (zero for culled Gaussians, as in the fixture)
    geo = harness.engine_geometry_grads(g.groups(), cs, torch.as_tensor(gt).cuda().contiguous())
    for key in ("v_mean3d", "v_scale", "v_quat"):
        out[key] = geo[key].reshape(-1)
    for gi, nm in enumerate(("means", "scales", "quats", "features_dc", "features_rest", "opacities")):
        out[f"param_{nm}"] = model.params[gi].cpu().numpy()
    out["vis_counts"] = model.vis_counts.cpu().numpy()
    out["xys_grad_norm"] = model.xys_grad_norm.cpu().numpy()
    out["max_2d_size"] = model.max_2d_size.cpu().numpy()
    check_against_golden(name, out, int(off[-1]))
