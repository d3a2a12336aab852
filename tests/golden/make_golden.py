"""Generate the golden fixtures in tests/golden/ from the reference's own
kernels (oracle/_ref/libmsplat_ref.so, built from the reference sources by
oracle/ref_shim/build_ref.py).

Each fixture is one training step of a small seeded scene: the inputs are
regenerated from the recorded seed and sizes (msplat_b200.synthetic), the
reference's outputs are stored.  Run from the repository root:

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from msplat_b200 import engine, synthetic  # noqa: E402
from oracle import oracle  # noqa: E402
from tests import harness  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (gaussians, width, height, seed, log-scale mean, distance, degrees_to_use)
CASES = {
    "chunked_96x64": (1500, 96, 64, 11, math.log(0.03), 3.0, 3),           # 24 tiles: depth chunks
    "mono_ragged_345x299": (2500, 345, 299, 12, math.log(0.02), 3.0, 3),   # 418 tiles: monolithic
    "sh1_ragged_100x75": (800, 100, 75, 13, math.log(0.03), 3.0, 1),       # SH degree 1 in use
}
# step 1 with the default learning rates (Model::setupOptimizers)
ADAM_STEPS, ADAM_BC2 = (list(map(float, x)) for x in engine.adam_scalars(1, engine.LR_INIT))


def case_inputs(name):
    n, w, h, seed, mu, dist, dtu = CASES[name]
    g = synthetic.gaussians(n, seed, mean_range=1.0, log_scale_mu=mu, log_scale_sigma=0.3)
    cs = harness.setup_cam(synthetic.front_camera(w, h, dist))
    cs.degrees_to_use = dtu
    gt = synthetic.target_image(w, h, seed + 100)
    return g, cs, gt


def run_case(name, impl):
    g, cs, gt = case_inputs(name)
    run = oracle.Run(cs, g.n, adam_steps=ADAM_STEPS, adam_bc2=ADAM_BC2)
    params = [x.copy() for x in g.groups()]
    m = [np.zeros_like(x) for x in params]
    v = [np.zeros_like(x) for x in params]
    st = [np.zeros(g.n, np.float32) for _ in range(3)]
    run.train_step(params, m, v, gt, *st, impl=impl)
    T = cs.tile_bounds[0] * cs.tile_bounds[1]
    out = {
        "radii": run.radii.copy(), "xys": run.xys.copy(), "conics": run.conics.copy(),
        "colors": run.colors.copy(), "tile_bins": run.tile_bins[: 2 * T].copy(),
        "gaussian_ids": run.gaussian_ids[: run.num_isects].copy(), "out_img": run.out_img.copy(),
        "final_T": run.final_T.copy(), "final_idx": run.final_idx.copy(),
        "v_rendered": run.v_rendered.copy(), "v_xy": run.v_xy.copy(), "v_conic": run.v_conic.copy(),
        "v_rgb": run.v_rgb.copy(), "v_opacity": run.v_opacity.copy(),
        "v_mean3d": run.v_mean3d.copy(), "v_scale": run.v_scale.copy(), "v_quat": run.v_quat.copy(),
    }
    # Adam state after step 1 follows from the gradients; the parameters are kept
    for gi, nm in enumerate(("means", "scales", "quats", "features_dc", "features_rest", "opacities")):
        out[f"param_{nm}"] = params[gi]
    out["vis_counts"], out["xys_grad_norm"], out["max_2d_size"] = st
    return out, run


# Outputs the engine must reproduce bit for bit are stored as SHA-256 digests
# of their float32/int32 bytes; the rest (float-atomic sums and what follows
# from them) are stored as values and compared with a tolerance.
BITEXACT = ("radii", "xys", "conics", "colors", "tile_bins", "gaussian_ids", "out_img", "final_T",
            "final_idx", "v_rendered")


PER_GAUSSIAN = {"xys": 2, "conics": 3, "colors": 3}


def visible_subset(key, arr, radii):
    """Per-Gaussian outputs are defined only where radii > 0."""
    if key in PER_GAUSSIAN:
        return np.asarray(arr).reshape(-1, PER_GAUSSIAN[key])[np.asarray(radii) > 0]
    return arr


def digest(a) -> str:
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    if oracle.load_ref() is None:
        raise SystemExit("oracle/_ref/libmsplat_ref.so not built (oracle/ref_shim/build_ref.py)")
    oracle.set_threads(os.cpu_count() or 1)
    meta = {"generator": "tests/golden/make_golden.py", "source": "reference kernels via oracle/ref_shim",
            "adam_steps": ADAM_STEPS, "adam_bc2": ADAM_BC2, "cases": {}}
    for name in CASES:
        out, run = run_case(name, "reference")
        digests = {k: digest(visible_subset(k, out[k], out["radii"])) for k in BITEXACT}
        vals = {k: v for k, v in out.items() if k not in BITEXACT}
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **vals)
        meta["cases"][name] = {"args": list(CASES[name]), "k_max": int(run.P.k_max),
                               "intersections": int(run.num_isects), "loss": run.loss,
                               "sha256": digests}
        print(name, "k_max", run.P.k_max, "isects", run.num_isects)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1)


if __name__ == "__main__":
    main()
