"""The oracle against golden fixtures produced by the reference's own
kernels (tests/golden/make_golden.py), and -- when the reference build
oracle/_ref exists -- against the reference build directly."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from oracle import oracle
from tests import harness
from tests.golden import make_golden as mg

HERE = os.path.dirname(os.path.abspath(__file__))
META = json.load(open(os.path.join(HERE, "golden", "golden.json")))
TOL_FIELDS = ("v_xy", "v_conic", "v_rgb", "v_opacity", "v_mean3d", "v_scale", "v_quat")


def check_against_golden(name, out, num_isects):
    case = META["cases"][name]
    assert num_isects == case["intersections"]
    for key, want in case["sha256"].items():
        got = mg.digest(mg.visible_subset(key, out[key], out["radii"]))
        assert got == want, f"{name}: {key} differs from the reference"
    gold = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    for key in TOL_FIELDS:
        bad, worst = harness.close(out[key], gold[key], 1e-4, 2e-6)
        assert bad == 0, f"{name}: {key} {bad} out of tolerance ({worst:.3g})"
    for key in gold.files:
        if key.startswith("param_") or key in ("vis_counts", "xys_grad_norm", "max_2d_size"):
            bad, worst = harness.close(out[key], gold[key], 1e-4, 1e-6)
            assert bad == 0, f"{name}: {key} {bad} out of tolerance ({worst:.3g})"


@pytest.mark.parametrize("name", sorted(mg.CASES))
def test_oracle_matches_reference_golden(name):
    out, run = mg.run_case(name, "oracle")
    check_against_golden(name, out, run.num_isects)


@pytest.mark.parametrize("name", sorted(mg.CASES))
def test_reference_build_reproduces_golden(name):
    if oracle.load_ref() is None:
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    out, run = mg.run_case(name, "reference")
    check_against_golden(name, out, run.num_isects)
