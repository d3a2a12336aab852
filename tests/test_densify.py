"""Densification (msplat_densify): the CPU oracle against the reference's
own kernels compiled through the MSL shim, bit for bit, on seeded inputs
with every flag setting the training schedule uses."""
from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import oracle
from tests import densify_case

HAS_REF = os.path.exists(oracle.REF_PATH)
# thresholds that, for densify_case's statistics, split and duplicate both
THRESH = {"grad": 60.0, "size": 0.04}

SETTINGS = [dict(check_screen=True, check_huge=True), dict(check_screen=False, check_huge=True),
            dict(check_screen=True, check_huge=False), dict(check_screen=False, check_huge=False)]


def _run(n, seed, impl, **kw):
    bufs, ea, es, gnorm, vis, max2d, samples = densify_case.make(n, seed)
    res = oracle.densify(bufs, ea, es, n, gnorm, vis, max2d, samples, half_max_dim=648.5,
                         grad_thresh=THRESH["grad"], size_thresh=THRESH["size"], impl=impl, **kw)
    return res, bufs, ea, es


def test_oracle_densify_grows_and_culls():
    (count, split, dup, keep), bufs, _, _ = _run(4000, 1, "oracle")
    assert split.sum() > 50 and dup.sum() > 50, (split.sum(), dup.sum())
    assert 0 < count < 4000 + 2 * split.sum() + dup.sum()
    assert keep[:count].dtype == np.int32 and keep.sum() == count
    assert np.isfinite(bufs[0][:count]).all()


@pytest.mark.skipif(not HAS_REF, reason="reference build (oracle/_ref) not present")
@pytest.mark.parametrize("setting", range(len(SETTINGS)))
def test_oracle_densify_matches_reference(setting):
    kw = SETTINGS[setting]
    (c1, s1, d1, k1), b1, m1, v1 = _run(3000, 2 + setting, "oracle", **kw)
    (c2, s2, d2, k2), b2, m2, v2 = _run(3000, 2 + setting, "reference", **kw)
    assert c1 == c2
    np.testing.assert_array_equal(s1, s2)
    np.testing.assert_array_equal(d1, d2)
    np.testing.assert_array_equal(k1, k2)
    for g in range(6):
        np.testing.assert_array_equal(b1[g][:c1], b2[g][:c1], err_msg=f"params {g}")
        np.testing.assert_array_equal(m1[g][:c1], m2[g][:c1], err_msg=f"exp_avg {g}")
        np.testing.assert_array_equal(v1[g][:c1], v2[g][:c1], err_msg=f"exp_avg_sq {g}")
