"""bench.py helpers that need no GPU: the on-disk scene cache returns the
seeded scene bit for bit, and the exchange byte counts of the batched-view
report follow the peer and NCCL protocols."""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402
from msplat_b200 import synthetic  # noqa: E402


def test_scene_cache_round_trip(tmp_path, monkeypatch):
    monkeypatch.setenv("MSPLAT_BENCH_SCENE_CACHE", str(tmp_path))
    want, wcams = synthetic.scene("C0", seed=3)
    first, _ = bench.scene("C0", seed=3)            # drawn, then written
    assert os.path.exists(tmp_path / "C0_seed3.npz")
    second, cams = bench.scene("C0", seed=3)        # read back
    for a, b, c in zip(want.groups(), first.groups(), second.groups()):
        np.testing.assert_array_equal(a, b)
        np.testing.assert_array_equal(a, c)
        assert c.dtype == np.float32
    assert len(cams) == len(wcams)
    np.testing.assert_array_equal(cams[0].cam_to_world, wcams[0].cam_to_world)
    assert not [p for p in os.listdir(tmp_path) if p.endswith(".tmp.npz")]


def test_exchange_bytes():
    n = 1000
    assert bench.exchange_bytes(n, 1, False, "peer") == 0
    # peer, full layout: read 60 gradient floats and write 59 parameter
    # floats of (world-1)/world of the Gaussians
    assert bench.exchange_bytes(n, 2, False, "peer") == int(0.5 * n * 119 * 4)
    # compact layout: 15 gradient floats
    assert bench.exchange_bytes(n, 8, True, "peer") == int(7 / 8 * n * 74 * 4)
    # ring all-reduce of the 60-float buffer
    assert bench.exchange_bytes(n, 4, False, "nccl") == int(2 * 0.75 * n * 60 * 4)


def test_exchange_roofline():
    n = 6_000_000
    assert bench.exchange_roofline(n, 1, False, "peer", 1.0) is None
    r = bench.exchange_roofline(n, 8, True, "peer", 2.967)
    # compact at 8 ranks: the parameter write-back (59 floats) is the larger way
    assert r["bytes_out"] == int(7 / 8 * n * 59 * 4) and r["bytes_in"] == int(7 / 8 * n * 15 * 4)
    assert abs(r["bound_ms"] - r["bytes_out"] / 770e9 * 1e3) < 1e-3
    assert 0.5 < r["frac"] < 0.6
    r = bench.exchange_roofline(n, 4, False, "peer", 3.907)
    assert r["bytes_in"] > r["bytes_out"]          # 60 gradient floats in, 59 out
