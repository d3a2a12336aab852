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
    # compact at 8 ranks: each way, 15 gradient floats and 59 parameter
    # floats of 7/8 of the Gaussians
    assert r["bytes_out"] == r["bytes_in"] == int(7 / 8 * n * 74 * 4)
    assert abs(r["bound_ms"] - r["bytes_out"] / 770e9 * 1e3) < 1e-3
    assert 0.65 < r["frac"] < 0.7
    r = bench.exchange_roofline(n, 4, False, "peer", 3.907)
    assert r["bytes_in"] == int(3 / 4 * n * 119 * 4)


def _ncu_csv(path, kernel, values):
    hdr = ('"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream",'
           '"Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit",'
           '"Metric Value"\n')
    rows = []
    for metric, unit, val in values:
        rows.append(f'"0","11","python3","127.0.0.1","{kernel}","1","7","(256, 1, 1)",'
                    f'"(4346, 1, 1)","0","10.0","Command line profiler metrics","{metric}",'
                    f'"{unit}","{val}"\n')
    path.write_text("==PROF== Connected to process 11\n" + hdr + "".join(rows))


def test_counter_summary_round_trip(tmp_path, monkeypatch):
    """--summarize-ncu writes the per-kernel summary bench.py reads back;
    the build hash decides whether a run may use it."""
    csvs = []
    for kern, rd in (("void raster_forward_kernel<0>(const StepParams *, int)", 1000),
                     ("msp::sort_tiles_kernel(const msp::StepParams *, const int *)", 2000)):
        p = tmp_path / f"{rd}.csv"
        _ncu_csv(p, kern, [("dram__bytes_read.sum", "byte", f"{rd:,}"),
                           ("dram__bytes_write.sum", "byte", "500"),
                           ("smsp__inst_executed.sum", "inst", "123,456"),
                           ("gpu__time_duration.sum", "nsecond", "98765")])
        csvs.append(str(p))
    hf = tmp_path / "h.json"
    hf.write_text('loading\n{"build_hash": "%s", "view": 5, "warmup": 5}\n' % bench.build_hash())
    out = str(tmp_path / "counters.txt")
    bench.summarize_ncu(csvs, str(hf), out)
    ctr = bench.load_counters(out)
    assert ctr["view"] == 5 and ctr["build"] == bench.build_hash()
    k = ctr["kernels"]
    assert set(k) == {"raster_forward_kernel", "sort_tiles_kernel"}
    assert k["raster_forward_kernel"]["dram_read_bytes"] == 1000
    assert k["sort_tiles_kernel"]["warp_instructions"] == 123456
    assert k["sort_tiles_kernel"]["duration_ns"] == 98765
    monkeypatch.setattr(bench, "COUNTERS_FILE", out)
    assert bench.counters_status(ctr)["matches_this_build"]
    assert not bench.counters_status(dict(ctr, build="0" * 12))["matches_this_build"]
    roof = bench.issue_rooflines({"rast_fwd": 0.4, "bin_sort": 0.1}, 1965.0, k,
                                 {"rast_fwd": 2.0})
    fwd = [r for r in roof if r["stage"] == "rast_fwd"][0]
    assert fwd["warp_instructions"] == 2 * 123456 and fwd["work_scale"] == 2.0


def test_balanced_views_split_the_batch_evenly():
    costs = [31, 34, 32, 33, 30, 35, 29, 36]
    for world in (1, 2, 4, 8):
        groups = bench.balanced_views(costs, world)
        assert sorted(v for g in groups for v in g) == list(range(8))
        assert all(len(g) == 8 // world for g in groups)
    two = bench.balanced_views(costs, 2)
    loads = [sum(costs[v] for v in g) for g in two]
    assert abs(loads[0] - loads[1]) <= 2          # round-robin would give 8
    assert bench.balanced_views(costs, 2) == two  # deterministic
