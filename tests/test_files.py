"""Model files on the host (no GPU): the engine's checkpoint, PLY and .splat
writers and readers (msplat_b200/csrc/io.cu, called through the C-ABI on
host arrays) against the reference's own code compiled from its sources
(oracle/_ref/libmsplat_ref_io.so), the committed fixtures that code wrote,
and the checkpoint restatement of Model::saveCheckpoint."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

from msplat_b200 import _lib
from oracle import files
from tests import io_case
from tests.golden.make_io_golden import step_of

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "io")
needs_ref = pytest.mark.skipif(not files.RefIO.available(),
                               reason="oracle/_ref/libmsplat_ref_io.so not built")


def _ptrs(arrs):
    return (C.c_void_p * 6)(*[a.ctypes.data if a is not None else None for a in arrs])


def _case(name):
    n, rb, seed, keep, scale, trans = io_case.CASES[name]
    return io_case.gaussians(n, rb, seed), rb, keep, scale, trans


def eng_save_ply(path, step, params, keep=False, scale=1.0, trans=(0, 0, 0)):
    rc = _lib.load().msplat_save_ply(str(path).encode(), step, params[0].shape[0],
                                     params[4].shape[1], _ptrs(params), int(keep), scale,
                                     _lib.farr(trans))
    _lib.check(rc, "msplat_save_ply")


def eng_save_splat(path, params, keep=False, scale=1.0, trans=(0, 0, 0)):
    rc = _lib.load().msplat_save_splat(str(path).encode(), params[0].shape[0], _ptrs(params),
                                       int(keep), scale, _lib.farr(trans))
    _lib.check(rc, "msplat_save_splat")


def eng_load_ply(path, capacity, rest_bases, keep=False, scale=1.0, trans=(0, 0, 0)):
    lib = _lib.load()
    n, step, rb = C.c_int(), C.c_int(), C.c_int()
    _lib.check(lib.msplat_read_ply_header(str(path).encode(), C.byref(n), C.byref(step),
                                          C.byref(rb)), "msplat_read_ply_header")
    assert rb.value == rest_bases
    out = [np.full(s, np.nan, np.float32) for s in files.group_shapes(capacity, rest_bases)]
    rc = lib.msplat_load_ply(str(path).encode(), capacity, _ptrs(out), int(keep), scale,
                             _lib.farr(trans))
    if rc < 0:
        _lib.check(rc, "msplat_load_ply")
    assert rc == step.value
    return [a[:n.value] for a in out], rc, out


def eng_save_ckpt(path, step, params, m, v, sh_degree=3, adam_steps=5,
                  lr=(1, 2, 3, 4, 5, 6), lr0=0.00016, lr1=0.0000016):
    rc = _lib.load().msplat_save_checkpoint(
        str(path).encode(), step, params[0].shape[0], sh_degree, adam_steps, _lib.farr(lr), lr0,
        lr1, params[4].shape[1], _ptrs(params), _ptrs(m), _ptrs(v))
    _lib.check(rc, "msplat_save_checkpoint")


# ---- PLY / .splat --------------------------------------------------------------------

@needs_ref
def test_ply_restatement_matches_reference(tmp_path):
    """The byte-level PLY restatement is pinned to the reference's writer."""
    for name in ("deg3", "deg0"):
        params, *_ = _case(name)
        files.RefIO().save_ply(tmp_path / "r.ply", 42, params)
        assert (tmp_path / "r.ply").read_bytes() == files.ply_bytes(42, params)


@pytest.mark.parametrize("name", sorted(io_case.CASES))
def test_ply_and_splat_match_reference_fixtures(tmp_path, name):
    params, rb, keep, scale, trans = _case(name)
    eng_save_ply(tmp_path / "e.ply", step_of(name), params, keep, scale, trans)
    eng_save_splat(tmp_path / "e.splat", params, keep, scale, trans)
    assert (tmp_path / "e.ply").read_bytes() == open(os.path.join(GOLDEN, f"{name}.ply"), "rb").read()
    assert (tmp_path / "e.splat").read_bytes() == open(os.path.join(GOLDEN, f"{name}.splat"), "rb").read()


@needs_ref
@pytest.mark.parametrize("keep", [False, True])
def test_ply_and_splat_match_reference_live(tmp_path, keep):
    """Fresh seeds through both writers, with and without the CRS transform;
    features_rest may be NULL for .splat."""
    ref = files.RefIO()
    for seed in range(3):
        params = io_case.gaussians(200 + 50 * seed, 15, 300 + seed)
        scale, trans = 0.5 + seed, (seed * 3.0, -1.5, 0.25)
        ref.save_ply(tmp_path / "r.ply", seed, params, keep, scale, trans)
        eng_save_ply(tmp_path / "e.ply", seed, params, keep, scale, trans)
        assert (tmp_path / "e.ply").read_bytes() == (tmp_path / "r.ply").read_bytes()
        ref.save_splat(tmp_path / "r.splat", params, keep, scale, trans)
        no_rest = list(params)
        no_rest[4] = None
        eng_save_splat(tmp_path / "e.splat", no_rest, keep, scale, trans)
        assert (tmp_path / "e.splat").read_bytes() == (tmp_path / "r.splat").read_bytes()


def test_splat_record_layout(tmp_path):
    """32-byte records ordered by size x sigmoid(opacity), largest first
    (save_gaussians.cpp:64-96); the u8 fields clamped."""
    params, *_ = _case("deg3")
    eng_save_splat(tmp_path / "e.splat", params)
    rec = np.frombuffer((tmp_path / "e.splat").read_bytes(), np.uint8).reshape(-1, 32)
    n = params[0].shape[0]
    assert rec.shape[0] == n
    pos = rec[:, :12].copy().view("<f4")
    size = rec[:, 12:24].copy().view("<f4")
    order = size.sum(1) * (rec[:, 27] / 255.0)
    assert np.all(np.diff(order) <= 0.02 * order[:-1] + 0.02)   # alpha is quantised
    src = {tuple(p): i for i, p in enumerate(params[0])}
    idx = np.array([src[tuple(p)] for p in pos])
    assert sorted(idx) == list(range(n))
    np.testing.assert_allclose(size, np.exp(params[1][idx]), rtol=1e-6)
    q = np.clip(params[2][idx] * 128 + 128, 0, 255).astype(np.uint8)
    assert np.array_equal(rec[:, 28:32], q)
    assert rec[:, 24:27].max() == 255 and rec[:, 24:27].min() == 0


@needs_ref
@pytest.mark.parametrize("name", sorted(io_case.CASES))
def test_load_ply_matches_reference(tmp_path, name):
    params, rb, keep, scale, trans = _case(name)
    path = os.path.join(GOLDEN, f"{name}.ply")
    ref, ref_step = files.RefIO().load_ply(path, 64, rb, keep, scale, trans)
    got, step, full = eng_load_ply(path, 64, rb, keep, scale, trans)
    assert step == ref_step == 0   # the writer's comment is not the one the reader parses
    for a, b in zip(got, ref):
        assert a.tobytes() == b.tobytes()
    n = params[0].shape[0]
    assert all(np.isnan(a[n:]).all() for a in full)   # rows past N untouched
    if not keep:
        for a, b in zip(got, params):
            assert a.tobytes() == b.tobytes()


def test_ply_round_trip_and_step_comment(tmp_path):
    """save -> load gives the same arrays; a PLY whose header carries
    "comment Generated by msplat at iteration <k>" loads with step k."""
    params, rb, *_ = _case("deg3")
    eng_save_ply(tmp_path / "a.ply", 9, params)
    got, step, _ = eng_load_ply(tmp_path / "a.ply", 40, rb)
    assert step == 0
    assert all(a.tobytes() == b.tobytes() for a, b in zip(got, params))
    blob = (tmp_path / "a.ply").read_bytes().replace(
        b"comment msplat v9\n", b"comment Generated by msplat at iteration 1234\n")
    (tmp_path / "b.ply").write_bytes(blob)
    got, step, _ = eng_load_ply(tmp_path / "b.ply", 40, rb)
    assert step == 1234
    parsed, pstep = files.read_ply(blob)
    assert pstep == 1234 and all(a.tobytes() == b.tobytes() for a, b in zip(parsed, params))


def test_ply_errors(tmp_path):
    lib = _lib.load()
    n = C.c_int()
    out = _ptrs([None] * 6)
    (tmp_path / "x.ply").write_bytes(b"not a ply\n")
    assert lib.msplat_read_ply_header(str(tmp_path / "x.ply").encode(), C.byref(n), None, None) < 0
    assert b"PLY" in lib.msplat_last_error()
    assert lib.msplat_load_ply(str(tmp_path / "missing.ply").encode(), 4, out, 0, 1.0,
                               _lib.farr((0, 0, 0))) < 0
    params, *_ = _case("deg3")
    eng_save_ply(tmp_path / "a.ply", 1, params)
    assert lib.msplat_load_ply(str(tmp_path / "a.ply").encode(), 10, out, 0, 1.0,
                               _lib.farr((0, 0, 0))) < 0      # 37 rows do not fit in 10
    (tmp_path / "t.ply").write_bytes((tmp_path / "a.ply").read_bytes()[:-100])
    full = [np.zeros(s, np.float32) for s in files.group_shapes(40, 15)]
    assert lib.msplat_load_ply(str(tmp_path / "t.ply").encode(), 40, _ptrs(full), 0, 1.0,
                               _lib.farr((0, 0, 0))) < 0      # truncated vertex data


# ---- .msplat checkpoints -------------------------------------------------------------

@pytest.mark.parametrize("name", sorted(io_case.CASES))
def test_checkpoint_bytes_and_round_trip(tmp_path, name):
    params, rb, *_ = _case(name)
    n = params[0].shape[0]
    m, v = io_case.moments(params, 5)
    lr = (0.1, 0.2, 0.3, 0.4, 0.5, 0.6)
    eng_save_ckpt(tmp_path / "c.msplat", 777, params, m, v, 3, 41, lr, 0.00016, 0.0000016)
    blob = (tmp_path / "c.msplat").read_bytes()
    assert blob == files.checkpoint_bytes(777, n, 3, 41, lr, 0.00016, 0.0000016, params, m, v)
    lib = _lib.load()
    step, num, deg, ast, bases = (C.c_int() for _ in range(5))
    lrs = (C.c_float * 6)()
    l0, l1 = C.c_float(), C.c_float()
    _lib.check(lib.msplat_read_checkpoint_header(
        str(tmp_path / "c.msplat").encode(), C.byref(step), C.byref(num), C.byref(deg),
        C.byref(ast), lrs, C.byref(l0), C.byref(l1), C.byref(bases)), "header")
    assert (step.value, num.value, deg.value, ast.value, bases.value) == (777, n, 3, 41, rb)
    assert list(lrs) == list(np.float32(lr)) and l0.value == np.float32(0.00016)
    cap = 4 * n
    out = [[np.full(s, np.nan, np.float32) for s in files.group_shapes(cap, rb)] for _ in range(3)]
    rc = lib.msplat_load_checkpoint(str(tmp_path / "c.msplat").encode(), cap, *map(_ptrs, out))
    assert rc == 777
    for got, want in zip(out, (params, m, v)):
        for a, b in zip(got, want):
            assert a[:n].tobytes() == b.tobytes() and np.isnan(a[n:]).all()
    parsed = files.read_checkpoint(blob)
    assert parsed["size"] == len(blob) and parsed["num_active"] == n


def test_checkpoint_errors(tmp_path):
    params, rb, *_ = _case("deg3")
    m, v = io_case.moments(params, 1)
    eng_save_ckpt(tmp_path / "c.msplat", 5, params, m, v)
    blob = (tmp_path / "c.msplat").read_bytes()
    lib = _lib.load()
    n = params[0].shape[0]
    outs = [[np.zeros(s, np.float32) for s in files.group_shapes(n, rb)] for _ in range(3)]

    def load(data, cap=n):
        (tmp_path / "x.msplat").write_bytes(data)
        return lib.msplat_load_checkpoint(str(tmp_path / "x.msplat").encode(), cap,
                                          *map(_ptrs, outs))
    assert load(blob) == 5
    assert load(b"XXXX" + blob[4:]) < 0
    assert b"not a valid msplat checkpoint" in lib.msplat_last_error()
    assert load(blob[:4] + (2).to_bytes(4, "little") + blob[8:]) < 0
    assert b"unsupported checkpoint version 2" in lib.msplat_last_error()
    assert load(blob[:-8]) < 0                       # truncated inside the last tensor
    assert load(blob, cap=n - 1) < 0                 # too many Gaussians for the buffers
    bad = bytearray(blob)
    bad[56 + 4:56 + 12] = (n + 1).to_bytes(8, "little")   # means tensor claims n+1 rows
    assert load(bytes(bad)) < 0
    assert lib.msplat_load_checkpoint(str(tmp_path / "none.msplat").encode(), n,
                                      *map(_ptrs, outs)) < 0
