"""Dataset loaders on the host (no GPU): the engine's native COLMAP,
Nerfstudio and Polycam readers, point clouds, pose normalisation and splits
(msplat_b200/csrc/dataset.cu through the C-ABI, images not loaded) against
the reference's own loaders compiled from its sources
(oracle/_ref/libmsplat_ref_data.so): cameras, poses, paths, points and the
CRS transform bit-exact."""
from __future__ import annotations

import ctypes as C
import os
import struct

import numpy as np
import pytest

from msplat_b200 import _lib
from msplat_b200.dataset import Dataset
from oracle import data as ref_data
from tests import dataset_case

pytestmark = pytest.mark.skipif(not ref_data.available(),
                                reason="oracle/_ref/libmsplat_ref_data.so not built")


def _open(path):
    return Dataset(path, load_images=False)


@pytest.mark.parametrize("layout", sorted(dataset_case.LAYOUTS))
def test_loader_matches_reference(tmp_path, layout):
    dataset_case.LAYOUTS[layout](str(tmp_path))
    ref = ref_data.RefDataset(str(tmp_path))
    ds = _open(str(tmp_path))
    assert len(ds.cameras) == ref.num_cameras > 0
    for i, cam in enumerate(ds.cameras):
        want = ref.camera(i)
        assert cam.file_path == want["path"]
        assert (cam.width, cam.height) == (want["width"], want["height"])
        for k in ("fx", "fy", "cx", "cy", "k1", "k2", "k3", "p1", "p2"):
            assert np.float32(getattr(cam, k)).tobytes() == want[k].tobytes(), (i, k)
        assert cam.cam_to_world.tobytes() == want["cam_to_world"].tobytes(), i
    xyz, rgb = ds.points()
    rxyz, rrgb = ref.points()
    assert xyz.shape[0] == rxyz.shape[0] > 0
    assert xyz.tobytes() == rxyz.tobytes() and rgb.tobytes() == rrgb.tobytes()
    s, t = ds.transform()
    rs, rt = ref.transform()
    assert np.float32(s) == rs and np.array(t, np.float32).tobytes() == rt.tobytes()
    n = len(ds.cameras)
    for every in (1, 2, 3, 8):
        tr = (C.c_int * n)()
        te = (C.c_int * n)()
        a, b = C.c_int(), C.c_int()
        _lib.check(_lib.load().msplat_dataset_split(ds._h, every, tr, C.byref(a), te, C.byref(b)), "split")
        assert (list(tr[:a.value]), list(te[:b.value])) == ref.split(every)
    for val in ("random", os.path.basename(ds.cameras[-1].file_path), "no-such-image"):
        assert ds.validation_camera(val) == ref.validation(val)
    # the normalised camera centres lie in [-1, 1] with one at the bound
    centres = np.array([c.cam_to_world[:3, 3] for c in ds.cameras])
    assert abs(np.abs(centres).max() - 1.0) < 1e-6


def test_eval_split_mirrors_reference_dataset(tmp_path):
    dataset_case.write_colmap(str(tmp_path))
    ds = Dataset(str(tmp_path), eval_mode=True, test_every=3, load_images=False)
    tr, te = ref_data.RefDataset(str(tmp_path)).split(3)
    assert [c.index for c in ds.train_cams] == tr and [c.index for c in ds.test_cams] == te
    assert ds.num_train == len(tr) and ds.num_test == len(te)
    np.testing.assert_array_equal(ds.camera_pose(0), ds.train_cams[0].cam_to_world)
    with pytest.raises(IndexError):
        ds.camera_pose(ds.num_train)


def test_unknown_layout_and_bad_camera_model(tmp_path):
    with pytest.raises(_lib.EngineError, match="Unrecognized dataset format"):
        _open(str(tmp_path))
    assert ref_data.RefDataset.lib().ref_dataset_open(str(tmp_path).encode(), b"") is None
    dataset_case.write_colmap(str(tmp_path))
    cams = tmp_path / "sparse" / "0" / "cameras.bin"
    cams.write_bytes(struct.pack("<QIIQQ", 1, 1, 5, 64, 48) + struct.pack("<8d", *[1.0] * 8))
    with pytest.raises(_lib.EngineError, match="Unsupported COLMAP camera model: 5"):
        _open(str(tmp_path))
    with pytest.raises(RuntimeError, match="Unsupported COLMAP camera model: 5"):
        ref_data.RefDataset(str(tmp_path))


def test_points_ply_variants(tmp_path):
    """Point-cloud PLYs: ascii with float colours, binary double xyz with
    16-bit colours, no colour at all (grey 128)."""
    rng = np.random.default_rng(5)
    xyz = rng.normal(0, 1, (50, 3))
    rgb = rng.integers(0, 256, (50, 3))
    for i, kw in enumerate([dict(binary=False, rgb_type="float"),
                            dict(binary=True, xyz_type="double", rgb_type="ushort", extra=True),
                            dict(binary=True, rgb=None)]):
        root = tmp_path / f"v{i}"
        dataset_case.write_nerfstudio(str(root))
        args = dict(kw)
        colours = args.pop("rgb", rgb)
        dataset_case.write_points_ply(str(root / "pc.ply"), xyz, colours, **args)
        ds, ref = _open(str(root)), ref_data.RefDataset(str(root))
        got, want = ds.points(), ref.points()
        assert got[0].tobytes() == want[0].tobytes() and got[1].tobytes() == want[1].tobytes()
        if colours is None:
            assert (got[1] == 128).all()
