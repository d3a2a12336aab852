"""The reference's own trainer C API (core/src/msplat_api.mm over
core/src/model.cpp), compiled from its sources into
oracle/_ref/libmsplat_ref_trainer.so (oracle/ref_shim/build_ref.py
build_trainer) and running the reference's kernels on the CPU through the
MSL shim.

TEST INFRASTRUCTURE ONLY: the end-to-end checker for the engine's native
trainer (include/msplat_c_api.h).  Same C signatures as the product's, so
one wrapper drives either library.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_TRAINER_PATH = os.path.join(HERE, "_ref", "libmsplat_ref_trainer.so")


class Config(C.Structure):
    _fields_ = [
        ("iterations", C.c_int), ("shDegree", C.c_int), ("shDegreeInterval", C.c_int),
        ("ssimWeight", C.c_float), ("numDownscales", C.c_int), ("resolutionSchedule", C.c_int),
        ("refineEvery", C.c_int), ("warmupLength", C.c_int), ("resetAlphaEvery", C.c_int),
        ("densifyGradThresh", C.c_float), ("densifySizeThresh", C.c_float),
        ("stopScreenSizeAt", C.c_int), ("splitScreenSize", C.c_float), ("keepCrs", C.c_bool),
        ("downscaleFactor", C.c_float), ("bgColor", C.c_float * 3),
    ]


class Stats(C.Structure):
    _fields_ = [("iteration", C.c_int), ("splatCount", C.c_int), ("msPerStep", C.c_float)]


class Metrics(C.Structure):
    _fields_ = [("psnr", C.c_float), ("ssim", C.c_float), ("l1", C.c_float),
                ("numTest", C.c_int), ("numGaussians", C.c_int)]


class Pixels(C.Structure):
    _fields_ = [("data", C.POINTER(C.c_float)), ("width", C.c_int), ("height", C.c_int)]


def default_config(**kw) -> Config:
    c = Config(30000, 3, 1000, 0.2, 2, 3000, 100, 500, 30, 0.0002, 0.01, 4000, 0.05, False, 1.0,
               (C.c_float * 3)(0.6130, 0.0101, 0.3984))
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def available() -> bool:
    return os.path.exists(REF_TRAINER_PATH)


def bind(lib: C.CDLL) -> C.CDLL:
    """Attach the C API's signatures to `lib` (either implementation)."""
    p, fp = C.c_void_p, C.POINTER(C.c_float)
    sig = {
        "msplat_dataset_create": (p, [C.c_char_p, C.c_float, C.c_bool, C.c_int]),
        "msplat_dataset_destroy": (None, [p]),
        "msplat_dataset_num_train": (C.c_int, [p]),
        "msplat_dataset_num_test": (C.c_int, [p]),
        "msplat_dataset_camera_pose": (None, [p, C.c_int, fp]),
        "msplat_trainer_create": (p, [p, Config]),
        "msplat_trainer_destroy": (None, [p]),
        "msplat_trainer_step": (Stats, [p]),
        "msplat_trainer_evaluate": (Metrics, [p]),
        "msplat_trainer_render": (Pixels, [p, C.c_int, C.c_bool]),
        "msplat_trainer_render_pose": (Pixels, [p, fp, C.c_int]),
        "msplat_trainer_render_pose_to_buffer": (None, [p, fp, C.c_int, C.POINTER(C.c_ubyte),
                                                        C.POINTER(C.c_int), C.POINTER(C.c_int)]),
        "msplat_trainer_export_ply": (None, [p, C.c_char_p]),
        "msplat_trainer_export_splat": (None, [p, C.c_char_p]),
        "msplat_trainer_save_checkpoint": (None, [p, C.c_char_p]),
        "msplat_trainer_load_checkpoint": (C.c_int, [p, C.c_char_p]),
        "msplat_trainer_splat_count": (C.c_int, [p]),
        "msplat_trainer_iteration": (C.c_int, [p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


class Session:
    """A dataset + trainer pair on one implementation of the C API."""

    def __init__(self, lib: C.CDLL, path: str, config: Config, downscale: float = 1.0,
                 eval_mode: bool = False, test_every: int = 8):
        self.lib = lib
        self.ds = lib.msplat_dataset_create(str(path).encode(), downscale, eval_mode, test_every)
        assert self.ds, "dataset creation failed"
        self.t = lib.msplat_trainer_create(self.ds, config)
        assert self.t, "trainer creation failed"

    def close(self):
        if self.t:
            self.lib.msplat_trainer_destroy(self.t)
            self.lib.msplat_dataset_destroy(self.ds)
            self.t = self.ds = None

    def step(self):
        s = self.lib.msplat_trainer_step(self.t)
        return s.iteration, s.splatCount

    def render(self, index: int, test: bool = False) -> np.ndarray:
        pb = self.lib.msplat_trainer_render(self.t, index, test)
        return self._take(pb)

    def render_pose(self, pose, ref: int = 0) -> np.ndarray:
        pose = np.ascontiguousarray(pose, np.float32)
        return self._take(self.lib.msplat_trainer_render_pose(
            self.t, pose.ctypes.data_as(C.POINTER(C.c_float)), ref))

    def render_rgba(self, pose, ref: int = 0) -> np.ndarray:
        pose = np.ascontiguousarray(pose, np.float32)
        fp = pose.ctypes.data_as(C.POINTER(C.c_float))
        w, h = C.c_int(), C.c_int()
        self.lib.msplat_trainer_render_pose_to_buffer(self.t, fp, ref, None, C.byref(w), C.byref(h))
        out = np.zeros((h.value, w.value, 4), np.uint8)
        self.lib.msplat_trainer_render_pose_to_buffer(
            self.t, fp, ref, out.ctypes.data_as(C.POINTER(C.c_ubyte)), C.byref(w), C.byref(h))
        return out

    def evaluate(self):
        m = self.lib.msplat_trainer_evaluate(self.t)
        return m.psnr, m.ssim, m.l1, m.numTest, m.numGaussians

    @staticmethod
    def _take(pb) -> np.ndarray:
        assert pb.data, "render failed"
        n = pb.width * pb.height * 3
        out = np.ctypeslib.as_array(pb.data, (n,)).reshape(pb.height, pb.width, 3).copy()
        C.CDLL(None).free(C.cast(pb.data, C.c_void_p))
        return out


def reference() -> C.CDLL:
    return bind(C.CDLL(REF_TRAINER_PATH))
