"""Datasets: the reference's Python `Dataset` (python/bindings.cpp:60-98) over
the engine's native loaders (msplat_dataset_* in include/msplat_engine.h).

`Dataset(path, downscale_factor, eval_mode, test_every)` detects the layout
(COLMAP, Nerfstudio, Polycam), loads every training image straight into
device memory (decoded, downscaled and undistorted on the GPU) and splits
train / test cameras as the reference does.  Each `Camera` gives the
intrinsics and pose the training step needs and its ground truth as a
device tensor (`gt(k)`, the image downscaled by k, made once and kept).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib


class _DeviceArray:
    """A borrowed (h, w, 3) float32 device buffer for torch.as_tensor."""

    def __init__(self, ptr: int, h: int, w: int):
        self.__cuda_array_interface__ = {
            "shape": (h, w, 3), "typestr": "<f4", "data": (int(ptr), False), "version": 3,
            "strides": None,
        }


class Camera:
    """Camera (core/include/input_data.hpp:20-40) of an open dataset."""

    def __init__(self, dataset: "Dataset", index: int):
        self._ds = dataset
        self.index = index
        self.refresh()

    def refresh(self) -> None:
        info = _lib.CameraInfo()
        _lib.check(_lib.load().msplat_dataset_camera(self._ds._h, self.index, C.byref(info)),
                   "msplat_dataset_camera")
        self.width, self.height = info.width, info.height
        self.fx, self.fy, self.cx, self.cy = info.fx, info.fy, info.cx, info.cy
        self.k1, self.k2, self.k3, self.p1, self.p2 = info.k1, info.k2, info.k3, info.p1, info.p2
        self.cam_to_world = np.array(list(info.cam_to_world), np.float32).reshape(4, 4)
        self.file_path = _lib.load().msplat_dataset_camera_path(self._ds._h, self.index).decode()

    def gt(self, downscale: int = 1):
        """Camera::getGPUImage: the resident ground truth, (H, W, 3) float32
        on the device, a view that lives as long as the dataset."""
        import torch
        ptr, w, h = C.c_void_p(), C.c_int(), C.c_int()
        _lib.check(_lib.load().msplat_dataset_gt(self._ds._h, self.index, int(downscale),
                                                 C.byref(ptr), C.byref(w), C.byref(h)),
                   "msplat_dataset_gt")
        return torch.as_tensor(_DeviceArray(ptr.value, h.value, w.value), device="cuda")


class Dataset:
    """Dataset(path, downscale_factor=1.0, eval_mode=False, test_every=8)."""

    def __init__(self, path: str, downscale_factor: float = 1.0, eval_mode: bool = False,
                 test_every: int = 8, load_images: bool = True, colmap_image_path: str = ""):
        lib = _lib.load()
        self.downscale_factor = float(downscale_factor)
        self._c = None
        if load_images and not colmap_image_path:
            # the trainer-level dataset (msplat_dataset_create): images loaded, split made
            self._c = lib.msplat_dataset_create(str(path).encode(), self.downscale_factor,
                                                bool(eval_mode), int(test_every))
            if not self._c:
                raise _lib.EngineError("Dataset: " + lib.msplat_last_error().decode())
            self._h = lib.msplat_dataset_data(self._c)
            n = lib.msplat_dataset_num_cameras(self._h)
            self.cameras = [Camera(self, i) for i in range(n)]
            idx = (C.c_int * max(n, 1))()
            tr = [idx[i] for i in range(lib.msplat_dataset_indices(self._c, 0, idx, n))]
            te = [idx[i] for i in range(lib.msplat_dataset_indices(self._c, 1, idx, n))]
        else:
            h = C.c_void_p()
            _lib.check(lib.msplat_dataset_open(str(path).encode(), colmap_image_path.encode(),
                                               C.byref(h)), "msplat_dataset_open")
            self._h = h.value
            if load_images:
                _lib.check(lib.msplat_dataset_load_images(self._h, self.downscale_factor),
                           "msplat_dataset_load_images")
            n = lib.msplat_dataset_num_cameras(self._h)
            self.cameras = [Camera(self, i) for i in range(n)]
            tr, te = list(range(n)), []
            if eval_mode:
                a_ = (C.c_int * max(n, 1))()
                b_ = (C.c_int * max(n, 1))()
                a, b = C.c_int(), C.c_int()
                _lib.check(lib.msplat_dataset_split(self._h, int(test_every), a_, C.byref(a), b_,
                                                    C.byref(b)), "msplat_dataset_split")
                tr, te = list(a_[:a.value]), list(b_[:b.value])
        self.train_cams = [self.cameras[i] for i in tr]
        self.test_cams = [self.cameras[i] for i in te]

    def close(self) -> None:
        lib = _lib.load()
        if getattr(self, "_c", None):
            lib.msplat_dataset_destroy(self._c)   # owns the engine dataset
            self._c = None
            self._h = None
        elif getattr(self, "_h", None):
            lib.msplat_dataset_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 -- interpreter shutdown
            pass

    @property
    def num_train(self) -> int:
        return len(self.train_cams)

    @property
    def num_test(self) -> int:
        return len(self.test_cams)

    def camera_pose(self, index: int) -> np.ndarray:
        if index < 0 or index >= len(self.train_cams):
            raise IndexError("Camera index out of range")
        return self.train_cams[index].cam_to_world.copy()

    def points(self):
        """InputData::points after normalisation: (xyz (N,3) f32, rgb (N,3) u8)."""
        xyz, rgb = C.POINTER(C.c_float)(), C.POINTER(C.c_ubyte)()
        n = _lib.load().msplat_dataset_points(self._h, C.byref(xyz), C.byref(rgb))
        if n <= 0:
            return np.zeros((0, 3), np.float32), np.zeros((0, 3), np.uint8)
        return (np.ctypeslib.as_array(xyz, (n, 3)).copy(), np.ctypeslib.as_array(rgb, (n, 3)).copy())

    def transform(self):
        """(scale, translation[3]) applied by autoScaleAndCenter."""
        s = C.c_float()
        t = (C.c_float * 3)()
        _lib.check(_lib.load().msplat_dataset_transform(self._h, C.byref(s), t), "transform")
        return float(s.value), tuple(t)

    def validation_camera(self, val_image: str = "random") -> int:
        return _lib.load().msplat_dataset_validation_camera(self._h, val_image.encode())

    def device_bytes(self) -> int:
        return int(_lib.load().msplat_dataset_device_bytes(self._h))


def load_dataset(path: str, downscale_factor: float = 1.0, eval_mode: bool = False,
                 test_every: int = 8) -> Dataset:
    return Dataset(path, downscale_factor, eval_mode, test_every)
