"""The reference's data front end, compiled from its sources into
oracle/_ref/libmsplat_ref_data.so (oracle/ref_shim/build_ref.py build_data):
dataset loaders (COLMAP, Nerfstudio, Polycam), autoScaleAndCenter, the
train/test splits, Camera::loadImage / getGPUImage, resizeArea,
undistortImage and the evaluation metrics (ssim_eval, psnr, l1_loss).

TEST INFRASTRUCTURE ONLY (tests/ use it as the checker for
msplat_b200/csrc/dataset.cu and kernels_image.cu).  Images reach the
reference through "<image path>.rgb8" sidecar files (see
oracle/ref_shim/ref_data.cpp), since its decoder is CoreGraphics.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DATA_PATH = os.path.join(HERE, "_ref", "libmsplat_ref_data.so")

_FP = C.POINTER(C.c_float)
_IP = C.POINTER(C.c_int)


def available() -> bool:
    return os.path.exists(REF_DATA_PATH)


def write_rgb8(image_path: str, pixels: np.ndarray) -> None:
    """The sidecar the reference build reads in place of decoding
    `image_path`: "<w> <h>\\n" and the (h, w, 3) uint8 pixels."""
    h, w = pixels.shape[:2]
    with open(image_path + ".rgb8", "wb") as f:
        f.write(f"{w} {h}\n".encode())
        f.write(np.ascontiguousarray(pixels, np.uint8).tobytes())


class RefDataset:
    """InputData loaded by the reference (inputDataFromX)."""

    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            lib = C.CDLL(REF_DATA_PATH)
            lib.ref_data_last_error.restype = C.c_char_p
            lib.ref_dataset_open.restype = C.c_void_p
            lib.ref_dataset_open.argtypes = [C.c_char_p, C.c_char_p]
            lib.ref_dataset_close.argtypes = [C.c_void_p]
            lib.ref_dataset_num_cameras.argtypes = [C.c_void_p]
            lib.ref_dataset_camera.argtypes = [C.c_void_p, C.c_int, _FP]
            lib.ref_dataset_camera_path.restype = C.c_char_p
            lib.ref_dataset_camera_path.argtypes = [C.c_void_p, C.c_int]
            lib.ref_dataset_points.restype = C.c_longlong
            lib.ref_dataset_points.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
            lib.ref_dataset_transform.argtypes = [C.c_void_p, _FP, _FP]
            lib.ref_dataset_split.argtypes = [C.c_void_p, C.c_int, _IP, _IP, _IP, _IP]
            lib.ref_dataset_validation.argtypes = [C.c_void_p, C.c_char_p]
            lib.ref_camera_load_image.argtypes = [C.c_void_p, C.c_int, C.c_float]
            lib.ref_camera_gt.argtypes = [C.c_void_p, C.c_int, C.c_int, _FP, C.c_longlong, _IP, _IP]
            lib.ref_resize_area.argtypes = [_FP, C.c_int, C.c_int, _FP, C.c_int, C.c_int]
            lib.ref_undistort.argtypes = [_FP, C.c_int, C.c_int] + [C.c_float] * 9 + [_FP, _FP, _IP]
            lib.ref_eval.argtypes = [_FP, _FP, C.c_int, C.c_int, C.c_int, C.c_float, _FP]
            cls._lib = lib
        return cls._lib

    def __init__(self, path: str, image_path: str = ""):
        lib = self.lib()
        self.h = lib.ref_dataset_open(str(path).encode(), image_path.encode())
        if not self.h:
            raise RuntimeError(lib.ref_data_last_error().decode())

    def close(self):
        if self.h:
            self.lib().ref_dataset_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    @property
    def num_cameras(self) -> int:
        return self.lib().ref_dataset_num_cameras(self.h)

    def camera(self, i: int) -> dict:
        out = np.zeros(27, np.float32)
        self.lib().ref_dataset_camera(self.h, i, out.ctypes.data_as(_FP))
        keys = ("fx", "fy", "cx", "cy", "k1", "k2", "k3", "p1", "p2")
        cam = {"width": int(out[0]), "height": int(out[1])}
        cam.update({k: np.float32(out[2 + j]) for j, k in enumerate(keys)})
        cam["cam_to_world"] = out[11:27].reshape(4, 4).copy()
        cam["path"] = self.lib().ref_dataset_camera_path(self.h, i).decode()
        return cam

    def points(self):
        n = self.lib().ref_dataset_points(self.h, None, None)
        xyz = np.zeros((n, 3), np.float32)
        rgb = np.zeros((n, 3), np.uint8)
        self.lib().ref_dataset_points(self.h, xyz.ctypes.data, rgb.ctypes.data)
        return xyz, rgb

    def transform(self):
        s = C.c_float()
        t = (C.c_float * 3)()
        self.lib().ref_dataset_transform(self.h, C.byref(s), t)
        return np.float32(s.value), np.array(list(t), np.float32)

    def split(self, test_every: int):
        n = self.num_cameras
        tr, te = np.zeros(n, np.int32), np.zeros(n, np.int32)
        a, b = C.c_int(), C.c_int()
        self.lib().ref_dataset_split(self.h, test_every, tr.ctypes.data_as(_IP), C.byref(a),
                                     te.ctypes.data_as(_IP), C.byref(b))
        return tr[:a.value].tolist(), te[:b.value].tolist()

    def validation(self, val_image: str = "random") -> int:
        return self.lib().ref_dataset_validation(self.h, val_image.encode())

    def load_image(self, i: int, downscale_factor: float) -> None:
        if self.lib().ref_camera_load_image(self.h, i, downscale_factor) != 0:
            raise RuntimeError(self.lib().ref_data_last_error().decode())

    def gt(self, i: int, k: int) -> np.ndarray:
        cam = self.camera(i)
        cap = cam["width"] * cam["height"] * 3
        out = np.zeros(cap, np.float32)
        w, h = C.c_int(), C.c_int()
        rc = self.lib().ref_camera_gt(self.h, i, k, out.ctypes.data_as(_FP), cap, C.byref(w),
                                      C.byref(h))
        assert rc == 0
        return out[:w.value * h.value * 3].reshape(h.value, w.value, 3)


def resize_area(src: np.ndarray, dw: int, dh: int) -> np.ndarray:
    src = np.ascontiguousarray(src, np.float32)
    out = np.zeros((dh, dw, 3), np.float32)
    RefDataset.lib().ref_resize_area(src.ctypes.data_as(_FP), src.shape[1], src.shape[0],
                                     out.ctypes.data_as(_FP), dw, dh)
    return out


def undistort(src: np.ndarray, fx, fy, cx, cy, k1, k2, p1, p2, k3):
    """undistortImage: (cropped image, (fx, fy, cx, cy))."""
    src = np.ascontiguousarray(src, np.float32)
    h, w = src.shape[:2]
    out = np.zeros(w * h * 3, np.float32)
    intr = np.zeros(4, np.float32)
    size = np.zeros(2, np.int32)
    RefDataset.lib().ref_undistort(src.ctypes.data_as(_FP), w, h, fx, fy, cx, cy, k1, k2, p1, p2,
                                   k3, out.ctypes.data_as(_FP), intr.ctypes.data_as(_FP),
                                   size.ctypes.data_as(_IP))
    rw, rh = int(size[0]), int(size[1])
    return out[:rw * rh * 3].reshape(rh, rw, 3), tuple(intr)


def eval_metrics(rendered: np.ndarray, gt: np.ndarray, window: int = 11, sigma: float = 1.5):
    """(psnr, ssim, l1) as the reference's evaluate() computes them."""
    r = np.ascontiguousarray(rendered, np.float32)
    g = np.ascontiguousarray(gt, np.float32)
    out = np.zeros(3, np.float32)
    RefDataset.lib().ref_eval(r.ctypes.data_as(_FP), g.ctypes.data_as(_FP), r.shape[0], r.shape[1],
                              window, sigma, out.ctypes.data_as(_FP))
    return out[0], out[1], out[2]
