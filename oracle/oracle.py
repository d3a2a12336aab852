"""ctypes front end of the CPU oracle (oracle/libmsplat_oracle.so).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline leg use it as the checker; the engine never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmsplat_oracle.so")


class Params(C.Structure):
    _fields_ = [
        ("num_points", C.c_int32), ("img_w", C.c_int32), ("img_h", C.c_int32),
        ("tiles_x", C.c_int32), ("tiles_y", C.c_int32), ("degree", C.c_int32),
        ("degrees_to_use", C.c_int32), ("k_max", C.c_int32),
        ("viewmat", C.c_float * 16), ("projmat", C.c_float * 16),
        ("fx", C.c_float), ("fy", C.c_float), ("cx", C.c_float), ("cy", C.c_float),
        ("glob_scale", C.c_float), ("clip_thresh", C.c_float),
        ("cam_pos", C.c_float * 3), ("background", C.c_float * 3),
        ("ssim_weight", C.c_float), ("loss_inv_n", C.c_float), ("inv_max_dim", C.c_float),
        ("adam_step_size", C.c_float * 6), ("adam_bc2_sqrt", C.c_float * 6),
        ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float),
    ]


_FP = C.POINTER(C.c_float)
_IP = C.POINTER(C.c_int32)


class State(C.Structure):
    _fields_ = [
        ("xys", _FP), ("depths", _FP), ("radii", _IP), ("conics", _FP), ("num_tiles_hit", _IP),
        ("colors", _FP), ("aabb", _FP), ("tile_bins", _IP), ("gaussian_ids", _IP),
        ("isect_capacity", C.c_int64), ("num_isects", C.c_int64),
        ("out_img", _FP), ("final_T", _FP), ("final_idx", _IP), ("v_rendered", _FP),
        ("loss", C.c_double), ("v_xy", _FP), ("v_conic", _FP), ("v_rgb", _FP),
        ("v_opacity", _FP), ("v_mean3d", _FP), ("v_scale", _FP), ("v_quat", _FP),
        ("max_tile_count", C.c_int32),
    ]


_lib = None
_ref = None
REF_PATH = os.path.join(HERE, "_ref", "libmsplat_ref.so")


def load_ref():
    """The reference's own kernels built through the MSL shim
    (oracle/ref_shim/build_ref.py); None when it was not built."""
    global _ref
    if _ref is None and os.path.exists(REF_PATH):
        lib = C.CDLL(REF_PATH)
        for name in ("ref_train_step", "ref_render", "ref_tile_cap", "ref_densify"):
            getattr(lib, name).restype = C.c_int
        lib.ref_set_threads.argtypes = [C.c_int]
        _ref = lib
    return _ref


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        lib = C.CDLL(LIB_PATH)
        lib.msp_expf.restype = C.c_float
        lib.msp_expf.argtypes = [C.c_float]
        lib.orc_set_threads.argtypes = [C.c_int]
        lib.orc_chunk_k_max.restype = C.c_int32
        lib.orc_chunk_k_max.argtypes = [C.c_int32, C.c_int32]
        for name in ("orc_train_step", "orc_render", "orc_densify"):
            getattr(lib, name).restype = C.c_int
        _lib = lib
    return _lib


def _fp(a):
    return a.ctypes.data_as(_FP) if a is not None else None


def _ip(a):
    return a.ctypes.data_as(_IP) if a is not None else None


class Run:
    """Holds the oracle's parameter block and every intermediate it dumps."""

    def __init__(self, cam, n: int, ssim_weight: float = 0.2, background=(0.6130, 0.0101, 0.3984),
                 adam_steps=None, adam_bc2=None, glob_scale=1.0, clip_thresh=0.01,
                 isect_capacity=None, degrees_to_use=None):
        lib = load()
        P = Params()
        P.num_points = n
        P.img_w, P.img_h = cam.width, cam.height
        P.tiles_x, P.tiles_y = cam.tile_bounds[0], cam.tile_bounds[1]
        P.degree = cam.degree
        P.degrees_to_use = cam.degrees_to_use if degrees_to_use is None else degrees_to_use
        P.k_max = lib.orc_chunk_k_max(n, P.tiles_x * P.tiles_y)
        P.viewmat[:] = [float(x) for x in cam.viewmat]
        P.projmat[:] = [float(x) for x in cam.projmat]
        P.fx, P.fy, P.cx, P.cy = cam.fx, cam.fy, cam.cx, cam.cy
        P.glob_scale, P.clip_thresh = glob_scale, clip_thresh
        P.cam_pos[:] = [float(x) for x in cam.cam_pos]
        P.background[:] = list(background)
        P.ssim_weight = ssim_weight
        h, w = cam.height, cam.width
        P.loss_inv_n = float(np.float32(1.0) / np.float32(h * w * 3))
        P.inv_max_dim = float(np.float32(1.0) / np.float32(max(h, w)))
        if adam_steps is not None:
            P.adam_step_size[:] = [float(x) for x in adam_steps]
            P.adam_bc2_sqrt[:] = [float(x) for x in adam_bc2]
        P.beta1, P.beta2, P.eps = 0.9, 0.999, 1e-8
        self.P = P
        T = P.tiles_x * P.tiles_y
        cap = 16 * n if isect_capacity is None else isect_capacity
        f, i = np.float32, np.int32
        self.xys = np.zeros(n * 2, f); self.depths = np.zeros(n, f)
        self.radii = np.zeros(n, i); self.conics = np.zeros(n * 3, f)
        self.num_tiles_hit = np.zeros(n, i); self.colors = np.zeros(n * 3, f)
        self.aabb = np.zeros(n * 2, f); self.tile_bins = np.zeros(T * 2, i)
        self.gaussian_ids = np.zeros(max(cap, 1), i)
        self.out_img = np.zeros(h * w * 3, f); self.final_T = np.zeros(h * w, f)
        self.final_idx = np.zeros(h * w, i); self.v_rendered = np.zeros(h * w * 3, f)
        self.v_xy = np.zeros(n * 2, f); self.v_conic = np.zeros(n * 3, f)
        self.v_rgb = np.zeros(n * 3, f); self.v_opacity = np.zeros(n, f)
        self.v_mean3d = np.zeros(n * 3, f); self.v_scale = np.zeros(n * 3, f)
        self.v_quat = np.zeros(n * 4, f)
        S = State()
        for name in ("xys", "depths", "conics", "colors", "aabb", "out_img", "final_T",
                     "v_rendered", "v_xy", "v_conic", "v_rgb", "v_opacity", "v_mean3d",
                     "v_scale", "v_quat"):
            setattr(S, name, _fp(getattr(self, name)))
        for name in ("radii", "num_tiles_hit", "tile_bins", "gaussian_ids", "final_idx"):
            setattr(S, name, _ip(getattr(self, name)))
        S.isect_capacity = cap
        self.S = S

    @property
    def num_isects(self) -> int:
        return int(self.S.num_isects)

    @property
    def loss(self) -> float:
        return float(self.S.loss)

    def render(self, groups, impl: str = "oracle") -> int:
        """impl "oracle" runs the C restatement, "reference" the reference's
        kernels through the shim (returns 1 when a tile overflowed its cap)."""
        arrs = [np.ascontiguousarray(g, dtype=np.float32) for g in groups]
        ptrs = (_FP * 6)(*[_fp(a) for a in arrs])
        if impl == "reference":
            return int(load_ref().ref_render(C.byref(self.P), C.byref(self.S), ptrs))
        rc = load().orc_render(C.byref(self.P), C.byref(self.S), ptrs)
        if rc != 0:
            raise RuntimeError("oracle: intersection capacity too small")
        return 0

    def train_step(self, params, exp_avg, exp_avg_sq, gt, vis_counts, grad_norm, max_2d,
                   impl: str = "oracle") -> int:
        """Updates params / moments / statistics in place (float32 arrays)."""
        pp = (_FP * 6)(*[_fp(a) for a in params])
        mm = (_FP * 6)(*[_fp(a) for a in exp_avg])
        vv = (_FP * 6)(*[_fp(a) for a in exp_avg_sq])
        args = (C.byref(self.P), C.byref(self.S), pp, mm, vv, _fp(gt), _fp(vis_counts),
                _fp(grad_norm), _fp(max_2d))
        if impl == "reference":
            return int(load_ref().ref_train_step(*args))
        rc = load().orc_train_step(*args)
        if rc != 0:
            raise RuntimeError("oracle: intersection capacity too small")
        return 0


def expf(x: float) -> float:
    return float(load().msp_expf(float(x)))


def set_threads(n: int) -> None:
    load().orc_set_threads(int(n))


def chunk_k_max(n: int, num_tiles: int) -> int:
    return int(load().orc_chunk_k_max(n, num_tiles))


def densify(bufs, exp_avg, exp_avg_sq, n: int, xys_grad_norm, vis_counts, max_2d_size,
            random_samples, half_max_dim: float, grad_thresh: float = 0.0002,
            size_thresh: float = 0.01, screen_thresh: float = 0.05, check_screen: bool = True,
            cull_alpha_thresh: float = 0.1, cull_scale_thresh: float = 0.5,
            cull_screen_size: float = 0.15, check_huge: bool = True, impl: str = "oracle"):
    """msplat_densify on float32 numpy buffers of >= 3n rows (updated in
    place, group order means, scales, quats, features_dc, features_rest,
    opacities).  impl "oracle" runs the C restatement, "reference" the
    reference's kernels through the shim.  Returns (new_count, split flags,
    duplicate flags, keep flags)."""
    cap = min(b.shape[0] for b in bufs)
    fr_stride = int(np.prod(bufs[4].shape[1:]))
    split = np.zeros(max(n, 1), np.int32)
    dup = np.zeros(max(n, 1), np.int32)
    keep = np.zeros(max(3 * n, 1), np.int32)
    pb = (_FP * 6)(*[_fp(b) for b in bufs])
    pm = (_FP * 6)(*[_fp(b) for b in exp_avg])
    pv = (_FP * 6)(*[_fp(b) for b in exp_avg_sq])
    lib = load_ref() if impl == "reference" else load()
    fn = lib.ref_densify if impl == "reference" else lib.orc_densify
    fn.argtypes = [C.c_int, C.c_int, C.c_float, C.c_float, C.c_float, C.c_int, C.c_float,
                   C.c_float, C.c_float, C.c_int, _FP, _FP, _FP, C.c_float, _FP * 6, C.c_int,
                   _FP * 6, _FP * 6, _FP, _IP, _IP, _IP]
    rc = fn(n, cap, grad_thresh, size_thresh, screen_thresh, int(check_screen),
            cull_alpha_thresh, cull_scale_thresh, cull_screen_size, int(check_huge),
            _fp(xys_grad_norm), _fp(vis_counts), _fp(max_2d_size), half_max_dim, pb, fr_stride,
            pm, pv, _fp(random_samples), _ip(split), _ip(dup), _ip(keep))
    if rc < 0:
        raise RuntimeError("densify: 3N exceeds the buffers' capacity")
    return int(rc), split[:n], dup[:n], keep[:3 * n]
