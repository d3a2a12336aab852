"""Python host for the engine's C-ABI: the per-step host work of
Model::fullIteration (core/src/model.cpp:546-597) over torch CUDA tensors.

`GaussianModel` owns the six parameter groups and their Adam moments on the
device (the reference's Model keeps them in 4N-capacity buffers and hands
the engine views; here the tensors are exactly N rows).  `train_step` and
`render` call msplat_train_step / msplat_render through ctypes; torch only
allocates device memory and supplies the stream.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import _lib
from .camera import CamSetup

f32 = np.float32

# Per-group learning rates, Model::setupOptimizers (model.cpp:138): means,
# scales, quats, features_dc, features_rest, opacities.
LR_INIT = (0.00016, 0.005, 0.001, 0.0025, 0.000125, 0.05)
MEANS_LR_FINAL = 0.0000016
DEFAULT_BG = (0.6130, 0.0101, 0.3984)  # Model::Model default background (model.cpp:114)


def _torch():
    import torch  # noqa: WPS433 -- torch is only the allocator/stream provider
    return torch


def bind_stream() -> None:
    """Run engine work on torch's current CUDA stream.  When that is the
    legacy default stream (handle 0, which the C-ABI reads as "the engine's
    own stream"), torch is first moved to a dedicated stream so torch ops,
    CUDA events and engine kernels share one stream."""
    torch = _torch()
    lib = _lib.load()
    cur = torch.cuda.current_stream()
    if cur.cuda_stream == 0:
        cur = torch.cuda.Stream()
        torch.cuda.set_stream(cur)
    _lib.check(lib.msplat_set_stream(C.c_void_p(cur.cuda_stream)), "msplat_set_stream")


def adam_scalars(step_count: int, lr, beta1: float = 0.9, beta2: float = 0.999):
    """Per-group lr/bc1 and sqrt(bc2) as Model::fullIteration forms them
    (model.cpp:558-571): bc = 1 - std::pow(float beta, int t), where the
    power is taken in double, then every value is a float."""
    b1 = float(f32(beta1))
    b2 = float(f32(beta2))
    bc1 = f32(1.0 - b1 ** step_count)
    bc2 = f32(1.0 - b2 ** step_count)
    steps = [f32(f32(x) / bc1) for x in lr]
    bc2s = [f32(math.sqrt(float(bc2)))] * len(lr)
    return steps, bc2s


class GaussianModel:
    """Device-resident Gaussians + Adam state + densification statistics."""

    def __init__(self, groups, device: str = "cuda", lr=LR_INIT):
        torch = _torch()
        self.params = [torch.as_tensor(np.ascontiguousarray(g)).to(device).contiguous()
                       for g in groups]
        self.exp_avg = [torch.zeros_like(p) for p in self.params]
        self.exp_avg_sq = [torch.zeros_like(p) for p in self.params]
        n = self.params[0].shape[0]
        self.vis_counts = torch.zeros(n, dtype=torch.float32, device=device)
        self.xys_grad_norm = torch.zeros(n, dtype=torch.float32, device=device)
        self.max_2d_size = torch.zeros(n, dtype=torch.float32, device=device)
        self.lr = [float(x) for x in lr]
        self.beta1, self.beta2, self.eps = 0.9, 0.999, 1e-8
        self.step_count = 0

    @property
    def n(self) -> int:
        return int(self.params[0].shape[0])

    @property
    def rest_bases(self) -> int:
        return int(self.params[4].shape[1])

    def adam_scalars(self):
        return adam_scalars(self.step_count, self.lr, self.beta1, self.beta2)

    def schedule_means_lr(self, step: int, max_steps: int) -> None:
        """Model::schedulersStep (model.cpp:179-182)."""
        t = min(max(f32(step) / f32(max_steps), f32(0.0)), f32(1.0))
        self.lr[0] = float(f32(math.exp(float(f32(math.log(float(f32(LR_INIT[0])))) * (f32(1.0) - t)
                                               + f32(math.log(float(f32(MEANS_LR_FINAL)))) * t))))


def _ptr(t) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def _ptr_array(ts):
    return (C.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def train_step(model: GaussianModel, cam: CamSetup, gt, ssim_weight: float = 0.2,
               background=DEFAULT_BG, glob_scale: float = 1.0, clip_thresh: float = 0.01):
    """One msplat_train_step; returns the engine's loss value (see
    msplat_train_step in include/msplat_engine.h)."""
    lib = _lib.load()
    model.step_count += 1
    steps, bc2s = model.adam_scalars()
    h, w = cam.height, cam.width
    loss_inv_n = float(f32(1.0) / f32(h * w * 3))
    inv_max_dim = float(f32(1.0) / f32(max(h, w)))
    radii = C.c_void_p()
    loss = C.c_float()
    p = model.params
    rc = lib.msplat_train_step(
        model.n, _ptr(p[0]), _ptr(p[1]), glob_scale, _ptr(p[2]),
        _lib.farr(cam.viewmat), _lib.farr(cam.projmat), cam.fx, cam.fy, cam.cx, cam.cy,
        h, w, _lib.iarr(cam.tile_bounds), clip_thresh, cam.degree, cam.degrees_to_use,
        _lib.farr(cam.cam_pos), _ptr(p[3]), _ptr(p[4]), _ptr(p[5]), _lib.farr(background),
        _ptr(gt), None, ssim_weight, loss_inv_n, model.rest_bases, 6,
        _ptr_array(p), _ptr_array(model.exp_avg), _ptr_array(model.exp_avg_sq),
        _lib.farr(steps), _lib.farr(bc2s), model.beta1, model.beta2, model.eps,
        _ptr(model.vis_counts), _ptr(model.xys_grad_norm), _ptr(model.max_2d_size), inv_max_dim,
        C.byref(radii), C.byref(loss))
    _lib.check(rc, "msplat_train_step")
    return float(loss.value)


def render(model: GaussianModel, cam: CamSetup, background=DEFAULT_BG, glob_scale: float = 1.0,
           clip_thresh: float = 0.01) -> int:
    """msplat_render; returns the device address of the (H,W,3) image."""
    lib = _lib.load()
    out = C.c_void_p()
    p = model.params
    rc = lib.msplat_render(
        model.n, _ptr(p[0]), _ptr(p[1]), glob_scale, _ptr(p[2]),
        _lib.farr(cam.viewmat), _lib.farr(cam.projmat), cam.fx, cam.fy, cam.cx, cam.cy,
        cam.height, cam.width, _lib.iarr(cam.tile_bounds), clip_thresh, cam.degree,
        cam.degrees_to_use, _lib.farr(cam.cam_pos), _ptr(p[3]), _ptr(p[4]), _ptr(p[5]),
        _lib.farr(background), C.byref(out))
    _lib.check(rc, "msplat_render")
    return int(out.value)


def download(dev_ptr: int, count: int, dtype) -> np.ndarray:
    """Copy `count` elements of `dtype` from device memory (synchronous)."""
    lib = _lib.load()
    out = np.empty(count, dtype=dtype)
    if count:
        _lib.check(lib.msplat_copy(C.c_void_p(out.ctypes.data), C.c_void_p(dev_ptr), out.nbytes, 1, 1),
                   "msplat_copy")
    return out


def debug_buffer(name: str, count: int, dtype) -> np.ndarray:
    """Download the first `count` elements of a named engine buffer."""
    lib = _lib.load()
    ptr = C.c_void_p()
    cap = C.c_longlong()
    _lib.check(lib.msplat_debug_buffer(name.encode(), C.byref(ptr), C.byref(cap)), "debug_buffer")
    return download(ptr.value, count, dtype)
