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
    """Device-resident Gaussians + Adam state + densification statistics.

    As Model does (core/src/model.cpp:128-195), every group lives in a
    backing buffer with room for `capacity` rows (4N at first) and the
    parameters, moments and statistics are views of the first num_active
    rows; densification grows the buffers (ensure_capacity) and changes
    num_active.
    """

    def __init__(self, groups, device: str = "cuda", lr=LR_INIT, capacity: int | None = None):
        torch = _torch()
        arrs = [np.ascontiguousarray(g, dtype=np.float32) for g in groups]
        n = int(arrs[0].shape[0])
        cap = max(int(capacity) if capacity is not None else 4 * n, n, 1)
        self._device = device
        self._bufs = [torch.zeros((cap,) + a.shape[1:], dtype=torch.float32, device=device)
                      for a in arrs]
        for buf, a in zip(self._bufs, arrs):
            buf[:n].copy_(torch.as_tensor(a))
        self._m = [torch.zeros_like(b) for b in self._bufs]
        self._v = [torch.zeros_like(b) for b in self._bufs]
        self._stats = [torch.zeros(cap, dtype=torch.float32, device=device) for _ in range(3)]
        self.num_active = n
        self.lr = [float(x) for x in lr]
        self.means_lr_init, self.means_lr_final = float(LR_INIT[0]), float(MEANS_LR_FINAL)
        self.beta1, self.beta2, self.eps = 0.9, 0.999, 1e-8
        self.step_count = 0
        # Model::shDegree: the SH degree the features_rest bases were sized for
        self.sh_degree = int(round(math.sqrt(arrs[4].shape[1] + 1))) - 1
        # CRS of the input data (Model::keepCrs, scale, translation), used by the exports
        self.keep_crs, self.crs_scale, self.crs_translation = False, 1.0, (0.0, 0.0, 0.0)
        self._refresh()

    def _refresh(self) -> None:
        n = self.num_active
        self.params = [b[:n] for b in self._bufs]
        self.exp_avg = [m[:n] for m in self._m]
        self.exp_avg_sq = [v[:n] for v in self._v]
        self.vis_counts, self.xys_grad_norm, self.max_2d_size = [s[:n] for s in self._stats]

    @property
    def n(self) -> int:
        return int(self.params[0].shape[0])

    @property
    def capacity(self) -> int:
        return int(self._bufs[0].shape[0])

    @property
    def rest_bases(self) -> int:
        return int(self.params[4].shape[1])

    def adam_scalars(self):
        return adam_scalars(self.step_count, self.lr, self.beta1, self.beta2)

    def schedule_means_lr(self, step: int, max_steps: int) -> None:
        """Model::schedulersStep (model.cpp:179-182)."""
        t = min(max(f32(step) / f32(max_steps), f32(0.0)), f32(1.0))
        lo, hi = f32(self.means_lr_init), f32(self.means_lr_final)
        self.lr[0] = float(f32(math.exp(float(f32(math.log(float(lo))) * (f32(1.0) - t)
                                               + f32(math.log(float(hi))) * t))))

    def ensure_capacity(self, needed: int) -> None:
        """Model::ensureCapacity (model.cpp:197-225): grow every backing
        buffer to max(needed, 2 x capacity), keeping the active rows."""
        if needed <= self.capacity:
            return
        torch = _torch()
        cap = max(int(needed), 2 * self.capacity)
        n = self.num_active

        def grow(buf):
            out = torch.zeros((cap,) + tuple(buf.shape[1:]), dtype=buf.dtype, device=buf.device)
            out[:n].copy_(buf[:n])
            return out
        self._bufs = [grow(b) for b in self._bufs]
        self._m = [grow(m) for m in self._m]
        self._v = [grow(v) for v in self._v]
        self._stats = [grow(st) for st in self._stats]
        self._refresh()

    def densify(self, step: int, grad_thresh: float, size_thresh: float, screen_thresh: float,
                check_screen: bool, check_huge: bool, half_max_dim: float,
                random_samples=None, cull_alpha_thresh: float = 0.1,
                cull_scale_thresh: float = 0.5, cull_screen_size: float = 0.15) -> int:
        """msplat_densify over this model (the densification branch of
        Model::afterTrain, model.cpp:243-275).  random_samples: [2N, 3]
        standard normals on the device; by default drawn from a generator
        seeded with the step (the reference seeds std::mt19937 with it).
        Returns the new number of Gaussians."""
        torch = _torch()
        n = self.num_active
        self.ensure_capacity(3 * n)
        if random_samples is None:
            gen = torch.Generator(device=self._device).manual_seed(int(step))
            random_samples = torch.randn(2 * n, 3, generator=gen, device=self._device)
        samples = random_samples.contiguous()   # held until the call returns
        b = self._bufs
        fr_stride = int(np.prod(b[4].shape[1:]))
        rc = _lib.load().msplat_densify(
            n, self.capacity, grad_thresh, size_thresh, screen_thresh, int(check_screen),
            cull_alpha_thresh, cull_scale_thresh, cull_screen_size, int(check_huge),
            _ptr(self._stats[1]), _ptr(self._stats[0]), _ptr(self._stats[2]), half_max_dim,
            _ptr(b[0]), _ptr(b[1]), _ptr(b[2]), _ptr(b[3]), _ptr(b[4]), _ptr(b[5]), fr_stride,
            _ptr_array(self._m), _ptr_array(self._v), None, None, None, None, None, None, None,
            None, _ptr(samples))
        if rc < 0:
            _lib.check(rc, "msplat_densify")
        self.num_active = int(rc)
        self._refresh()
        return self.num_active

    def reset_opacity(self) -> None:
        """The opacity reset of Model::afterTrain (model.cpp:280-290)."""
        _lib.check(_lib.load().msplat_reset_opacity(_ptr(self.params[5]), _ptr(self.exp_avg[5]),
                                                    _ptr(self.exp_avg_sq[5]), self.n),
                   "msplat_reset_opacity")

    def reset_stats(self) -> None:
        for st in self._stats:
            st.zero_()

    # ---- model files (msplat_save_checkpoint & co.) ---------------------

    @classmethod
    def _blank(cls, n: int, rest_bases: int, device: str, capacity: int) -> "GaussianModel":
        shapes = [(n, 3), (n, 3), (n, 4), (n, 3), (n, rest_bases, 3), (n, 1)]
        return cls([np.zeros(s, np.float32) for s in shapes], device=device, capacity=capacity)

    def _crs_args(self):
        return int(self.keep_crs), float(self.crs_scale), _lib.farr(self.crs_translation)

    def save_checkpoint(self, path: str, step: int) -> None:
        """Model::saveCheckpoint (core/src/model.cpp:361-399)."""
        _lib.check(_lib.load().msplat_save_checkpoint(
            str(path).encode(), int(step), self.num_active, self.sh_degree, self.step_count,
            _lib.farr(self.lr), self.means_lr_init, self.means_lr_final, self.rest_bases,
            _ptr_array(self.params), _ptr_array(self.exp_avg), _ptr_array(self.exp_avg_sq)),
            "msplat_save_checkpoint")

    @classmethod
    def load_checkpoint(cls, path: str, device: str = "cuda"):
        """Model::loadCheckpoint (model.cpp:401-488): a model with the
        checkpoint's parameters, Adam moments, step count and learning
        rates in 4N-capacity buffers.  Returns (model, step)."""
        lib = _lib.load()
        step, n, deg, adam_steps, rb = (C.c_int() for _ in range(5))
        lr = (C.c_float * 6)()
        lr0, lr1 = C.c_float(), C.c_float()
        _lib.check(lib.msplat_read_checkpoint_header(
            str(path).encode(), C.byref(step), C.byref(n), C.byref(deg), C.byref(adam_steps), lr,
            C.byref(lr0), C.byref(lr1), C.byref(rb)), "msplat_read_checkpoint_header")
        model = cls._blank(n.value, rb.value, device, capacity=4 * n.value)
        rc = lib.msplat_load_checkpoint(str(path).encode(), model.capacity, _ptr_array(model._bufs),
                                        _ptr_array(model._m), _ptr_array(model._v))
        if rc < 0:
            _lib.check(rc, "msplat_load_checkpoint")
        model.lr = [float(x) for x in lr]
        model.means_lr_init, model.means_lr_final = float(lr0.value), float(lr1.value)
        model.step_count = adam_steps.value
        model.sh_degree = deg.value
        return model, int(rc)

    def save_ply(self, path: str, step: int) -> None:
        """Model::savePly -> saveGaussianPly (core/src/loaders/save_gaussians.cpp:10-54)."""
        _lib.check(_lib.load().msplat_save_ply(
            str(path).encode(), int(step), self.n, self.rest_bases, _ptr_array(self.params),
            *self._crs_args()), "msplat_save_ply")

    def save_splat(self, path: str) -> None:
        """Model::saveSplat -> saveGaussianSplat (save_gaussians.cpp:56-97)."""
        _lib.check(_lib.load().msplat_save_splat(
            str(path).encode(), self.n, _ptr_array(self.params), *self._crs_args()),
            "msplat_save_splat")

    def save(self, path: str, step: int) -> None:
        """Model::save (model.cpp:298-305): .splat by extension, else PLY."""
        if str(path).endswith(".splat"):
            self.save_splat(path)
        else:
            self.save_ply(path, step)

    @classmethod
    def load_ply(cls, path: str, device: str = "cuda", keep_crs: bool = False,
                 crs_scale: float = 1.0, crs_translation=(0.0, 0.0, 0.0)):
        """Model::loadPly (model.cpp:319-329) -> loadGaussianPly: a model with
        fresh Adam state.  Returns (model, step)."""
        lib = _lib.load()
        n, step, rb = C.c_int(), C.c_int(), C.c_int()
        _lib.check(lib.msplat_read_ply_header(str(path).encode(), C.byref(n), C.byref(step),
                                              C.byref(rb)), "msplat_read_ply_header")
        model = cls._blank(n.value, rb.value, device, capacity=4 * n.value)
        model.keep_crs, model.crs_scale = bool(keep_crs), float(crs_scale)
        model.crs_translation = tuple(float(x) for x in crs_translation)
        rc = lib.msplat_load_ply(str(path).encode(), model.capacity, _ptr_array(model._bufs),
                                 *model._crs_args())
        if rc < 0:
            _lib.check(rc, "msplat_load_ply")
        return model, int(rc)


class Schedule:
    """The refinement schedule of Model::afterTrain (model.cpp:236-296),
    with the reference's defaults (msplat_api.hpp:16-33)."""

    def __init__(self, max_steps: int = 30000, num_cameras: int = 1, refine_every: int = 100,
                 warmup_length: int = 500, reset_alpha_every: int = 30,
                 densify_grad_thresh: float = 0.0002, densify_size_thresh: float = 0.01,
                 stop_screen_size_at: int = 4000, split_screen_size: float = 0.05):
        self.num_cameras = num_cameras
        self.refine_every = refine_every
        self.warmup_length = warmup_length
        self.reset_alpha_every = reset_alpha_every
        self.stop_split_at = max_steps // 2
        self.densify_grad_thresh = densify_grad_thresh
        self.densify_size_thresh = densify_size_thresh
        self.stop_screen_size_at = stop_screen_size_at
        self.split_screen_size = split_screen_size

    def after_train(self, model: GaussianModel, step: int, width: int, height: int) -> dict:
        """Runs the densification / opacity reset due at `step` (after the
        step's training) and resets the statistics on refinement steps.
        Returns what happened."""
        done = {"densified": None, "opacity_reset": False}
        if not (step % self.refine_every == 0 and step > self.warmup_length):
            return done
        reset_interval = self.reset_alpha_every * self.refine_every
        if step < self.stop_split_at and step % reset_interval > self.num_cameras + self.refine_every:
            before = model.n
            after = model.densify(
                step, self.densify_grad_thresh, self.densify_size_thresh, self.split_screen_size,
                check_screen=step < self.stop_screen_size_at,
                check_huge=step > self.refine_every * self.reset_alpha_every,
                half_max_dim=float(f32(0.5) * f32(max(width, height))))
            done["densified"] = (before, after)
        if step < self.stop_split_at and step % reset_interval == self.refine_every:
            model.reset_opacity()
            done["opacity_reset"] = True
        model.reset_stats()
        return done


class DevicePtr:
    """A raw device address where the step functions expect a tensor (they
    only read its data_ptr()), e.g. a buffer from msplat_stage_input."""

    def __init__(self, address: int):
        self.address = int(address)

    def data_ptr(self) -> int:
        return self.address


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
