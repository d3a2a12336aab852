"""The reference's Python training API (python/bindings.cpp:24-418,
python/msplat/__init__.py) over the native trainer C API
(include/msplat_c_api.h, msplat_b200/csrc/trainer.cu): TrainingConfig,
TrainingStats, GaussianTrainer, sync, cleanup.  Same names, keyword
arguments, defaults and error behaviour; the work runs on the GPU.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .dataset import Dataset


class TrainingConfig:
    """TrainingConfig (bindings.cpp:24-43) with the reference's defaults."""

    _FIELDS = (
        ("iterations", 30000), ("sh_degree", 3), ("sh_degree_interval", 1000),
        ("ssim_weight", 0.2), ("num_downscales", 2), ("resolution_schedule", 3000),
        ("refine_every", 100), ("warmup_length", 500), ("reset_alpha_every", 30),
        ("densify_grad_thresh", 0.0002), ("densify_size_thresh", 0.01),
        ("stop_screen_size_at", 4000), ("split_screen_size", 0.05), ("keep_crs", False),
        ("downscale_factor", 1.0), ("output", "splat.ply"), ("save_every", -1),
        ("bg_color", (0.6130, 0.0101, 0.3984)),
    )

    def __init__(self, iterations=30000, sh_degree=3, sh_degree_interval=1000, ssim_weight=0.2,
                 num_downscales=2, resolution_schedule=3000, refine_every=100, warmup_length=500,
                 reset_alpha_every=30, densify_grad_thresh=0.0002, densify_size_thresh=0.01,
                 stop_screen_size_at=4000, split_screen_size=0.05, keep_crs=False,
                 downscale_factor=1.0, output="splat.ply", save_every=-1,
                 bg_color=(0.6130, 0.0101, 0.3984)):
        if len(bg_color) != 3:
            raise ValueError("bg_color must have exactly 3 elements [R, G, B]")
        args = locals()
        for name, _ in self._FIELDS:
            setattr(self, name, args[name])
        self.bg_color = [float(x) for x in bg_color]

    def to_c(self) -> _lib.MsplatConfig:
        c = _lib.MsplatConfig()
        c.iterations = int(self.iterations)
        c.shDegree = int(self.sh_degree)
        c.shDegreeInterval = int(self.sh_degree_interval)
        c.ssimWeight = float(self.ssim_weight)
        c.numDownscales = int(self.num_downscales)
        c.resolutionSchedule = int(self.resolution_schedule)
        c.refineEvery = int(self.refine_every)
        c.warmupLength = int(self.warmup_length)
        c.resetAlphaEvery = int(self.reset_alpha_every)
        c.densifyGradThresh = float(self.densify_grad_thresh)
        c.densifySizeThresh = float(self.densify_size_thresh)
        c.stopScreenSizeAt = int(self.stop_screen_size_at)
        c.splitScreenSize = float(self.split_screen_size)
        c.keepCrs = bool(self.keep_crs)
        c.downscaleFactor = float(self.downscale_factor)
        for i in range(3):
            c.bgColor[i] = float(self.bg_color[i])
        return c

    def __repr__(self):
        body = ", ".join(f"{n}={getattr(self, n)!r}" for n, _ in self._FIELDS)
        return f"TrainingConfig({body})"


class TrainingStats:
    """Per-step statistics (bindings.cpp:47-51)."""

    def __init__(self, iteration: int, splat_count: int, ms_per_step: float):
        self.iteration = iteration
        self.splat_count = splat_count
        self.ms_per_step = ms_per_step

    def __repr__(self):
        return (f"TrainingStats(iteration={self.iteration}, splats={self.splat_count}, "
                f"ms={self.ms_per_step:.6f})")


def _pixels(pb: _lib.MsplatPixelBuffer) -> np.ndarray:
    if not pb.data:
        raise RuntimeError("render failed: " + _lib.load().msplat_last_error().decode())
    try:
        n = pb.width * pb.height * 3
        return np.ctypeslib.as_array(pb.data, (n,)).reshape(pb.height, pb.width, 3).copy()
    finally:
        C.CDLL(None).free(C.cast(pb.data, C.c_void_p))


class GaussianTrainer:
    """GaussianTrainer(dataset, config) (bindings.cpp:102-282)."""

    def __init__(self, dataset: Dataset, config: TrainingConfig):
        if dataset._c is None:
            raise ValueError("the dataset was opened without images (load_images=False)")
        self._dataset = dataset   # keep_alive, as the binding does
        self.config = config
        lib = _lib.load()
        self._t = lib.msplat_trainer_create(dataset._c, config.to_c())
        if not self._t:
            raise RuntimeError("GaussianTrainer: " + lib.msplat_last_error().decode())

    def close(self) -> None:
        if getattr(self, "_t", None):
            _lib.load().msplat_trainer_destroy(self._t)
            self._t = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 -- interpreter shutdown
            pass

    def step(self) -> TrainingStats:
        s = _lib.load().msplat_trainer_step(self._t)
        if s.iteration == 0:
            raise RuntimeError("step failed: " + _lib.load().msplat_last_error().decode())
        return TrainingStats(s.iteration, s.splatCount, s.msPerStep)

    def train(self, callback, callback_every: int = 100) -> None:
        while self.iteration < self.config.iterations:
            stats = self.step()
            if callback_every > 0 and stats.iteration % callback_every == 0:
                callback(stats)

    def evaluate(self) -> dict:
        if self._dataset.num_test == 0:
            raise RuntimeError("No test cameras. Load dataset with eval_mode=True.")
        m = _lib.load().msplat_trainer_evaluate(self._t)
        if m.numTest == 0:
            raise RuntimeError("evaluate failed: " + _lib.load().msplat_last_error().decode())
        return {"psnr": float(m.psnr), "ssim": float(m.ssim), "l1": float(m.l1),
                "num_test": int(m.numTest), "num_gaussians": int(m.numGaussians)}

    def render(self, cam_idx: int, use_test: bool = False) -> np.ndarray:
        cams = self._dataset.test_cams if use_test else self._dataset.train_cams
        if cam_idx < 0 or cam_idx >= len(cams):
            raise IndexError("Camera index out of range")
        return _pixels(_lib.load().msplat_trainer_render(self._t, cam_idx, bool(use_test)))

    def render_from_pose(self, cam_to_world, ref_cam_idx: int = 0) -> np.ndarray:
        pose = np.ascontiguousarray(cam_to_world, np.float32)
        if pose.size != 16:
            raise ValueError("cam_to_world must have 16 elements (4x4 matrix)")
        if ref_cam_idx < 0 or ref_cam_idx >= self._dataset.num_train:
            raise IndexError("ref_cam_idx out of range")
        return _pixels(_lib.load().msplat_trainer_render_pose(
            self._t, pose.ctypes.data_as(C.POINTER(C.c_float)), ref_cam_idx))

    def render_from_pose_rgba8(self, cam_to_world, ref_cam_idx: int = 0) -> np.ndarray:
        """renderFromPoseToBuffer (msplat_api.mm:205-233): (H, W, 4) uint8."""
        pose = np.ascontiguousarray(cam_to_world, np.float32)
        fp = pose.ctypes.data_as(C.POINTER(C.c_float))
        w, h = C.c_int(), C.c_int()
        lib = _lib.load()
        lib.msplat_trainer_render_pose_to_buffer(self._t, fp, ref_cam_idx, None, C.byref(w), C.byref(h))
        if w.value <= 0:
            raise IndexError("ref_cam_idx out of range")
        out = np.zeros((h.value, w.value, 4), np.uint8)
        lib.msplat_trainer_render_pose_to_buffer(self._t, fp, ref_cam_idx,
                                                 out.ctypes.data_as(C.POINTER(C.c_ubyte)),
                                                 C.byref(w), C.byref(h))
        return out

    def export_ply(self, path: str) -> None:
        _lib.load().msplat_trainer_export_ply(self._t, str(path).encode())

    def export_splat(self, path: str) -> None:
        _lib.load().msplat_trainer_export_splat(self._t, str(path).encode())

    def save_checkpoint(self, path: str) -> None:
        _lib.load().msplat_trainer_save_checkpoint(self._t, str(path).encode())

    def load_checkpoint(self, path: str) -> None:
        # the binding assigns the iteration and keeps its camera order
        if _lib.load().msplat_trainer_load_checkpoint_ex(self._t, str(path).encode(), 0) < 0:
            raise RuntimeError("load_checkpoint: " + _lib.load().msplat_last_error().decode())

    @property
    def splat_count(self) -> int:
        return _lib.load().msplat_trainer_splat_count(self._t)

    @property
    def iteration(self) -> int:
        return _lib.load().msplat_trainer_iteration(self._t)


def sync() -> None:
    """Wait for all queued GPU work."""
    _lib.load().msplat_sync()


def cleanup() -> None:
    """Release the engine's cached device buffers."""
    _lib.load().msplat_cleanup()
