"""Data-parallel training: one process per GPU, each rank trains its own view
of the same (replicated) Gaussians every step.

The reference trains one view per step on one device (Trainer::step,
core/src/msplat_api.mm:106-129).  Across ranks the step splits at the one
point where views interact -- the optimiser:

  1. msplat_train_step_grads: forward, loss and backward of this rank's
     view; the per-Gaussian gradient (59 floats at SH degree 3) and a
     visibility flag go into one flat buffer instead of into Adam;
  2. one all-reduce (sum) of that buffer over NVLink (NCCL);
  3. msplat_adam_apply with grad_scale = 1/world: every rank applies the
     same Adam update to its own replica, so replicas stay identical.
     features_dc / features_rest move for Gaussians that ANY rank saw,
     the multi-view form of the reference's visible-only SH update.

With world = 1 the two halves reproduce msplat_train_step bit for bit.
Densification statistics stay per rank during training; sync_stats() sums
vis_counts / xys_grad_norm and takes the max of max_2d_size across ranks
before a densification pass reads them.

The compute calls go through an `ops` object (EngineOps, the CUDA engine),
so the collective protocol can be exercised with gloo ranks on the CPU.
"""
from __future__ import annotations

import ctypes as C
import datetime
import os

import numpy as np

from . import _lib
from .engine import DEFAULT_BG, GaussianModel, _ptr, _ptr_array

f32 = np.float32

# Per-Gaussian floats of each gradient group, in buffer order: means,
# scales, quats, features_dc, features_rest (per SH-rest basis x3),
# opacities; one visibility flag follows the six groups.
GROUP_WIDTHS = (3, 3, 4, 3, None, 1)


def grad_floats(n: int, rest_bases: int) -> int:
    """Length of the flat gradient buffer of msplat_train_step_grads."""
    return (15 + 3 * rest_bases) * n


def grad_views(buf, n: int, rest_bases: int):
    """Views of the flat buffer: the six groups' gradients and `vis`."""
    widths = [w if w is not None else 3 * rest_bases for w in GROUP_WIDTHS]
    out, off = [], 0
    for w in widths:
        out.append(buf[off:off + w * n].view(n, w))
        off += w * n
    return out, buf[off:off + n]


class EngineOps:
    """The CUDA engine's two halves of a data-parallel step."""

    def alloc(self, count: int):
        import torch
        return torch.empty(count, dtype=torch.float32, device="cuda")

    def grads(self, model: GaussianModel, cam, gt, out, ssim_weight, background, glob_scale,
              clip_thresh) -> float:
        lib = _lib.load()
        h, w = cam.height, cam.width
        loss_inv_n = float(f32(1.0) / f32(h * w * 3))
        inv_max_dim = float(f32(1.0) / f32(max(h, w)))
        p = model.params
        radii = C.c_void_p()
        loss = C.c_float()
        rc = lib.msplat_train_step_grads(
            model.n, _ptr(p[0]), _ptr(p[1]), glob_scale, _ptr(p[2]),
            _lib.farr(cam.viewmat), _lib.farr(cam.projmat), cam.fx, cam.fy, cam.cx, cam.cy,
            h, w, _lib.iarr(cam.tile_bounds), clip_thresh, cam.degree, cam.degrees_to_use,
            _lib.farr(cam.cam_pos), _ptr(p[3]), _ptr(p[4]), _ptr(p[5]), _lib.farr(background),
            _ptr(gt), ssim_weight, loss_inv_n, model.rest_bases, _ptr(out),
            _ptr(model.vis_counts), _ptr(model.xys_grad_norm), _ptr(model.max_2d_size),
            inv_max_dim, C.byref(radii), C.byref(loss))
        _lib.check(rc, "msplat_train_step_grads")
        return float(loss.value)

    def adam_apply(self, model: GaussianModel, cam, grad, scale: float) -> None:
        lib = _lib.load()
        steps, bc2s = model.adam_scalars()
        rc = lib.msplat_adam_apply(
            model.n, model.rest_bases, cam.degree, cam.degrees_to_use, _ptr(grad), scale, 0,
            model.n, 6, _ptr_array(model.params), _ptr_array(model.exp_avg),
            _ptr_array(model.exp_avg_sq), _lib.farr(steps), _lib.farr(bc2s), model.beta1,
            model.beta2, model.eps)
        _lib.check(rc, "msplat_adam_apply")


class DataParallel:
    """Replicated Gaussians, one view per rank per step, gradient all-reduce.

    Creates the default process group from the torchrun environment when
    none exists (NCCL on GPUs; `backend` overrides, e.g. "gloo" on CPU) and
    destroys it in shutdown() only if it created it.
    """

    def __init__(self, model: GaussianModel, rank: int, world: int, ops=None,
                 backend: str | None = None, timeout_s: float = 120.0):
        import torch
        import torch.distributed as dist
        self.model, self.rank, self.world = model, rank, world
        self.ops = ops if ops is not None else EngineOps()
        self._owns_group = False
        if not dist.is_initialized():
            be = backend or ("nccl" if torch.cuda.is_available() else "gloo")
            kw = dict(backend=be, rank=rank, world_size=world,
                      timeout=datetime.timedelta(seconds=timeout_s))
            if be == "nccl":
                kw["device_id"] = torch.device("cuda", torch.cuda.current_device())
            dist.init_process_group(**kw)
            self._owns_group = True
        self.backend = dist.get_backend()
        self.grad = self.ops.alloc(grad_floats(model.n, model.rest_bases))
        self.last_loss = 0.0

    def train_step(self, cam, gt, ssim_weight: float = 0.2, background=DEFAULT_BG,
                   glob_scale: float = 1.0, clip_thresh: float = 0.01) -> float:
        """One data-parallel step; every rank passes its own view."""
        import torch.distributed as dist
        self.model.step_count += 1
        self.last_loss = self.ops.grads(self.model, cam, gt, self.grad, ssim_weight, background,
                                        glob_scale, clip_thresh)
        if self.world > 1:
            dist.all_reduce(self.grad, op=dist.ReduceOp.SUM)
        self.ops.adam_apply(self.model, cam, self.grad, 1.0 / self.world)
        return self.last_loss

    def sync_stats(self) -> None:
        """Combine the ranks' densification statistics (before densifying)."""
        import torch.distributed as dist
        if self.world == 1:
            return
        dist.all_reduce(self.model.vis_counts, op=dist.ReduceOp.SUM)
        dist.all_reduce(self.model.xys_grad_norm, op=dist.ReduceOp.SUM)
        dist.all_reduce(self.model.max_2d_size, op=dist.ReduceOp.MAX)

    def barrier(self) -> None:
        import torch.distributed as dist
        if self.backend == "nccl":
            import torch
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()

    def max_over_ranks(self, value: float) -> float:
        import torch
        import torch.distributed as dist
        dev = "cuda" if self.backend == "nccl" else "cpu"
        t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def shutdown(self) -> None:
        import torch.distributed as dist
        if self._owns_group and dist.is_initialized():
            dist.destroy_process_group()
        self._owns_group = False


def rank_and_world() -> tuple[int, int]:
    """RANK / WORLD_SIZE from the torchrun environment (0, 1 without it)."""
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
