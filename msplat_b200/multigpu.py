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

A step may also train a batch of several views per rank (the batched-view
configuration: 8 views per step on 1, 2, 4 or 8 GPUs): the rank's first
view writes the gradient buffer, the others add to it
(msplat_train_step_grads_accumulate), every view's loss is normalised by
the rank's view count, and the exchange above completes the mean over the
batch.  train_batch() is the same step on one device.
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


def grad_floats_compact(n: int) -> int:
    """Length of the compact gradient buffer (msplat_train_step_grads_compact):
    means, scales, quats, v_rgb, opacities, visibility, camera position."""
    return 15 * n + 4


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

    def _grads(self, fn: str, model: GaussianModel, cam, gt, out, ssim_weight, background,
               glob_scale, clip_thresh, batch: int) -> float:
        lib = _lib.load()
        h, w = cam.height, cam.width
        # the mean over the pixels and channels of `batch` views (a division
        # by a power-of-two batch is exact)
        loss_inv_n = float(f32(f32(1.0) / f32(h * w * 3)) / f32(batch))
        inv_max_dim = float(f32(1.0) / f32(max(h, w)))
        p = model.params
        radii = C.c_void_p()
        loss = C.c_float()
        rc = getattr(lib, fn)(
            model.n, _ptr(p[0]), _ptr(p[1]), glob_scale, _ptr(p[2]),
            _lib.farr(cam.viewmat), _lib.farr(cam.projmat), cam.fx, cam.fy, cam.cx, cam.cy,
            h, w, _lib.iarr(cam.tile_bounds), clip_thresh, cam.degree, cam.degrees_to_use,
            _lib.farr(cam.cam_pos), _ptr(p[3]), _ptr(p[4]), _ptr(p[5]), _lib.farr(background),
            _ptr(gt), ssim_weight, loss_inv_n, model.rest_bases, _ptr(out),
            _ptr(model.vis_counts), _ptr(model.xys_grad_norm), _ptr(model.max_2d_size),
            inv_max_dim, C.byref(radii), C.byref(loss))
        _lib.check(rc, fn)
        return float(loss.value)

    def grads(self, model: GaussianModel, cam, gt, out, ssim_weight, background, glob_scale,
              clip_thresh, accumulate: bool = False, batch: int = 1) -> float:
        """This view's gradients into `out` (full layout); with `accumulate`
        added to what it holds.  `batch`: views per rank in the step."""
        fn = "msplat_train_step_grads_accumulate" if accumulate else "msplat_train_step_grads"
        return self._grads(fn, model, cam, gt, out, ssim_weight, background, glob_scale,
                           clip_thresh, batch)

    def grads_compact(self, model: GaussianModel, cam, gt, out, ssim_weight, background,
                      glob_scale, clip_thresh) -> float:
        return self._grads("msplat_train_step_grads_compact", model, cam, gt, out, ssim_weight,
                           background, glob_scale, clip_thresh, 1)

    def adam_apply(self, model: GaussianModel, cam, grad, scale: float) -> None:
        lib = _lib.load()
        steps, bc2s = model.adam_scalars()
        rc = lib.msplat_adam_apply(
            model.n, model.rest_bases, cam.degree, cam.degrees_to_use, _ptr(grad), scale, 0,
            model.n, 6, _ptr_array(model.params), _ptr_array(model.exp_avg),
            _ptr_array(model.exp_avg_sq), _lib.farr(steps), _lib.farr(bc2s), model.beta1,
            model.beta2, model.eps)
        _lib.check(rc, "msplat_adam_apply")


def accumulate_views(ops, model: GaussianModel, cams, gts, out, compact: bool = False,
                     ssim_weight: float = 0.2, background=DEFAULT_BG, glob_scale: float = 1.0,
                     clip_thresh: float = 0.01) -> float:
    """Gradient of one rank's share of a batched step: its views in order,
    the first written into `out`, the others added to it, each with the loss
    normalised by the rank's view count (the exchange's 1/world completes the
    mean over the batch).  Returns the sum of the views' losses so scaled."""
    if compact and len(cams) != 1:
        raise ValueError("the compact gradient layout carries one view per rank")
    loss = 0.0
    for k, (cam, gt) in enumerate(zip(cams, gts)):
        if compact:
            loss += ops.grads_compact(model, cam, gt, out, ssim_weight, background, glob_scale,
                                      clip_thresh)
        else:
            loss += ops.grads(model, cam, gt, out, ssim_weight, background, glob_scale,
                              clip_thresh, accumulate=k > 0, batch=len(cams))
    return loss


def train_batch(model: GaussianModel, cams, gts, grad, ops=None, ssim_weight: float = 0.2,
                background=DEFAULT_BG, glob_scale: float = 1.0,
                clip_thresh: float = 0.01) -> float:
    """One step on a batch of views on a single device: the gradient of the
    mean loss over the views (accumulated in `grad`, a grad_floats buffer),
    then one Adam update.  With one view it equals msplat_train_step within
    the parity bar (the fused step is faster there)."""
    ops = ops if ops is not None else EngineOps()
    model.step_count += 1
    loss = accumulate_views(ops, model, cams, gts, grad, False, ssim_weight, background,
                            glob_scale, clip_thresh)
    ops.adam_apply(model, cams[0], grad, 1.0)
    return loss


class DeviceBuffer:
    """A whole cudaMalloc allocation (msplat_gpu_alloc), so that its CUDA IPC
    handle maps exactly this buffer in the peers; torch sees it through the
    CUDA array interface without a copy.  Freed only by free()."""

    def __init__(self, count: int, typestr: str = "<f4", zero: bool = True):
        lib = _lib.load()
        self.count = int(count)
        self.ptr = lib.msplat_gpu_alloc(4 * max(self.count, 1), 1 if zero else 0)
        if not self.ptr:
            raise _lib.EngineError(f"msplat_gpu_alloc: {lib.msplat_last_error().decode()}")
        self.__cuda_array_interface__ = {"shape": (self.count,), "typestr": typestr,
                                         "data": (self.ptr, False), "version": 3}

    def tensor(self, shape=None):
        import torch
        t = torch.as_tensor(self, device="cuda")
        return t.view(shape) if shape is not None else t

    def handle(self) -> bytes:
        h = C.create_string_buffer(64)
        _lib.check(_lib.load().msplat_ipc_get_handle(C.c_void_p(self.ptr), h),
                   "msplat_ipc_get_handle")
        return h.raw

    def free(self) -> None:
        if self.ptr:
            _lib.load().msplat_gpu_free(C.c_void_p(self.ptr))
            self.ptr = 0


def _open_handle(h: bytes) -> int:
    out = C.c_void_p()
    _lib.check(_lib.load().msplat_ipc_open_handle(C.create_string_buffer(h, 64), C.byref(out)),
               "msplat_ipc_open_handle")
    return int(out.value)


class DataParallel:
    """Replicated Gaussians, views_per_rank views per rank per step.

    mode "peer" (GPUs): the gradient buffers, parameter arrays and flag
    arrays of all ranks are mapped into every process, and one kernel per
    rank sums its 1/world shard of the gradients over NVLink, applies Adam to
    it and writes it into every replica (msplat_dp_reduce_adam).  With
    `compact` (the default) the ranks exchange each Gaussian's colour
    gradient v_rgb instead of its 48 SH gradients, which the owner rebuilds
    from every rank's camera position (15 instead of 60 floats per Gaussian).
    mode "nccl": one all-reduce of the gradient buffer, then Adam on every
    replica (msplat_adam_apply).  The stand-in ops of the CPU tests use it.

    Creates the default process group from the torchrun environment when
    none exists (NCCL on GPUs; `backend` overrides, e.g. "gloo" on CPU) and
    destroys it in shutdown() only if it created it.
    """

    def __init__(self, model: GaussianModel, rank: int, world: int, ops=None,
                 backend: str | None = None, timeout_s: float = 120.0, mode: str | None = None,
                 peer_timeout_s: float = 10.0, compact: bool = True, views_per_rank: int = 1):
        import torch
        import torch.distributed as dist
        self.model, self.rank, self.world = model, rank, world
        self.ops = ops if ops is not None else EngineOps()
        self._owns_group = False
        self.mode = mode or ("peer" if ops is None and torch.cuda.is_available() else "nccl")
        if self.mode not in ("peer", "nccl"):
            raise ValueError(f"unknown data-parallel mode {self.mode!r}")
        self.peer_timeout_s = float(peer_timeout_s)
        # peer mode: exchange v_rgb instead of the 48 SH gradients per Gaussian
        # (one view per rank: v_rgb is tied to its view's camera)
        self.views_per_rank = int(views_per_rank)
        if self.views_per_rank < 1:
            raise ValueError("views_per_rank must be >= 1")
        self.compact = bool(compact) and self.mode == "peer" and self.views_per_rank == 1
        self._bufs = []
        if not dist.is_initialized():
            be = backend or ("nccl" if torch.cuda.is_available() else "gloo")
            kw = dict(backend=be, rank=rank, world_size=world,
                      timeout=datetime.timedelta(seconds=timeout_s))
            if be == "nccl":
                kw["device_id"] = torch.device("cuda", torch.cuda.current_device())
            dist.init_process_group(**kw)
            self._owns_group = True
        self.backend = dist.get_backend()
        self.last_loss = 0.0
        if self.mode == "peer":
            self._setup_peer()
        else:
            self.grad = self.ops.alloc(grad_floats(model.n, model.rest_bases))

    def _setup_peer(self) -> None:
        """Move the parameters into shareable allocations and map every
        rank's buffers into this process."""
        import torch
        import torch.distributed as dist
        m = self.model
        gbuf = DeviceBuffer(grad_floats_compact(m.n) if self.compact
                            else grad_floats(m.n, m.rest_bases))
        fbuf = DeviceBuffer(2 * self.world, typestr="<u4")
        pbufs = [DeviceBuffer(p.numel()) for p in m.params]
        self._bufs = [gbuf, fbuf] + pbufs
        torch.cuda.synchronize()
        for i, (buf, p) in enumerate(zip(pbufs, m.params)):
            t = buf.tensor(p.shape)
            t.copy_(p)
            m.params[i] = t
        self.grad = gbuf.tensor()
        mine = [b.handle() for b in self._bufs]
        every = [None] * self.world
        dist.all_gather_object(every, mine)
        ptrs = []
        for q in range(self.world):
            ptrs.append([b.ptr for b in self._bufs] if q == self.rank
                        else [_open_handle(h) for h in every[q]])
        self._grads_arr = (C.c_void_p * self.world)(*[ptrs[q][0] for q in range(self.world)])
        self._flags_arr = (C.c_void_p * self.world)(*[ptrs[q][1] for q in range(self.world)])
        self._params_arr = (C.c_void_p * (6 * self.world))(
            *[ptrs[q][2 + g] for q in range(self.world) for g in range(6)])
        self.epoch = 0
        torch.cuda.synchronize()
        self.barrier()

    def train_step(self, cam, gt, ssim_weight: float = 0.2, background=DEFAULT_BG,
                   glob_scale: float = 1.0, clip_thresh: float = 0.01) -> float:
        """One data-parallel step; every rank passes its own view."""
        return self.train_views([cam], [gt], ssim_weight, background, glob_scale, clip_thresh)

    def train_views(self, cams, gts, ssim_weight: float = 0.2, background=DEFAULT_BG,
                    glob_scale: float = 1.0, clip_thresh: float = 0.01) -> float:
        """One data-parallel step over a batch of world * views_per_rank
        views; every rank passes its own views_per_rank of them.  Adam
        follows the gradient of the mean loss over the whole batch."""
        if len(cams) != self.views_per_rank or len(gts) != len(cams):
            raise ValueError(f"expected {self.views_per_rank} views per rank, got {len(cams)}")
        self.model.step_count += 1
        try:
            self.last_loss = accumulate_views(self.ops, self.model, cams, gts, self.grad,
                                              self.compact, ssim_weight, background, glob_scale,
                                              clip_thresh)
            self.apply(cams[0])
        except PeerLostError:
            self.model.step_count -= 1   # the step did not happen
            raise
        return self.last_loss

    def apply(self, cam) -> None:
        """The optimiser half of a step, from the gradients in self.grad
        (this rank's view); model.step_count must already count the step."""
        import torch.distributed as dist
        if self.mode == "peer":
            m = self.model
            steps, bc2s = m.adam_scalars()
            self.epoch += 1
            rc = _lib.load().msplat_dp_reduce_adam(
                self.rank, self.world, m.n, m.rest_bases, cam.degree, cam.degrees_to_use,
                self._grads_arr, self._params_arr, _ptr_array(m.exp_avg), _ptr_array(m.exp_avg_sq),
                self._flags_arr, self.epoch, _lib.farr(steps), _lib.farr(bc2s), m.beta1, m.beta2,
                m.eps, 1 if self.compact else 0, self.peer_timeout_s)
            _lib.check(rc, "msplat_dp_reduce_adam")
            return
        if self.world > 1:
            try:
                dist.all_reduce(self.grad, op=dist.ReduceOp.SUM)
            except RuntimeError as e:   # timed out, or a peer's connection closed
                raise PeerLostError(
                    f"rank {self.rank}: the gradient exchange of step {self.model.step_count} "
                    f"failed (a peer exited or stalled past the process group's timeout); "
                    f"no parameter was updated: {e}") from e
        self.ops.adam_apply(self.model, cam, self.grad, 1.0 / self.world)

    def peer_errors(self, reset: bool = False) -> int:
        """Error bits of the peer-memory steps so far (0 = none; waits for
        the GPU): 1 a peer's gradients, 2 a peer's updated shard never came."""
        return int(_lib.load().msplat_dp_errors(1 if reset else 0))

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
        """Hands the parameters back to torch-owned memory, unmaps the peers'
        buffers and frees this rank's (peer mode), then ends the group if this
        object created it."""
        import torch
        import torch.distributed as dist
        if self._bufs:
            torch.cuda.synchronize()
            self.barrier()
            self.model.params = [p.clone() for p in self.model.params]
            self.grad = None
            torch.cuda.synchronize()
            _lib.load().msplat_ipc_close_all()
            self.barrier()
            for b in self._bufs:
                b.free()
            self._bufs = []
        if self._owns_group and dist.is_initialized():
            dist.destroy_process_group()
        self._owns_group = False


class PeerLostError(RuntimeError):
    """A data-parallel step could not complete because another rank left or
    stalled between steps; the local replica is left as before the step."""


def rank_and_world() -> tuple[int, int]:
    """RANK / WORLD_SIZE from the torchrun environment (0, 1 without it)."""
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
