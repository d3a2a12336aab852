"""Checkers for the model files the engine writes: .msplat checkpoints,
Gaussian PLY and .splat.

TEST INFRASTRUCTURE ONLY (tests/ and the golden-fixture script use it; the
engine never does).

* PLY and .splat: the reference's own writers and reader
  (core/src/loaders/save_gaussians.cpp) compiled from its source into
  oracle/_ref/libmsplat_ref_io.so (oracle/ref_shim/build_ref.py build_io),
  reached through `RefIO`; plus a byte-level restatement of the PLY layout
  (`ply_bytes`, no CRS transform) and parsers for round-trip checks.
* .msplat: a restatement of Model::saveCheckpoint (core/src/model.cpp:
  333-399) in `checkpoint_bytes`, and its reader.  model.cpp does not build
  on its own (it needs the Metal runtime bindings and the un-vendored
  nanoflann k-d tree), so this restatement is pinned only by the format as
  the source states it.
"""
from __future__ import annotations

import ctypes as C
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_IO_PATH = os.path.join(HERE, "_ref", "libmsplat_ref_io.so")

CKPT_MAGIC = 0x4C50534D   # model.cpp:335
CKPT_VERSION = 1          # model.cpp:336
GROUPS = ("means", "scales", "quats", "features_dc", "features_rest", "opacities")


def group_shapes(n: int, rest_bases: int):
    return [(n, 3), (n, 3), (n, 4), (n, 3), (n, rest_bases, 3), (n, 1)]


# ---- .msplat -----------------------------------------------------------------

def _tensor_bytes(a: np.ndarray) -> bytes:
    """writeTensor (model.cpp:338-348): u32 ndim, i64 shape, u64 bytes, data."""
    a = np.ascontiguousarray(a, dtype="<f4")
    out = struct.pack("<I", a.ndim) + struct.pack(f"<{a.ndim}q", *a.shape)
    return out + struct.pack("<Q", a.nbytes) + a.tobytes()


def checkpoint_bytes(step, num_active, sh_degree, adam_step_count, adam_lr, means_lr_init,
                     means_lr_final, params, exp_avg, exp_avg_sq) -> bytes:
    """Model::saveCheckpoint (model.cpp:361-399)."""
    out = struct.pack("<6I", CKPT_MAGIC, CKPT_VERSION, step, num_active, sh_degree,
                      adam_step_count)
    out += np.asarray(adam_lr, dtype="<f4").tobytes()
    out += struct.pack("<2f", means_lr_init, means_lr_final)
    for group in (params, exp_avg, exp_avg_sq):
        for a in group:
            out += _tensor_bytes(a)
    return out


def read_checkpoint(blob: bytes) -> dict:
    """Model::loadCheckpoint's reads (model.cpp:401-435)."""
    magic, version, step, num, deg, adam_steps = struct.unpack_from("<6I", blob, 0)
    if magic != CKPT_MAGIC:
        raise ValueError("Not a valid msplat checkpoint file")
    if version != CKPT_VERSION:
        raise ValueError(f"Unsupported checkpoint version: {version}")
    off = 24
    lr = list(struct.unpack_from("<6f", blob, off))
    off += 24
    lr_init, lr_final = struct.unpack_from("<2f", blob, off)
    off += 8
    tensors = []
    for _ in range(18):
        (ndim,) = struct.unpack_from("<I", blob, off)
        off += 4
        shape = struct.unpack_from(f"<{ndim}q", blob, off)
        off += 8 * ndim
        (nbytes,) = struct.unpack_from("<Q", blob, off)
        off += 8
        tensors.append(np.frombuffer(blob, "<f4", int(nbytes) // 4, off).reshape(shape).copy())
        off += int(nbytes)
    return {"step": step, "num_active": num, "sh_degree": deg, "adam_step_count": adam_steps,
            "adam_lr": lr, "means_lr_init": lr_init, "means_lr_final": lr_final,
            "params": tensors[:6], "exp_avg": tensors[6:12], "exp_avg_sq": tensors[12:18],
            "size": off}


# ---- PLY -------------------------------------------------------------------------

def ply_header(step: int, n: int, rest_bases: int) -> bytes:
    """saveGaussianPly's header (save_gaussians.cpp:19-29)."""
    lines = ["ply", "format binary_little_endian 1.0", f"comment msplat v{step}",
             f"element vertex {n}", "property float x", "property float y", "property float z",
             "property float nx", "property float ny", "property float nz"]
    lines += [f"property float f_dc_{i}" for i in range(3)]
    lines += [f"property float f_rest_{i}" for i in range(3 * rest_bases)]
    lines += ["property float opacity"] + [f"property float scale_{i}" for i in range(3)]
    lines += [f"property float rot_{i}" for i in range(4)] + ["end_header"]
    return ("\n".join(lines) + "\n").encode()


def ply_bytes(step: int, params) -> bytes:
    """saveGaussianPly without the CRS transform (save_gaussians.cpp:10-54):
    per vertex x y z, three zero normals, f_dc, f_rest as [3, B], opacity,
    scale_0..2, rot_0..3, all little-endian f32."""
    means, scales, quats, dc, rest, op = (np.asarray(a, np.float32) for a in params)
    n, rb = means.shape[0], rest.shape[1]
    rows = np.concatenate([
        means, np.zeros((n, 3), np.float32), dc, rest.transpose(0, 2, 1).reshape(n, 3 * rb),
        op.reshape(n, 1), scales, quats], axis=1)
    return ply_header(step, n, rb) + rows.astype("<f4").tobytes()


def read_ply(blob: bytes):
    """Parse a Gaussian PLY as loadGaussianPly does (save_gaussians.cpp:99-180)
    without the CRS transform.  Returns (params, step)."""
    end = blob.index(b"end_header\n") + len(b"end_header\n")
    step, n, n_dc, n_fr = 0, 0, 0, 0
    for line in blob[:end].decode().split("\n"):
        if line.startswith("comment Generated by msplat at iteration "):
            step = int(line.split()[-1])
        if line.startswith("element vertex "):
            n = int(line.split()[-1])
        n_dc += line.startswith("property float f_dc_")
        n_fr += line.startswith("property float f_rest_")
    rb = n_fr // 3
    rows = np.frombuffer(blob, "<f4", offset=end).reshape(n, 3 + 3 + n_dc + n_fr + 1 + 3 + 4)
    c = 6
    dc = rows[:, c:c + n_dc]
    c += n_dc
    rest = rows[:, c:c + n_fr].reshape(n, 3, rb).transpose(0, 2, 1)
    c += n_fr
    op = rows[:, c:c + 1]
    scales = rows[:, c + 1:c + 4]
    quats = rows[:, c + 4:c + 8]
    params = [rows[:, :3], scales, quats, dc, rest, op]
    return [np.ascontiguousarray(a, np.float32) for a in params], step


# ---- the reference's own writers/reader ---------------------------------------------

class RefIO:
    """oracle/_ref/libmsplat_ref_io.so: the reference's saveGaussianPly,
    saveGaussianSplat and loadGaussianPly on host arrays."""

    def __init__(self, path: str = REF_IO_PATH):
        lib = C.CDLL(path)
        pp = C.POINTER(C.c_void_p)
        fp = C.POINTER(C.c_float)
        lib.ref_save_ply.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, pp, C.c_int, C.c_float, fp]
        lib.ref_save_splat.argtypes = [C.c_char_p, C.c_int, pp, C.c_int, C.c_float, fp]
        lib.ref_load_ply.argtypes = [C.c_char_p, C.c_int, C.c_float, fp, C.c_int, pp,
                                     C.POINTER(C.c_int), C.POINTER(C.c_int)]
        lib.ref_io_last_error.restype = C.c_char_p
        self.lib = lib

    @staticmethod
    def available(path: str = REF_IO_PATH) -> bool:
        return os.path.exists(path)

    @staticmethod
    def _arrays(params):
        arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in params]
        return arrs, (C.c_void_p * 6)(*[a.ctypes.data for a in arrs])

    def _check(self, rc):
        if rc < 0:
            raise RuntimeError(self.lib.ref_io_last_error().decode())
        return rc

    def save_ply(self, path, step, params, keep_crs=False, scale=1.0, translation=(0, 0, 0)):
        arrs, ptrs = self._arrays(params)
        t = (C.c_float * 3)(*translation)
        self._check(self.lib.ref_save_ply(str(path).encode(), step, arrs[0].shape[0],
                                          arrs[4].shape[1], ptrs, int(keep_crs), scale, t))

    def save_splat(self, path, params, keep_crs=False, scale=1.0, translation=(0, 0, 0)):
        arrs, ptrs = self._arrays(params)
        t = (C.c_float * 3)(*translation)
        self._check(self.lib.ref_save_splat(str(path).encode(), arrs[0].shape[0], ptrs,
                                            int(keep_crs), scale, t))

    def load_ply(self, path, capacity, rest_bases, keep_crs=False, scale=1.0,
                 translation=(0, 0, 0)):
        out = [np.zeros(s, np.float32) for s in group_shapes(capacity, rest_bases)]
        ptrs = (C.c_void_p * 6)(*[a.ctypes.data for a in out])
        n, rb = C.c_int(), C.c_int()
        t = (C.c_float * 3)(*translation)
        step = self._check(self.lib.ref_load_ply(str(path).encode(), int(keep_crs), scale, t,
                                                 capacity, ptrs, C.byref(n), C.byref(rb)))
        assert rb.value == rest_bases
        return [a[:n.value] for a in out], step
