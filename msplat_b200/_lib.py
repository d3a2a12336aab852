"""ctypes binding of libmsplat_b200.so (C-ABI in include/msplat_engine.h).

The library is built in-tree by msplat_b200/build.py.  Loading fails loudly
when it is missing: the engine has no CPU path.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# MSPLAT_B200_LIB selects another build of the same library (e.g. a tuning
# variant built elsewhere); by default the in-tree build.
LIB_PATH = os.environ.get("MSPLAT_B200_LIB") or os.path.join(_HERE, "libmsplat_b200.so")

_f = C.c_float
_i = C.c_int
_u = C.c_uint
_p = C.c_void_p
_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int)


class CameraInfo(C.Structure):
    """MsplatCameraInfo (include/msplat_engine.h)."""
    _fields_ = [
        ("width", C.c_int), ("height", C.c_int),
        ("fx", C.c_float), ("fy", C.c_float), ("cx", C.c_float), ("cy", C.c_float),
        ("k1", C.c_float), ("k2", C.c_float), ("k3", C.c_float), ("p1", C.c_float),
        ("p2", C.c_float), ("cam_to_world", C.c_float * 16),
    ]

class MsplatConfig(C.Structure):
    """MsplatConfig (include/msplat_c_api.h)."""
    _fields_ = [
        ("iterations", C.c_int), ("shDegree", C.c_int), ("shDegreeInterval", C.c_int),
        ("ssimWeight", C.c_float), ("numDownscales", C.c_int), ("resolutionSchedule", C.c_int),
        ("refineEvery", C.c_int), ("warmupLength", C.c_int), ("resetAlphaEvery", C.c_int),
        ("densifyGradThresh", C.c_float), ("densifySizeThresh", C.c_float),
        ("stopScreenSizeAt", C.c_int), ("splitScreenSize", C.c_float), ("keepCrs", C.c_bool),
        ("downscaleFactor", C.c_float), ("bgColor", C.c_float * 3),
    ]


class MsplatStats(C.Structure):
    _fields_ = [("iteration", C.c_int), ("splatCount", C.c_int), ("msPerStep", C.c_float)]


class MsplatEvalMetrics(C.Structure):
    _fields_ = [("psnr", C.c_float), ("ssim", C.c_float), ("l1", C.c_float),
                ("numTest", C.c_int), ("numGaussians", C.c_int)]


class MsplatPixelBuffer(C.Structure):
    _fields_ = [("data", C.POINTER(C.c_float)), ("width", C.c_int), ("height", C.c_int)]


# name -> (restype, argtypes); mirrors include/msplat_engine.h and msplat_c_api.h
SIGNATURES = {
    "msplat_last_error": (C.c_char_p, []),
    "msplat_set_stream": (_i, [_p]),
    "msplat_get_stream": (_p, []),
    "msplat_device": (_p, []),
    "msplat_gpu_alloc": (_p, [C.c_size_t, _i]),
    "msplat_gpu_free": (None, [_p]),
    "msplat_copy": (_i, [_p, _p, C.c_size_t, _i, _i]),
    "msplat_commit": (None, []),
    "msplat_gpu_sync": (None, []),
    "cleanup_msplat_metal": (None, []),
    "cleanup_msplat_cuda": (None, []),
    "msplat_set_metallib_path": (None, [C.c_char_p]),
    "msplat_enable_gpu_timing": (None, [_i]),
    "msplat_drain_gpu_times": (_i, [C.POINTER(C.c_double), _i]),
    "msplat_drain_stage_times": (_i, [C.POINTER(C.c_double), _i, _i, _ip, C.POINTER(C.c_char_p)]),
    "msplat_train_step": (_i, [
        _i, _p, _p, _f, _p,            # num_points, means3d, scales, glob_scale, quats
        _fp, _fp, _f, _f, _f, _f,      # viewmat, projmat, fx, fy, cx, cy
        _u, _u, _ip, _f,               # img_height, img_width, tile_bounds, clip_thresh
        _u, _u, _fp,                   # degree, degrees_to_use, cam_pos
        _p, _p, _p, _fp,               # features_dc, features_rest, opacities, background
        _p, _p, _f, _f,                # gt, window2d, ssim_weight, loss_inv_n
        _i, _i, C.POINTER(_p), C.POINTER(_p), C.POINTER(_p),  # rest bases, groups, params, m, v
        _fp, _fp, _f, _f, _f,          # step sizes, bc2 sqrts, beta1, beta2, eps
        _p, _p, _p, _f,                # vis_counts, xys_grad_norm, max_2d_size, inv_max_dim
        C.POINTER(_p), _fp,            # radii_out, loss_out
    ]),
    "msplat_render": (_i, [
        _i, _p, _p, _f, _p, _fp, _fp, _f, _f, _f, _f, _u, _u, _ip, _f, _u, _u, _fp,
        _p, _p, _p, _fp, C.POINTER(_p),
    ]),
    "msplat_train_step_grads": (_i, [
        _i, _p, _p, _f, _p, _fp, _fp, _f, _f, _f, _f, _u, _u, _ip, _f, _u, _u, _fp,
        _p, _p, _p, _fp, _p, _f, _f, _i, _p, _p, _p, _p, _f, C.POINTER(_p), _fp,
    ]),
    "msplat_train_step_grads_compact": (_i, [
        _i, _p, _p, _f, _p, _fp, _fp, _f, _f, _f, _f, _u, _u, _ip, _f, _u, _u, _fp,
        _p, _p, _p, _fp, _p, _f, _f, _i, _p, _p, _p, _p, _f, C.POINTER(_p), _fp,
    ]),
    "msplat_train_step_grads_accumulate": (_i, [
        _i, _p, _p, _f, _p, _fp, _fp, _f, _f, _f, _f, _u, _u, _ip, _f, _u, _u, _fp,
        _p, _p, _p, _fp, _p, _f, _f, _i, _p, _p, _p, _p, _f, C.POINTER(_p), _fp,
    ]),
    "msplat_adam_apply": (_i, [
        _i, _i, _u, _u, _p, _f, _i, _i, _i, C.POINTER(_p), C.POINTER(_p), C.POINTER(_p),
        _fp, _fp, _f, _f, _f,
    ]),
    "msplat_dp_reduce_adam": (_i, [
        _i, _i, _i, _i, _u, _u, C.POINTER(_p), C.POINTER(_p), C.POINTER(_p), C.POINTER(_p),
        C.POINTER(_p), _u, _fp, _fp, _f, _f, _f, _i, C.c_double,
    ]),
    "msplat_dp_errors": (_i, [_i]),
    "msplat_ipc_get_handle": (_i, [_p, _p]),
    "msplat_ipc_open_handle": (_i, [_p, C.POINTER(_p)]),
    "msplat_ipc_close_all": (_i, []),
    "msplat_densify": (_i, [
        _i, _i, _f, _f, _f, _i, _f, _f, _f, _i, _p, _p, _p, _f, _p, _p, _p, _p, _p, _p, _i,
        C.POINTER(_p), C.POINTER(_p), _p, _p, _p, _p, _p, _p, _p, _p, _p,
    ]),
    "msplat_reset_opacity": (_i, [_p, _p, _p, _i]),
    "msplat_stage_input": (_i, [_p, C.c_size_t, C.POINTER(_p)]),
    "msplat_save_checkpoint": (_i, [
        C.c_char_p, _i, _i, _i, _i, _fp, _f, _f, _i, C.POINTER(_p), C.POINTER(_p), C.POINTER(_p),
    ]),
    "msplat_read_checkpoint_header": (_i, [
        C.c_char_p, _ip, _ip, _ip, _ip, _fp, _fp, _fp, _ip,
    ]),
    "msplat_load_checkpoint": (_i, [C.c_char_p, _i, C.POINTER(_p), C.POINTER(_p), C.POINTER(_p)]),
    "msplat_save_ply": (_i, [C.c_char_p, _i, _i, _i, C.POINTER(_p), _i, _f, _fp]),
    "msplat_save_splat": (_i, [C.c_char_p, _i, C.POINTER(_p), _i, _f, _fp]),
    "msplat_read_ply_header": (_i, [C.c_char_p, _ip, _ip, _ip]),
    "msplat_load_ply": (_i, [C.c_char_p, _i, C.POINTER(_p), _i, _f, _fp]),
    "msplat_bytes_to_rgb": (_i, [_p, _i, _i, _i, _p]),
    "msplat_resize_area": (_i, [_p, _i, _i, _p, _i, _i]),
    "msplat_undistort_roi": (_i, [_i, _i, _f, _f, _f, _f, _f, _f, _f, _f, _f, _ip]),
    "msplat_undistort": (_i, [_p, _i, _i, _f, _f, _f, _f, _f, _f, _f, _f, _f, _ip, _p]),
    "msplat_image_info": (_i, [C.c_char_p, _ip, _ip]),
    "msplat_image_decode": (_i, [C.c_char_p, _p, C.c_longlong, _ip, _ip]),
    "msplat_dataset_open": (_i, [C.c_char_p, C.c_char_p, C.POINTER(_p)]),
    "msplat_dataset_close": (None, [_p]),
    "msplat_dataset_num_cameras": (_i, [_p]),
    "msplat_dataset_camera": (_i, [_p, _i, C.POINTER(CameraInfo)]),
    "msplat_dataset_camera_path": (C.c_char_p, [_p, _i]),
    "msplat_dataset_points": (C.c_longlong, [_p, C.POINTER(_fp), C.POINTER(C.POINTER(C.c_ubyte))]),
    "msplat_dataset_transform": (_i, [_p, _fp, _fp]),
    "msplat_dataset_split": (_i, [_p, _i, _ip, _ip, _ip, _ip]),
    "msplat_dataset_validation_camera": (_i, [_p, C.c_char_p]),
    "msplat_dataset_load_images": (_i, [_p, _f]),
    "msplat_dataset_load_image": (_i, [_p, _i, _f]),
    "msplat_dataset_gt": (_i, [_p, _i, _i, C.POINTER(_p), _ip, _ip]),
    "msplat_dataset_device_bytes": (C.c_longlong, [_p]),
    "msplat_eval_metrics": (_i, [_p, _p, _i, _i, _i, _f, _fp, _fp, _fp]),
    "msplat_knn_mean_distance": (_i, [_p, C.c_longlong, _i, _p]),
    "msplat_dataset_data": (_p, [_p]),
    "msplat_dataset_indices": (_i, [_p, _i, _ip, _i]),
    "msplat_dataset_create": (_p, [C.c_char_p, _f, C.c_bool, _i]),
    "msplat_dataset_destroy": (None, [_p]),
    "msplat_dataset_num_train": (_i, [_p]),
    "msplat_dataset_num_test": (_i, [_p]),
    "msplat_dataset_camera_pose": (None, [_p, _i, _fp]),
    "msplat_trainer_create": (_p, [_p, MsplatConfig]),
    "msplat_trainer_destroy": (None, [_p]),
    "msplat_trainer_step": (MsplatStats, [_p]),
    "msplat_trainer_train": (None, [_p]),
    "msplat_trainer_evaluate": (MsplatEvalMetrics, [_p]),
    "msplat_trainer_render": (MsplatPixelBuffer, [_p, _i, C.c_bool]),
    "msplat_trainer_render_pose": (MsplatPixelBuffer, [_p, _fp, _i]),
    "msplat_trainer_render_pose_to_buffer": (None, [_p, _fp, _i, C.POINTER(C.c_ubyte), _ip, _ip]),
    "msplat_trainer_export_ply": (None, [_p, C.c_char_p]),
    "msplat_trainer_export_splat": (None, [_p, C.c_char_p]),
    "msplat_trainer_save_checkpoint": (None, [_p, C.c_char_p]),
    "msplat_trainer_load_checkpoint": (_i, [_p, C.c_char_p]),
    "msplat_trainer_load_checkpoint_ex": (_i, [_p, C.c_char_p, _i]),
    "msplat_trainer_splat_count": (_i, [_p]),
    "msplat_trainer_iteration": (_i, [_p]),
    "msplat_sync": (None, []),
    "msplat_cleanup": (None, []),
    "msplat_init_gaussians": (_i, [_p, _p, C.c_longlong, _i, _p, _p, _p, _p, _p, _p]),
    "msplat_render_noalloc": (_i, [
        _i, _p, _p, _f, _p, _fp, _fp, _f, _f, _f, _f, _u, _u, _ip, _f, _u, _u, _fp,
        _p, _p, _p, _fp, _p, _p,
    ]),
    "msplat_last_loss": (_f, [_i]),
    "msplat_num_intersections": (C.c_longlong, []),
    "msplat_device_errors": (_i, []),
    "msplat_debug_buffer": (_i, [C.c_char_p, C.POINTER(_p), C.POINTER(C.c_longlong)]),
    "msplat_kernel_launches": (C.c_longlong, [_i]),
    "msplat_last_binning": (_i, []),
    "msplat_count_raster_work": (_i, [C.POINTER(C.c_ulonglong)]),
    "msplat_shared_alloc": (_p, [C.c_size_t, _i]),
    "msplat_shared_free": (None, [_p]),
    "msplat_shared_prefetch": (_i, [_p, C.c_size_t]),
}

_lib = None


def load() -> C.CDLL:
    """Load the engine library (once) and attach argument types."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python msplat_b200/build.py` "
            "(the engine is CUDA-only and has no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class EngineError(RuntimeError):
    pass


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = load().msplat_last_error().decode(errors="replace")
        raise EngineError(f"{what} failed ({rc}): {msg}")


def farr(values) -> C.Array:
    vals = [float(v) for v in values]
    return (C.c_float * len(vals))(*vals)


def iarr(values) -> C.Array:
    vals = [int(v) for v in values]
    return (C.c_int * len(vals))(*vals)
