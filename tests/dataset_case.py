"""Seeded miniature datasets in the three layouts the loaders accept, written
to a temporary directory: COLMAP (binary cameras/images/points3D), Nerfstudio
(transforms.json + PLY points) and Polycam (per-keyframe camera JSONs or one
cameras.json, + PLY points).  Images are PNG (written by PIL) with the same
pixels in a ".rgb8" sidecar for the reference build (oracle/data.py).

The COLMAP set covers every camera model the reference reads, unnormalised
quaternions, image names out of order, 2D-point tracks to skip, an image
whose file is smaller than its camera says (the intrinsics are rescaled) and
an OPENCV camera with distortion (undistorted and cropped on load)."""
from __future__ import annotations

import json
import os
import struct

import numpy as np
from PIL import Image

from oracle import data as ref_data


def image_pixels(w: int, h: int, seed: int) -> np.ndarray:
    """Smooth colour ramps plus noise, so resampling errors would show."""
    rng = np.random.default_rng(seed)
    y, x = np.mgrid[0:h, 0:w].astype(np.float32)
    base = np.stack([x / max(w - 1, 1), y / max(h - 1, 1), 0.5 + 0.5 * np.sin(x * 0.3 + y * 0.2)], -1)
    noise = rng.normal(0, 0.08, (h, w, 3))
    return np.clip((base + noise) * 255.0 + 0.5, 0, 255).astype(np.uint8)


def write_image(path: str, pixels: np.ndarray) -> None:
    Image.fromarray(pixels, "RGB").save(path)
    ref_data.write_rgb8(path, pixels)


# COLMAP camera models: id -> (model, width, height, params)
COLMAP_CAMERAS = {
    1: (1, 64, 48, [60.0, 58.5, 31.7, 24.2]),                 # PINHOLE
    2: (0, 64, 48, [55.25, 32.0, 23.5]),                      # SIMPLE_PINHOLE
    3: (2, 128, 96, [110.0, 64.0, 48.0, 0.0]),                # SIMPLE_RADIAL, file is 64x48
    4: (3, 64, 48, [57.0, 32.5, 24.5, 0.0, 0.0]),             # RADIAL (no distortion)
    7: (4, 72, 56, [66.0, 65.0, 36.2, 27.9, -0.08, 0.02, 0.0015, -0.001]),   # OPENCV, distorted
}


def write_colmap(root: str, seed: int = 0, layout: str = "sparse0", points: str = "bin",
                 n_points: int = 300) -> dict:
    rng = np.random.default_rng(seed)
    sparse = os.path.join(root, "sparse", "0") if layout == "sparse0" else root
    os.makedirs(sparse, exist_ok=True)
    img_dir = os.path.join(root, "images")
    os.makedirs(img_dir, exist_ok=True)
    with open(os.path.join(sparse, "cameras.bin"), "wb") as f:
        f.write(struct.pack("<Q", len(COLMAP_CAMERAS)))
        for cid, (model, w, h, params) in COLMAP_CAMERAS.items():
            f.write(struct.pack("<IIQQ", cid, model, w, h))
            f.write(struct.pack(f"<{len(params)}d", *params))
    names = [f"frame_{k:03d}.png" for k in (5, 2, 9, 0, 7, 3, 8, 1)]
    cam_of = [1, 2, 3, 4, 7, 1, 2, 7]
    with open(os.path.join(sparse, "images.bin"), "wb") as f:
        f.write(struct.pack("<Q", len(names)))
        for i, (name, cid) in enumerate(zip(names, cam_of)):
            q = rng.normal(0, 1, 4) * rng.uniform(0.5, 2.0)     # not unit length
            t = rng.normal(0, 3, 3)
            f.write(struct.pack("<I", 100 + i))
            f.write(struct.pack("<4d", *q))
            f.write(struct.pack("<3d", *t))
            f.write(struct.pack("<I", cid))
            f.write(name.encode() + b"\0")
            n2d = int(rng.integers(0, 5))
            f.write(struct.pack("<Q", n2d))
            for _ in range(n2d):
                f.write(struct.pack("<ddq", *rng.normal(0, 10, 2), int(rng.integers(-1, 50))))
            w, h = COLMAP_CAMERAS[cid][1:3]
            if cid == 3:
                w, h = w // 2, h // 2
            write_image(os.path.join(img_dir, name), image_pixels(w, h, seed * 100 + i))
    xyz = rng.normal(0, 2, (n_points, 3))
    rgb = rng.integers(0, 256, (n_points, 3)).astype(np.uint8)
    if points == "bin":
        with open(os.path.join(sparse, "points3D.bin"), "wb") as f:
            f.write(struct.pack("<Q", n_points))
            for i in range(n_points):
                f.write(struct.pack("<Q3d", 1000 + i, *xyz[i]))
                f.write(rgb[i].tobytes())
                f.write(struct.pack("<d", rng.uniform(0, 1)))
                tl = int(rng.integers(0, 4))
                f.write(struct.pack("<Q", tl))
                f.write(rng.integers(0, 100, 2 * tl).astype("<u4").tobytes())
    elif points == "ply":
        write_points_ply(os.path.join(sparse, "points3D.ply"), xyz, rgb, binary=True)
    return {"names": sorted(names), "n_points": n_points if points else 0}


def write_points_ply(path, xyz, rgb, binary=True, xyz_type="float", rgb_type="uchar",
                     extra=False):
    n = len(xyz)
    props = [("x", xyz_type), ("y", xyz_type), ("z", xyz_type)]
    if extra:
        props.append(("nx", "float"))
    if rgb is not None:
        props += [("red", rgb_type), ("green", rgb_type), ("blue", rgb_type)]
    head = ["ply", "format " + ("binary_little_endian 1.0" if binary else "ascii 1.0"),
            f"element vertex {n}"] + [f"property {t} {nm}" for nm, t in props] + ["end_header"]
    np_t = {"float": "<f4", "double": "<f8", "uchar": "u1", "ushort": "<u2"}
    with open(path, "wb") as f:
        f.write(("\n".join(head) + "\n").encode())
        for i in range(n):
            vals = list(xyz[i]) + ([0.25] if extra else [])
            if rgb is not None:
                c = rgb[i]
                vals += [v / 255.0 for v in c] if rgb_type == "float" else (
                    [int(v) * 257 for v in c] if rgb_type == "ushort" else [int(v) for v in c])
            if binary:
                for (nm, t), v in zip(props, vals):
                    f.write(np.array([v], np_t[t]).tobytes())
            else:
                f.write((" ".join(repr(float(v)) if t in ("float", "double") else str(int(v))
                                  for (nm, t), v in zip(props, vals)) + "\n").encode())


def write_nerfstudio(root: str, seed: int = 1) -> dict:
    rng = np.random.default_rng(seed)
    os.makedirs(os.path.join(root, "imgs"), exist_ok=True)
    frames = []
    for k in (3, 0, 2, 1):
        name = f"imgs/view_{k}"
        w, h = (48, 40) if k != 2 else (40, 32)
        write_image(os.path.join(root, name + ".png"), image_pixels(w, h, seed * 10 + k))
        c2w = np.eye(4)
        c2w[:3, :3] = np.linalg.qr(rng.normal(size=(3, 3)))[0]
        c2w[:3, 3] = rng.normal(0, 2, 3)
        fr = {"file_path": name, "transform_matrix": c2w.tolist()}
        if k == 2:
            fr.update({"w": 40, "h": 32, "fl_x": 35.5, "cx": 20.25})
        if k == 1:
            fr.update({"k1": -0.03, "p2": 0.0007})
        frames.append(fr)
    xyz = rng.normal(0, 1, (120, 3))
    rgb = rng.integers(0, 256, (120, 3))
    write_points_ply(os.path.join(root, "pc.ply"), xyz, rgb, binary=False, rgb_type="uchar")
    meta = {"w": 48, "h": 40, "fl_x": 41.0, "fl_y": 40.5, "cx": 24.0, "cy": 20.0,
            "ply_file_path": "pc.ply", "frames": frames}
    with open(os.path.join(root, "transforms.json"), "w") as f:
        json.dump(meta, f, indent=1)
    return {"n": len(frames)}


def write_polycam(root: str, seed: int = 2, layout: int = 1) -> dict:
    rng = np.random.default_rng(seed)
    if layout == 1:
        cams = os.path.join(root, "keyframes", "corrected_cameras")
        imgs = os.path.join(root, "keyframes", "corrected_images")
        os.makedirs(cams, exist_ok=True)
        os.makedirs(imgs, exist_ok=True)
        for k in (11, 4, 7):
            R = np.linalg.qr(rng.normal(size=(3, 3)))[0]
            j = {"width": 40, "height": 30, "fx": 33.0 + k, "fy": 32.5 + k}
            if k != 4:
                j.update({"cx": 19.5, "cy": 15.25})
            j.update({f"R_{r}{c}": float(R[r, c]) for r in range(3) for c in range(3)})
            j.update({"t_20": float(rng.normal()), "t_21": float(rng.normal()), "t_22": float(rng.normal())})
            with open(os.path.join(cams, f"{k}.json"), "w") as f:
                json.dump(j, f)
            write_image(os.path.join(imgs, f"{k}.png"), image_pixels(40, 30, seed * 10 + k))
        ply = os.path.join(root, "keyframes", "point_cloud.ply")
    else:
        os.makedirs(os.path.join(root, "im"), exist_ok=True)
        frames = []
        for k in range(3):
            c2w = np.eye(4)
            c2w[:3, :3] = np.linalg.qr(rng.normal(size=(3, 3)))[0]
            c2w[:3, 3] = rng.normal(0, 1, 3)
            write_image(os.path.join(root, "im", f"{k}.png"), image_pixels(36, 28, seed * 10 + k))
            frames.append({"width": 36, "height": 28, "fx": 30.0, "fy": 30.0,
                           "transform_matrix": c2w.tolist(), "file_path": f"im/{k}.png"})
        with open(os.path.join(root, "cameras.json"), "w") as f:
            json.dump({"frames": frames}, f)
        ply = os.path.join(root, "point_cloud.ply")
    xyz = rng.normal(0, 1, (80, 3))
    rgb = rng.integers(0, 256, (80, 3))
    write_points_ply(ply, xyz, rgb, binary=True, xyz_type="double", rgb_type="ushort", extra=True)
    return {}


LAYOUTS = {
    "colmap": lambda root: write_colmap(root),
    "colmap_flat_ply": lambda root: write_colmap(root, seed=3, layout="flat", points="ply"),
    "nerfstudio": write_nerfstudio,
    "polycam_keyframes": lambda root: write_polycam(root, layout=1),
    "polycam_json": lambda root: write_polycam(root, seed=4, layout=2),
}
