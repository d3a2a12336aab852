"""Training images on the device: PNG decoding (every colour type, bit depth,
filter and interlacing) bit-exact; JPEG through nvJPEG against PIL's decoder
within a stated tolerance; area downscaling and undistortion bit-exact with
the reference's resizeArea / undistortImage (compiled from its sources); and
whole datasets loaded onto the device (Camera::loadImage + getGPUImage)
bit-exact with the reference, intrinsics included."""
from __future__ import annotations

import ctypes as C
import io

import numpy as np
import pytest

from msplat_b200 import _lib, engine
from msplat_b200.dataset import Dataset
from oracle import data as ref_data
from tests import dataset_case, png_case

pytestmark = pytest.mark.gpu
needs_ref = pytest.mark.skipif(not ref_data.available(),
                               reason="oracle/_ref/libmsplat_ref_data.so not built")


@pytest.fixture(scope="module", autouse=True)
def gpu():
    import torch
    assert torch.cuda.is_available(), "image GPU tests need a CUDA device"
    engine.bind_stream()
    yield


def _decode(path):
    import torch
    lib = _lib.load()
    w, h = C.c_int(), C.c_int()
    _lib.check(lib.msplat_image_info(str(path).encode(), C.byref(w), C.byref(h)), "image_info")
    out = torch.full((h.value, w.value, 3), float("nan"), device="cuda")
    w2, h2 = C.c_int(), C.c_int()
    _lib.check(lib.msplat_image_decode(str(path).encode(), C.c_void_p(out.data_ptr()), out.numel(),
                                       C.byref(w2), C.byref(h2)), "image_decode")
    assert (w2.value, h2.value) == (w.value, h.value)
    return out.cpu().numpy()


def _as_float(rgb8):
    return rgb8.astype(np.float32) / np.float32(255.0)


PNG_KINDS = [(2, 8), (6, 8), (0, 8), (4, 8), (0, 1), (0, 2), (0, 4), (3, 1), (3, 2), (3, 4),
             (3, 8), (2, 16), (6, 16), (0, 16), (4, 16)]


@pytest.mark.parametrize("interlace", [False, True])
def test_png_decode_bit_exact(tmp_path, interlace):
    for k, (color, depth) in enumerate(PNG_KINDS):
        h, w = (37, 53) if k % 2 else (8, 9)
        s = png_case.random_samples(h, w, color, depth, 40 + k)
        pal = np.random.default_rng(k).integers(0, 256, (1 << depth, 3)) if color == 3 else None
        path = tmp_path / f"k{k}.png"
        path.write_bytes(png_case.png_bytes(s, color, depth, interlace, pal))
        got = _decode(path)
        want = _as_float(png_case.expected_rgb8(s, color, depth, pal))
        assert got.tobytes() == want.tobytes(), (color, depth, interlace)


def test_png_matches_pil_and_errors(tmp_path):
    from PIL import Image
    px = dataset_case.image_pixels(61, 43, 9)
    Image.fromarray(px).save(tmp_path / "a.png")
    assert _decode(tmp_path / "a.png").tobytes() == _as_float(px).tobytes()
    lib = _lib.load()
    (tmp_path / "x.bmp").write_bytes(b"BM" + bytes(100))
    w = C.c_int()
    assert lib.msplat_image_info(str(tmp_path / "x.bmp").encode(), C.byref(w), None) < 0
    assert lib.msplat_image_info(str(tmp_path / "none.png").encode(), C.byref(w), None) < 0
    blob = (tmp_path / "a.png").read_bytes()
    (tmp_path / "t.png").write_bytes(blob[: len(blob) // 2])     # truncated stream
    import torch
    buf = torch.zeros(61 * 43 * 3, device="cuda")
    assert lib.msplat_image_decode(str(tmp_path / "t.png").encode(), C.c_void_p(buf.data_ptr()),
                                   buf.numel(), None, None) < 0
    assert lib.msplat_image_decode(str(tmp_path / "a.png").encode(), C.c_void_p(buf.data_ptr()),
                                   100, None, None) < 0           # too small a buffer


# nvJPEG and libjpeg (PIL) use different IDCT arithmetic, and for 4:2:0
# chroma libjpeg interpolates ("fancy" triangular upsampling) where nvJPEG
# replicates; the decoded bytes differ by a few levels, and by more in the
# chroma of subsampled images with per-pixel colour noise.  So: every
# channel on a 4:4:4 or grey file and on a smooth 4:2:0 file, and luma only
# on a noisy 4:2:0 file.
JPEG_MAX_LEVELS = 12
JPEG_MEAN_LEVELS = {False: 0.75, True: 1.5}   # by chroma subsampling


def _smooth_pixels(w, h):
    y, x = np.mgrid[0:h, 0:w].astype(np.float32)
    rgb = np.stack([x / (w - 1), y / (h - 1), 0.5 + 0.4 * np.sin(x * 0.05 + y * 0.03)], -1)
    return np.clip(rgb * 255.0 + 0.5, 0, 255).astype(np.uint8)


@pytest.mark.parametrize("mode,subsampling,noisy", [("RGB", 0, True), ("RGB", 2, False),
                                                    ("RGB", 2, True), ("L", 0, True)])
def test_jpeg_decode_against_pil(tmp_path, mode, subsampling, noisy):
    from PIL import Image
    px = dataset_case.image_pixels(203, 131, 11) if noisy else _smooth_pixels(203, 131)
    im = Image.fromarray(px).convert(mode)
    kw = {"subsampling": subsampling} if mode == "RGB" else {}
    im.save(tmp_path / "a.jpg", quality=92, **kw)
    ref = np.array(Image.open(tmp_path / "a.jpg").convert("RGB")).astype(np.float64)
    got = _decode(tmp_path / "a.jpg")
    # every value is a byte / 255
    got8 = np.rint(got * 255.0)
    assert got.tobytes() == _as_float(got8.astype(np.uint8)).tobytes()
    if mode == "RGB" and subsampling == 2 and noisy:
        luma = np.array([0.299, 0.587, 0.114])
        got8, ref = got8 @ luma, ref @ luma
    levels = np.abs(got8 - ref)
    assert levels.max() <= JPEG_MAX_LEVELS, levels.max()
    assert levels.mean() <= JPEG_MEAN_LEVELS[subsampling == 2], levels.mean()


def _dev(a):
    import torch
    return torch.as_tensor(np.ascontiguousarray(a, np.float32), device="cuda")


@needs_ref
@pytest.mark.parametrize("src,dst", [((97, 61), (48, 30)), ((97, 61), (32, 20)), ((64, 48), (16, 12)),
                                     ((97, 61), (13, 7)), ((50, 40), (37, 29)), ((31, 17), (31, 17))])
def test_resize_area_bit_exact(src, dst):
    import torch
    img = np.random.default_rng(src[0] + dst[0]).random((src[1], src[0], 3), dtype=np.float32)
    out = torch.zeros((dst[1], dst[0], 3), device="cuda")
    _lib.check(_lib.load().msplat_resize_area(C.c_void_p(_dev(img).data_ptr()), src[0], src[1],
                                              C.c_void_p(out.data_ptr()), dst[0], dst[1]), "resize")
    torch.cuda.synchronize()
    assert out.cpu().numpy().tobytes() == ref_data.resize_area(img, *dst).tobytes()


@needs_ref
@pytest.mark.parametrize("dist", [(-0.08, 0.02, 0.0015, -0.001, 0.0), (0.12, -0.05, 0.0, 0.0, 0.01),
                                  (-0.3, 0.1, 0.004, 0.003, -0.02), (1e-4, 0.0, 0.0, 0.0, 0.0)])
def test_undistort_bit_exact(dist):
    import torch
    w, h, fx, fy, cx, cy = 96, 72, 80.0, 78.5, 47.3, 36.1
    k1, k2, p1, p2, k3 = dist
    img = np.random.default_rng(7).random((h, w, 3), dtype=np.float32)
    want, intr = ref_data.undistort(img, fx, fy, cx, cy, k1, k2, p1, p2, k3)
    roi = (C.c_int * 4)()
    lib = _lib.load()
    _lib.check(lib.msplat_undistort_roi(w, h, fx, fy, cx, cy, k1, k2, p1, p2, k3, roi), "roi")
    assert (roi[2], roi[3]) == (want.shape[1], want.shape[0])
    out = torch.zeros((roi[3], roi[2], 3), device="cuda")
    _lib.check(lib.msplat_undistort(C.c_void_p(_dev(img).data_ptr()), w, h, fx, fy, cx, cy, k1, k2,
                                    p1, p2, k3, roi, C.c_void_p(out.data_ptr())), "undistort")
    torch.cuda.synchronize()
    assert out.cpu().numpy().tobytes() == want.tobytes()
    assert np.float32(cx - roi[0]) == intr[2] and np.float32(cy - roi[1]) == intr[3]


@needs_ref
@pytest.mark.parametrize("layout", sorted(dataset_case.LAYOUTS))
@pytest.mark.parametrize("downscale", [1.0, 2.0, 2.5])
def test_dataset_images_bit_exact(tmp_path, layout, downscale):
    import torch
    dataset_case.LAYOUTS[layout](str(tmp_path))
    ds = Dataset(str(tmp_path), downscale_factor=downscale)
    ref = ref_data.RefDataset(str(tmp_path))
    for i, cam in enumerate(ds.cameras):
        ref.load_image(i, downscale)
        want = ref.camera(i)
        assert (cam.width, cam.height) == (want["width"], want["height"])
        for k in ("fx", "fy", "cx", "cy", "k1", "k2", "k3", "p1", "p2"):
            assert np.float32(getattr(cam, k)).tobytes() == want[k].tobytes(), (i, k)
        for k in (1, 2, 4):
            got = cam.gt(k)
            torch.cuda.synchronize()
            assert got.cpu().numpy().tobytes() == ref.gt(i, k).tobytes(), (i, k)
    assert ds.device_bytes() > 0
    ds.close()
