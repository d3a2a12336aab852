"""Held-out metrics on the device (msplat_eval_metrics): PSNR, SSIM and L1
of a rendered image against its ground truth, against the reference's own
ssim_eval / psnr / l1_loss compiled from its sources.  Per-pixel arithmetic
is the reference's; only the order of the double-precision sums differs, so
each metric agrees to within one float ulp (and is usually identical)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from msplat_b200 import _lib, engine
from oracle import data as ref_data

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_data.available(),
                                 reason="oracle/_ref/libmsplat_ref_data.so not built")]


@pytest.fixture(scope="module", autouse=True)
def gpu():
    import torch
    assert torch.cuda.is_available()
    engine.bind_stream()
    yield


def device_metrics(r, g, window=11, sigma=1.5):
    import torch
    rt = torch.as_tensor(np.ascontiguousarray(r, np.float32), device="cuda")
    gt = torch.as_tensor(np.ascontiguousarray(g, np.float32), device="cuda")
    out = [C.c_float() for _ in range(3)]
    _lib.check(_lib.load().msplat_eval_metrics(
        C.c_void_p(rt.data_ptr()), C.c_void_p(gt.data_ptr()), r.shape[0], r.shape[1], window,
        sigma, *[C.byref(o) for o in out]), "msplat_eval_metrics")
    return tuple(np.float32(o.value) for o in out)


def _ulps(a, b):
    return abs(int(np.float32(a).view(np.int32)) - int(np.float32(b).view(np.int32)))


@pytest.mark.parametrize("h,w", [(1, 1), (7, 5), (64, 96), (61, 97), (299, 345), (840, 1297)])
def test_metrics_match_reference(h, w):
    rng = np.random.default_rng(h * 1000 + w)
    gt = rng.random((h, w, 3), dtype=np.float32)
    rendered = np.clip(gt + rng.normal(0, 0.05, gt.shape), 0, 1).astype(np.float32)
    got = device_metrics(rendered, gt)
    want = ref_data.eval_metrics(rendered, gt)
    for name, a, b in zip(("psnr", "ssim", "l1"), got, want):
        assert _ulps(a, b) <= 1, (name, a, b)


@pytest.mark.parametrize("window,sigma", [(11, 1.5), (7, 1.0), (1, 1.5), (10, 2.0)])
def test_window_variants(window, sigma):
    rng = np.random.default_rng(window)
    gt = rng.random((45, 70, 3), dtype=np.float32)
    rendered = (gt * 0.7 + 0.1).astype(np.float32)
    got = device_metrics(rendered, gt, window, sigma)
    want = ref_data.eval_metrics(rendered, gt, window, sigma)
    for a, b in zip(got, want):
        assert _ulps(a, b) <= 1


def test_identical_images_and_errors():
    img = np.random.default_rng(0).random((33, 40, 3), dtype=np.float32)
    psnr, ssim, l1 = device_metrics(img, img)
    assert np.isinf(psnr) and l1 == 0.0 and abs(ssim - 1.0) < 1e-6
    lib = _lib.load()
    assert lib.msplat_eval_metrics(None, None, 4, 4, 11, 1.5, None, None, None) < 0
    assert lib.msplat_eval_metrics(C.c_void_p(1), C.c_void_p(1), 4, 4, 13, 1.5, None, None, None) < 0
