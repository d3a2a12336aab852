"""The CUDA backend seam library (msplat_b200/seam/build_seam.py) builds from
the reference's sources, links the engine and exports the reference's C API
(no compute calls: this runs without a GPU)."""
from __future__ import annotations

import os
import re
import subprocess

import pytest

from msplat_b200 import _lib
from msplat_b200.seam import build_seam

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_seam_library_exports_the_reference_c_api():
    if not build_seam.available() and not os.path.exists(build_seam.LIB):
        pytest.skip("reference sources absent and the seam library was not built")
    if build_seam.available():
        if not os.path.exists(_lib.LIB_PATH):
            from msplat_b200 import build
            build.build()
        build_seam.build()
    out = subprocess.run(["nm", "-D", "--defined-only", build_seam.LIB], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    header = open(os.path.join(ROOT, "include", "msplat_c_api.h")).read()
    api = set(re.findall(r"\b(msplat_(?:dataset|trainer)_\w+)\s*\(", header))
    # msplat_dataset_camera_pose is this repository's addition to the C API
    api.discard("msplat_dataset_camera_pose")
    assert api and api <= exported, sorted(api - exported)
    # the engine is a dependency, resolved beside the package
    deps = subprocess.run(["ldd", build_seam.LIB], capture_output=True, text=True).stdout
    assert "libmsplat_b200.so" in deps and "not found" not in deps
