"""The C++ API (include/msplat_api.hpp, the reference's msplat::Trainer
surface): compiles against the library on the CPU; on a GPU, the program
tests/cpp_api_check.cpp trains, evaluates, renders, exports and resumes
through it."""
from __future__ import annotations

import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "msplat_b200")


def _compile(out):
    cmd = ["g++", "-std=c++17", "-O1", "-I" + os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "cpp_api_check.cpp"), "-o", out, "-L" + LIB_DIR,
           "-lmsplat_b200", "-Wl,-rpath," + LIB_DIR]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_cpp_api_compiles_and_links(tmp_path):
    _compile(str(tmp_path / "api_check"))


@pytest.mark.gpu
def test_cpp_api_runs(tmp_path):
    from tests import dataset_case
    data = tmp_path / "scene"
    dataset_case.write_colmap(str(data), n_points=400)
    exe = str(tmp_path / "api_check")
    _compile(exe)
    r = subprocess.run([exe, str(data), str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert (tmp_path / "scene.ply").stat().st_size > 1000
    # no refinement step within 12 iterations: the 400 initial Gaussians
    assert (tmp_path / "scene.splat").stat().st_size == 32 * 400
