"""The engine's C-ABI library builds, loads and exports every symbol its
header declares (no compute calls: this runs without a GPU)."""
from __future__ import annotations

import os
import re
import subprocess

import pytest

from msplat_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def declared_functions(path: str) -> list:
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    names = re.findall(r"\b([A-Za-z_]\w*)\s*\(", text)
    skip = {"sizeof", "defined", "if", "return", "extern"}
    out = []
    for m in re.finditer(r"^[A-Za-z_][\w \t\*]*?\b([A-Za-z_]\w*)\s*\([^;{]*\)\s*;", text, re.M):
        if m.group(1) not in skip:
            out.append(m.group(1))
    return sorted(set(out) & set(names))


@pytest.fixture(scope="module")
def lib_path():
    if not os.path.exists(_lib.LIB_PATH):
        build.build()
    return _lib.LIB_PATH


def test_headers_exist():
    assert HEADERS, "include/*.h missing"


def test_every_declared_symbol_exported(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for h in HEADERS:
        if os.path.basename(h) != "msplat_engine.h":
            continue
        decl = declared_functions(h)
        assert len(decl) >= 20
        missing = [d for d in decl if d not in exported]
        assert not missing, f"{os.path.basename(h)}: not exported: {missing}"


def test_ctypes_signatures_cover_header(lib_path):
    decl = declared_functions(os.path.join(ROOT, "include", "msplat_engine.h"))
    assert set(decl) <= set(_lib.SIGNATURES), set(decl) - set(_lib.SIGNATURES)
    lib = _lib.load()
    for name in decl:
        assert hasattr(lib, name)


def test_last_error_is_a_string(lib_path):
    assert isinstance(_lib.load().msplat_last_error(), bytes)


def test_no_device_fails_loudly(lib_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    assert lib.msplat_device() is None
    assert b"no CUDA device" in lib.msplat_last_error()
