"""Build libmsplat_model_cuda.so: the reference's own Model, Trainer, C API
and data front end, compiled unmodified from the reference's sources, over
the CUDA engine through the backend seam of this directory.

What a maintainer of the reference would do to switch its backend from
Metal to this engine: compile core/src/*.cpp, the loaders and msplat_api.mm
(plain C++ despite its extension) with bindings_cuda.cpp in place of
core/metal/msplat_metal.mm and image_io.cpp's CoreGraphics half, and link
libmsplat_b200.so.  The reference checkout is read where it lies
($MSPLAT_REFERENCE, else a "reference" directory beside this repository);
outputs go to msplat_b200/seam/_build/ only.  nanoflann (the reference
fetches v1.5.5 at configure time) is replaced by include/kdtree_tensor.hpp,
which runs the k-nearest-neighbour search on the GPU; nlohmann/json (also
fetched at configure time) is taken from an unmodified copy in the Python
environment (cudnn_frontend ships one).
"""
from __future__ import annotations

import glob
import os
import site
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(BUILD, "libmsplat_model_cuda.so")
REFERENCE = os.environ.get("MSPLAT_REFERENCE") or os.path.join(os.path.dirname(REPO),
                                                                "reference")

REF_SOURCES = [("core", "src", "model.cpp"), ("core", "src", "ssim.cpp"),
               ("core", "src", "input_data.cpp"), ("core", "src", "loaders", "load_colmap.cpp"),
               ("core", "src", "loaders", "load_ply.cpp"),
               ("core", "src", "loaders", "load_nerfstudio.cpp"),
               ("core", "src", "loaders", "load_polycam.cpp"),
               ("core", "src", "loaders", "save_gaussians.cpp"),
               ("core", "src", "msplat_api.mm")]
# the reference's host arithmetic (camera set-up, schedules) as written: no
# FMA contraction, no fast math
COMMON = ["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC",
          "-Wno-return-type", "-Wno-unused-result"]
# headers the reference's sources reach transitively through libc++ on macOS
FORCE_INCLUDES = ["-include", "cmath", "-include", "stdexcept", "-include", "unordered_map",
                  "-include", "cstring", "-include", "algorithm"]


def available() -> bool:
    return all(os.path.exists(os.path.join(REFERENCE, *p)) for p in REF_SOURCES)


def nlohmann_include() -> str:
    for root in site.getsitepackages() + [sys.prefix]:
        for hit in glob.glob(os.path.join(root, "**", "nlohmann", "json.hpp"), recursive=True):
            return os.path.dirname(os.path.dirname(hit))
    raise FileNotFoundError("nlohmann/json.hpp not found")


def _ref_includes() -> list:
    # the stand-in kdtree_tensor.hpp first, then the reference's headers
    return [f"-I{os.path.join(HERE, 'include')}", f"-I{HERE}",
            f"-I{os.path.join(REFERENCE, 'core', 'include')}",
            f"-I{os.path.join(REFERENCE, 'core', 'metal')}", f"-I{nlohmann_include()}"]


def _jobs() -> list:
    jobs = []
    for parts in REF_SOURCES:
        src = os.path.join(REFERENCE, *parts)
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        lang = ["-x", "c++"] if src.endswith(".mm") else []
        jobs.append((src, obj, COMMON + ["-c"] + FORCE_INCLUDES + _ref_includes() + lang +
                     [src, "-o", obj]))
    src = os.path.join(HERE, "bindings_cuda.cpp")
    obj = os.path.join(BUILD, "bindings_cuda.o")
    jobs.append((src, obj, COMMON + ["-c"] + _ref_includes() + [src, "-o", obj]))
    # the engine half sees only the engine's header
    src = os.path.join(HERE, "seam_engine.cpp")
    obj = os.path.join(BUILD, "seam_engine.o")
    jobs.append((src, obj, COMMON + ["-c", f"-I{HERE}", f"-I{os.path.join(REPO, 'include')}",
                                     src, "-o", obj]))
    return jobs


def build(verbose: bool = False) -> str:
    if not available():
        raise FileNotFoundError(f"reference sources not found under {REFERENCE}")
    engine = os.path.join(PKG, "libmsplat_b200.so")
    if not os.path.exists(engine):
        raise FileNotFoundError(f"{engine} missing: build the engine first")
    os.makedirs(BUILD, exist_ok=True)
    headers = glob.glob(os.path.join(HERE, "*.h")) + glob.glob(os.path.join(HERE, "include", "*"))
    headers.append(os.path.join(REPO, "include", "msplat_engine.h"))

    def stale(obj, src):
        return (not os.path.exists(obj) or
                any(os.path.getmtime(d) > os.path.getmtime(obj) for d in [src] + headers))

    def run(job):
        src, obj, cmd = job
        if not stale(obj, src):
            return None
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        return None if r.returncode == 0 else f"{src}:\n{r.stderr[-4000:]}"

    jobs = _jobs()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        errors = [e for e in ex.map(run, jobs) if e]
    if errors:
        raise RuntimeError("seam build failed:\n" + "\n".join(errors))
    objs = [o for _, o, _ in jobs]
    if (not os.path.exists(LIB) or
            any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs + [engine])):
        cmd = ["g++", "-shared", "-o", LIB, *objs, f"-L{PKG}", "-lmsplat_b200",
               "-Wl,-rpath,$ORIGIN/../..", "-Wl,-Bsymbolic"]
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"seam link failed:\n{r.stderr[-4000:]}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
