"""Build the engine's shared library, libmsplat_b200.so, in-tree.

nvcc compiles every .cu under csrc/ for sm_100a (B200) only.  The forward
files are compiled with --fmad=false: the engine's projection, binning,
forward raster and loss must produce the same bits as the CPU oracle, and
explicit fmaf() calls mark the fused multiply-adds the reference kernels ask
for.  The backward file (gradients and Adam, held to a tolerance) is
compiled with FMA contraction; the forward decisions it replays are written
with explicit non-fused operations.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libmsplat_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
          f"-I{INCLUDE}"]
FMA_CONTRACTED = {"kernels_bwd.cu", "dp_peer.cu"}   # every other file: --fmad=false


def fmad_flag(src: str) -> str:
    return "--fmad=true" if os.path.basename(src) in FMA_CONTRACTED else "--fmad=false"


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps() -> list[str]:
    out = []
    for d in (CSRC, INCLUDE):
        out += [os.path.join(d, f) for f in os.listdir(d) if f.endswith((".h", ".cuh"))]
    return out


def _stale(target: str, inputs: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(i) > t for i in inputs)


def build(verbose: bool = False, force: bool = False, out: str = LIB, build_dir: str = BUILD,
          defines: tuple = ()) -> str:
    """Compile every csrc/*.cu for sm_100a and link `out`.  `defines`
    (-DNAME=VALUE strings) and a separate `build_dir` make a variant build."""
    os.makedirs(build_dir, exist_ok=True)
    nvcc = _nvcc()
    deps = _deps()
    objs, jobs = [], []
    for src in sources():
        obj = os.path.join(build_dir, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + deps):
            jobs.append([nvcc, *ARCH, *CFLAGS, *defines, fmad_flag(src), "-c", src, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    if force or jobs or _stale(out, objs):
        run([nvcc, *ARCH, "-shared", "-o", out, *objs, "-cudart", "static", "-lz", "-ldl"])
    return out


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
