"""Build the reference's own kernels (msplat core/metal/msplat_metal.metal) as
a CPU library, oracle/_ref/libmsplat_ref.so, through the MSL shim.

TEST INFRASTRUCTURE ONLY.  Reads the reference where it lies (read-only);
writes only under oracle/_ref/ (git-ignored; it travels to the GPU box).
Nothing of the reference is copied into the repository.

Mechanical transforms applied to the kernel source before compiling it as
C++ (each keeps the reference's arithmetic):
  1. the Metal header include and `using namespace metal` are dropped;
     address-space qualifiers become C++ (constant -> const, device/thread ->
     nothing, kernel -> nothing) and [[attributes]] are removed;
  2. overloads that differ only in address space (identical bodies) are kept
     once;
  3. only the kernels msplat_train_step / msplat_render / msplat_densify
     dispatch are kept;
  4. each `threadgroup T name[...]` becomes a reference to per-threadgroup
     storage of the shim (filled with 0x7F bytes per threadgroup);
  5. MAX_TILE_ELEMS (the per-tile cap, 2048) becomes overridable; the default
     build raises it (REF_TILE_CAP) so no tile overflows;
  6. in rasterize_backward*_kernel every lane reads the batch entry that the
     reference reads on lane 0 and then broadcasts (the `if (wr == 0)` guard
     of that load only, not of the atomics), which gives the broadcast a
     defined value when lane 0 has returned;
  7. in rasterize_backward_chunked_kernel a thread whose pixel has no
     contributor in the chunk no longer returns early (only empty chunks
     return): the reference's early return leaves that thread's share of the
     cooperative batch load unwritten (other lanes then read stale
     threadgroup memory as Gaussian data) and, when the thread is lane 0,
     drops its SIMD-group's atomics.  Kept in the loop, the thread adds
     nothing, since every index exceeds its bin_final.
"""
from __future__ import annotations

import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE = os.path.dirname(HERE)
OUT = os.path.join(ORACLE, "_ref")
# The reference checkout: $MSPLAT_REFERENCE, else a "reference" directory
# beside this repository.
REFERENCE = os.environ.get("MSPLAT_REFERENCE") or os.path.join(
    os.path.dirname(os.path.dirname(ORACLE)), "reference")
METAL = os.path.join(REFERENCE, "core", "metal", "msplat_metal.metal")
REF_TILE_CAP = int(os.environ.get("REF_TILE_CAP", "16384"))

KERNELS = {
    "project_and_sh_forward_kernel", "scatter_to_prealloc_bins_kernel", "prefix_sum_kernel",
    "bitonic_sort_per_tile_kernel", "nd_rasterize_forward_kernel",
    "rasterize_forward_chunked_kernel", "rasterize_forward_merge_kernel", "ssim_h_fwd_kernel",
    "ssim_fused_v_fwd_h_bwd_kernel", "ssim_v_bwd_kernel", "rasterize_backward_kernel",
    "compute_chunk_prefix_suffix_kernel", "rasterize_backward_chunked_kernel",
    "project_and_sh_backward_kernel", "fused_adam_kernel", "accumulate_grad_stats_kernel",
    # msplat_densify
    "densify_classify_kernel", "block_reduce_kernel", "block_scan_propagate_kernel",
    "densify_append_split_kernel", "densify_append_dup_kernel", "densify_cull_classify_kernel",
    "compact_scatter_kernel", "compact_copy_back_kernel",
}
BWD_KERNELS = {"rasterize_backward_kernel", "rasterize_backward_chunked_kernel"}


def strip_comments(s: str) -> str:
    s = re.sub(r"/\*.*?\*/", "", s, flags=re.S)
    return re.sub(r"//[^\n]*", "", s)


def split_top_level(src: str):
    """Yield ('pp', line) / ('item', text) top-level units."""
    i, n = 0, len(src)
    buf = []
    while i < n:
        if src[i] == "#" and (i == 0 or src[i - 1] == "\n"):
            j = src.find("\n", i)
            j = n if j < 0 else j
            if "".join(buf).strip():
                yield ("item", "".join(buf))
                buf = []
            yield ("pp", src[i:j])
            i = j + 1
            continue
        c = src[i]
        buf.append(c)
        if c == ";" and not any(ch == "{" for ch in "".join(buf)):
            yield ("item", "".join(buf))
            buf = []
        elif c == "{":
            depth = 1
            i += 1
            while i < n and depth:
                buf.append(src[i])
                depth += {"{": 1, "}": -1}.get(src[i], 0)
                i += 1
            # struct definitions end with ';'
            k = i
            while k < n and src[k] in " \t\n":
                k += 1
            if k < n and src[k] == ";":
                buf.append(";")
                i = k + 1
            yield ("item", "".join(buf))
            buf = []
            continue
        i += 1
    if "".join(buf).strip():
        yield ("item", "".join(buf))


ADDR = re.compile(r"\b(device|thread|constant|threadgroup)\b")


def signature_key(head: str) -> str:
    h = re.sub(r"\[\[[^\]]*\]\]", "", head)
    h = re.sub(r"\bconstant\b", "const", h)
    h = re.sub(r"\b(device|thread|inline)\b", "", h)
    h = re.sub(r"\b[A-Za-z_]\w*\s*(?=[,)])", "", h)  # drop parameter names
    return re.sub(r"\s+", "", h)


TG_DECL = re.compile(r"threadgroup\s+([\w:]+)\s+([^;]+);")


def rewrite_tg(body: str, counter: list) -> str:
    def repl(m):
        typ, decls = m.group(1), m.group(2)
        out = []
        for d in re.split(r",\s*(?![^\[]*\])", decls):
            dm = re.match(r"\s*(\w+)\s*((?:\[[^\]]+\])+)\s*$", d)
            if not dm:
                raise ValueError(f"unhandled threadgroup declaration: {d!r}")
            name, dims = dm.group(1), dm.group(2)
            counter[0] += 1
            out.append(f"{typ} (&{name}){dims} = msl::tg_array<{typ}{dims}, {counter[0]}>();")
        return " ".join(out)
    return TG_DECL.sub(repl, body)


def transform(src: str) -> str:
    src = strip_comments(src)
    src = src.replace("#include <metal_stdlib>", "")
    src = re.sub(r"using\s+namespace\s+metal\s*;", "", src)
    out, seen = [], set()
    counter = [0]
    for kind, text in split_top_level(src):
        if kind == "pp":
            m = re.match(r"#define\s+MAX_TILE_ELEMS\s+(\d+)", text)
            if m:
                out.append(f"#ifndef MAX_TILE_ELEMS\n#define MAX_TILE_ELEMS {m.group(1)}\n#endif")
            else:
                out.append(text)
            continue
        t = text.strip()
        if "{" in t and "(" in t.split("{", 1)[0] and not t.startswith("struct"):
            head, body = t.split("{", 1)
            name = re.search(r"(\w+)\s*\(", head).group(1)
            is_kernel = re.search(r"\bkernel\b", head) is not None
            if is_kernel and name not in KERNELS:
                continue
            if not is_kernel:
                key = signature_key(head)
                if key in seen:
                    continue
                seen.add(key)
            body = rewrite_tg(body, counter)
            if name in BWD_KERNELS:
                # only the batch-entry load that feeds simd_broadcast, not the
                # lane-0 atomics that follow the reductions
                body, n_sub = re.subn(r"if\s*\(\s*wr\s*==\s*0\s*\)\s*\{(\s*b_conic\s*=)",
                                      r"if (true) {\1", body)
                if n_sub != 1:
                    raise ValueError(f"{name}: expected one broadcast load block, found {n_sub}")
            if name == "rasterize_backward_chunked_kernel":
                # threads without a contributor in the chunk stay in the
                # threadgroup (they still load their batch entries and add
                # nothing: every index exceeds their bin_final)
                body, n_sub = re.subn(
                    r"if\s*\(\s*chunk_start\s*>=\s*chunk_end\s*\|\|\s*bin_final\s*<\s*chunk_start\s*\)",
                    "if (chunk_start >= chunk_end)", body)
                if n_sub != 1:
                    raise ValueError("chunked backward: early-return test not found")
            t = head + "{" + body
        out.append(t)
    code = "\n".join(out)
    code = re.sub(r"\[\[[^\]]*\]\]", "", code)
    return code


PRELUDE = """// Generated by oracle/ref_shim/build_ref.py from the reference's
// core/metal/msplat_metal.metal -- do not edit, do not commit.
#include "msl_shim.hpp"
namespace msl {
#define kernel
#define device
#define thread
#define constant const
"""
EPILOGUE = """
#undef kernel
#undef device
#undef thread
#undef constant
}  // namespace msl
"""


def build(verbose: bool = False) -> str:
    if not os.path.exists(METAL):
        raise FileNotFoundError(f"reference kernels not found at {METAL}")
    os.makedirs(OUT, exist_ok=True)
    gen = os.path.join(OUT, "msplat_metal_ref.inc")
    code = PRELUDE + transform(open(METAL).read()) + EPILOGUE
    if not os.path.exists(gen) or open(gen).read() != code:
        with open(gen, "w") as f:
            f.write(code)
    lib = os.path.join(OUT, "libmsplat_ref.so")
    srcs = [os.path.join(HERE, "ref_driver.cpp"), os.path.join(HERE, "msl_runtime.cpp")]
    deps = srcs + [gen, os.path.join(HERE, "msl_shim.hpp"), os.path.join(HERE, "msl_runtime.hpp"),
                   os.path.join(ORACLE, "msplat_oracle.h")]
    if os.path.exists(lib) and all(os.path.getmtime(d) <= os.path.getmtime(lib) for d in deps):
        return lib
    cmd = ["g++", "-std=c++20", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC",
           "-shared", "-Wno-attributes", "-Wno-unknown-pragmas", f"-DMAX_TILE_ELEMS={REF_TILE_CAP}",
           f"-I{HERE}", f"-I{OUT}", f"-I{ORACLE}", "-o", lib, *srcs]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"reference shim build failed:\n{r.stderr[-6000:]}")
    return lib


IO_SOURCE = os.path.join(REFERENCE, "core", "src", "loaders", "save_gaussians.cpp")


def build_io(verbose: bool = False) -> str:
    """oracle/_ref/libmsplat_ref_io.so: the reference's save_gaussians.cpp
    (PLY / .splat writers, PLY reader) compiled as it is, with ref_io.cpp
    supplying host versions of the three runtime calls it makes."""
    if not os.path.exists(IO_SOURCE):
        raise FileNotFoundError(f"reference Gaussian I/O not found at {IO_SOURCE}")
    os.makedirs(OUT, exist_ok=True)
    lib = os.path.join(OUT, "libmsplat_ref_io.so")
    srcs = [os.path.join(HERE, "ref_io.cpp"), IO_SOURCE]
    if os.path.exists(lib) and all(os.path.getmtime(d) <= os.path.getmtime(lib) for d in srcs):
        return lib
    cmd = ["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
           "-Wno-return-type", f"-I{os.path.join(REFERENCE, 'core', 'include')}",
           f"-I{os.path.join(REFERENCE, 'core', 'metal')}", "-o", lib, *srcs]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"reference I/O build failed:\n{r.stderr[-6000:]}")
    return lib


DATA_SOURCES = [os.path.join(REFERENCE, "core", "src", *p) for p in (
    ("input_data.cpp",), ("loaders", "load_colmap.cpp"), ("loaders", "load_ply.cpp"),
    ("loaders", "load_nerfstudio.cpp"), ("loaders", "load_polycam.cpp"))]
IMAGE_IO = os.path.join(REFERENCE, "core", "src", "loaders", "image_io.cpp")
SSIM_CPP = os.path.join(REFERENCE, "core", "src", "ssim.cpp")


def nlohmann_include() -> str:
    """A directory holding nlohmann/json.hpp (the reference fetches it at
    configure time; an unmodified copy ships inside cudnn_frontend)."""
    import glob
    import site
    roots = site.getsitepackages() + [sys.prefix]
    for root in roots:
        for hit in glob.glob(os.path.join(root, "**", "nlohmann", "json.hpp"), recursive=True):
            return os.path.dirname(os.path.dirname(hit))
    raise FileNotFoundError("nlohmann/json.hpp not found")


def strip_function(src: str, signature: str) -> str:
    """Remove the definition that starts with `signature` (brace matched)."""
    i = src.find(signature)
    if i < 0:
        raise ValueError(f"{signature!r} not found")
    j = src.index("{", i)
    depth = 0
    for k in range(j, len(src)):
        depth += {"{": 1, "}": -1}.get(src[k], 0)
        if depth == 0:
            return src[:i] + src[k + 1:]
    raise ValueError("unbalanced braces")


def extract_function(src: str, signature: str) -> str:
    """The definition that starts with `signature` (brace matched)."""
    i = src.find(signature)
    if i < 0:
        raise ValueError(f"{signature!r} not found")
    j = src.index("{", i)
    depth = 0
    for k in range(j, len(src)):
        depth += {"{": 1, "}": -1}.get(src[k], 0)
        if depth == 0:
            return src[i:k + 1]
    raise ValueError("unbalanced braces")


MODEL_CPP = os.path.join(REFERENCE, "core", "src", "model.cpp")


def model_metrics_source() -> str:
    """psnr and l1_loss of model.cpp (the rest of that file needs the Metal
    runtime and nanoflann), taken verbatim."""
    src = open(MODEL_CPP).read()
    funcs = [extract_function(src, "float psnr(const MTensor& rendered, const MTensor& gt)"),
             extract_function(src, "float l1_loss(const MTensor& rendered, const MTensor& gt)")]
    return "#include <cmath>\n#include \"model.hpp\"\n\n" + "\n\n".join(funcs) + "\n"


def image_io_transform(src: str) -> str:
    """image_io.cpp without its CoreGraphics half: the two platform includes
    and the CoreGraphics decoder / encoder (imreadRGB, imwriteRGB) are
    dropped; resizeArea and undistortImage are kept as written."""
    src = "\n".join(line for line in src.split("\n")
                     if not re.match(r"\s*#include <(CoreGraphics|ImageIO)/", line))
    src = strip_function(src, "Image imreadRGB(const std::string &path)")
    return strip_function(src, "void imwriteRGB(const std::string &path, const Image &img)")


def build_data(verbose: bool = False) -> str:
    """oracle/_ref/libmsplat_ref_data.so: the reference's dataset loaders,
    pose normalisation, splits, Camera image pipeline, the resize /
    undistort code of image_io.cpp and the evaluation metrics (ssim.cpp,
    psnr / l1_loss of model.cpp); ref_data.cpp stands in for the
    CoreGraphics decoder and the Metal runtime calls."""
    for src in DATA_SOURCES + [IMAGE_IO, SSIM_CPP, MODEL_CPP]:
        if not os.path.exists(src):
            raise FileNotFoundError(f"reference source not found: {src}")
    os.makedirs(OUT, exist_ok=True)
    gens = []
    for name, code in (("image_io_ref.cpp", image_io_transform(open(IMAGE_IO).read())),
                       ("model_metrics_ref.cpp", model_metrics_source())):
        gen = os.path.join(OUT, name)
        if not os.path.exists(gen) or open(gen).read() != code:
            with open(gen, "w") as f:
                f.write(code)
        gens.append(gen)
    lib = os.path.join(OUT, "libmsplat_ref_data.so")
    srcs = [os.path.join(HERE, "ref_data.cpp")] + gens + DATA_SOURCES + [SSIM_CPP]
    if os.path.exists(lib) and all(os.path.getmtime(d) <= os.path.getmtime(lib) for d in srcs):
        return lib
    cmd = ["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
           "-Wno-return-type", f"-I{os.path.join(REFERENCE, 'core', 'include')}",
           # headers the sources reach transitively through libc++ on macOS
           "-include", "cmath", "-include", "stdexcept", "-include", "unordered_map",
           f"-I{os.path.join(REFERENCE, 'core', 'metal')}", f"-I{nlohmann_include()}", "-o", lib,
           *srcs]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"reference data build failed:\n{r.stderr[-6000:]}")
    return lib


TRAINER_SOURCES = [os.path.join(REFERENCE, "core", "src", *p) for p in (
    ("model.cpp",), ("ssim.cpp",), ("loaders", "save_gaussians.cpp"))] + DATA_SOURCES
API_SOURCE = os.path.join(REFERENCE, "core", "src", "msplat_api.mm")


def build_trainer(verbose: bool = False) -> str:
    """oracle/_ref/libmsplat_ref_trainer.so: the reference's Model
    (model.cpp), Trainer and C API (msplat_api.mm -- plain C++ despite its
    extension) and data front end, over ref_backend.cpp, which implements
    the backend seam (bindings.h) with the reference's kernels built through
    the MSL shim (libmsplat_ref.so, linked).  nanoflann is absent; the
    stand-in kdtree_tensor.hpp in stub_include/ searches exhaustively."""
    ref_lib = build(verbose)
    build_data(verbose)   # writes the generated image_io_ref.cpp
    for src in TRAINER_SOURCES + [API_SOURCE]:
        if not os.path.exists(src):
            raise FileNotFoundError(f"reference source not found: {src}")
    lib = os.path.join(OUT, "libmsplat_ref_trainer.so")
    gen = os.path.join(OUT, "image_io_ref.cpp")
    srcs = [os.path.join(HERE, "ref_backend.cpp"), gen] + TRAINER_SOURCES
    deps = srcs + [API_SOURCE, ref_lib, os.path.join(HERE, "stub_include", "kdtree_tensor.hpp")]
    if os.path.exists(lib) and all(os.path.getmtime(d) <= os.path.getmtime(lib) for d in deps):
        return lib
    cmd = ["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC",
           "-shared", "-Wno-return-type", "-Wno-unused-result",
           f"-I{os.path.join(HERE, 'stub_include')}",
           f"-I{os.path.join(REFERENCE, 'core', 'include')}",
           "-include", "cmath", "-include", "stdexcept", "-include", "unordered_map",
           "-include", "cstring", "-include", "algorithm",
           f"-I{os.path.join(REFERENCE, 'core', 'metal')}",
           f"-I{nlohmann_include()}", f"-I{ORACLE}", "-o", lib, *srcs,
           "-x", "c++", API_SOURCE, "-x", "none",
           f"-L{OUT}", "-lmsplat_ref", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"reference trainer build failed:\n{r.stderr[-6000:]}")
    return lib


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
    print(build_io(verbose="-v" in sys.argv))
    print(build_data(verbose="-v" in sys.argv))
    print(build_trainer(verbose="-v" in sys.argv))
