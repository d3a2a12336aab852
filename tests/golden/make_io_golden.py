"""Generate the model-file fixtures in tests/golden/io/ with the reference's
own writers (core/src/loaders/save_gaussians.cpp compiled into
oracle/_ref/libmsplat_ref_io.so by oracle/ref_shim/build_ref.py).

For each case of tests/io_case.py: <case>.ply (step `step_of(case)` in its
header) and <case>.splat written by the reference from the seeded Gaussians,
which the tests regenerate from the case's seed.  Run from the repository
root:

    python tests/golden/make_io_golden.py
"""
from __future__ import annotations

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import files  # noqa: E402
from tests import io_case  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "io")


def step_of(name: str) -> int:
    return 1000 + 7 * sorted(io_case.CASES).index(name)


def main() -> None:
    os.makedirs(OUT, exist_ok=True)
    ref = files.RefIO()
    for name, (n, rb, seed, keep, scale, trans) in io_case.CASES.items():
        params = io_case.gaussians(n, rb, seed)
        ref.save_ply(os.path.join(OUT, f"{name}.ply"), step_of(name), params, keep, scale, trans)
        ref.save_splat(os.path.join(OUT, f"{name}.splat"), params, keep, scale, trans)
        print(name, n, "gaussians")


if __name__ == "__main__":
    main()
