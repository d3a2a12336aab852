"""How a render's device error word becomes a status (msplat_b200/csrc/
errors.h, used by msplat_render_noalloc): every nonzero word is a failure,
an intersection overflow alone is MSPLAT_ERR_OVERFLOW and anything else --
a shared-memory copy that timed out, unknown bits -- MSPLAT_ERR_CUDA.
Compiled and run on the CPU (the header has no CUDA dependency)."""
from __future__ import annotations

import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#include <cstdio>
#include "errors.h"
int main() {
    const int words[] = {0, 1, 2, 3, 4, 5, 0x100, -1};
    for (int w : words) {
        const char* what = (const char*)1;
        int rc = msp::render_status(w, &what);
        std::printf("%d %d %d\n", w, rc, what ? 1 : 0);
    }
    return 0;
}
"""


def test_render_status_fails_on_every_nonzero_word(tmp_path):
    src = tmp_path / "status.cpp"
    src.write_text(PROGRAM)
    exe = str(tmp_path / "status")
    r = subprocess.run(["g++", "-std=c++17", "-I" + os.path.join(ROOT, "msplat_b200", "csrc"),
                        str(src), "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {int(a): (int(b), int(c)) for a, b, c in (ln.split() for ln in out if ln)}
    OK, CUDA, OVERFLOW = 0, -2, -3
    assert got[0] == (OK, 0)
    assert got[1] == (OVERFLOW, 1)          # overflow alone: retry smaller
    assert got[2] == (CUDA, 1)              # stage timeout: the image lost a block
    assert got[3] == (CUDA, 1)              # both
    for w in (4, 5, 0x100, -1):             # bits this build does not define
        assert got[w] == (CUDA, 1), w
