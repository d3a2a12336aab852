"""Derivation of the exp() polynomial shared by the CUDA engine
(msplat_b200/csrc/msp_math.cuh), the CPU oracle (oracle/msplat_oracle.c) and
the reference shim (oracle/ref_shim/msl_runtime.cpp).

e^r on |r| <= ln2/2 (plus a margin for the rounding of k) is written as
1 + r + r^2 q(r) with q of degree 4; q's five coefficients are the discrete
Chebyshev (minimax) fit of the relative error, posed as a linear programme
over 8,000 Chebyshev-distributed points and solved with HiGHS, then rounded
to float32.  Run it to print the coefficients the three sources hold:

    python oracle/derive_exp_coefficients.py

With float32 Horner evaluation and the Cody & Waite reduction the resulting
expf is within 0.90 ulp of exp() over every float input (checked
exhaustively against double exp; tests/test_oracle.py samples it).
"""
from __future__ import annotations

import numpy as np


def fit(half_width: float = 0.3466 + 2e-5, points: int = 8001) -> np.ndarray:
    from scipy.optimize import linprog

    r = np.cos(np.linspace(0.0, np.pi, points)) * half_width
    r = r[np.abs(r) > 1e-6]
    f = np.exp(r)
    taylor = np.array([1 / 2, 1 / 6, 1 / 24, 1 / 120, 1 / 720])
    basis = np.stack([r ** k for k in range(2, 7)], 1)
    resid = f - 1.0 - r - basis @ taylor      # fit the correction to Taylor
    w = 1.0 / f                               # relative error
    scale = 1e9                               # keep the LP well inside HiGHS tolerances
    n = basis.shape[1]
    a_ub = np.vstack([np.hstack([scale * w[:, None] * basis, -np.ones((len(r), 1))]),
                      np.hstack([-scale * w[:, None] * basis, -np.ones((len(r), 1))])])
    b_ub = np.concatenate([scale * w * resid, -scale * w * resid])
    res = linprog(np.r_[np.zeros(n), 1.0], A_ub=a_ub, b_ub=b_ub,
                  bounds=[(None, None)] * (n + 1), method="highs",
                  options=dict(primal_feasibility_tolerance=1e-10,
                               dual_feasibility_tolerance=1e-10))
    if not res.success:
        raise RuntimeError(res.message)
    return taylor + res.x[:n]


if __name__ == "__main__":
    for k, c in zip(range(2, 7), fit()):
        c32 = float(np.float32(c))
        print(f"c{k} = {c32!r:<24} ({c32.hex()})")
