"""Generate the float32 coefficients of exp_c's 2^f polynomial (spec_accept.cu).

exp_c(x) = 2^n * P(f) with n = rint(x * log2 e) and f in [-1/2, 1/2].  P is
the degree-5 polynomial P(f) = 1 + c1 f + ... + c5 f^5 (P(0) = 1 exactly, so
exp_c(0) = 1) that minimises the largest relative error |P(f) / 2^f - 1|
over a uniform grid of 20,001 points of [-1/2, 1/2].

Method: discrete Chebyshev (minimax) approximation solved as a linear
program (Stiefel, "Note on Jordan elimination, linear programming and
Tchebycheff approximation", Numer. Math. 2, 1960): minimise t subject to
-t <= r_i(c) <= t at every grid point, where r_i is linear in the unknown
coefficients c1..c5.  scipy's HiGHS solver finds the optimum; each
coefficient is then rounded to the nearest float32.  The result (printed as
C hex literals) is what spec_accept.cu's kExpCoef and the CPU restatement of
the acceptance kernel hold; a test re-runs this script and compares.

    python learn-nano-vllm_b200/csrc/gen_exp2_coef.py
"""
import numpy as np
from scipy.optimize import linprog

DEGREE = 5
GRID_POINTS = 20001


def fit(degree=DEGREE, points=GRID_POINTS):
    """Minimax relative-error coefficients [1, c1, ..., c_degree] in float64,
    and the optimal relative error on the grid."""
    f = np.linspace(-0.5, 0.5, points)
    inv = 1.0 / np.exp2(f)
    # relative error r(f) = (1 + sum_k c_k f^k) / 2^f - 1 = V c + b
    V = np.stack([f ** k for k in range(1, degree + 1)], axis=1) * inv[:, None]
    b = inv - 1.0
    ones = np.ones((points, 1))
    A = np.vstack([np.hstack([V, -ones]), np.hstack([-V, -ones])])
    rhs = np.concatenate([-b, b])
    cost = np.zeros(degree + 1)
    cost[-1] = 1.0
    res = linprog(cost, A_ub=A, b_ub=rhs, bounds=[(None, None)] * (degree + 1), method="highs")
    if not res.success:
        raise RuntimeError(f"linear program failed: {res.message}")
    return np.concatenate([[1.0], res.x[:degree]]), float(res.x[degree])


def coefficients_f32():
    """The coefficients rounded to float32."""
    c, _ = fit()
    return [np.float32(x) for x in c]


def hex_literals():
    """C hex literals of the float32 coefficients, trailing zero digits dropped."""
    out = []
    for x in coefficients_f32():
        mant, exp = float(x).hex().split("p")
        head, frac = mant.split(".")
        out.append(f"{head}.{frac.rstrip('0') or '0'}p{exp}")
    return out


if __name__ == "__main__":
    c, t = fit()
    print(f"minimax relative error on the grid (float64 coefficients): {t:.3e}")
    print(", ".join(h + "f" for h in hex_literals()))
