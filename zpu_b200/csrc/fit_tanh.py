"""Derives the f32 coefficients of the fused kernels' tanh (region.cuh).

The method (written for this library): a minimax polynomial by
Lawson-weighted least squares on a dense point set, minimising the RELATIVE
error of tanh, with every coefficient rounded to f32 before the error is
measured:

    |x| < 0.9:  tanh(x) = x + x z P(z), z = x^2, P of degree 5.

(Above 0.9 the kernels use tanh(x) = 1 - 2 / (1 + e^(2x)) with the SFU's
ex2 / rcp, which needs no coefficients.)

    python zpu_b200/csrc/fit_tanh.py   # prints the coefficients and the error

Run offline; the kernels carry the printed constants.
"""
import numpy as np


def lawson(A, target, weight, iters=400):
    """min_c max_i weight_i |A_i c - target_i| with f32-rounded c."""
    wt = np.ones(len(target))
    best = None
    for _ in range(iters):
        s = (wt * weight)[:, None]
        c, *_ = np.linalg.lstsq(A * s, target * s[:, 0], rcond=None)
        c32 = c.astype(np.float32).astype(np.float64)
        err = np.abs(A @ c32 - target) * weight
        m = err.max()
        if best is None or m < best[0]:
            best = (m, c32)
        wt *= (err / m + 1e-3) ** 0.5
        wt /= wt.mean()
    return best


def tanh_small(split=0.9, deg=5):
    x = np.unique(np.concatenate([np.linspace(1e-4, split, 20000),
                                  split / 2 * (1 - np.cos(np.linspace(0, np.pi, 20000)))]))
    x = x[x > 0]
    z = x * x
    f = np.tanh(x)
    # tanh = x + x z P(z): fit P to (f - x)/(x z), weighted to the relative error of f
    A = z[:, None] ** np.arange(deg + 1)
    m, c = lawson(A, (f - x) / (x * z), x * z / f)
    return m / 2.0 ** -24, c


if __name__ == "__main__":
    e, c = tanh_small()
    print("tanh, |x| < 0.9, degree 5 in z: max rel err %.3f ulp" % e)
    print("  " + ", ".join("%.9ef" % v for v in c))
