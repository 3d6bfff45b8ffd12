"""Fit of the FMA-pipe exp2 polynomial used by ex2_poly() in mms_common.cuh.

    python mamba-metal-scan_b200/csrc/exp2_fit.py

Method (Cody and Waite's argument reduction; a minimax fit computed here):
2^x = 2^j * 2^f with j = round(x) and f = x - j in [-1/2, 1/2]. 2^f is
approximated by p(f) = 1 + f*q(f), q of degree 4, so p(0) = 1 exactly and the
error vanishes at f = 0, where the scan's decays near 1 put most arguments.
q minimises the maximum relative error |p(f) - 2^f| / 2^f on [-1/2, 1/2]; it
is found by Lawson's iteratively reweighted least squares on a dense grid.
The coefficients are then rounded to float32 and the float32 Horner
evaluation is checked on a dense grid of float32 arguments.

Prints the five float32 coefficients (as C hex-float literals) and the
measured maximum relative error of the float32 evaluation.
"""
from __future__ import annotations

import numpy as np

DEG_Q = 4          # p has degree 5


def fit(n: int = 400_001, iters: int = 300) -> np.ndarray:
    f = np.linspace(-0.5, 0.5, n)
    f = f[f != 0.0]
    target = np.expm1(f * np.log(2.0)) / f          # q exact = (2^f - 1) / f
    w_rel = np.abs(f) / np.exp2(f)                  # p - 2^f = f (q - target); relative to 2^f
    V = np.vander(f, DEG_Q + 1, increasing=True)
    wt = np.full_like(f, 1.0 / f.size)
    c = None
    for _ in range(iters):
        W = np.sqrt(wt) * w_rel
        c, *_ = np.linalg.lstsq(V * W[:, None], target * W, rcond=None)
        err = np.abs((V @ c - target) * w_rel)
        wt = wt * err
        wt /= wt.sum()
    return c


def eval_f32(c32: np.ndarray, f: np.ndarray) -> np.ndarray:
    """p(f) by float32 Horner with fused multiply-adds (each step rounded once)."""
    f64 = f.astype(np.float64)
    p = np.float64(c32[-1])
    for k in range(len(c32) - 2, -1, -1):
        p = (p * f64 + np.float64(c32[k])).astype(np.float32).astype(np.float64)
    return (p * f64 + 1.0).astype(np.float32)


def main() -> None:
    c = fit()
    c32 = c.astype(np.float32)
    rng = np.random.default_rng(0)
    f = np.concatenate([np.linspace(-0.5, 0.5, 2_000_001),
                        rng.uniform(-0.5, 0.5, 2_000_000),
                        np.geomspace(1e-12, 0.5, 200_000), -np.geomspace(1e-12, 0.5, 200_000)])
    f = f.astype(np.float32)
    got = eval_f32(c32, f).astype(np.float64)
    want = np.exp2(f.astype(np.float64))
    rel = np.abs(got - want) / want
    for k, v in enumerate(c32, start=1):
        print(f"c{k} = {float(v).hex()}f  // {float(v):.9g}")
    print(f"max relative error of the float32 evaluation on [-1/2, 1/2]: {rel.max():.3e} "
          f"({rel.max() / 2.0**-23:.2f} ulp of 1)")


if __name__ == "__main__":
    main()
