"""The FMA-pipe exp2 polynomial (ex2_poly in csrc/mms_common.cuh).

The forward computes a share of its decays 2^x, x = -dt*Aneg*log2(e), with a
polynomial on the FMA pipe instead of MUFU ex2 (Cody and Waite's split
2^x = 2^j * 2^f, j = round(x), f in [-1/2, 1/2]; 2^f = 1 + f*q(f) with q a
degree-4 minimax fit computed by csrc/exp2_fit.py). These tests:

  * CPU: restate the fp32 evaluation step by step in numpy (every operation
    rounded to fp32 once, as the device's fma / add do) with the
    coefficients read from the header, and bound its error against float64
    exp2 over the argument range the scan produces, [-125, 0], plus a
    margin of positive arguments: relative error <= 2e-7 (1.7 ulp of 1);
  * GPU: the device's scalar and packed-pair paths (mms_probe_exp2) equal
    that restatement bit for bit, and MUFU ex2.approx meets the same bound
    (the two paths of the forward are interchangeable within it).
"""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest
import torch

HEADER = Path(__file__).resolve().parents[1] / "mamba-metal-scan_b200" / "csrc" / "mms_common.cuh"
REL_BOUND = 2e-7


def _coefficients():
    text = HEADER.read_text()
    c = {k: float.fromhex(v) for k, v in re.findall(r"EXP2_(C\d) = (0x[0-9a-fp.+-]+)f", text)}
    return [np.float32(c[f"C{k}"]) for k in range(1, 6)]


def poly_f32(x: np.ndarray) -> np.ndarray:
    """ex2_poly restated in float32, one rounding per operation."""
    f32 = np.float32
    c1, c2, c3, c4, c5 = _coefficients()
    x = np.clip(x.astype(f32), f32(-125.0), f32(125.0))
    rnd = f32(12582912.0)
    t = (x + rnd).astype(f32)
    j = (t - rnd).astype(f32)
    f = (x - j).astype(f32)

    def fma(a, b, c):
        # a*b + c rounded once to fp32: the product of two fp32 values is exact
        # in the 64-bit significand of long double, and the sum is rounded
        # there before the final rounding, far from fp32's rounding points
        ld = np.longdouble
        return (a.astype(ld) * b.astype(ld) + ld(c)).astype(f32)

    p = fma(np.full_like(f, c5), f, c4)
    p = fma(p, f, c3)
    p = fma(p, f, c2)
    p = fma(p, f, c1)
    p = fma(p, f, f32(1.0))
    bits = p.view(np.int32) + (t.view(np.int32) << 23)
    return bits.astype(np.int32).view(f32)


def _arguments():
    rng = np.random.default_rng(0)
    return np.concatenate([np.linspace(-125.0, 0.0, 2_000_001), rng.uniform(-125.0, 5.0, 1_000_000),
                           -np.geomspace(1e-9, 125.0, 200_000), np.arange(-125, 6, dtype=np.float64),
                           np.arange(-125, 6) + 0.5]).astype(np.float32)


def test_polynomial_is_within_its_bound_of_exp2():
    x = _arguments()
    got = poly_f32(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() <= REL_BOUND, rel.max()
    assert np.all(poly_f32(np.array([0.0], np.float32)) == 1.0)


def test_polynomial_saturates_outside_its_range():
    x = np.array([-200.0, -126.0, -125.0, 125.0, 130.0], np.float32)
    y = poly_f32(x)
    assert np.all(np.isfinite(y)) and np.all(y > 0)
    assert y[0] == y[1] == y[2] and y[3] == y[4]


@pytest.mark.gpu
def test_device_paths_match_the_restatement_and_the_bound():
    from mamba_metal import _native
    lib = _native.load()
    x = _arguments()
    xd = torch.from_numpy(x).cuda()
    want = np.exp2(x.astype(np.float64))
    ref = poly_f32(x)
    for kind in (0, 1, 2):
        y = torch.empty_like(xd)
        rc = lib.mms_probe_exp2(xd.data_ptr(), y.data_ptr(), xd.numel(), kind,
                                torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        got = y.cpu().numpy()
        if kind:
            assert np.array_equal(got.view(np.int32), ref.view(np.int32)), kind
        else:
            keep = x >= -126.0            # ex2.approx.ftz flushes results below 2^-126 to zero
            rel = np.abs(got[keep] - want[keep]) / want[keep]
            assert rel.max() <= REL_BOUND, rel.max()
