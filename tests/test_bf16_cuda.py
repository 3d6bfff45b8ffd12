"""Parity gates for bf16 storage (mms_fwd_bf16 / mms_bwd_bf16, selective_scan_bf16).

The reference is float32-only (mamba_metal/scan.py:350-354), so no reference
test pins bf16 results. Two checks stand in:

* against the float64 oracle run on the same bf16 values (x, dt and dy
  rounded to bf16, then widened): y, dx and ddt are stored as bf16, so their
  normalised error is bounded by bf16 rounding (2^-9 relative per element;
  tolerance BF16_TOL = 2^-8); dAneg, dB and dC are fp32 outputs of fp32
  arithmetic on those values and keep the fp32 scan's 1e-4;
* against the fp32 entry points on the widened inputs, where both run the
  same kernels (whole-state or G-lane forward, 8- or 4-state backward, time
  segments): every fp32
  output is bit-identical and every bf16 output equals the fp32 one rounded
  to nearest even. So the storage type changes the loads and the final
  rounding and nothing else.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _inputs import SEED, inputs, max_rel
from mamba_metal import _native, selective_scan, selective_scan_bf16
from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"
BF16_TOL = 2.0 ** -8
GRAD_TOL = 1e-4

# (Bt, T, D, N): whole-state forward with and without time segments, T not a
# multiple of the 8-step chunk or the 16-step tile, D not a multiple of the
# 128-channel CTA, d_state 12; the G-lane forward and 4-state backward at
# every other lane count (d_state 4, 8, 20, 32, 64), with time segments.
CASES = [
    (16, 64, 2304, 16),
    (2, 77, 40, 16),
    (3, 50, 24, 12),
    (1, 3000, 64, 16),
    (1, 9, 8, 16),
    (2, 33, 24, 4),
    (2, 77, 40, 8),
    (3, 40, 32, 20),
    (2, 100, 64, 32),
    (1, 50, 16, 64),
    (1, 2000, 32, 32),
]
# shapes where the fp32 entry points run the same kernels as the bf16 ones
SAME_PATH = [(16, 64, 2304, 16), (12, 40, 2048, 12), (1, 3000, 64, 16), (2, 100, 64, 32),
             (1, 64, 40, 8), (1, 2000, 32, 32)]


def _bf16_inputs(bt, t_len, d, n, seed):
    x, dt, aneg, b_in, c_in, dy = inputs(bt, t_len, d, n, dist="c0", seed=seed)
    xb, dtb, dyb = (t.to(torch.bfloat16) for t in (x, dt, dy))
    return xb, dtb, aneg, b_in, c_in, dyb


def _run_bf16(xb, dtb, aneg, b_in, c_in, dyb):
    leaves = [t.to(DEV).requires_grad_(True) for t in (xb, dtb, aneg, b_in, c_in)]
    y, h = selective_scan_bf16(*leaves, return_state=True)
    grads = torch.autograd.grad(y, leaves, grad_outputs=dyb.to(DEV))
    return y, h, grads


@pytest.mark.parametrize("bt,t_len,d,n", CASES)
def test_bf16_scan_matches_the_float64_oracle(bt, t_len, d, n):
    xb, dtb, aneg, b_in, c_in, dyb = _bf16_inputs(bt, t_len, d, n, SEED + 7 * d + t_len)
    y, h, grads = _run_bf16(xb, dtb, aneg, b_in, c_in, dyb)
    assert y.dtype == torch.bfloat16 and y.shape == (bt, t_len, d)
    assert grads[0].dtype == torch.bfloat16 and grads[1].dtype == torch.bfloat16
    assert all(g.dtype == torch.float32 for g in grads[2:])
    x64, dt64, a64, b64, c64, dy64 = (t.double().numpy() for t in (xb, dtb, aneg, b_in, c_in, dyb))
    y64, h64 = oracle.scan_fwd(x64, dt64, a64, b64, c64, chunk=8)
    assert max_rel(y, y64) <= BF16_TOL, max_rel(y, y64)
    assert max_rel(h, h64[:, -1]) <= GRAD_TOL, max_rel(h, h64[:, -1])
    want = oracle.scan_bwd(x64, dt64, a64, b64, c64, dy64)
    for name, g, w, tol in zip(("dx", "ddt", "dAneg", "dB", "dC"), grads, want,
                               (BF16_TOL, BF16_TOL, GRAD_TOL, GRAD_TOL, GRAD_TOL)):
        assert np.isfinite(g.float().cpu().numpy()).all(), name
        assert max_rel(g, w) <= tol, (name, max_rel(g, w))


@pytest.mark.parametrize("bt,t_len,d,n", SAME_PATH)
def test_bf16_storage_only_rounds_the_fp32_results(bt, t_len, d, n):
    xb, dtb, aneg, b_in, c_in, dyb = _bf16_inputs(bt, t_len, d, n, SEED + 11 * d + t_len)
    y, h, grads = _run_bf16(xb, dtb, aneg, b_in, c_in, dyb)
    leaves = [t.float().to(DEV).requires_grad_(True) for t in (xb, dtb, aneg, b_in, c_in)]
    y32, h32 = selective_scan(*leaves, impl="cuda", chunk=8, return_state=True)
    g32 = torch.autograd.grad(y32, leaves, grad_outputs=dyb.float().to(DEV))
    assert torch.equal(y, y32.to(torch.bfloat16))
    assert torch.equal(h, h32)
    assert torch.equal(grads[0], g32[0].to(torch.bfloat16))
    assert torch.equal(grads[1], g32[1].to(torch.bfloat16))
    for g, w in zip(grads[2:], g32[2:]):
        assert torch.equal(g, w)


def test_bf16_results_repeat_bit_for_bit():
    xb, dtb, aneg, b_in, c_in, dyb = _bf16_inputs(2, 200, 64, 16, SEED)
    first = _run_bf16(xb, dtb, aneg, b_in, c_in, dyb)
    second = _run_bf16(xb, dtb, aneg, b_in, c_in, dyb)
    assert torch.equal(first[0], second[0])
    for a, b in zip(first[2], second[2]):
        assert torch.equal(a, b)


def test_bf16_gradients_follow_the_input_dtypes():
    """bf16 Aneg, B, C are widened for the kernels; their gradients come back as bf16."""
    xb, dtb, aneg, b_in, c_in, dyb = _bf16_inputs(2, 40, 32, 16, SEED + 1)
    leaves = [t.to(DEV, torch.bfloat16).requires_grad_(True) for t in (xb, dtb, aneg, b_in, c_in)]
    y = selective_scan_bf16(*leaves)
    grads = torch.autograd.grad(y, leaves, grad_outputs=dyb.to(DEV))
    assert all(g.dtype == torch.bfloat16 for g in grads)


def test_bf16_shape_rules_raise_before_any_launch():
    xb, dtb, aneg, b_in, c_in, _ = _bf16_inputs(1, 16, 16, 6, SEED)
    args = [t.to(DEV) for t in (xb, dtb, aneg, b_in, c_in)]
    with pytest.raises(ValueError, match="d_state"):
        selective_scan_bf16(*args)
    xb, dtb, aneg, b_in, c_in, _ = _bf16_inputs(1, 16, 12, 16, SEED)
    args = [t.to(DEV) for t in (xb, dtb, aneg, b_in, c_in)]
    with pytest.raises(ValueError, match="% 8"):
        selective_scan_bf16(*args)
    xb, dtb, aneg, b_in, c_in, _ = _bf16_inputs(1, 16, 16, 16, SEED)
    args = [t.to(DEV) for t in (xb, dtb, aneg, b_in, c_in)]
    with pytest.raises(ValueError, match="stride 8"):
        selective_scan_bf16(*args, chunk=16)
    with pytest.raises(RuntimeError, match="bf16"):
        selective_scan_bf16(args[0].float(), *args[1:])
    # the C ABI answers the same shapes with its own status, before launching
    lib = _native.load()
    p = [t.data_ptr() for t in args] + [args[0].data_ptr(), args[2].data_ptr()]
    assert lib.mms_fwd_bf16(*p, 1, 16, 12, 16, 8, None) == _native.MMS_ERR_UNSUPPORTED_BF16
