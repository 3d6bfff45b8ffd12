"""Failure detection of the TMA-staged kernels (GPU), without any fault.

Every kernel that stages its inputs by TMA waits on a per-stage completion
barrier with a bounded poll. When a wait runs out the CTA leaves as a whole
(the decision is a block-wide vote), after its thread 0 has waited, again
bounded, for the copies it still has in flight, and a device flag makes
mms_device_status() return MMS_ERR_TIMEOUT.

These tests make that happen the allowed way: the test hook
mms_debug_set_wait(polls, skip_item) lowers the poll limit and makes every CTA
withhold the copies of one staged item, so its wait can only run out. Each
case checks that the call returns promptly, that the status reports the
timeout, and that after the hook is reset the same call runs normally and
matches the float64 oracle (the context stayed usable).
"""
from __future__ import annotations

import time

import pytest
import torch

from _inputs import inputs, max_rel
from mamba_metal import _native
from oracle import oracle

pytestmark = pytest.mark.gpu

POLLS = 1 << 10


def _with_withheld_item(fn, skip_item):
    lib = _native.load()
    assert _native.device_status() == _native.MMS_OK
    assert lib.mms_debug_set_wait(POLLS, skip_item) == _native.MMS_OK
    try:
        t0 = time.perf_counter()
        fn()
        status = _native.device_status()          # synchronises
        elapsed = time.perf_counter() - t0
    finally:
        lib.mms_debug_set_wait(0, -1)
    return status, elapsed


# (B, T, D, N, K, withheld item): the channel-pair backward at strides 8
# and 16, one CTA each (64 channels of one row), and at d_state 32 (two CTAs
# of 32 channels)
BWD_CASES = [(1, 64, 64, 16, 8, 3), (1, 64, 64, 16, 16, 2), (1, 64, 64, 32, 8, 4)]


@pytest.mark.parametrize("bt,t_len,d,n,chunk,skip", BWD_CASES)
def test_backward_wait_that_runs_out_is_reported_and_leaves_the_context_usable(
        bt, t_len, d, n, chunk, skip):
    x, dt, aneg, b_in, c_in, dy = inputs(bt, t_len, d, n, "c0", seed=9, device="cuda")
    _, ckpt = _native.fwd(x, dt, aneg, b_in, c_in, chunk)
    torch.cuda.synchronize()
    status, elapsed = _with_withheld_item(
        lambda: _native.bwd(x, dt, aneg, b_in, c_in, dy, ckpt, chunk), skip)
    assert status == _native.MMS_ERR_TIMEOUT
    assert elapsed < 2.0, f"the timed-out call took {elapsed:.2f} s"
    grads = _native.bwd(x, dt, aneg, b_in, c_in, dy, ckpt, chunk)
    assert _native.device_status() == _native.MMS_OK
    g64 = oracle.scan_bwd(*(t.cpu().numpy() for t in (x, dt, aneg, b_in, c_in, dy)))
    for g, w in zip(grads, g64):
        assert max_rel(g, w) <= 1e-4


def test_forward_wait_that_runs_out_is_reported_and_leaves_the_context_usable():
    """The whole-state forward (TMA staging, bulk stores) on 148 CTAs of two
    16-step tiles each; every CTA withholds its second tile."""
    bt, t_len, d, n, chunk = 1, 32, 148 * 128, 16, 8
    x, dt, aneg, b_in, c_in, _ = inputs(bt, t_len, d, n, "c0", seed=11, device="cuda")
    status, elapsed = _with_withheld_item(lambda: _native.fwd(x, dt, aneg, b_in, c_in, chunk), 1)
    assert status == _native.MMS_ERR_TIMEOUT
    assert elapsed < 2.0, f"the timed-out call took {elapsed:.2f} s"
    y, _ = _native.fwd(x, dt, aneg, b_in, c_in, chunk)
    assert _native.device_status() == _native.MMS_OK
    y64, _ = oracle.scan_fwd(*(t.cpu().numpy() for t in (x, dt, aneg, b_in, c_in)), chunk=chunk)
    assert max_rel(y, y64) <= 1e-5


def test_the_hook_rejects_a_negative_item():
    assert _native.load().mms_debug_set_wait(0, -2) == _native.MMS_ERR_INVALID_ARG
