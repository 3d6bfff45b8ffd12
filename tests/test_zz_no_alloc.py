"""mms_bwd_noalloc: the backward for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc at run time (a plugin inside a host
framework that reserved all GPU memory, or a path that cannot afford
cudaMalloc's implicit device synchronisation). mms_bwd_noalloc gives them the
backward with its scratch taken from a static device array compiled into the
library. This file calls it through the C ABI and checks it against mms_bwd
(the entry point with a caller workspace) on two calls in a row, because the
second call finds the first call's leftovers in the shared scratch array.

The file is named to be collected last: if it fails, a run that stops at the
first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from _inputs import inputs, max_rel
from mamba_metal import _native

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-4            # the normalised tolerance of the other GPU gradient tests
SCRATCH = 16 << 20          # MMS_NOALLOC_SCRATCH_BYTES in include/mms_scan.h


def _grads(bt, t_len, d, n):
    return [torch.empty(bt, t_len, d, device="cuda"), torch.empty(bt, t_len, d, device="cuda"),
            torch.empty(d, n, device="cuda"), torch.empty(bt, t_len, n, device="cuda"),
            torch.empty(bt, t_len, n, device="cuda")]


@pytest.mark.parametrize("chunk", [8, 64, 200])
def test_noalloc_backward_matches_the_workspace_backward_twice(chunk):
    lib = _native.load()
    bt, t_len, d, n = 3, 300, 200, 16
    x, dt, aneg, b_in, c_in, dy = inputs(bt, t_len, d, n, "c0", seed=77 + chunk, device="cuda")
    y, ckpt = _native.fwd(x, dt, aneg, b_in, c_in, chunk)
    need = lib.mms_bwd_workspace_size(bt, t_len, d, n, chunk)
    assert 0 < need <= SCRATCH
    stream = torch.cuda.current_stream().cuda_stream
    P = lambda t: t.data_ptr()  # noqa: E731
    ins = [P(t) for t in (x, dt, aneg, b_in, c_in, dy, ckpt)]

    want = _grads(bt, t_len, d, n)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    rc = lib.mms_bwd(*ins, *(P(t) for t in want), P(ws), need, bt, t_len, d, n, chunk, stream)
    assert rc == 0, _native.status_string(rc)

    for call in range(2):
        got = _grads(bt, t_len, d, n)
        for t in got:
            t.fill_(float("nan"))          # every output must be written
        rc = lib.mms_bwd_noalloc(*ins, *(P(t) for t in got), bt, t_len, d, n, chunk, stream)
        assert rc == 0, _native.status_string(rc)
        torch.cuda.synchronize()
        for name, g, w in zip(("dx", "ddt", "dAneg", "dB", "dC"), got, want):
            assert torch.isfinite(g).all(), (call, name)
            assert max_rel(g, w) <= GRAD_TOL, (call, name, max_rel(g, w))


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _native.load()
    bt, t_len, d, n, chunk = 16, 512, 2304, 16, 64
    assert lib.mms_bwd_workspace_size(bt, t_len, d, n, chunk) > SCRATCH
    x = torch.zeros(1, device="cuda")
    p = [ctypes.c_void_p(x.data_ptr())] * 12
    rc = lib.mms_bwd_noalloc(*p, bt, t_len, d, n, chunk, None)
    assert rc == _native.MMS_ERR_TOO_LARGE
    assert "16 MiB" in _native.status_string(rc)
