"""mms_bwd_noalloc: the backward for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc at run time (a plugin inside a host
framework that reserved all GPU memory, or a path that cannot afford
cudaMalloc's implicit device synchronisation). mms_bwd_noalloc gives them the
backward with its scratch taken from a static device array compiled into the
library. This file calls it through the C ABI, on shapes that fill most of
that 16 MiB array, and checks two calls in a row:

  * against the float64 oracle, at the gradient tolerance of the other GPU
    tests (max|got - want| / max|want| <= 1e-4);
  * against mms_bwd (the entry point with a caller workspace) bit for bit:
    both run the same kernels with the same plan, and the results are
    deterministic, so a read of stale scratch would show in the low bits.

Before the checked calls, one call on a different shape leaves other data in
the shared array, so the checks see a scratch array whose every word the
backward must write before it reads it.

The file is named to be collected last: if it fails, a run that stops at the
first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from _inputs import inputs, max_rel
from mamba_metal import _native
from oracle import oracle

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-4            # the normalised tolerance of the other GPU gradient tests
SCRATCH = 16 << 20          # MMS_NOALLOC_SCRATCH_BYTES in include/mms_scan.h
NAMES = ("dx", "ddt", "dAneg", "dB", "dC")


def _grads(bt, t_len, d, n):
    return [torch.empty(bt, t_len, d, device="cuda"), torch.empty(bt, t_len, d, device="cuda"),
            torch.empty(d, n, device="cuda"), torch.empty(bt, t_len, n, device="cuda"),
            torch.empty(bt, t_len, n, device="cuda")]


def _noalloc(lib, shape, seed):
    """Inputs, forward and one mms_bwd_noalloc call on `shape`; returns all."""
    bt, t_len, d, n, chunk = shape
    x, dt, aneg, b_in, c_in, dy = inputs(bt, t_len, d, n, "c0", seed=seed, device="cuda")
    y, ckpt = _native.fwd(x, dt, aneg, b_in, c_in, chunk)
    ins = [t.data_ptr() for t in (x, dt, aneg, b_in, c_in, dy, ckpt)]
    got = _grads(bt, t_len, d, n)
    for t in got:
        t.fill_(float("nan"))              # every output must be written
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.mms_bwd_noalloc(*ins, *(t.data_ptr() for t in got), bt, t_len, d, n, chunk, stream)
    assert rc == 0, _native.status_string(rc)
    return (x, dt, aneg, b_in, c_in, dy, ckpt), ins, got


# (B, T, D, N, K) filling 97-100 % of the scratch; the stride picks the kernel:
# channel-pair (K = 8 and 64), general with segment-start states (K = 200)
SHAPES = [(12, 300, 2048, 16, 8), (15, 512, 1024, 16, 64), (12, 512, 1024, 16, 200)]
# a different shape run first, so the array holds another call's data
OTHER = {8: (3, 100, 512, 16, 8), 64: (2, 200, 768, 16, 64), 200: (3, 333, 256, 16, 200)}


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_noalloc_backward_matches_the_oracle_and_the_workspace_backward_twice(shape):
    lib = _native.load()
    bt, t_len, d, n, chunk = shape
    need = lib.mms_bwd_workspace_size(bt, t_len, d, n, chunk)
    assert SCRATCH // 2 < need <= SCRATCH
    _noalloc(lib, OTHER[chunk], seed=5)   # leaves other data in the shared scratch

    tensors, ins, got = _noalloc(lib, shape, seed=77 + chunk)
    torch.cuda.synchronize()
    g64 = oracle.scan_bwd(*(t.cpu().numpy() for t in tensors[:6]))

    want = _grads(bt, t_len, d, n)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.mms_bwd(*ins, *(t.data_ptr() for t in want), ws.data_ptr(), need,
                     bt, t_len, d, n, chunk, stream)
    assert rc == 0, _native.status_string(rc)

    for call in range(2):
        if call:
            _, _, got = _noalloc(lib, shape, seed=77 + chunk)
        torch.cuda.synchronize()
        assert _native.device_status() == _native.MMS_OK
        for name, g, w, o in zip(NAMES, got, want, g64):
            assert torch.equal(g, w), (call, name, "differs from mms_bwd")
            assert max_rel(g, o) <= GRAD_TOL, (call, name, max_rel(g, o))


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _native.load()
    bt, t_len, d, n, chunk = 16, 512, 2304, 16, 64
    assert lib.mms_bwd_workspace_size(bt, t_len, d, n, chunk) > SCRATCH
    x = torch.zeros(1, device="cuda")
    p = [ctypes.c_void_p(x.data_ptr())] * 12
    rc = lib.mms_bwd_noalloc(*p, bt, t_len, d, n, chunk, None)
    assert rc == _native.MMS_ERR_TOO_LARGE
    assert "16 MiB" in _native.status_string(rc)
