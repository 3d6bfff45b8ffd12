"""Parity at the exact shapes bench.py times (GPU, full size).

Every number bench.py reports comes from one of these kernel launches, so each
one is compared with the float64 C oracle at the north star's tolerances
(max|got - want| / max|want|: 1e-5 for y and the returned state, 1e-4 for
each of the five gradients):

  c1   B16 T512 D2304 N16 at checkpoint stride 8 (the headline) and at the
       reference's stride 64, and the second run with return_state=True
       (BASELINE config 1);
  c3b  B1 T16384 D2048 N64 (config 3 with d_state 64, one sequence per GPU);
  c4   B4 T4096 D8192 N16 on one GPU, and the per-GPU shards of its d_inner
       split over 2, 4 and 8 GPUs (D 4096, 2048, 1024), which are the kernel
       instances the multi-GPU bench runs;
  c1 with bf16 storage of the channel arrays (bench.py's `bf16` leg), against
       the oracle on the same bf16-rounded values (y, dx, ddt within the bf16
       rounding bound 2^-8, dAneg, dB, dC within 1e-4).

The launches go through the C ABI (mamba_metal._native, the calls bench.py
times); the return_state case goes through the public selective_scan API.
Inputs use the benchmark configs' distributions with fixed seeds.
"""
from __future__ import annotations

import functools

import numpy as np
import pytest
import torch

from _inputs import inputs, max_rel
from mamba_metal import _native, selective_scan
from oracle import oracle

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

FWD_TOL = 1e-5
GRAD_TOL = 1e-4
BF16_TOL = 2.0 ** -8
NAMES = ("dx", "ddt", "dAneg", "dB", "dC")


@functools.lru_cache(maxsize=2)
def _case(bt, t_len, d, n, seed):
    """Host inputs and the float64 oracle's y and five gradients."""
    ins = inputs(bt, t_len, d, n, "c0", seed=seed)
    cpu = [t.numpy() for t in ins]
    y64, _ = oracle.scan_fwd(*cpu[:5], chunk=max(t_len, 1))
    g64 = oracle.scan_bwd(*cpu)
    return ins, y64, g64


def _check(y, grads, y64, g64, label):
    e = max_rel(y, y64)
    assert e <= FWD_TOL, f"{label} y: {e:.3e}"
    for name, g, w in zip(NAMES, grads, g64):
        e = max_rel(g, w)
        assert e <= GRAD_TOL, f"{label} {name}: {e:.3e}"


def _run_abi(ins, chunk):
    x, dt, aneg, b_in, c_in, dy = (t.cuda() for t in ins)
    y, ckpt = _native.fwd(x, dt, aneg, b_in, c_in, chunk)
    grads = _native.bwd(x, dt, aneg, b_in, c_in, dy, ckpt, chunk)
    torch.cuda.synchronize()
    assert _native.device_status() == _native.MMS_OK
    return y, ckpt, grads


@pytest.mark.parametrize("chunk", [8, 64])
def test_config1_matches_the_float64_oracle(chunk):
    ins, y64, g64 = _case(16, 512, 2304, 16, 101)
    y, ckpt, grads = _run_abi(ins, chunk)
    _check(y, grads, y64, g64, f"c1 K{chunk}")


def test_config1_return_state_run_matches_the_float64_oracle():
    """BASELINE config 1's second run: return_state=True through the public API."""
    ins, y64, g64 = _case(16, 512, 2304, 16, 101)
    x, dt, aneg, b_in, c_in, dy = (t.cuda() for t in ins)
    leaves = [t.clone().requires_grad_(True) for t in (x, dt, aneg, b_in, c_in)]
    y, h = selective_scan(*leaves, impl="cuda", return_state=True)
    assert h.shape == (16, 2304, 16)
    grads = torch.autograd.grad(y, leaves, grad_outputs=dy)
    _check(y.detach(), grads, y64, g64, "c1 return_state")
    _, ck64 = oracle.scan_fwd(*(t.numpy() for t in ins[:5]), chunk=512)
    assert max_rel(h, ck64[:, -1]) <= FWD_TOL


def test_config3b_matches_the_float64_oracle():
    ins, y64, g64 = _case(1, 16384, 2048, 64, 303)
    y, ckpt, grads = _run_abi(ins, 8)
    _check(y, grads, y64, g64, "c3b")


@pytest.mark.parametrize("shards", [1, 2, 4, 8])
def test_config4_and_its_channel_shards_match_the_float64_oracle(shards):
    """Config 4 whole, and the first rank's d_inner shard of an N-GPU split
    (B and C replicated, so a shard's dB / dC are its partial sums over its
    channels: checked against the oracle run on the shard alone)."""
    from mamba_metal.sharded import channel_shard
    ins, y64, g64 = _case(4, 4096, 8192, 16, 404)
    if shards > 1:
        sl = channel_shard(8192, shards, 0)
        x, dt, aneg, b_in, c_in, dy = ins
        ins = (x[:, :, sl].contiguous(), dt[:, :, sl].contiguous(), aneg[sl].contiguous(),
               b_in, c_in, dy[:, :, sl].contiguous())
        y64 = y64[:, :, sl]
        g64 = (g64[0][:, :, sl], g64[1][:, :, sl], g64[2][sl]) + tuple(
            oracle.scan_bwd(*(t.numpy() for t in ins))[3:])
    y, ckpt, grads = _run_abi(ins, 8)
    _check(y, grads, y64, g64, f"c4 / {shards}")


def test_config1_bf16_storage_matches_the_float64_oracle():
    ins = inputs(16, 512, 2304, 16, "c0", seed=505)
    x, dt, aneg, b_in, c_in, dy = ins
    xb, dtb, dyb = (t.to(torch.bfloat16) for t in (x, dt, dy))
    cpu = [xb.double().numpy(), dtb.double().numpy(), aneg.numpy(), b_in.numpy(), c_in.numpy(),
           dyb.double().numpy()]
    y64, _ = oracle.scan_fwd(*cpu[:5], chunk=512)
    g64 = oracle.scan_bwd(*cpu)
    dev = [t.cuda() for t in (xb, dtb, aneg, b_in, c_in, dyb)]
    y, ckpt = _native.fwd_bf16(*dev[:5], 8)
    grads = _native.bwd_bf16(*dev, ckpt, 8)
    torch.cuda.synchronize()
    assert y.dtype == torch.bfloat16 and grads[0].dtype == torch.bfloat16
    assert max_rel(y, y64) <= BF16_TOL
    for name, g, w in zip(NAMES, grads, g64):
        tol = BF16_TOL if name in ("dx", "ddt") else GRAD_TOL
        e = max_rel(g, w)
        assert e <= tol, f"c1 bf16 {name}: {e:.3e}"
    assert np.isfinite(y.float().cpu().numpy()).all()
