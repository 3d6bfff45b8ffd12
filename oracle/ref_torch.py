"""The reference's CPU path, restated in PyTorch -- test/baseline infrastructure only.

This is the reference's `impl="torch"` scan (`selective_scan_ref`,
mamba_metal/scan.py:313-333 of Anamaya1729/mamba-metal-scan): a Python loop
over time of (B, D, N) tensor ops, differentiated by autograd. It is used as

  * the CPU baseline that bench.py times (`cpu_baseline`, kind "port", and the
    `--impl reference` arm), with as many intra-op threads as the host has;
  * a second, autograd-based checker in tests/ next to the C oracle.

It is pinned against the golden vectors that tests/golden/make_golden.py
produced by running the reference itself.
"""
from __future__ import annotations

import torch


def scan_ref(x, dt, aneg, b_in, c_in, return_state: bool = False):
    """y (B,T,D) [, h_last (B,D,N)] by the left-to-right recurrence (scan.py:321-333)."""
    bt, t_len, d = x.shape
    n = aneg.shape[1]
    state = x.new_zeros(bt, d, n)
    ys = []
    for t in range(t_len):
        step = dt[:, t, :].unsqueeze(-1)                                # (B,D,1)
        decay = torch.exp(-step * aneg.unsqueeze(0))                    # (B,D,N)
        inject = step * b_in[:, t, :].unsqueeze(1) * x[:, t, :].unsqueeze(-1)
        state = decay * state + inject
        ys.append((c_in[:, t, :].unsqueeze(1) * state).sum(-1))
    y = torch.stack(ys, dim=1)
    return (y, state) if return_state else y


def fwd_bwd(x, dt, aneg, b_in, c_in, dy):
    """One forward + autograd backward; returns (y, dx, ddt, dAneg, dB, dC)."""
    leaves = [t.detach().clone().requires_grad_(True) for t in (x, dt, aneg, b_in, c_in)]
    y = scan_ref(*leaves)
    grads = torch.autograd.grad(y, leaves, grad_outputs=dy)
    return (y.detach(),) + tuple(g.detach() for g in grads)
