"""Parity gates for the fused _proj prologue (mms_fwd_proj / mms_bwd_proj).

The model computes dt = dt_min + (dt_max - dt_min)*sigmoid(dt_proj(x)) and
Aneg = softplus(A) with PyTorch ops before the scan (reference
mamba_metal/model.py:191-201). selective_scan_proj computes both inside the
kernels. Arbiter: the float64 oracle on the float64 prologue, with the chain
rule applied in float64 for the logit and A gradients. Same normalised
tolerances as the scan: 1e-5 forward, 1e-4 gradients. The shapes cover every
kernel path the prologue runs through: the whole-state and G-lane forwards,
time segments (local pass + combine), the channel-pair backward (4, 8 and
16 lanes per pair), the cp.async 8-state backward (unaligned arrays at
stride 8) and the 4-state backwards at other d_state and strides.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _inputs import SEED, max_rel
from mamba_metal import selective_scan_proj
from mamba_metal.scan import proj_ref
from oracle import oracle

pytestmark = pytest.mark.gpu

FWD_TOL, GRAD_TOL = 1e-5, 1e-4
DT_MIN, DT_MAX = 0.001, 0.1
DEV = "cuda"

CASES = [
    (16, 64, 2304, 16, 8),     # whole-state forward, channel-pair backward
    (2, 100, 40, 16, 8),       # G-lane forward + time segments, channel-pair backward
    (2, 130, 33, 16, 8),       # D % 4 != 0: cp.async paths (8-state backward)
    (3, 64, 20, 12, 8),        # d_state 12
    (2, 77, 21, 32, 64),       # d_state 32, stride 64 (4-state backward, recompute)
    (2, 100, 64, 32, 8),       # d_state 32: channel-pair backward, 8 lanes per pair
    (1, 150, 48, 64, 16),      # d_state 64: channel-pair backward, 16 lanes per pair
    (1, 200, 40, 8, 7),        # d_state 8, stride 7
    (1, 3000, 64, 16, 8),      # long: many time segments
]


def _inputs(bt, t_len, d, n, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(bt, t_len, d, generator=g)
    logit = torch.randn(bt, t_len, d, generator=g)
    a = torch.arange(1, n + 1, dtype=torch.float32).repeat(d, 1) \
        * (1 + 0.1 * torch.rand(d, n, generator=g)) - 2.0
    b_in = torch.randn(bt, t_len, n, generator=g)
    c_in = torch.randn(bt, t_len, n, generator=g)
    dy = torch.randn(bt, t_len, d, generator=g)
    return x, logit, a, b_in, c_in, dy


def _oracle(x, logit, a, b_in, c_in, dy, chunk):
    x64, z, a64, b64, c64, dy64 = (t.double() for t in (x, logit, a, b_in, c_in, dy))
    sig = torch.sigmoid(z)
    dt = DT_MIN + (DT_MAX - DT_MIN) * sig
    aneg = torch.nn.functional.softplus(a64)
    y, _ = oracle.scan_fwd(x64.numpy(), dt.numpy(), aneg.numpy(), b64.numpy(), c64.numpy(),
                           chunk=chunk)
    dx, ddt, daneg, db, dc = oracle.scan_bwd(x64.numpy(), dt.numpy(), aneg.numpy(), b64.numpy(),
                                             c64.numpy(), dy64.numpy())
    dz = ddt * ((DT_MAX - DT_MIN) * sig * (1 - sig)).numpy()
    da = daneg * torch.sigmoid(a64).numpy()
    return y, (dx, dz, da, db, dc)


@pytest.mark.parametrize("bt,t_len,d,n,chunk", CASES)
def test_fused_prologue_matches_the_float64_oracle(bt, t_len, d, n, chunk):
    x, logit, a, b_in, c_in, dy = _inputs(bt, t_len, d, n, SEED + d + t_len)
    leaves = [t.to(DEV).requires_grad_(True) for t in (x, logit, a, b_in, c_in)]
    y = selective_scan_proj(*leaves, DT_MIN, DT_MAX, impl="cuda", chunk=chunk)
    grads = torch.autograd.grad(y, leaves, grad_outputs=dy.to(DEV))
    y64, g64 = _oracle(x, logit, a, b_in, c_in, dy, chunk)
    assert max_rel(y, y64) <= FWD_TOL, max_rel(y, y64)
    for name, g, w in zip(("dx", "dlogit", "dA", "dB", "dC"), grads, g64):
        assert max_rel(g, w) <= GRAD_TOL, (name, max_rel(g, w))


def test_fused_prologue_equals_the_unfused_composition():
    """Same scan, prologue in the kernels or as PyTorch ops before them."""
    x, logit, a, b_in, c_in, dy = (t.to(DEV) for t in _inputs(4, 96, 512, 16, 5))
    l1 = [t.clone().requires_grad_(True) for t in (x, logit, a, b_in, c_in)]
    y1, h1 = selective_scan_proj(*l1, DT_MIN, DT_MAX, impl="cuda", return_state=True)
    g1 = torch.autograd.grad(y1, l1, grad_outputs=dy)
    from mamba_metal import selective_scan
    l2 = [t.clone().requires_grad_(True) for t in (x, logit, a, b_in, c_in)]
    dt, aneg = proj_ref(l2[1], l2[2], DT_MIN, DT_MAX)
    y2, h2 = selective_scan(l2[0], dt, aneg, l2[3], l2[4], impl="cuda", return_state=True)
    g2 = torch.autograd.grad(y2, l2, grad_outputs=dy)
    assert max_rel(y1, y2) <= FWD_TOL and max_rel(h1, h2) <= FWD_TOL
    for a_, b_ in zip(g1, g2):
        assert max_rel(a_, b_) <= GRAD_TOL


def test_model_with_and_without_the_fused_prologue():
    from mamba_metal.model import MambaConfig, TinyMamba
    kw = dict(vocab_size=200, d_model=64, n_layers=2, d_ff=128, max_seq_len=64, d_state=16,
              d_conv=4, scan_impl="cuda")
    torch.manual_seed(SEED)
    m1 = TinyMamba(MambaConfig(**kw, fuse_proj=True)).to(DEV)
    m2 = TinyMamba(MambaConfig(**kw, fuse_proj=False)).to(DEV)
    m2.load_state_dict(m1.state_dict())
    idx = torch.randint(0, 200, (3, 40), generator=torch.Generator().manual_seed(1)).to(DEV)
    losses, grads = [], []
    for m in (m1, m2):
        _, loss = m(idx, idx)
        loss.backward()
        losses.append(loss.item())
        grads.append({k: p.grad.clone() for k, p in m.named_parameters()})
    assert abs(losses[0] - losses[1]) <= 1e-5 * abs(losses[1])
    for k in grads[0]:
        assert torch.allclose(grads[0][k], grads[1][k], atol=1e-5, rtol=1e-3), k


def test_fused_prologue_argument_errors():
    x, logit, a, b_in, c_in, _ = (t.to(DEV) for t in _inputs(1, 8, 8, 4, 0))
    with pytest.raises(ValueError, match="dt_min < dt_max"):
        selective_scan_proj(x, logit, a, b_in, c_in, 0.1, 0.1, impl="cuda")
    from mamba_metal import _native
    lib = _native.load()
    args = [None] * 5
    assert lib.mms_fwd_proj(*args, 0.2, 0.1, None, None, 1, 8, 8, 4, 8, None) \
        == _native.MMS_ERR_INVALID_ARG
