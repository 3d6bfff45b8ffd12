"""Parity gates for the gate epilogue kernels (mms_gate_fwd / mms_gate_bwd).

out = (y + D_skip) * silu(z) is the Mamba block's epilogue (reference
mamba_metal/model.py:255-256, PyTorch ops there). The kernels are checked
against float64 PyTorch autograd of the same expression, including the
strided z the block passes (a half of in_proj's output), ragged channel
counts and empty inputs; and the model with the fused gate against the model
without it. Normalised tolerance 1e-5 forward, 1e-5 for dy and dz, 1e-4 for
the D_skip gradient (a sum over B*T terms).
"""
from __future__ import annotations

import pytest
import torch

from _inputs import SEED, max_rel
from mamba_metal import _native, gated_output
from mamba_metal.scan import gate_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(bt, t_len, d, seed, strided):
    g = torch.Generator().manual_seed(seed)
    y = torch.randn(bt, t_len, d, generator=g)
    zz = torch.randn(bt, t_len, 2 * d, generator=g) * 3
    z = zz[..., d:] if strided else zz[..., d:].contiguous()
    dskip = torch.randn(d, generator=g)
    dout = torch.randn(bt, t_len, d, generator=g)
    return y, z, dskip, dout


@pytest.mark.parametrize("bt,t_len,d,strided", [(16, 512, 2304, True), (2, 33, 40, False),
                                                (3, 17, 37, True), (1, 1, 1, False),
                                                (4, 300, 1432, True)])
def test_gate_matches_float64_autograd(bt, t_len, d, strided):
    y, z, dskip, dout = _case(bt, t_len, d, SEED + d, strided)
    leaves64 = [t.double().requires_grad_(True) for t in (y, z, dskip)]
    out64 = gate_ref(*leaves64)
    g64 = torch.autograd.grad(out64, leaves64, grad_outputs=dout.double())
    yd, zd, dd = y.to(DEV), z.to(DEV), dskip.to(DEV)
    if strided:            # keep the row stride on the device too
        zfull = torch.empty(bt, t_len, 2 * d, device=DEV)
        zfull[..., d:] = zd
        zd = zfull[..., d:]
    leaves = [t.requires_grad_(True) for t in (yd, zd, dd)]
    out = gated_output(*leaves)
    g = torch.autograd.grad(out, leaves, grad_outputs=dout.to(DEV))
    assert max_rel(out, out64) <= 1e-5
    for name, a, b, tol in zip(("dy", "dz", "dD"), g, g64, (1e-5, 1e-5, 1e-4)):
        assert max_rel(a, b) <= tol, (name, max_rel(a, b))


def test_gate_is_deterministic():
    y, z, dskip, dout = (t.to(DEV) for t in _case(8, 128, 512, 3, False))
    a = _native.gate_bwd(dout, y, z, dskip)
    b = _native.gate_bwd(dout, y, z, dskip)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_gate_empty_and_errors():
    y = torch.zeros(2, 0, 8, device=DEV)
    assert gated_output(y, y, torch.zeros(8, device=DEV)).shape == y.shape
    with pytest.raises(ValueError):
        gated_output(torch.zeros(2, 3, 8, device=DEV), torch.zeros(2, 3, 8, device=DEV),
                     torch.zeros(7, device=DEV))
    lib = _native.load()
    assert lib.mms_gate_fwd(None, None, 8, None, None, 1, 1, 8, None) == _native.MMS_ERR_INVALID_ARG


def test_model_with_and_without_the_fused_gate():
    from mamba_metal.model import MambaConfig, TinyMamba
    kw = dict(vocab_size=200, d_model=64, n_layers=2, d_ff=128, max_seq_len=64, d_state=16,
              d_conv=4, scan_impl="cuda")
    torch.manual_seed(SEED)
    m1 = TinyMamba(MambaConfig(**kw, fuse_gate=True)).to(DEV)
    m2 = TinyMamba(MambaConfig(**kw, fuse_gate=False)).to(DEV)
    m2.load_state_dict(m1.state_dict())
    idx = torch.randint(0, 200, (3, 40), generator=torch.Generator().manual_seed(2)).to(DEV)
    losses, grads = [], []
    for m in (m1, m2):
        _, loss = m(idx, idx)
        loss.backward()
        losses.append(loss.item())
        grads.append({k: p.grad.clone() for k, p in m.named_parameters()})
    assert abs(losses[0] - losses[1]) <= 1e-5 * abs(losses[1])
    for k in grads[0]:
        assert torch.allclose(grads[0][k], grads[1][k], atol=1e-5, rtol=1e-3), k
