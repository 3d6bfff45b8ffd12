"""Parity gates for the decode step kernel (mms_step) on the GPU.

The step is h = exp(-dt*Aneg)*h + dt*B*x, y = sum_n C*h on a cached state, in
place (the reference runs it as PyTorch ops, mamba_metal/model.py:228-241).
It is checked (1) against the float64 step on random states, (2) over 128
consecutive steps from a return_state cache at batch 256, d_inner 2304,
d_state 16 against the full-context rerun of the forward scan, and (3) in the
model, where the recurrent cache must reproduce the full rerun's logits.
Tolerances as for the forward scan: max|got - want| / max|want| <= 1e-5.
"""
from __future__ import annotations

import pytest
import torch

from _inputs import SEED, inputs, max_rel
from mamba_metal import _native, selective_scan, selective_scan_step, selective_scan_step_ref
from oracle import oracle

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-5
DEV = "cuda"


@pytest.mark.parametrize("bt,d,n", [(1, 1, 4), (3, 37, 8), (5, 100, 12), (4, 64, 16),
                                    (2, 33, 20), (2, 70, 32), (3, 17, 64), (256, 2304, 16)])
def test_step_matches_the_float64_step(bt, d, n):
    x, dt, aneg, b_in, c_in, _ = inputs(bt, 1, d, n, dist="c0", seed=SEED + n + d)
    h0 = torch.randn(bt, d, n, generator=torch.Generator().manual_seed(5))
    y64, h64 = selective_scan_step_ref(*(t.double() for t in (x[:, 0], dt[:, 0], aneg,
                                                             b_in[:, 0], c_in[:, 0], h0)))
    h = h0.to(DEV)
    y = selective_scan_step(x[:, 0].to(DEV), dt[:, 0].to(DEV), aneg.to(DEV),
                            b_in[:, 0].to(DEV), c_in[:, 0].to(DEV), h)
    torch.cuda.synchronize()
    assert y.shape == (bt, d)
    assert max_rel(y, y64) <= FWD_TOL, max_rel(y, y64)
    assert max_rel(h, h64) <= FWD_TOL, max_rel(h, h64)


def test_128_decode_steps_match_the_full_context_rerun():
    """Config-4 decode case: B=256, d_inner=2304, d_state=16, 128 steps from a cache."""
    bt, d, n, prefix, steps = 256, 2304, 16, 16, 128
    x, dt, aneg, b_in, c_in, _ = inputs(bt, prefix + steps, d, n, dist="c0", seed=99,
                                        device=DEV)
    y_full, h_full = selective_scan(x, dt, aneg, b_in, c_in, impl="cuda", return_state=True)
    _, h = selective_scan(x[:, :prefix], dt[:, :prefix], aneg, b_in[:, :prefix],
                          c_in[:, :prefix], impl="cuda", return_state=True)
    h = h.contiguous().clone()
    ys = []
    for t in range(prefix, prefix + steps):
        ys.append(selective_scan_step(x[:, t].contiguous(), dt[:, t].contiguous(), aneg,
                                      b_in[:, t].contiguous(), c_in[:, t].contiguous(), h))
    y_dec = torch.stack(ys, dim=1)
    assert max_rel(y_dec, y_full[:, prefix:]) <= FWD_TOL
    assert max_rel(h, h_full) <= FWD_TOL
    # and against the float64 oracle on a slice of the batch
    sl = slice(0, 4)
    y64, ck64 = oracle.scan_fwd(*(t[sl].cpu().numpy() for t in (x, dt)), aneg.cpu().numpy(),
                                *(t[sl].cpu().numpy() for t in (b_in, c_in)), chunk=8)
    assert max_rel(y_dec[sl], y64[:, prefix:]) <= FWD_TOL
    assert max_rel(h[sl], ck64[:, -1]) <= FWD_TOL


def test_step_is_deterministic_and_in_place():
    x, dt, aneg, b_in, c_in, _ = inputs(8, 1, 300, 16, dist="c0", seed=3, device=DEV)
    h1 = torch.randn(8, 300, 16, device=DEV)
    h2 = h1.clone()
    ptr = h1.data_ptr()
    args = (x[:, 0], dt[:, 0], aneg, b_in[:, 0], c_in[:, 0])
    ya = selective_scan_step(*args, h1)
    yb = selective_scan_step(*args, h2)
    assert h1.data_ptr() == ptr
    assert torch.equal(ya, yb) and torch.equal(h1, h2)


def test_step_argument_errors():
    x, dt, aneg, b_in, c_in, _ = inputs(2, 1, 8, 4, device=DEV)
    args = (x[:, 0], dt[:, 0], aneg, b_in[:, 0], c_in[:, 0])
    with pytest.raises(ValueError, match="state h"):
        selective_scan_step(*args, torch.zeros(2, 8, 4, device=DEV, dtype=torch.float64))
    with pytest.raises(ValueError, match="contiguous"):
        selective_scan_step(*args, torch.zeros(2, 4, 8, device=DEV).transpose(1, 2))
    with pytest.raises(ValueError, match="d_state"):
        selective_scan_step(x[:, 0], dt[:, 0], torch.ones(8, 6, device=DEV),
                            torch.ones(2, 6, device=DEV), torch.ones(2, 6, device=DEV),
                            torch.zeros(2, 8, 6, device=DEV))
    with pytest.raises(RuntimeError, match="CUDA"):
        selective_scan_step(*(t.cpu() for t in args), torch.zeros(2, 8, 4), impl="cuda")
    lib = _native.load()
    assert lib.mms_step(None, None, None, None, None, None, None, 2, 8, 4, None) \
        == _native.MMS_ERR_INVALID_ARG


def test_model_cache_uses_the_step_kernel():
    from mamba_metal.model import MambaConfig, TinyMamba
    cfg = MambaConfig(vocab_size=200, d_model=64, n_layers=2, d_ff=128, max_seq_len=64,
                      d_state=16, d_conv=4, scan_chunk=8, scan_impl="auto")
    torch.manual_seed(SEED)
    model = TinyMamba(cfg).to(DEV).eval()
    g = torch.Generator().manual_seed(SEED)
    full = torch.randint(0, 200, (4, 30), generator=g).to(DEV)
    with torch.no_grad():
        cache: dict = {}
        model(full[:, :22], cache=cache)
        calls = []
        orig = _native.step

        def spy(*a):
            calls.append(1)
            return orig(*a)

        _native.step = spy
        try:
            cached = [model(full[:, t:t + 1], cache=cache)[0][:, -1] for t in range(22, 30)]
        finally:
            _native.step = orig
        naive = [model(full[:, :t + 1])[0][:, -1] for t in range(22, 30)]
    assert len(calls) == 8 * cfg.n_layers
    for a, b in zip(cached, naive):
        assert torch.allclose(a, b, atol=1e-5)
