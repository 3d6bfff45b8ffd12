"""Host-side model logic on the CPU (no GPU needed).

Mirrors what the reference's model suite checks (Anamaya1729/mamba-metal-scan,
tests/test_model.py:39-146) against this package's own restatement of the
model: the log-depth scan equals the plain recurrence (also chunked and at
lengths that are not powers of two), the block fits the transformer's
parameter budget, logits are causal, and the recurrent cache reproduces the
full-context rerun. The decode step's PyTorch form is checked against the
forward scan's returned state.
"""
from __future__ import annotations

import pytest
import torch

from _inputs import SEED, inputs, max_rel
from mamba_metal import selective_scan, selective_scan_step, selective_scan_step_ref
from mamba_metal.model import (MambaConfig, TinyMamba, d_inner_for_budget, mamba_block_params,
                               parallel_scan, scan_recurrence, transformer_block_params)

VOCAB = 200


def small_cfg(**over):
    kw = dict(vocab_size=VOCAB, d_model=64, n_layers=2, d_ff=128, max_seq_len=64,
              d_state=8, d_conv=4, scan_chunk=0)
    kw.update(over)
    return MambaConfig(**kw)


def tokens(batch=4, seq=32, seed=SEED):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, VOCAB, (batch, seq), generator=g)


def _ab(bt, t_len, d, n, seed=SEED):
    g = torch.Generator().manual_seed(seed)
    a = torch.rand(bt, t_len, d, n, generator=g) * 0.5 + 0.5
    b = torch.randn(bt, t_len, d, n, generator=g)
    return a, b


@pytest.mark.parametrize("t_len", [1, 2, 7, 32, 33, 100])
def test_parallel_scan_equals_the_recurrence(t_len):
    a, b = _ab(2, t_len, 6, 4)
    want = scan_recurrence(a, b)
    assert torch.allclose(parallel_scan(a, b), want, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("chunk", [1, 5, 16, 64])
def test_chunked_parallel_scan_carries_the_state(chunk):
    a, b = _ab(2, 53, 5, 4, seed=3)
    assert torch.allclose(parallel_scan(a, b, chunk=chunk), scan_recurrence(a, b),
                          atol=1e-5, rtol=1e-5)


def test_block_fits_the_transformer_parameter_budget():
    for d_model, d_ff, n in ((384, 1536, 16), (640, 2560, 16), (64, 128, 8)):
        budget = transformer_block_params(d_model, d_ff)
        d_inner = d_inner_for_budget(budget, d_model, n, 4)
        assert d_inner % 8 == 0
        assert mamba_block_params(d_model, d_inner, n, 4) <= budget
        if d_inner > 8:
            assert mamba_block_params(d_model, d_inner + 8, n, 4) > budget
    # config 2's scan shape: d_model 640, d_ff 2560 -> d_inner 1432
    assert d_inner_for_budget(transformer_block_params(640, 2560), 640, 16, 4) == 1432
    model = TinyMamba(small_cfg())
    per_block = mamba_block_params(64, model.d_inner, 8, 4)
    assert sum(p.numel() for p in model.blocks[0].parameters()) == per_block


def test_shapes_dtypes_and_loss():
    model = TinyMamba(small_cfg(scan_impl="torch"))
    idx = tokens(3, 20)
    logits, loss = model(idx, idx)
    assert logits.shape == (3, 20, VOCAB) and logits.dtype == torch.float32
    assert loss.ndim == 0 and torch.isfinite(loss)


@pytest.mark.parametrize("impl", ["torch", "auto"])
def test_future_tokens_do_not_change_past_logits(impl):
    torch.manual_seed(SEED)
    model = TinyMamba(small_cfg(scan_impl=impl)).eval()
    idx = tokens(2, 24)
    other = idx.clone()
    other[:, 12:] = (other[:, 12:] + 7) % VOCAB
    with torch.no_grad():
        a, _ = model(idx)
        b, _ = model(other)
    assert torch.allclose(a[:, :12], b[:, :12], atol=1e-6)
    assert not torch.allclose(a[:, 12:], b[:, 12:])


@pytest.mark.parametrize("impl", ["torch", "auto"])
def test_recurrent_cache_matches_full_recomputation(impl):
    torch.manual_seed(SEED)
    model = TinyMamba(small_cfg(scan_impl=impl, scan_chunk=8)).eval()
    full = tokens(4, 26)
    x, nxt = full[:, :20], full[:, 20:]
    with torch.no_grad():
        cache: dict = {}
        model(x, cache=cache)
        cached = [model(nxt[:, t:t + 1], cache=cache)[0][:, -1] for t in range(nxt.shape[1])]
        naive = [model(torch.cat([x, nxt[:, :t + 1]], dim=1))[0][:, -1]
                 for t in range(nxt.shape[1])]
    for a, b in zip(cached, naive):
        assert torch.allclose(a, b, atol=1e-5)


def test_decode_step_continues_the_scan():
    """h and y of selective_scan_step after a prefix equal the scan over prefix + 1 step."""
    x, dt, aneg, b_in, c_in, _ = inputs(3, 17, 10, 8, dist="c0", seed=11, dtype=torch.float64)
    y_full, h_full = selective_scan(x, dt, aneg, b_in, c_in, impl="torch", return_state=True)
    _, h = selective_scan(x[:, :-1], dt[:, :-1], aneg, b_in[:, :-1], c_in[:, :-1],
                          impl="torch", return_state=True)
    h = h.clone()
    y = selective_scan_step(x[:, -1], dt[:, -1], aneg, b_in[:, -1], c_in[:, -1], h, impl="torch")
    assert max_rel(y, y_full[:, -1]) < 1e-13 and max_rel(h, h_full) < 1e-13
    y2, h2 = selective_scan_step_ref(x[:, -1], dt[:, -1], aneg, b_in[:, -1], c_in[:, -1],
                                     torch.zeros_like(h))
    assert h2.shape == h.shape and y2.shape == y.shape


def test_decode_step_dispatch_off_cuda():
    x, dt, aneg, b_in, c_in, _ = inputs(2, 1, 8, 4)
    h = torch.zeros(2, 8, 4)
    args = (x[:, 0], dt[:, 0], aneg, b_in[:, 0], c_in[:, 0], h)
    assert selective_scan_step(*args, impl="auto") is None
    for impl in ("cuda", "metal"):
        with pytest.raises(RuntimeError, match="CUDA"):
            selective_scan_step(*args, impl=impl)
    with pytest.raises(ValueError, match="scan_impl"):
        selective_scan_step(*args, impl="nope")
