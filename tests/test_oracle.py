"""Pin the oracle before trusting it (CPU).

The C oracle (oracle/scan_oracle.c) and the PyTorch port of the reference's
CPU path (oracle/ref_torch.py) are checked against the golden vectors that
tests/golden/make_golden.py recorded by running the reference's own
`selective_scan_ref` forward + autograd backward (float32 and float64), and
against an independent numpy recurrence. A planted mistake shows that the
comparisons can fail.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from _inputs import inputs, max_rel
from oracle import oracle, ref_torch

GOLDEN = sorted((Path(__file__).resolve().parent / "golden").glob("*.npz"))
OUT = ("y", "h_last", "dx", "ddt", "daneg", "db", "dc")


def _load(path):
    z = np.load(path)
    ins = tuple(z[k] for k in ("x", "dt", "aneg", "b", "c", "dy"))
    return z, ins


def _oracle_all(ins, dtype, chunk=64):
    y, ckpt = oracle.scan_fwd(*ins[:5], chunk=chunk, dtype=dtype)
    grads = oracle.scan_bwd(*ins, dtype=dtype)
    return [y, ckpt[:, -1]] + list(grads)


def test_golden_set_is_present():
    names = {p.stem for p in GOLDEN}
    assert "c0_2x256x64x16" in names and len(names) >= 10


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
def test_c_oracle_float64_matches_the_reference_float64(path):
    z, ins = _load(path)
    for name, got in zip(OUT, _oracle_all(ins, np.float64)):
        e = max_rel(got, z[f"{name}_f64"])
        assert e < 1e-11, f"{path.stem} {name}: {e:.3e}"


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
def test_c_oracle_float32_matches_the_reference_float32(path):
    z, ins = _load(path)
    for name, got in zip(OUT, _oracle_all(ins, np.float32)):
        e = max_rel(got, z[f"{name}_f32"])
        assert e < 2e-6, f"{path.stem} {name}: {e:.3e}"


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
def test_reference_float32_is_within_the_north_star_tolerance_of_float64(path):
    """The tolerance the CUDA kernels are held to is met by the reference's own fp32 path."""
    z, _ = _load(path)
    for name in OUT:
        tol = 1e-5 if name in ("y", "h_last") else 1e-4
        assert max_rel(z[f"{name}_f32"], z[f"{name}_f64"]) < tol, name


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
def test_torch_port_matches_the_reference(path):
    z, ins = _load(path)
    t = [torch.from_numpy(a) for a in ins]
    torch.set_num_threads(1)
    y, state = ref_torch.scan_ref(*t[:5], return_state=True)
    outs = [y, state] + list(ref_torch.fwd_bwd(*t)[1:])
    for name, got in zip(OUT, outs):
        want = torch.from_numpy(z[f"{name}_f32"])
        if name in ("y", "h_last"):
            # same torch ops in the same order on the same host: bit for bit
            assert torch.equal(got, want), f"{path.stem} {name}"
        else:
            assert max_rel(got, want) < 1e-6, f"{path.stem} {name}"


def test_c_oracle_matches_an_independent_numpy_recurrence():
    for shape, dist in (((2, 33, 5, 8), "ref"), ((1, 97, 3, 4), "c0"), ((2, 40, 6, 64), "c0")):
        x, dt, aneg, b_in, c_in, _ = (a.numpy() for a in inputs(*shape, dist=dist, seed=7))
        y, ckpt = oracle.scan_fwd(x, dt, aneg, b_in, c_in, chunk=64)
        y2, h2 = oracle.recurrence_f64(x, dt, aneg, b_in, c_in)
        assert max_rel(y, y2) < 1e-13
        assert max_rel(ckpt[:, -1], h2) < 1e-13


def test_c_oracle_gradients_match_float64_autograd():
    x, dt, aneg, b_in, c_in, dy = inputs(2, 45, 6, 8, dist="c0", seed=21, dtype=torch.float64)
    leaves = [t.clone().requires_grad_(True) for t in (x, dt, aneg, b_in, c_in)]
    y = ref_torch.scan_ref(*leaves)
    want = torch.autograd.grad(y, leaves, grad_outputs=dy)
    got = oracle.scan_bwd(*(t.numpy() for t in (x, dt, aneg, b_in, c_in, dy)))
    for g, w in zip(got, want):
        assert max_rel(g, w) < 1e-12


@pytest.mark.parametrize("chunk", [1, 7, 64, 100])
def test_c_oracle_checkpoints_are_chunk_end_states(chunk):
    x, dt, aneg, b_in, c_in, _ = (a.double().numpy() for a in inputs(1, 100, 3, 4, seed=5))
    _, ckpt = oracle.scan_fwd(x, dt, aneg, b_in, c_in, chunk=chunk)
    nchunk = (100 + chunk - 1) // chunk
    assert ckpt.shape == (1, nchunk, 3, 4)
    for c in range(nchunk):
        t_end = min((c + 1) * chunk, 100)
        _, h = oracle.recurrence_f64(x[:, :t_end], dt[:, :t_end], aneg, b_in[:, :t_end],
                                     c_in[:, :t_end])
        assert np.allclose(ckpt[:, c], h, rtol=0, atol=1e-13)


def test_a_planted_mistake_is_caught():
    """Perturb the oracle's result on the CPU: the gate that guards the kernels must fail."""
    path = GOLDEN[0]
    z, ins = _load(path)
    y, _ = oracle.scan_fwd(*ins[:5], chunk=64, dtype=np.float64)
    assert max_rel(y, z["y_f64"]) < 1e-11
    bad = y.copy()
    bad.reshape(-1)[bad.size // 2] += 1e-4 * np.abs(y).max()
    assert max_rel(bad, z["y_f64"]) > 1e-5
    # a wrong decay (dt*Aneg off by one ulp-ish scale) is also visible in the gradients
    dx, *_ = oracle.scan_bwd(*ins[:2], ins[2] * (1 + 1e-3), *ins[3:])
    assert max_rel(dx, z["dx_f64"]) > 1e-4


def test_oracle_rejects_bad_arguments():
    x, dt, aneg, b_in, c_in, _ = (a.numpy() for a in inputs(1, 4, 2, 4))
    with pytest.raises(ValueError):
        oracle.scan_fwd(x, dt, aneg, b_in, c_in, chunk=0)
