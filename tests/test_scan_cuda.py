"""Parity gates for the CUDA selective scan (GPU).

Port of the reference's MPS gates (tests/test_scan.py:74-230 of
Anamaya1729/mamba-metal-scan) to the CUDA kernels, plus the checks the
north star adds. The arbiter is the float64 C oracle (oracle/scan_oracle.c);
the reference's own fp32 outputs come from the committed golden vectors.

Tolerances, written as max|got - want| / max|want| (the error normalisation
under which even the reference's fp32 path meets them; elementwise relative
error is not met by the reference itself on near-zero elements):
    FWD_TOL  = 1e-5 for y (and the returned state)
    GRAD_TOL = 1e-4 for each of dx, ddt, dAneg, dB, dC
and, as in the reference suite, torch.allclose(atol=1e-4, rtol=1e-3) against
the fp32 reference path.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from _inputs import ATOL, RTOL, SEED, inputs, max_rel
from mamba_metal import selective_scan, selective_scan_cuda, selective_scan_metal
from mamba_metal.model import MambaConfig, TinyMamba
from oracle import oracle

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-5
GRAD_TOL = 1e-4
DEV = "cuda"
GRAD_NAMES = ("dx", "ddt", "dAneg", "dB", "dC")
GOLDEN = Path(__file__).resolve().parent / "golden"

# The reference's shapes (T not a multiple of 64, D not a multiple of a CTA,
# batch 1, a single step, d_state 8 and 16, an 18M-model d_inner), config 0,
# and every d_state group width the kernels instantiate.
SHAPES = [
    (2, 64, 32, 16, "ref"),
    (1, 100, 17, 16, "ref"),
    (4, 63, 128, 16, "ref"),
    (1, 1, 16, 16, "ref"),
    (2, 130, 40, 8, "ref"),
    (3, 512, 856, 16, "ref"),
    (2, 256, 64, 16, "c0"),
    (2, 77, 33, 4, "c0"),
    (1, 90, 70, 12, "c0"),
    (2, 65, 21, 32, "c0"),
    (1, 129, 19, 64, "c0"),
]


def cuda_fwd_bwd(x, dt, aneg, b_in, c_in, dy, chunk=64):
    leaves = [t.detach().clone().requires_grad_(True) for t in (x, dt, aneg, b_in, c_in)]
    y = selective_scan_cuda(*leaves, chunk=chunk)
    grads = torch.autograd.grad(y, leaves, grad_outputs=dy)
    return y.detach(), grads


def oracle64(x, dt, aneg, b_in, c_in, dy, chunk=64):
    cpu = [t.detach().cpu().numpy() for t in (x, dt, aneg, b_in, c_in, dy)]
    y, ckpt = oracle.scan_fwd(*cpu[:5], chunk=chunk)
    grads = oracle.scan_bwd(*cpu)
    return y, ckpt, grads


def assert_parity(y, grads, y64, grads64, label=""):
    e = max_rel(y, y64)
    assert e <= FWD_TOL, f"{label} y: normalised error {e:.3e} > {FWD_TOL}"
    for name, g, g64 in zip(GRAD_NAMES, grads, grads64):
        assert tuple(g.shape) == g64.shape, name
        e = max_rel(g, g64)
        assert e <= GRAD_TOL, f"{label} {name}: normalised error {e:.3e} > {GRAD_TOL}"


@pytest.mark.parametrize("chunk", [64, 8])
@pytest.mark.parametrize("bt,t_len,d,n,dist", SHAPES)
def test_forward_and_gradients_match_the_float64_oracle(bt, t_len, d, n, dist, chunk):
    x, dt, aneg, b_in, c_in, dy = inputs(bt, t_len, d, n, dist, seed=SEED + d, device=DEV)
    y, grads = cuda_fwd_bwd(x, dt, aneg, b_in, c_in, dy, chunk=chunk)
    assert y.shape == (bt, t_len, d) and y.dtype == torch.float32
    y64, _, g64 = oracle64(x, dt, aneg, b_in, c_in, dy, chunk=chunk)
    assert_parity(y, grads, y64, g64, f"{(bt, t_len, d, n)} chunk {chunk}")


# Shapes with B*D large enough for the forward's whole-state kernel (one thread
# per channel, d_state 12 or 16), with aligned and unaligned D.
WIDE = [(2, 130, 9500, 16, 8), (2, 77, 9501, 12, 64), (1, 300, 19000, 16, 7)]


@pytest.mark.parametrize("bt,t_len,d,n,chunk", WIDE)
def test_wide_channel_counts_match_the_float64_oracle(bt, t_len, d, n, chunk):
    x, dt, aneg, b_in, c_in, dy = inputs(bt, t_len, d, n, "c0", seed=d, device=DEV)
    y, grads = cuda_fwd_bwd(x, dt, aneg, b_in, c_in, dy, chunk=chunk)
    y64, ckpt64, g64 = oracle64(x, dt, aneg, b_in, c_in, dy, chunk=chunk)
    assert_parity(y, grads, y64, g64, f"{(bt, t_len, d, n)} chunk {chunk}")
    from mamba_metal import _native
    _, ckpt = _native.fwd(x, dt, aneg, b_in, c_in, chunk)
    assert max_rel(ckpt, ckpt64) <= FWD_TOL


# Long sequences with few channels: the kernels cut the sequence into time
# segments that run in parallel and chain their entry states and adjoint
# carries (csrc/mms_seg.cu). `slow` shrinks dt 50x so states and adjoints
# survive across many segments and a wrong carry cannot hide behind decay.
LONG = [(1, 4096, 256, 16, 8, False), (1, 4096, 256, 16, 8, True), (1, 3001, 130, 12, 8, True),
        (2, 2000, 64, 64, 8, True), (1, 5000, 96, 16, 64, True), (1, 1234, 40, 8, 7, True),
        (1, 4096, 64, 4, 100, True), (3, 700, 16, 16, 8, True)]


@pytest.mark.parametrize("bt,t_len,d,n,chunk,slow", LONG)
def test_long_sequences_match_the_float64_oracle(bt, t_len, d, n, chunk, slow):
    x, dt, aneg, b_in, c_in, dy = inputs(bt, t_len, d, n, "c0", seed=t_len + d, device=DEV)
    if slow:
        dt = dt * 0.02
    y, grads = cuda_fwd_bwd(x, dt, aneg, b_in, c_in, dy, chunk=chunk)
    y64, ckpt64, g64 = oracle64(x, dt, aneg, b_in, c_in, dy, chunk=chunk)
    assert_parity(y, grads, y64, g64, f"{(bt, t_len, d, n)} chunk {chunk} slow {slow}")
    from mamba_metal import _native
    _, ckpt = _native.fwd(x, dt, aneg, b_in, c_in, chunk)
    assert max_rel(ckpt, ckpt64) <= FWD_TOL


# The channel-pair backward at d_state 12 (4 lanes per pair, states 12..15
# padded) and 20..64 (8 or 16 lanes per channel pair): every stride class, a
# channel count that leaves a CTA partly empty, and long sequences that also
# run time segments.
PAIRS = [(2, 200, 64, 12, 8, False), (1, 1500, 32, 12, 24, True),
         (2, 200, 64, 32, 8, False), (1, 333, 48, 20, 16, False), (2, 150, 40, 48, 24, False),
         (1, 257, 32, 64, 64, False), (1, 100, 36, 64, 8, False), (2, 130, 24, 28, 40, False),
         (1, 3000, 96, 32, 16, True), (1, 2500, 32, 64, 8, True)]


@pytest.mark.parametrize("bt,t_len,d,n,chunk,slow", PAIRS)
def test_channel_pair_backward_at_wide_state_matches_the_float64_oracle(bt, t_len, d, n, chunk, slow):
    x, dt, aneg, b_in, c_in, dy = inputs(bt, t_len, d, n, "c0", seed=7 * t_len + n, device=DEV)
    if slow:
        dt = dt * 0.02
    y, grads = cuda_fwd_bwd(x, dt, aneg, b_in, c_in, dy, chunk=chunk)
    y64, _, g64 = oracle64(x, dt, aneg, b_in, c_in, dy, chunk=chunk)
    assert_parity(y, grads, y64, g64, f"{(bt, t_len, d, n)} chunk {chunk} slow {slow}")


def test_config3_shape_matches_the_float64_oracle():
    """One sequence of config 3 per GPU: B=1, T=16384, d_inner=2048, d_state=16."""
    x, dt, aneg, b_in, c_in, dy = inputs(1, 16384, 2048, 16, "c0", seed=3, device=DEV)
    y, grads = cuda_fwd_bwd(x, dt, aneg, b_in, c_in, dy, chunk=8)
    y64, _, g64 = oracle64(x, dt, aneg, b_in, c_in, dy, chunk=8)
    assert_parity(y, grads, y64, g64, "config 3")


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("*.npz")), ids=lambda p: p.stem)
def test_golden_vectors_from_the_reference(path):
    """The reference's own outputs (fp32 and fp64), recorded by tests/golden/make_golden.py."""
    z = np.load(path)
    x, dt, aneg, b_in, c_in, dy = (torch.from_numpy(z[k]).to(DEV)
                                   for k in ("x", "dt", "aneg", "b", "c", "dy"))
    leaves = [t.clone().requires_grad_(True) for t in (x, dt, aneg, b_in, c_in)]
    y, state = selective_scan_cuda(*leaves, return_state=True)
    grads = torch.autograd.grad(y, leaves, grad_outputs=dy)
    outs = [y, state] + list(grads)
    for name, got in zip(("y", "h_last", "dx", "ddt", "daneg", "db", "dc"), outs):
        want32 = torch.from_numpy(z[f"{name}_f32"]).to(DEV)
        assert torch.allclose(got.detach(), want32, atol=ATOL, rtol=RTOL), \
            f"{path.stem} {name}: max delta {(got - want32).abs().max().item():.3e}"
        tol = FWD_TOL if name in ("y", "h_last") else GRAD_TOL
        e = max_rel(got, z[f"{name}_f64"])
        assert e <= tol, f"{path.stem} {name}: normalised error vs fp64 {e:.3e} > {tol}"


def test_gradients_match_finite_differences():
    """The reference's gate (tests/test_scan.py:133-161): real derivatives, not just consistent."""
    bt, t_len, d, n = 1, 24, 12, 8
    x, dt, aneg, b_in, c_in, dy = inputs(bt, t_len, d, n, "ref", seed=SEED + 11, device=DEV)
    base = (x, dt, aneg, b_in, c_in)

    def f(i, j, v):
        inp = [t.clone() for t in base]
        inp[i].reshape(-1)[j] = v
        return (selective_scan_cuda(*inp) * dy).double().sum()

    _, grads = cuda_fwd_bwd(*base, dy)
    g = torch.Generator(device="cpu").manual_seed(SEED)
    worst = 0.0
    for i, tensor in enumerate(base):
        flat = tensor.reshape(-1)
        for j in torch.randperm(flat.numel(), generator=g)[:6].tolist():
            h = 1e-3 * max(1.0, abs(flat[j].item()))
            num = (f(i, j, flat[j] + h) - f(i, j, flat[j] - h)) / (2 * h)
            ana = grads[i].reshape(-1)[j].double()
            scale = max(1.0, abs(num.item()), abs(ana.item()))
            worst = max(worst, (num - ana).abs().item() / scale)
    assert worst < 0.05, f"finite-difference mismatch: {worst:.3f}"


@pytest.mark.parametrize("chunk", [1, 7, 8, 9, 16, 64, 65, 100, 511, 512])
def test_checkpoint_stride_is_an_implementation_detail(chunk):
    """Reference gate (tests/test_scan.py:213-221), extended to the gradients."""
    x, dt, aneg, b_in, c_in, dy = inputs(2, 512, 96, 16, "ref", seed=SEED + 5, device=DEV)
    y, grads = cuda_fwd_bwd(x, dt, aneg, b_in, c_in, dy, chunk=chunk)
    y64, ckpt64, g64 = oracle64(x, dt, aneg, b_in, c_in, dy, chunk=chunk)
    assert_parity(y, grads, y64, g64, f"chunk {chunk}")


def test_checkpoints_match_the_oracle():
    """ckpt[:, c] is h at the end of chunk c, the last one at t = T-1 (scan.py:120-125)."""
    from mamba_metal import _native
    x, dt, aneg, b_in, c_in, _ = inputs(2, 200, 40, 16, "c0", seed=3, device=DEV)
    for chunk in (1, 7, 64, 200, 300):
        _, ckpt = _native.fwd(x, dt, aneg, b_in, c_in, chunk)
        _, ckpt64 = oracle.scan_fwd(*(t.cpu().numpy() for t in (x, dt, aneg, b_in, c_in)),
                                    chunk=chunk)
        assert ckpt.shape == ckpt64.shape
        assert max_rel(ckpt, ckpt64) <= FWD_TOL, chunk


def test_returned_state_is_the_recurrence_state():
    x, dt, aneg, b_in, c_in, _ = inputs(1, 100, 16, 16, "ref", seed=SEED + 7, device=DEV)
    y, state = selective_scan_metal(x, dt, aneg, b_in, c_in, return_state=True)
    y64, h64 = oracle.recurrence_f64(*(t.cpu().numpy() for t in (x, dt, aneg, b_in, c_in)))
    assert state.shape == h64.shape and not state.requires_grad
    assert max_rel(state, h64) <= FWD_TOL
    assert max_rel(y, y64) <= FWD_TOL


def test_results_are_bitwise_deterministic():
    x, dt, aneg, b_in, c_in, dy = inputs(4, 300, 200, 16, "c0", seed=9, device=DEV)
    y1, g1 = cuda_fwd_bwd(x, dt, aneg, b_in, c_in, dy)
    y2, g2 = cuda_fwd_bwd(x, dt, aneg, b_in, c_in, dy)
    assert torch.equal(y1, y2)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def test_dispatch_on_cuda_tensors():
    x, dt, aneg, b_in, c_in, _ = inputs(1, 8, 16, 4, device=DEV)
    ref = selective_scan(x, dt, aneg, b_in, c_in, impl="torch")
    for impl in ("auto", "cuda", "metal"):
        y = selective_scan(x, dt, aneg, b_in, c_in, impl=impl)
        assert torch.allclose(y, ref, atol=ATOL, rtol=RTOL), impl
    with pytest.raises(ValueError, match="scan_impl"):
        selective_scan(x, dt, aneg, b_in, c_in, impl="nonsense")


def test_input_errors_are_raised_not_launched():
    x, dt, aneg, b_in, c_in, _ = inputs(1, 8, 16, 8, device=DEV)
    with pytest.raises(RuntimeError, match="fp32"):
        selective_scan_cuda(x.double(), dt, aneg, b_in, c_in)
    with pytest.raises(RuntimeError, match="CUDA"):
        selective_scan_cuda(x.cpu(), dt, aneg, b_in, c_in)
    with pytest.raises(ValueError, match="shapes"):
        selective_scan_cuda(x[0], dt, aneg, b_in, c_in)
    with pytest.raises(ValueError):
        selective_scan_cuda(x, dt, aneg[:-1], b_in, c_in)
    with pytest.raises(ValueError):
        selective_scan_cuda(x, dt, aneg, b_in[:, :-1], c_in)
    x6, dt6, aneg6, b6, c6, _ = inputs(1, 8, 16, 6, device=DEV)
    with pytest.raises(ValueError, match="d_state"):
        selective_scan_cuda(x6, dt6, aneg6, b6, c6)
    x68, dt68, aneg68, b68, c68, _ = inputs(1, 8, 16, 68, device=DEV)
    with pytest.raises(ValueError, match="d_state"):
        selective_scan_cuda(x68, dt68, aneg68, b68, c68)
    with pytest.raises(ValueError, match="chunk"):
        selective_scan_cuda(x, dt, aneg, b_in, c_in, chunk=0)


def test_strided_and_offset_inputs_are_accepted():
    """Non-contiguous views and storage offsets are made contiguous and aligned first."""
    x, dt, aneg, b_in, c_in, dy = inputs(2, 50, 24, 8, "c0", seed=4, device=DEV)
    big_b = torch.zeros(2, 50, 9, device=DEV)
    big_b[..., 1:] = b_in                                   # strided rows
    c_off = torch.zeros(c_in.numel() + 1, device=DEV)[1:].view_as(c_in)
    c_off.copy_(c_in)                                       # contiguous, 4 bytes off 16
    assert c_off.data_ptr() % 16 != 0
    xt = x.transpose(1, 2).contiguous().transpose(1, 2)     # non-contiguous
    y, grads = cuda_fwd_bwd(xt, dt, aneg, big_b[..., 1:], c_off, dy)
    y64, _, g64 = oracle64(x, dt, aneg, b_in, c_in, dy)
    assert_parity(y, grads, y64, g64)


def test_empty_inputs():
    for shape in ((0, 5, 8), (2, 0, 8), (2, 5, 0)):
        bt, t_len, d = shape
        x = torch.zeros(bt, t_len, d, device=DEV, requires_grad=True)
        dt = torch.zeros(bt, t_len, d, device=DEV)
        aneg = torch.ones(d, 4, device=DEV)
        b_in = torch.zeros(bt, t_len, 4, device=DEV)
        c_in = torch.zeros(bt, t_len, 4, device=DEV)
        y, state = selective_scan_cuda(x, dt, aneg, b_in, c_in, return_state=True)
        assert y.shape == shape and state.shape == (bt, d, 4)
        assert torch.count_nonzero(state) == 0
        y.sum().backward()
        assert x.grad.shape == x.shape


# ------------------------------------------------------------------ model level

def _tinymamba(scan_impl):
    cfg = MambaConfig(vocab_size=200, d_model=64, n_layers=2, d_ff=128, max_seq_len=64,
                      d_state=8, d_conv=4, scan_chunk=0, scan_impl=scan_impl)
    torch.manual_seed(SEED)
    return TinyMamba(cfg).to(DEV).eval()


def _loss_and_grads(model, idx):
    model.zero_grad(set_to_none=True)
    _, loss = model(idx, idx)
    loss.backward()
    return loss.detach(), [(n, p.grad.detach().clone()) for n, p in model.named_parameters()]


def test_end_to_end_torch_vs_cuda():
    """Reference gate (tests/test_scan.py:176-202): same loss and every parameter gradient."""
    g = torch.Generator().manual_seed(SEED)
    idx = torch.randint(0, 200, (2, 48), generator=g).to(DEV)
    ref = _tinymamba("torch")
    cud = _tinymamba("cuda")
    cud.load_state_dict(ref.state_dict())
    loss_r, grads_r = _loss_and_grads(ref, idx.clone())
    loss_c, grads_c = _loss_and_grads(cud, idx.clone())
    assert torch.allclose(loss_r, loss_c, atol=ATOL, rtol=RTOL)
    worst = 0.0
    for (name, gr), (_, gc) in zip(grads_r, grads_c):
        scale = max(1.0, gr.abs().max().item())
        worst = max(worst, (gr - gc).abs().max().item() / scale)
        assert torch.allclose(gr, gc, atol=ATOL, rtol=RTOL), name
    assert worst < 1e-3


def test_auto_selects_cuda_in_the_model():
    model = _tinymamba("auto")
    idx = torch.randint(0, 200, (2, 16), device=DEV)
    from mamba_metal import _native
    calls = []
    orig = _native.fwd

    def spy(*a, **k):
        calls.append(1)
        return orig(*a, **k)

    _native.fwd = spy
    try:
        model(idx, idx)
    finally:
        _native.fwd = orig
    assert len(calls) == 2          # one CUDA forward per layer


def test_recurrent_cache_matches_full_recomputation_on_cuda():
    """Reference gate (tests/test_model.py:123-146) with the CUDA scan priming the cache."""
    cfg = MambaConfig(vocab_size=200, d_model=64, n_layers=2, d_ff=128, max_seq_len=64,
                      d_state=8, d_conv=4, scan_chunk=8, scan_impl="cuda")
    torch.manual_seed(SEED)
    model = TinyMamba(cfg).to(DEV).eval()
    g = torch.Generator().manual_seed(SEED)
    full = torch.randint(0, 200, (4, 26), generator=g).to(DEV)
    x, step = full[:, :20], full[:, 20:]
    with torch.no_grad():
        cache: dict = {}
        model(x, cache=cache)
        cached = [model(step[:, t:t + 1], cache=cache)[0][:, -1] for t in range(step.shape[1])]
        naive = [model(torch.cat([x, step[:, :t + 1]], dim=1))[0][:, -1]
                 for t in range(step.shape[1])]
    for a, b in zip(cached, naive):
        assert torch.allclose(a, b, atol=1e-5)


def test_no_kernel_reported_a_timeout():
    """The backward's TMA stages wait on barriers with a bounded poll; none ran out."""
    from mamba_metal import _native
    x, dt, aneg, b_in, c_in, dy = inputs(16, 512, 2304, 16, "c0", seed=9, device=DEV)
    cuda_fwd_bwd(x, dt, aneg, b_in, c_in, dy, chunk=8)
    assert _native.device_status() == _native.MMS_OK


def test_backward_from_a_fresh_thread_matches_the_float64_oracle():
    """The first scan on a thread that has made no CUDA call yet (as PyTorch's
    autograd worker is at its first backward): the kernels' TMA tensor maps
    need the device's context made current on that thread."""
    import threading
    from mamba_metal import _native
    x, dt, aneg, b_in, c_in, dy = inputs(2, 64, 32, 16, "ref", seed=SEED + 7, device=DEV)
    out = {}

    def run():
        try:
            for chunk in (64, 8):
                y, ckpt = _native.fwd(x, dt, aneg, b_in, c_in, chunk)
                out[chunk] = (y, _native.bwd(x, dt, aneg, b_in, c_in, dy, ckpt, chunk))
            torch.cuda.synchronize()
        except Exception as e:          # surfaced in the main thread below
            out["error"] = e

    th = threading.Thread(target=run)
    th.start()
    th.join()
    assert "error" not in out, out.get("error")
    y64, _, g64 = oracle64(x, dt, aneg, b_in, c_in, dy)
    for chunk in (64, 8):
        y, grads = out[chunk]
        assert_parity(y, grads, y64, g64, f"fresh thread, chunk {chunk}")
