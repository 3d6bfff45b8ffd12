"""Fused selective scan for Mamba on NVIDIA B200 (sm_100a), forward and backward.

Drop-in for the reference package's `mamba_metal.scan`
(Anamaya1729/mamba-metal-scan, mamba_metal/scan.py): same function names,
arguments, return values and errors; the Metal kernels are replaced by
hand-written CUDA kernels in libmms_scan.so, called through its C ABI.

    dA[t,d,n] = exp(-dt[t,d] * Aneg[d,n])
    h[t,d,n]  = dA[t,d,n] * h[t-1,d,n] + dt[t,d] * B[t,n] * x[t,d]    h[-1] = 0
    y[t,d]    = sum_n C[t,n] * h[t,d,n]

Shapes: x, dt (B, T, D); Aneg (D, N); B, C (B, T, N); y (B, T, D).

The forward keeps h on chip and writes only a checkpoint of h every `chunk`
steps; the backward recomputes from those checkpoints and returns gradients
for all five inputs. Kernels, launch geometry and reductions are described in
mamba-metal-scan_b200/csrc/. Dispatch (reference scan.py:424-447):

  'cuda'   the CUDA kernels; raises unless every input is a CUDA tensor.
  'metal'  accepted alias of 'cuda', so configs written for the reference
           keep working; there is no Metal backend in this build.
  'torch'  selective_scan_ref, the pure-PyTorch recurrence, on any device.
  'auto'   the CUDA kernels on CUDA tensors, otherwise None so the caller can
           fall back to its own path (TinyMamba uses parallel_scan).

On CUDA tensors 'auto', 'cuda' and 'metal' always run the native library; if
it is missing they raise RuntimeError rather than fall back.
"""
from __future__ import annotations

import torch

from mamba_metal import _native

# K: the forward checkpoints h every K steps. The reference uses 64 (sized for a
# 36 GB laptop); 8 lets the backward start every 8-step group from a stored
# state instead of recomputing 64-step segments, for 8x the checkpoint memory
# (still 1/8 of one (B, T, D, N) tensor). Any K >= 1 gives the same results.
SSM_CHUNK = 8
DBLOCK = 64           # accepted for API compatibility; the CUDA kernels size their own CTAs

_IMPLS = ("auto", "cuda", "metal", "torch")


# ------------------------------------------------------- reference (pure torch)

def selective_scan_ref(x: torch.Tensor, dt: torch.Tensor, aneg: torch.Tensor,
                       b_in: torch.Tensor, c_in: torch.Tensor,
                       return_state: bool = False):
    """The recurrence left to right in PyTorch ops (reference scan.py:313-333).

    Differentiable through autograd, any device, dtype and d_state. This is
    the 'torch' implementation; it keeps one (B, D, N) state per step alive
    for autograd, so it is meant for small shapes and for checking.
    """
    bt, t_len, d = x.shape
    n = aneg.shape[1]
    h = x.new_zeros(bt, d, n)
    ys = []
    for i in range(t_len):
        dt_i = dt[:, i, :].unsqueeze(-1)
        h = torch.exp(-dt_i * aneg.unsqueeze(0)) * h \
            + dt_i * b_in[:, i, :].unsqueeze(1) * x[:, i, :].unsqueeze(-1)
        ys.append((c_in[:, i, :].unsqueeze(1) * h).sum(-1))
    y = torch.stack(ys, dim=1) if ys else x.new_zeros(bt, 0, d)
    return (y, h) if return_state else y


# ------------------------------------------------------------------- the kernels

def _aligned(t: torch.Tensor, nbytes: int) -> torch.Tensor:
    """Contiguous, with a data pointer aligned for the kernels' vector loads."""
    t = t.contiguous()
    if t.data_ptr() % nbytes:
        t = t.clone()
    return t


def _validate(x, dt, aneg, b_in, c_in, impl_name: str):
    tensors = (x, dt, aneg, b_in, c_in)
    if not all(t.is_cuda for t in tensors):
        raise RuntimeError(
            f"scan_impl={impl_name!r} runs the CUDA kernels and needs every input on a "
            f"CUDA device (this build has no MPS/Metal backend); saw devices "
            f"{x.device}, {dt.device}, {aneg.device}, {b_in.device}, {c_in.device}")
    if len({t.device for t in tensors}) != 1:
        raise RuntimeError("selective_scan inputs are on different CUDA devices: "
                           + ", ".join(str(t.device) for t in tensors))
    if not all(t.dtype == torch.float32 for t in tensors):
        raise RuntimeError(f"scan_impl={impl_name!r} is fp32-only (the kernels are float32); got "
                           + ", ".join(str(t.dtype) for t in tensors))
    if x.dim() != 3 or dt.shape != x.shape or aneg.dim() != 2:
        raise ValueError(f"bad shapes: x {tuple(x.shape)}, dt {tuple(dt.shape)}, "
                         f"Aneg {tuple(aneg.shape)}")
    bt, t_len, d = x.shape
    n = aneg.shape[1]
    if aneg.shape[0] != d:
        raise ValueError(f"Aneg {tuple(aneg.shape)} does not match x's channel count {d}")
    if b_in.shape != (bt, t_len, n) or c_in.shape != (bt, t_len, n):
        raise ValueError(f"B {tuple(b_in.shape)} / C {tuple(c_in.shape)} must be "
                         f"({bt}, {t_len}, {n})")
    if n % 4 != 0 or n <= 0 or n > 64:
        raise ValueError(f"d_state must be a positive multiple of 4 no larger than 64 for the "
                         f"CUDA scan; got {n} (scan_impl='torch' takes any size)")


class SelectiveScanCUDA(torch.autograd.Function):
    """selective_scan_cuda(x, dt, Aneg, B, C) -> y, forward and backward.

    Same contract as the reference's SelectiveScanMetal (scan.py:338-411):
    inputs are made contiguous, (x, dt, Aneg, B, C, ckpt) are saved, the
    optional state is the last checkpoint returned detached, and backward
    returns the five input gradients plus None for chunk, dblock and
    return_state.
    """

    @staticmethod
    def forward(ctx, x, dt, aneg, b_in, c_in, chunk=SSM_CHUNK, dblock=DBLOCK,
                return_state=False, impl_name="cuda"):
        _validate(x, dt, aneg, b_in, c_in, impl_name)
        chunk = int(chunk)
        if chunk < 1:
            raise ValueError(f"chunk (the checkpoint stride) must be >= 1; got {chunk}")
        bt, t_len, d = x.shape
        n = aneg.shape[1]
        x = _aligned(x, 4)
        dt = _aligned(dt, 4)
        aneg = _aligned(aneg, 16)
        b_in = _aligned(b_in, 16)
        c_in = _aligned(c_in, 16)
        with torch.cuda.device(x.device):
            if bt == 0 or t_len == 0 or d == 0:
                y = x.new_zeros(bt, t_len, d)
                ckpt = x.new_zeros(bt, 0, d, n)
            else:
                y, ckpt = _native.fwd(x, dt, aneg, b_in, c_in, chunk)
        ctx.save_for_backward(x, dt, aneg, b_in, c_in, ckpt)
        ctx.chunk = chunk
        if return_state:
            # The last checkpoint is h at t = T-1; returned detached, as a
            # snapshot for the recurrent cache (reference scan.py:381-386).
            state = ckpt[:, -1].detach() if ckpt.shape[1] else x.new_zeros(bt, d, n)
            return y, state
        return y

    @staticmethod
    def backward(ctx, *grads):
        dy = grads[0]
        x, dt, aneg, b_in, c_in, ckpt = ctx.saved_tensors
        bt, t_len, d = x.shape
        if dy is None or bt == 0 or t_len == 0 or d == 0:
            return (torch.zeros_like(x), torch.zeros_like(dt), torch.zeros_like(aneg),
                    torch.zeros_like(b_in), torch.zeros_like(c_in), None, None, None, None)
        dy = _aligned(dy.float(), 4)
        with torch.cuda.device(x.device):
            dx, ddt, daneg, db, dc = _native.bwd(x, dt, aneg, b_in, c_in, dy, ckpt, ctx.chunk)
        return dx, ddt, daneg, db, dc, None, None, None, None


def selective_scan_cuda(x: torch.Tensor, dt: torch.Tensor, aneg: torch.Tensor,
                        b_in: torch.Tensor, c_in: torch.Tensor,
                        chunk: int = SSM_CHUNK,
                        dblock: int = DBLOCK,
                        return_state: bool = False):
    """y = selective_scan(x, dt, Aneg, B, C) with the CUDA kernels."""
    return SelectiveScanCUDA.apply(x, dt, aneg, b_in, c_in, chunk, dblock, return_state, "cuda")


def selective_scan_metal(x: torch.Tensor, dt: torch.Tensor, aneg: torch.Tensor,
                         b_in: torch.Tensor, c_in: torch.Tensor,
                         chunk: int = SSM_CHUNK,
                         dblock: int = DBLOCK,
                         return_state: bool = False):
    """The reference's entry point name, kept for drop-in use; runs the CUDA kernels."""
    return SelectiveScanCUDA.apply(x, dt, aneg, b_in, c_in, chunk, dblock, return_state, "metal")


def selective_scan(x: torch.Tensor, dt: torch.Tensor, aneg: torch.Tensor,
                   b_in: torch.Tensor, c_in: torch.Tensor,
                   impl: str = "auto",
                   chunk: int = SSM_CHUNK,
                   return_state: bool = False):
    """Dispatch the scan on `impl` (see the module docstring)."""
    if impl == "torch":
        return selective_scan_ref(x, dt, aneg, b_in, c_in, return_state=return_state)
    if impl not in _IMPLS:
        raise ValueError(f"unknown scan_impl {impl!r}; want 'auto', 'cuda', 'metal' or 'torch'")
    if x.is_cuda:
        return SelectiveScanCUDA.apply(x, dt, aneg, b_in, c_in, chunk, DBLOCK, return_state,
                                       "cuda" if impl == "auto" else impl)
    if impl in ("cuda", "metal"):
        raise RuntimeError(f"scan_impl={impl!r} needs CUDA tensors (this build has no MPS/Metal "
                           f"backend); got device {x.device.type!r}")
    return None


# ------------------------------------------------- fused _proj prologue (f2)

def proj_ref(dt_logit, a_param, dt_min: float, dt_max: float):
    """(dt, Aneg) as the reference model computes them (model.py:191-201)."""
    dt = dt_min + (dt_max - dt_min) * torch.sigmoid(dt_logit)
    return dt, torch.nn.functional.softplus(a_param)


class SelectiveScanProjCUDA(torch.autograd.Function):
    """The scan with dt and Aneg computed from their raw parameters in the kernels.

    forward(x, dt_logit, a_param, B, C, dt_min, dt_max, chunk, return_state):
    dt = dt_min + (dt_max - dt_min)*sigmoid(dt_logit), Aneg = softplus(a_param),
    then the scan; backward returns the gradients of x, dt_logit, a_param, B, C.
    Saves (x, dt_logit, a_param, B, C, ckpt): no (B, T, D) dt tensor exists.
    """

    @staticmethod
    def forward(ctx, x, dt_logit, a_param, b_in, c_in, dt_min, dt_max, chunk=SSM_CHUNK,
                return_state=False):
        _validate(x, dt_logit, a_param, b_in, c_in, "cuda")
        chunk = int(chunk)
        if chunk < 1:
            raise ValueError(f"chunk (the checkpoint stride) must be >= 1; got {chunk}")
        if not float(dt_max) > float(dt_min):
            raise ValueError(f"need dt_min < dt_max; got {dt_min}, {dt_max}")
        bt, t_len, d = x.shape
        n = a_param.shape[1]
        x, dt_logit = _aligned(x, 4), _aligned(dt_logit, 4)
        a_param, b_in, c_in = _aligned(a_param, 16), _aligned(b_in, 16), _aligned(c_in, 16)
        proj = (float(dt_min), float(dt_max))
        with torch.cuda.device(x.device):
            if bt == 0 or t_len == 0 or d == 0:
                y, ckpt = x.new_zeros(bt, t_len, d), x.new_zeros(bt, 0, d, n)
            else:
                y, ckpt = _native.fwd(x, dt_logit, a_param, b_in, c_in, chunk, proj=proj)
        ctx.save_for_backward(x, dt_logit, a_param, b_in, c_in, ckpt)
        ctx.chunk, ctx.proj = chunk, proj
        if return_state:
            state = ckpt[:, -1].detach() if ckpt.shape[1] else x.new_zeros(bt, d, n)
            return y, state
        return y

    @staticmethod
    def backward(ctx, *grads):
        dy = grads[0]
        x, dt_logit, a_param, b_in, c_in, ckpt = ctx.saved_tensors
        bt, t_len, d = x.shape
        if dy is None or bt == 0 or t_len == 0 or d == 0:
            return (torch.zeros_like(x), torch.zeros_like(dt_logit), torch.zeros_like(a_param),
                    torch.zeros_like(b_in), torch.zeros_like(c_in), None, None, None, None)
        dy = _aligned(dy.float(), 4)
        with torch.cuda.device(x.device):
            g = _native.bwd(x, dt_logit, a_param, b_in, c_in, dy, ckpt, ctx.chunk, proj=ctx.proj)
        return (*g, None, None, None, None)


def selective_scan_proj(x: torch.Tensor, dt_logit: torch.Tensor, a_param: torch.Tensor,
                        b_in: torch.Tensor, c_in: torch.Tensor, dt_min: float, dt_max: float,
                        impl: str = "auto", chunk: int = SSM_CHUNK, return_state: bool = False):
    """selective_scan with the model's _proj prologue fused in.

    Same as selective_scan(x, dt, Aneg, B, C) with
    dt = dt_min + (dt_max - dt_min)*sigmoid(dt_logit) and Aneg = softplus(a_param),
    differentiable with respect to dt_logit and a_param. On CUDA tensors the
    kernels compute dt and Aneg themselves (mms_fwd_proj / mms_bwd_proj), so
    the (B, T, D) dt tensor and its elementwise passes never exist; 'torch'
    composes proj_ref with selective_scan_ref; off-CUDA 'auto' returns None.
    """
    if impl == "torch":
        dt, aneg = proj_ref(dt_logit, a_param, dt_min, dt_max)
        return selective_scan_ref(x, dt, aneg, b_in, c_in, return_state=return_state)
    if impl not in _IMPLS:
        raise ValueError(f"unknown scan_impl {impl!r}; want 'auto', 'cuda', 'metal' or 'torch'")
    if x.is_cuda:
        return SelectiveScanProjCUDA.apply(x, dt_logit, a_param, b_in, c_in, dt_min, dt_max,
                                           chunk, return_state)
    if impl in ("cuda", "metal"):
        raise RuntimeError(f"scan_impl={impl!r} needs CUDA tensors (this build has no MPS/Metal "
                           f"backend); got device {x.device.type!r}")
    return None


# ---------------------------------------------------- bf16 storage (f4)

def _validate_bf16(x, dt, aneg, b_in, c_in, chunk: int):
    tensors = (x, dt, aneg, b_in, c_in)
    if not all(t.is_cuda for t in tensors) or len({t.device for t in tensors}) != 1:
        raise RuntimeError("selective_scan_bf16 needs every input on the same CUDA device; saw "
                           + ", ".join(str(t.device) for t in tensors))
    if x.dtype != torch.bfloat16 or dt.dtype != torch.bfloat16:
        raise RuntimeError(f"selective_scan_bf16 takes bf16 x and dt; got {x.dtype}, {dt.dtype}")
    if not all(t.is_floating_point() for t in (aneg, b_in, c_in)):
        raise RuntimeError("Aneg, B and C must be floating point")
    if x.dim() != 3 or dt.shape != x.shape or aneg.dim() != 2:
        raise ValueError(f"bad shapes: x {tuple(x.shape)}, dt {tuple(dt.shape)}, "
                         f"Aneg {tuple(aneg.shape)}")
    bt, t_len, d = x.shape
    n = aneg.shape[1]
    if aneg.shape[0] != d or b_in.shape != (bt, t_len, n) or c_in.shape != (bt, t_len, n):
        raise ValueError(f"Aneg {tuple(aneg.shape)}, B {tuple(b_in.shape)}, C {tuple(c_in.shape)} "
                         f"do not match x {tuple(x.shape)}")
    if n % 4 != 0 or n <= 0 or n > 64:
        raise ValueError(f"d_state must be a positive multiple of 4 no larger than 64; got {n}")
    if d % 8 != 0:
        raise ValueError(f"the bf16 scan needs d_inner % 8 == 0; got {d}")
    if chunk != 8:
        raise ValueError(f"the bf16 scan uses checkpoint stride 8; got chunk={chunk}")


class SelectiveScanBF16CUDA(torch.autograd.Function):
    """selective_scan_bf16(x, dt, Aneg, B, C) -> y (bf16), forward and backward.

    x, dt and y (and dy, dx, ddt) are stored as bf16; Aneg, B, C are used as
    fp32, as are the checkpoints and all arithmetic (mms_fwd_bf16 /
    mms_bwd_bf16). Gradients come back in each input's own dtype.
    """

    @staticmethod
    def forward(ctx, x, dt, aneg, b_in, c_in, chunk=SSM_CHUNK, return_state=False):
        chunk = int(chunk)
        _validate_bf16(x, dt, aneg, b_in, c_in, chunk)
        ctx.dtypes = (aneg.dtype, b_in.dtype, c_in.dtype)
        bt, t_len, d = x.shape
        n = aneg.shape[1]
        x = _aligned(x, 16)
        dt = _aligned(dt, 16)
        aneg = _aligned(aneg.float(), 16)
        b_in = _aligned(b_in.float(), 16)
        c_in = _aligned(c_in.float(), 16)
        with torch.cuda.device(x.device):
            if bt == 0 or t_len == 0 or d == 0:
                y = x.new_zeros(bt, t_len, d)
                ckpt = aneg.new_zeros(bt, 0, d, n)
            else:
                y, ckpt = _native.fwd_bf16(x, dt, aneg, b_in, c_in, chunk)
        ctx.save_for_backward(x, dt, aneg, b_in, c_in, ckpt)
        ctx.chunk = chunk
        if return_state:
            state = ckpt[:, -1].detach() if ckpt.shape[1] else aneg.new_zeros(bt, d, n)
            return y, state
        return y

    @staticmethod
    def backward(ctx, *grads):
        dy = grads[0]
        x, dt, aneg, b_in, c_in, ckpt = ctx.saved_tensors
        ta, tb, tc = ctx.dtypes
        bt, t_len, d = x.shape
        if dy is None or bt == 0 or t_len == 0 or d == 0:
            return (torch.zeros_like(x), torch.zeros_like(dt), torch.zeros_like(aneg, dtype=ta),
                    torch.zeros_like(b_in, dtype=tb), torch.zeros_like(c_in, dtype=tc), None, None)
        dy = _aligned(dy.to(torch.bfloat16), 16)
        with torch.cuda.device(x.device):
            dx, ddt, daneg, db, dc = _native.bwd_bf16(x, dt, aneg, b_in, c_in, dy, ckpt, ctx.chunk)
        return dx, ddt, daneg.to(ta), db.to(tb), dc.to(tc), None, None


def selective_scan_bf16(x: torch.Tensor, dt: torch.Tensor, aneg: torch.Tensor,
                        b_in: torch.Tensor, c_in: torch.Tensor,
                        chunk: int = SSM_CHUNK, return_state: bool = False):
    """The scan with bf16 x, dt and y (no counterpart in the fp32-only reference).

    Same recurrence and autograd contract as `selective_scan`; x and dt are
    bf16 CUDA tensors, Aneg, B and C any float dtype (used as fp32), y is
    bf16. Covers every d_state of the fp32 scan with d_inner a multiple of 8
    and checkpoint stride 8 (bf16 rows are staged in 16-byte pieces; the
    backward uses the stride-8 kernels); other shapes raise ValueError.
    """
    return SelectiveScanBF16CUDA.apply(x, dt, aneg, b_in, c_in, chunk, return_state)


# ------------------------------------------------------ gate epilogue (f3)

def gate_ref(y, z, d_skip):
    """(y + D_skip) * silu(z), the Mamba block's epilogue (reference model.py:255-256)."""
    return (y + d_skip) * torch.nn.functional.silu(z)


class GateCUDA(torch.autograd.Function):
    """out = (y + d_skip) * silu(z) as one kernel each way (mms_gate_fwd / _bwd).

    z may be a view with a row stride (the second half of in_proj's output);
    backward returns dy, dz and d_skip's gradient (a fixed-order sum).
    """

    @staticmethod
    def forward(ctx, y, z, d_skip):
        if not (y.is_cuda and z.is_cuda and d_skip.is_cuda):
            raise RuntimeError("the CUDA gate needs CUDA tensors")
        if y.dtype != torch.float32 or z.dtype != torch.float32 or d_skip.dtype != torch.float32:
            raise RuntimeError("the CUDA gate is fp32-only")
        if y.dim() != 3 or z.shape != y.shape or d_skip.shape != (y.shape[2],):
            raise ValueError(f"bad shapes: y {tuple(y.shape)}, z {tuple(z.shape)}, "
                             f"D_skip {tuple(d_skip.shape)}")
        y, d_skip = y.contiguous(), d_skip.contiguous()
        bt, t_len, d = y.shape
        # rows (b, t) must sit at one stride apart: contiguous channels, uniform rows
        if not (z.stride(2) == 1 and z.stride(1) >= d and z.stride(0) == t_len * z.stride(1)):
            z = z.contiguous()
        ctx.save_for_backward(y, z, d_skip)
        if y.numel() == 0:
            return torch.empty_like(y)
        with torch.cuda.device(y.device):
            return _native.gate_fwd(y, z, d_skip)

    @staticmethod
    def backward(ctx, dout):
        y, z, d_skip = ctx.saved_tensors
        if y.numel() == 0:
            return torch.zeros_like(y), torch.zeros_like(y), torch.zeros_like(d_skip)
        with torch.cuda.device(y.device):
            return _native.gate_bwd(dout.contiguous().float(), y, z, d_skip)


def gated_output(y: torch.Tensor, z: torch.Tensor, d_skip: torch.Tensor, impl: str = "auto"):
    """(y + d_skip) * silu(z): one CUDA kernel each way on CUDA tensors
    ('auto', 'cuda', 'metal'), PyTorch ops otherwise or with 'torch'."""
    if impl not in _IMPLS:
        raise ValueError(f"unknown scan_impl {impl!r}; want 'auto', 'cuda', 'metal' or 'torch'")
    if impl != "torch" and y.is_cuda:
        return GateCUDA.apply(y, z, d_skip)
    if impl in ("cuda", "metal"):
        raise RuntimeError(f"scan_impl={impl!r} needs CUDA tensors; got device {y.device.type!r}")
    return gate_ref(y, z, d_skip)


# ------------------------------------------------------------ decode (one token)

def selective_scan_step_ref(x, dt, aneg, b_in, c_in, h):
    """One recurrent step in PyTorch ops (reference model.py:228-241).

    x, dt (B, D); B, C (B, N); Aneg (D, N); h (B, D, N). Returns (y (B, D),
    new h); h itself is not modified.
    """
    dt_ = dt.unsqueeze(-1)
    h = h * torch.exp(-dt_ * aneg) + dt_ * b_in.unsqueeze(1) * x.unsqueeze(-1)
    return (h * c_in.unsqueeze(1)).sum(-1), h


def selective_scan_step(x: torch.Tensor, dt: torch.Tensor, aneg: torch.Tensor,
                        b_in: torch.Tensor, c_in: torch.Tensor, h: torch.Tensor,
                        impl: str = "auto"):
    """One decode step on a cached state: updates `h` in place, returns y (B, D).

        h = exp(-dt*Aneg) * h + dt*B*x;   y = sum_n C*h

    x, dt (B, D); B, C (B, N); Aneg (D, N); h (B, D, N), e.g. the state a
    `return_state=True` scan returned. Not differentiable: it is the
    inference path of the recurrent cache (reference model.py:228-241 runs
    the same arithmetic as PyTorch ops). On CUDA tensors 'auto'/'cuda'/'metal'
    run one fused kernel (mms_step); 'torch' runs selective_scan_step_ref and
    copies the result into h. Off-CUDA, 'auto' returns None like
    selective_scan.
    """
    if impl not in _IMPLS:
        raise ValueError(f"unknown scan_impl {impl!r}; want 'auto', 'cuda', 'metal' or 'torch'")
    if impl == "torch":
        y, h_new = selective_scan_step_ref(x, dt, aneg, b_in, c_in, h)
        h.copy_(h_new)
        return y
    if not x.is_cuda:
        if impl in ("cuda", "metal"):
            raise RuntimeError(f"scan_impl={impl!r} needs CUDA tensors (this build has no "
                               f"MPS/Metal backend); got device {x.device.type!r}")
        return None
    if x.dim() != 2 or dt.shape != x.shape or aneg.dim() != 2:
        raise ValueError(f"bad shapes: x {tuple(x.shape)}, dt {tuple(dt.shape)}, "
                         f"Aneg {tuple(aneg.shape)}")
    bt, d = x.shape
    n = aneg.shape[1]
    _validate(x.unsqueeze(1), dt.unsqueeze(1), aneg, b_in.unsqueeze(1), c_in.unsqueeze(1),
              impl)
    if h.shape != (bt, d, n) or h.dtype != torch.float32 or h.device != x.device:
        raise ValueError(f"state h must be float32 ({bt}, {d}, {n}) on {x.device}; "
                         f"got {h.dtype} {tuple(h.shape)} on {h.device}")
    if not h.is_contiguous() or h.data_ptr() % 16:
        raise ValueError("state h must be contiguous and 16-byte aligned (it is updated in place)")
    if bt == 0 or d == 0:
        return x.new_zeros(bt, d)
    with torch.cuda.device(x.device):
        return _native.step(_aligned(x, 4), _aligned(dt, 4), _aligned(aneg, 16),
                            _aligned(b_in, 16), _aligned(c_in, 16), h)
