"""TinyMamba: the small Mamba language model around the selective scan.

API-compatible with the reference package's `mamba_metal.model`
(Anamaya1729/mamba-metal-scan, mamba_metal/model.py): the same config fields,
module names and parameter shapes (so state_dicts load either way), the same
block arithmetic, and the same `scan_impl` switch. Only the scan itself is
native; everything else is ordinary PyTorch.

Block (reference model.py:161-256):
    x -> RMSNorm -> in_proj -> (x, z)
    x -> causal depthwise conv -> SiLU
    dt = dt_min + (dt_max - dt_min) * sigmoid(dt_proj(x)),  B = B_proj(x),
    C = C_proj(x),  Aneg = softplus(A)
    y = selective_scan(x, dt, Aneg, B, C) + D_skip
    out = residual + out_proj(y * SiLU(z))

`scan_impl` 'auto' runs the CUDA kernels on CUDA tensors and the associative
`parallel_scan` elsewhere; 'cuda'/'metal' force the kernels; 'torch' forces
the PyTorch recurrence. d_inner defaults to the largest multiple of 8 whose
block costs no more parameters than a transformer block of the same
d_model/d_ff (reference model.py:58-82).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from mamba_metal.scan import (SSM_CHUNK, gated_output, selective_scan, selective_scan_proj,
                              selective_scan_step, selective_scan_step_ref)


@dataclass
class MambaConfig:
    vocab_size: int
    d_model: int = 384
    n_layers: int = 10
    d_ff: int = 1536          # sizes d_inner through the transformer parameter budget
    max_seq_len: int = 512
    d_state: int = 16
    d_conv: int = 4
    d_inner: Optional[int] = None
    scan_chunk: int = 0       # time slice of the parallel_scan fallback; 0 = one pass
    ssm_chunk: int = SSM_CHUNK  # checkpoint stride of the CUDA scan (memory vs recompute)
    scan_impl: str = "auto"   # 'auto' | 'cuda' | 'metal' | 'torch'
    fuse_proj: bool = True    # CUDA scan computes dt and softplus(A) itself (selective_scan_proj)
    fuse_gate: bool = True    # (y + D_skip) * silu(z) as one CUDA kernel each way (gated_output)
    dt_min: float = 0.001
    dt_max: float = 0.1
    norm_eps: float = 1e-6


def transformer_block_params(d_model: int, d_ff: int) -> int:
    """Parameters of a pre-norm transformer block: attention (4 d^2), MLP, two norms."""
    attention = 4 * d_model * d_model
    mlp = 2 * d_model * d_ff
    norms = 2 * d_model
    return attention + mlp + norms


def mamba_block_params(d_model: int, d_inner: int, d_state: int, d_conv: int) -> int:
    """Parameters of one MambaBlock as built below."""
    in_proj = 2 * d_model * d_inner
    conv = d_inner * d_conv + d_inner
    dt_proj = d_inner * d_inner + d_inner
    ssm = 3 * d_inner * d_state            # A, B_proj, C_proj
    skip = d_inner
    out_proj = d_inner * d_model
    norm = d_model
    return in_proj + conv + dt_proj + ssm + skip + out_proj + norm


def d_inner_for_budget(target: int, d_model: int, d_state: int, d_conv: int) -> int:
    """Largest multiple of 8 (at least 8) whose MambaBlock fits in `target` parameters.

    mamba_block_params is d_inner^2 + c*d_inner + d_model with
    c = 3*d_model + d_conv + 3 + 3*d_state; take the positive root and round down.
    """
    c = 3 * d_model + d_conv + 3 + 3 * d_state
    disc = c * c + 4 * (target - d_model)
    root = (math.sqrt(disc) - c) / 2.0
    return max(8, 8 * int(root // 8))


class RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        dtype = x.dtype
        xf = x.float()
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (self.weight * xf).to(dtype)


# ------------------------------------------------------------------ the scans

def scan_recurrence(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """h_t = a_t * h_{t-1} + b_t over dim 1, one step at a time (h_{-1} = 0)."""
    h = torch.zeros_like(b[:, 0])
    hs = []
    for t in range(a.shape[1]):
        h = a[:, t] * h + b[:, t]
        hs.append(h)
    return torch.stack(hs, dim=1)


def _doubling_scan(a: torch.Tensor, b: torch.Tensor):
    """Inclusive scan of the affine maps h -> a*h + b over dim 1 in log2(T) rounds.

    Returns (A, H): A[t] = a_0*...*a_t and H[t] = the state after step t from
    a zero start. Round r combines every element with the one 2^r earlier;
    positions before the start see the identity map (a=1, b=0).
    """
    A, H = a, b
    T = a.shape[1]
    shift = 1
    while shift < T:
        A_prev = F.pad(A[:, :-shift], (0, 0) * (a.dim() - 2) + (shift, 0), value=1.0)
        H_prev = F.pad(H[:, :-shift], (0, 0) * (a.dim() - 2) + (shift, 0), value=0.0)
        H = A * H_prev + H
        A = A * A_prev
        shift *= 2
    return A, H


def parallel_scan(a: torch.Tensor, b: torch.Tensor, chunk: int = 0) -> torch.Tensor:
    """Same result as scan_recurrence, computed with a log-depth associative scan.

    chunk > 0 scans `chunk` steps at a time and folds in the state carried
    from the previous slice (h += A * carry), which bounds the memory of the
    intermediates without changing the result (reference model.py:139-156).
    """
    T = a.shape[1]
    if not chunk or T <= chunk:
        return _doubling_scan(a, b)[1]
    out, carry = [], None
    for s in range(0, T, chunk):
        A, H = _doubling_scan(a[:, s:s + chunk], b[:, s:s + chunk])
        if carry is not None:
            H = H + A * carry.unsqueeze(1)
        carry = H[:, -1]
        out.append(H)
    return torch.cat(out, dim=1)


# ------------------------------------------------------------------- the block

class MambaBlock(nn.Module):
    """Gated causal conv + diagonal selective SSM inside one residual."""

    def __init__(self, cfg: MambaConfig, d_inner: int):
        super().__init__()
        dm, ds, kc = cfg.d_model, cfg.d_state, cfg.d_conv
        self.d_inner = d_inner
        self.scan_chunk = cfg.scan_chunk
        self.ssm_chunk = cfg.ssm_chunk
        self.scan_impl = cfg.scan_impl
        self.fuse_proj = cfg.fuse_proj
        self.fuse_gate = cfg.fuse_gate
        self.dt_min, self.dt_max = cfg.dt_min, cfg.dt_max
        self.norm = RMSNorm(dm, cfg.norm_eps)
        self.in_proj = nn.Linear(dm, 2 * d_inner, bias=False)
        # padding kc-1 on both sides; keeping the first T outputs makes it causal
        self.conv = nn.Conv1d(d_inner, d_inner, kernel_size=kc, padding=kc - 1,
                              groups=d_inner, bias=True)
        self.dt_proj = nn.Linear(d_inner, d_inner, bias=True)
        self.A = nn.Parameter(torch.arange(1, ds + 1, dtype=torch.float32).repeat(d_inner, 1))
        self.B_proj = nn.Linear(d_inner, ds, bias=False)
        self.C_proj = nn.Linear(d_inner, ds, bias=False)
        self.D_skip = nn.Parameter(torch.ones(d_inner))
        self.out_proj = nn.Linear(d_inner, dm, bias=False)

    def _proj(self, x):
        """(dt, B, C, Aneg) from the post-conv, post-SiLU activations."""
        dt = self.dt_min + (self.dt_max - self.dt_min) * torch.sigmoid(self.dt_proj(x))
        return dt, self.B_proj(x), self.C_proj(x), F.softplus(self.A)

    def _ssm(self, x):
        """(a, b, C) of the recurrence h_t = a_t*h_{t-1} + b_t, materialised."""
        dt, B_t, C_t, Aneg = self._proj(x)
        a = torch.exp(-dt.unsqueeze(-1) * Aneg)
        b = dt.unsqueeze(-1) * B_t.unsqueeze(2) * x.unsqueeze(-1)
        return a, b, C_t

    def _scan(self, x, return_state=False):
        """y_t = sum_n C_tn h_tn; the fused scan when scan_impl allows it."""
        if self.fuse_proj and x.is_cuda and self.scan_impl != "torch":
            # dt and Aneg computed inside the kernels from dt_proj(x) and A
            return selective_scan_proj(x, self.dt_proj(x), self.A, self.B_proj(x), self.C_proj(x),
                                       self.dt_min, self.dt_max, impl=self.scan_impl,
                                       chunk=self.ssm_chunk, return_state=return_state)
        dt, B_t, C_t, Aneg = self._proj(x)
        r = selective_scan(x, dt, Aneg, B_t, C_t, impl=self.scan_impl, chunk=self.ssm_chunk,
                           return_state=return_state)
        if r is not None:
            return r
        a = torch.exp(-dt.unsqueeze(-1) * Aneg)
        b = dt.unsqueeze(-1) * B_t.unsqueeze(2) * x.unsqueeze(-1)
        h = parallel_scan(a, b, chunk=self.scan_chunk)
        y = (h * C_t.unsqueeze(2)).sum(-1)
        return (y, h[:, -1]) if return_state else y

    def _step(self, x, dt, Aneg, B_t, C_t, cache):
        """One token of the recurrence on cache["h"]; y (B, d_inner).

        Without autograd, on CUDA, the fused decode kernel updates the cached
        state in place (it owns that buffer: the scan's returned state is a
        detached checkpoint). With autograd, or off-CUDA, the step is the
        reference's differentiable PyTorch ops and the cache gets a new tensor.
        """
        h = cache["h"]
        needs_grad = torch.is_grad_enabled() and any(
            t.requires_grad for t in (x, dt, Aneg, B_t, C_t, h))
        if x.is_cuda and self.scan_impl != "torch" and not needs_grad:
            if not cache.get("h_owned"):
                h = h.clone(memory_format=torch.contiguous_format)
                cache["h"], cache["h_owned"] = h, True
            return selective_scan_step(x, dt, Aneg, B_t, C_t, h, impl=self.scan_impl)
        y, cache["h"] = selective_scan_step_ref(x, dt, Aneg, B_t, C_t, h)
        cache["h_owned"] = False
        return y

    def forward(self, x, cache=None):
        residual = x
        x, z = self.in_proj(self.norm(x)).chunk(2, dim=-1)
        kc = self.conv.kernel_size[0]
        if cache is not None and cache.get("h") is not None and x.shape[1] == 1:
            # one-token recurrent step against the cached conv window and state
            window = torch.cat([cache["conv"], x.transpose(1, 2)], dim=2)   # (B, d_inner, kc)
            x = F.silu(self.conv(window)[:, :, kc - 1:kc]).transpose(1, 2)
            cache["conv"] = window[:, :, 1:]
            dt, B_t, C_t, Aneg = self._proj(x)
            y = self._step(x[:, 0], dt[:, 0], Aneg, B_t[:, 0], C_t[:, 0], cache).unsqueeze(1)
        else:
            xc = x.transpose(1, 2)
            x = F.silu(self.conv(xc)[:, :, :xc.shape[2]]).transpose(1, 2)
            if cache is not None:
                tail = xc[:, :, -(kc - 1):]
                if tail.shape[2] < kc - 1:
                    tail = F.pad(tail, (kc - 1 - tail.shape[2], 0))
                cache["conv"] = tail
            # the last checkpoint of the scan is h[:, -1]: the cache costs nothing
            y, h_last = self._scan(x, return_state=True)
            if cache is not None:
                cache["h"], cache["h_owned"] = h_last, False
        if self.fuse_gate and y.is_cuda and self.scan_impl != "torch":
            return residual + self.out_proj(gated_output(y, z, self.D_skip, impl=self.scan_impl))
        y = y + self.D_skip
        return residual + self.out_proj(y * F.silu(z))


class TinyMamba(nn.Module):
    """A Mamba language model sized to a transformer's parameter budget."""

    def __init__(self, cfg: MambaConfig):
        super().__init__()
        self.cfg = cfg
        d_inner = cfg.d_inner
        if d_inner is None:
            d_inner = d_inner_for_budget(transformer_block_params(cfg.d_model, cfg.d_ff),
                                         cfg.d_model, cfg.d_state, cfg.d_conv)
        self.d_inner = d_inner
        self.tok = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.blocks = nn.ModuleList(MambaBlock(cfg, d_inner) for _ in range(cfg.n_layers))
        self.ln_f = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        self.head.weight = self.tok.weight          # tied
        self.apply(self._init)

    @staticmethod
    def _init(m):
        if isinstance(m, nn.Linear):
            nn.init.normal_(m.weight, mean=0.0, std=0.02)
            if m.bias is not None:
                nn.init.zeros_(m.bias)
        elif isinstance(m, nn.Embedding):
            nn.init.normal_(m.weight, mean=0.0, std=0.02)

    def forward(self, idx, targets=None, cache=None):
        if cache is not None and "blocks" not in cache:
            cache["blocks"] = [{} for _ in self.blocks]
        per_block = cache["blocks"] if cache is not None else [None] * len(self.blocks)
        x = self.tok(idx)
        for block, bc in zip(self.blocks, per_block):
            x = block(x, bc)
        logits = self.head(self.ln_f(x))
        loss = None
        if targets is not None:
            loss = F.cross_entropy(logits.reshape(-1, logits.size(-1)), targets.reshape(-1),
                                   ignore_index=-100)
        return logits, loss

    def count_params(self) -> int:
        """Unique parameters (the tied head counts once)."""
        return sum(p.numel() for p in self.parameters())
