"""Seeded input generators shared by the tests (same recipes as the golden script)."""
from __future__ import annotations

import numpy as np
import torch

SEED = 1337
ATOL, RTOL = 1e-4, 1e-3          # the reference test suite's kernel tolerance


def inputs(bt, t_len, d, n, dist="ref", seed=SEED, device="cpu", dtype=torch.float32):
    """(x, dt, Aneg, B, C, dy).

    "ref": the reference tests' generator (x ~ N(0,1), dt = 0.001 + 0.099*U,
           Aneg = softplus(arange(1..N) + 0.1), B, C = 0.5*N(0,1));
    "c0":  the benchmark configs' generator (dt = softplus(N(-2, 0.5^2)),
           Aneg[d,n] = (n+1)*(1+0.1*U), B, C ~ N(0,1)).
    """
    g = torch.Generator(device="cpu").manual_seed(seed)
    f32 = torch.float32
    x = torch.randn(bt, t_len, d, generator=g, dtype=f32)
    if dist == "ref":
        dt = 0.001 + 0.099 * torch.rand(bt, t_len, d, generator=g, dtype=f32)
        aneg = torch.nn.functional.softplus(torch.arange(1, n + 1, dtype=f32).repeat(d, 1) + 0.1)
        b_in = 0.5 * torch.randn(bt, t_len, n, generator=g, dtype=f32)
        c_in = 0.5 * torch.randn(bt, t_len, n, generator=g, dtype=f32)
    elif dist == "c0":
        dt = torch.nn.functional.softplus(-2.0 + 0.5 * torch.randn(bt, t_len, d, generator=g, dtype=f32))
        aneg = (torch.arange(1, n + 1, dtype=f32).unsqueeze(0)
                * (1.0 + 0.1 * torch.rand(d, n, generator=g, dtype=f32)))
        b_in = torch.randn(bt, t_len, n, generator=g, dtype=f32)
        c_in = torch.randn(bt, t_len, n, generator=g, dtype=f32)
    else:
        raise ValueError(dist)
    dy = torch.randn(bt, t_len, d, generator=g, dtype=f32)
    out = [t.contiguous().to(device=device, dtype=dtype) for t in (x, dt, aneg, b_in, c_in, dy)]
    return tuple(out)


def max_rel(a, b) -> float:
    """max|a-b| / max|b| in float64 (the normalised error the north star's tolerances use)."""
    a = np.asarray(a.detach().cpu().double() if torch.is_tensor(a) else a, np.float64)
    b = np.asarray(b.detach().cpu().double() if torch.is_tensor(b) else b, np.float64)
    scale = max(np.abs(b).max(initial=0.0), 1e-30)
    return float(np.abs(a - b).max(initial=0.0) / scale)
