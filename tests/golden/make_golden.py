"""Generate the golden vectors by running the REFERENCE itself.

    python tests/golden/make_golden.py /path/to/mamba-metal-scan

imports `selective_scan_ref` from the reference checkout given on the command
line (Anamaya1729/mamba-metal-scan, mamba_metal/scan.py:313-333), runs its
forward and autograd backward on seeded inputs in float32 and in float64, and
writes one compressed .npz per case next to this script. The reference cannot
travel to the GPU box, so the fixtures are committed; this script is how they
were made.

Input distributions:
  "ref"  the reference test suite's generator (tests/test_scan.py:31-40):
         x ~ N(0,1), dt = 0.001 + 0.099*U, Aneg = softplus(arange(1..N)+0.1),
         B, C = 0.5*N(0,1)
  "c0"   the benchmark configs' generator: x ~ N(0,1), dt = softplus(N(-2, 0.5^2)),
         Aneg[d,n] = (n+1)*(1+0.1*U), B, C ~ N(0,1)
In both, dy ~ N(0,1).
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# (name, B, T, D, N, distribution, seed)
CASES = [
    ("c0_2x256x64x16", 2, 256, 64, 16, "c0", 0),          # config 0, the oracle case
    ("ref_2x64x32x16", 2, 64, 32, 16, "ref", 1337 + 32),
    ("ref_1x100x17x16", 1, 100, 17, 16, "ref", 1337 + 17),
    ("ref_1x1x16x16", 1, 1, 16, 16, "ref", 1337 + 16),
    ("ref_2x130x40x8", 2, 130, 40, 8, "ref", 1337 + 40),
    ("ref_1x24x12x8", 1, 24, 12, 8, "ref", 1337 + 11),
    ("ref_1x97x3x4", 1, 97, 3, 4, "ref", 1337 + 97),
    ("c0_1x40x7x12", 1, 40, 7, 12, "c0", 12),
    ("c0_2x70x9x64", 2, 70, 9, 64, "c0", 64),
    ("c0_3x129x33x32", 3, 129, 33, 32, "c0", 32),
]


def make_inputs(bt, t_len, d, n, dist, seed):
    """float32 (x, dt, Aneg, B, C, dy) from a CPU torch.Generator."""
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
    return x, dt, aneg.contiguous(), b_in, c_in, dy


def _load_reference(ref_root: Path):
    spec = importlib.util.spec_from_file_location(
        "_reference_scan", ref_root / "mamba_metal" / "scan.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.selective_scan_ref


def _run(ref_fn, inputs, dy):
    leaves = [t.clone().requires_grad_(True) for t in inputs]
    y, h_last = ref_fn(*leaves, return_state=True)
    grads = torch.autograd.grad(y, leaves, grad_outputs=dy)
    return [y.detach(), h_last.detach()] + [g.detach() for g in grads]


OUT_NAMES = ("y", "h_last", "dx", "ddt", "daneg", "db", "dc")


def main(ref_root: str) -> None:
    ref_fn = _load_reference(Path(ref_root))
    torch.set_num_threads(1)            # fixed reduction order for the fp32 run
    for name, bt, t_len, d, n, dist, seed in CASES:
        x, dt, aneg, b_in, c_in, dy = make_inputs(bt, t_len, d, n, dist, seed)
        out32 = _run(ref_fn, (x, dt, aneg, b_in, c_in), dy)
        out64 = _run(ref_fn, tuple(t.double() for t in (x, dt, aneg, b_in, c_in)), dy.double())
        arrays = dict(x=x, dt=dt, aneg=aneg, b=b_in, c=c_in, dy=dy)
        arrays.update({f"{k}_f32": v for k, v in zip(OUT_NAMES, out32)})
        arrays.update({f"{k}_f64": v for k, v in zip(OUT_NAMES, out64)})
        np.savez_compressed(HERE / f"{name}.npz",
                            meta=np.array([bt, t_len, d, n, seed]),
                            dist=np.array(dist),
                            **{k: v.numpy() for k, v in arrays.items()})
        print(f"{name}: wrote {len(arrays)} arrays")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
