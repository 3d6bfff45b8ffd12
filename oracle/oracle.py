"""numpy front end of the C oracle (test infrastructure only).

`scan_fwd` / `scan_bwd` call oracle/scan_oracle.c in float64 (the arbiter)
or float32. The math follows the reference's kernels:
mamba_metal/scan.py:13-15 and :105-126 (forward, checkpoint every K steps),
:26-34 and :173-260 (backward). Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg use this module.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from oracle.build import build

_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        lib = ctypes.CDLL(str(build()))
        for suf, ct in (("f64", ctypes.c_double), ("f32", ctypes.c_float)):
            p = ctypes.POINTER(ct)
            getattr(lib, f"oracle_fwd_{suf}").argtypes = [p] * 7 + [ctypes.c_int] * 5
            getattr(lib, f"oracle_bwd_{suf}").argtypes = [p] * 11 + [ctypes.c_int] * 4
            getattr(lib, f"oracle_fwd_{suf}").restype = ctypes.c_int
            getattr(lib, f"oracle_bwd_{suf}").restype = ctypes.c_int
        lib.oracle_num_threads.restype = ctypes.c_int
        lib.oracle_set_num_threads.argtypes = [ctypes.c_int]
        _LIB = lib
    return _LIB


def num_threads() -> int:
    return _lib().oracle_num_threads()


def set_num_threads(n: int) -> None:
    _lib().oracle_set_num_threads(int(n))


def _prep(a, dtype):
    return np.ascontiguousarray(np.asarray(a), dtype=dtype)


def _ptr(a, dtype):
    ct = ctypes.c_double if dtype == np.float64 else ctypes.c_float
    return a.ctypes.data_as(ctypes.POINTER(ct))


def _suffix(dtype):
    if dtype == np.float64:
        return "f64"
    if dtype == np.float32:
        return "f32"
    raise ValueError(f"oracle supports float32/float64, not {dtype}")


def scan_fwd(x, dt, aneg, b_in, c_in, chunk: int = 64, dtype=np.float64):
    """Returns (y (B,T,D), ckpt (B, ceil(T/chunk), D, N)) in `dtype`."""
    dtype = np.dtype(dtype).type
    x, dt, aneg, b_in, c_in = (_prep(a, dtype) for a in (x, dt, aneg, b_in, c_in))
    bt, t_len, d = x.shape
    n = aneg.shape[1]
    if chunk < 1:
        raise ValueError(f"chunk must be >= 1, got {chunk}")
    nchunk = (t_len + chunk - 1) // chunk
    y = np.empty((bt, t_len, d), dtype)
    ckpt = np.zeros((bt, nchunk, d, n), dtype)
    fn = getattr(_lib(), f"oracle_fwd_{_suffix(dtype)}")
    rc = fn(*(_ptr(a, dtype) for a in (x, dt, aneg, b_in, c_in, y, ckpt)),
            bt, t_len, d, n, chunk)
    if rc:
        raise RuntimeError(f"oracle_fwd failed with status {rc}")
    return y, ckpt


def scan_bwd(x, dt, aneg, b_in, c_in, dy, dtype=np.float64):
    """Returns (dx, ddt, dAneg, dB, dC) in `dtype`."""
    dtype = np.dtype(dtype).type
    x, dt, aneg, b_in, c_in, dy = (_prep(a, dtype) for a in (x, dt, aneg, b_in, c_in, dy))
    bt, t_len, d = x.shape
    n = aneg.shape[1]
    dx = np.empty_like(x)
    ddt = np.empty_like(dt)
    daneg = np.empty_like(aneg)
    db = np.empty_like(b_in)
    dc = np.empty_like(c_in)
    fn = getattr(_lib(), f"oracle_bwd_{_suffix(dtype)}")
    rc = fn(*(_ptr(a, dtype) for a in (x, dt, aneg, b_in, c_in, dy, dx, ddt, daneg, db, dc)),
            bt, t_len, d, n)
    if rc:
        raise RuntimeError(f"oracle_bwd failed with status {rc}")
    return dx, ddt, daneg, db, dc


def recurrence_f64(x, dt, aneg, b_in, c_in):
    """The plain left-to-right recurrence in numpy float64 (small sizes only).

    scan.py:13-15: dA = exp(-dt*Aneg), h_t = dA*h_{t-1} + dt*B*x, y = sum_n C*h.
    Independent of the C code; used to pin the C oracle itself.
    """
    x, dt, aneg, b_in, c_in = (np.asarray(a, np.float64) for a in (x, dt, aneg, b_in, c_in))
    bt, t_len, d = x.shape
    n = aneg.shape[1]
    h = np.zeros((bt, d, n))
    ys = np.empty((bt, t_len, d))
    for t in range(t_len):
        da = np.exp(-dt[:, t, :, None] * aneg[None])
        h = da * h + dt[:, t, :, None] * b_in[:, t, None, :] * x[:, t, :, None]
        ys[:, t] = (c_in[:, t, None, :] * h).sum(-1)
    return ys, h
