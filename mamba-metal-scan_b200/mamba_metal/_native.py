"""ctypes binding of libmms_scan.so (C ABI in include/mms_scan.h).

The library is built in-tree (mamba-metal-scan_b200/build.py) into
mamba_metal/lib/. There is no fallback: if the library is missing or does not
load, every CUDA scan call raises RuntimeError naming the problem.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("MMS_SCAN_LIB", Path(__file__).resolve().parent / "lib" / "libmms_scan.so"))

MMS_OK = 0
MMS_ERR_INVALID_ARG = 1
MMS_ERR_UNSUPPORTED_N = 2
MMS_ERR_WORKSPACE = 3
MMS_ERR_MISALIGNED = 4
MMS_ERR_CUDA = 5
MMS_ERR_TOO_LARGE = 6
MMS_ERR_TIMEOUT = 7
MMS_ERR_UNSUPPORTED_BF16 = 8

# Every symbol include/mms_scan.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I = ctypes.c_int
SIGNATURES = {
    "mms_abi_version": ([], _I),
    "mms_status_string": ([_I], ctypes.c_char_p),
    "mms_last_cuda_error": ([], ctypes.c_char_p),
    "mms_fwd": ([_P] * 7 + [_I] * 5 + [_P], _I),
    "mms_bwd_workspace_size": ([_I] * 5, ctypes.c_size_t),
    "mms_bwd": ([_P] * 13 + [ctypes.c_size_t] + [_I] * 5 + [_P], _I),
    "mms_bwd_noalloc": ([_P] * 12 + [_I] * 5 + [_P], _I),
    "mms_step": ([_P] * 7 + [_I] * 3 + [_P], _I),
    "mms_device_status": ([], _I),
    "mms_gate_workspace_size": ([_I] * 3, ctypes.c_size_t),
    "mms_gate_fwd": ([_P, _P, ctypes.c_longlong] + [_P] * 2 + [_I] * 3 + [_P], _I),
    "mms_gate_bwd": ([_P] * 3 + [ctypes.c_longlong] + [_P] * 5 + [ctypes.c_size_t] + [_I] * 3
                     + [_P], _I),
    "mms_fwd_proj": ([_P] * 5 + [ctypes.c_float] * 2 + [_P] * 2 + [_I] * 5 + [_P], _I),
    "mms_bwd_proj": ([_P] * 7 + [ctypes.c_float] * 2 + [_P] * 6 + [ctypes.c_size_t] + [_I] * 5
                     + [_P], _I),
    "mms_fwd_bf16": ([_P] * 7 + [_I] * 5 + [_P], _I),
    "mms_bwd_bf16": ([_P] * 13 + [ctypes.c_size_t] + [_I] * 5 + [_P], _I),
    "mms_debug_set_wait": ([ctypes.c_uint, _I], _I),
    "mms_probe_pipe": ([_I] * 3 + [_P] * 4, _I),
    "mms_probe_ops_per_cta": ([_I] * 2, ctypes.c_longlong),
    "mms_probe_exp2": ([_P, _P, ctypes.c_longlong, _I, _P], _I),
}

# mms_probe_pipe kinds
PROBE_KINDS = {"ex2": 0, "ffma": 1, "ffma2": 2, "shfl": 3, "ex2_poly": 4, "ex2_poly2": 5}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raises RuntimeError if unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"the CUDA selective-scan library is not built: {LIB_PATH} is missing "
                    "(run `python mamba-metal-scan_b200/build.py`)")
            try:
                lib = ctypes.CDLL(str(LIB_PATH))
            except OSError as e:
                raise RuntimeError(f"cannot load {LIB_PATH}: {e}") from e
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def status_string(rc: int) -> str:
    return load().mms_status_string(rc).decode()


def _check(rc: int, what: str) -> None:
    if rc != MMS_OK:
        extra = f": {load().mms_last_cuda_error().decode()}" if rc == MMS_ERR_CUDA else ""
        raise RuntimeError(f"{what} failed: status {rc} ({status_string(rc)}){extra}")


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def fwd(x, dt, aneg, b_in, c_in, chunk: int, proj=None):
    """y (B,T,D) and ckpt (B, ceil(T/chunk), D, N) on the current stream.

    proj = (dt_min, dt_max): dt holds logits and aneg the raw A of the fused
    prologue (mms_fwd_proj)."""
    lib = load()
    bt, t_len, d = x.shape
    n = aneg.shape[1]
    nchunk = (t_len + chunk - 1) // chunk
    y = torch.empty(bt, t_len, d, device=x.device, dtype=torch.float32)
    ckpt = torch.empty(bt, nchunk, d, n, device=x.device, dtype=torch.float32)
    if proj is None:
        rc = lib.mms_fwd(_ptr(x), _ptr(dt), _ptr(aneg), _ptr(b_in), _ptr(c_in), _ptr(y),
                         _ptr(ckpt), bt, t_len, d, n, chunk, _stream(x.device))
        _check(rc, "mms_fwd")
    else:
        rc = lib.mms_fwd_proj(_ptr(x), _ptr(dt), _ptr(aneg), _ptr(b_in), _ptr(c_in),
                              float(proj[0]), float(proj[1]), _ptr(y), _ptr(ckpt),
                              bt, t_len, d, n, chunk, _stream(x.device))
        _check(rc, "mms_fwd_proj")
    return y, ckpt


def bwd_workspace_size(bt: int, t_len: int, d: int, n: int, chunk: int) -> int:
    return int(load().mms_bwd_workspace_size(bt, t_len, d, n, chunk))


def bwd(x, dt, aneg, b_in, c_in, dy, ckpt, chunk: int, workspace=None, proj=None):
    """(dx, ddt, dAneg, dB, dC) on the current stream (with proj: the
    gradients of the logits and of the raw A in place of ddt and dAneg)."""
    lib = load()
    bt, t_len, d = x.shape
    n = aneg.shape[1]
    dx = torch.empty_like(x)
    ddt = torch.empty_like(dt)
    daneg = torch.empty_like(aneg)
    db = torch.empty_like(b_in)
    dc = torch.empty_like(c_in)
    ws_bytes = bwd_workspace_size(bt, t_len, d, n, chunk)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), device=x.device, dtype=torch.uint8)
    if proj is None:
        rc = lib.mms_bwd(_ptr(x), _ptr(dt), _ptr(aneg), _ptr(b_in), _ptr(c_in), _ptr(dy),
                         _ptr(ckpt), _ptr(dx), _ptr(ddt), _ptr(daneg), _ptr(db), _ptr(dc),
                         _ptr(workspace), workspace.numel(),
                         bt, t_len, d, n, chunk, _stream(x.device))
        _check(rc, "mms_bwd")
    else:
        rc = lib.mms_bwd_proj(_ptr(x), _ptr(dt), _ptr(aneg), _ptr(b_in), _ptr(c_in), _ptr(dy),
                              _ptr(ckpt), float(proj[0]), float(proj[1]),
                              _ptr(dx), _ptr(ddt), _ptr(daneg), _ptr(db), _ptr(dc),
                              _ptr(workspace), workspace.numel(),
                              bt, t_len, d, n, chunk, _stream(x.device))
        _check(rc, "mms_bwd_proj")
    return dx, ddt, daneg, db, dc


def fwd_bf16(x, dt, aneg, b_in, c_in, chunk: int):
    """mms_fwd_bf16: x, dt bf16 (B,T,D), Aneg/B/C fp32; returns y bf16 (B,T,D)
    and the fp32 ckpt (B, ceil(T/chunk), D, N)."""
    lib = load()
    bt, t_len, d = x.shape
    n = aneg.shape[1]
    nchunk = (t_len + chunk - 1) // chunk
    y = torch.empty(bt, t_len, d, device=x.device, dtype=torch.bfloat16)
    ckpt = torch.empty(bt, nchunk, d, n, device=x.device, dtype=torch.float32)
    rc = lib.mms_fwd_bf16(_ptr(x), _ptr(dt), _ptr(aneg), _ptr(b_in), _ptr(c_in), _ptr(y),
                          _ptr(ckpt), bt, t_len, d, n, chunk, _stream(x.device))
    _check(rc, "mms_fwd_bf16")
    return y, ckpt


def bwd_bf16(x, dt, aneg, b_in, c_in, dy, ckpt, chunk: int, workspace=None):
    """mms_bwd_bf16: (dx, ddt) bf16 and (dAneg, dB, dC) fp32."""
    lib = load()
    bt, t_len, d = x.shape
    n = aneg.shape[1]
    dx = torch.empty_like(x)
    ddt = torch.empty_like(dt)
    daneg = torch.empty_like(aneg)
    db = torch.empty_like(b_in)
    dc = torch.empty_like(c_in)
    ws_bytes = bwd_workspace_size(bt, t_len, d, n, chunk)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), device=x.device, dtype=torch.uint8)
    rc = lib.mms_bwd_bf16(_ptr(x), _ptr(dt), _ptr(aneg), _ptr(b_in), _ptr(c_in), _ptr(dy),
                          _ptr(ckpt), _ptr(dx), _ptr(ddt), _ptr(daneg), _ptr(db), _ptr(dc),
                          _ptr(workspace), workspace.numel(),
                          bt, t_len, d, n, chunk, _stream(x.device))
    _check(rc, "mms_bwd_bf16")
    return dx, ddt, daneg, db, dc


def step(x, dt, aneg, b_in, c_in, h):
    """One decode step: updates h (B,D,N) in place, returns y (B,D)."""
    lib = load()
    bt, d = x.shape
    n = aneg.shape[1]
    y = torch.empty(bt, d, device=x.device, dtype=torch.float32)
    rc = lib.mms_step(_ptr(x), _ptr(dt), _ptr(aneg), _ptr(b_in), _ptr(c_in), _ptr(h), _ptr(y),
                      bt, d, n, _stream(x.device))
    _check(rc, "mms_step")
    return y


def device_status() -> int:
    """MMS_OK, or MMS_ERR_TIMEOUT if a kernel's bounded wait ran out since the last call."""
    return int(load().mms_device_status())


def gate_fwd(y, z, d_skip):
    """out = (y + d_skip) * silu(z) in one kernel; z may have a row stride."""
    lib = load()
    bt, t_len, d = y.shape
    out = torch.empty_like(y)
    rc = lib.mms_gate_fwd(_ptr(y), _ptr(z), z.stride(1), _ptr(d_skip), _ptr(out), bt, t_len, d,
                          _stream(y.device))
    _check(rc, "mms_gate_fwd")
    return out


def gate_bwd(dout, y, z, d_skip):
    """(dy, dz, d_dskip) of gate_fwd in one kernel (plus a fixed-order reduction)."""
    lib = load()
    bt, t_len, d = y.shape
    dy, dd = torch.empty_like(y), torch.empty_like(d_skip)
    dz = torch.empty(y.shape, device=y.device, dtype=torch.float32)
    nb = int(lib.mms_gate_workspace_size(bt, t_len, d))
    ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=y.device)
    rc = lib.mms_gate_bwd(_ptr(dout), _ptr(y), _ptr(z), z.stride(1), _ptr(d_skip), _ptr(dy),
                          _ptr(dz), _ptr(dd), _ptr(ws), nb, bt, t_len, d, _stream(y.device))
    _check(rc, "mms_gate_bwd")
    return dy, dz, dd


def pipe_rate(kind: str, device=None, iters: int = 4096, ctas_per_sm: int = 4) -> float:
    """Operations per SM per clock of one pipe (mms_probe_pipe), measured on the
    SM cycle counters: per SM, the operations of its CTAs over its longest CTA;
    the median over SMs. kind: one of PROBE_KINDS."""
    lib = load()
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    n_sm = torch.cuda.get_device_properties(device).multi_processor_count
    blocks = n_sm * ctas_per_sm
    sink = torch.empty(256, device=device)
    cycles = torch.empty(blocks, dtype=torch.int64, device=device)
    sm = torch.empty(blocks, dtype=torch.int32, device=device)
    k = PROBE_KINDS[kind]
    for _ in range(2):                       # the first launch warms the clocks up
        _check(lib.mms_probe_pipe(k, iters, blocks, _ptr(sink), _ptr(cycles), _ptr(sm),
                                  _stream(device)), "mms_probe_pipe")
    torch.cuda.synchronize(device)
    ops = int(lib.mms_probe_ops_per_cta(k, iters))
    per_sm = {}
    for c, s in zip(cycles.tolist(), sm.tolist()):
        n, m = per_sm.get(s, (0, 0))
        per_sm[s] = (n + 1, max(m, c))
    rates = sorted(n * ops / m for n, m in per_sm.values())
    return rates[len(rates) // 2]
