"""The drop-in boundary on the CPU: the C-ABI library and the Python dispatch.

No GPU is needed: the library is loaded and every symbol include/mms_scan.h
declares is resolved; argument errors are answered before any launch, so they
can be exercised with NULL pointers on a host without a device.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from _inputs import inputs
from mamba_metal import _native, selective_scan, selective_scan_bf16, selective_scan_ref
from mamba_metal.scan import SelectiveScanCUDA

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "mms_scan.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"\b(mms_[a-z_0-9]+)\s*\(", text)


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    names = declared_functions()
    assert set(names) == set(_native.SIGNATURES), names
    for name in names:
        assert hasattr(lib, name), name


def test_abi_version_and_status_strings():
    lib = _native.load()
    assert lib.mms_abi_version() == 105
    for rc in range(9):
        assert _native.status_string(rc) != "unknown status"
    assert _native.status_string(99) == "unknown status"


def test_bad_arguments_return_status_without_launching():
    lib = _native.load()
    null = None
    args = [null] * 7
    assert lib.mms_fwd(*args, 2, 8, 16, 6, 64, null) == _native.MMS_ERR_UNSUPPORTED_N
    assert lib.mms_fwd(*args, 2, 8, 16, 68, 64, null) == _native.MMS_ERR_UNSUPPORTED_N
    assert lib.mms_fwd(*args, 2, 8, 16, 16, 0, null) == _native.MMS_ERR_INVALID_ARG
    assert lib.mms_fwd(*args, 0, 8, 16, 16, 64, null) == _native.MMS_ERR_INVALID_ARG
    assert lib.mms_fwd(*args, 2, 8, 16, 16, 64, null) == _native.MMS_ERR_INVALID_ARG  # NULLs
    # misaligned (fake, never dereferenced) pointers
    fake = [ctypes.c_void_p(0x10000 + 4)] * 7
    assert lib.mms_fwd(*fake, 2, 8, 16, 16, 64, null) == _native.MMS_ERR_MISALIGNED
    bargs = [ctypes.c_void_p(0x10000)] * 12
    ws = ctypes.c_void_p(0x20000)
    need = lib.mms_bwd_workspace_size(2, 8, 16, 16, 64)
    assert need > 0
    assert lib.mms_bwd(*bargs, ws, need - 1, 2, 8, 16, 16, 64, null) == _native.MMS_ERR_WORKSPACE
    assert lib.mms_bwd(*bargs, None, need, 2, 8, 16, 16, 64, null) == _native.MMS_ERR_WORKSPACE
    assert lib.mms_bwd(*bargs, ctypes.c_void_p(0x20010), need, 2, 8, 16, 16, 64, null) \
        == _native.MMS_ERR_MISALIGNED
    assert lib.mms_bwd_workspace_size(2, 8, 16, 6, 64) == 0


def test_bf16_entry_points_check_their_shapes_first():
    """bf16 storage needs D % 8 == 0, and K == 8 for the backward (fake pointers:
    every call here must be refused before a launch)."""
    lib = _native.load()
    null = None
    fake = [ctypes.c_void_p(0x10000)] * 7
    unsup = _native.MMS_ERR_UNSUPPORTED_BF16
    assert lib.mms_fwd_bf16(*fake, 2, 8, 12, 16, 8, null) == unsup      # D % 8
    assert lib.mms_fwd_bf16(*fake, 2, 8, 20, 32, 1, null) == unsup      # D % 8
    assert lib.mms_fwd_bf16(*fake, 2, 8, 16, 6, 8, null) == _native.MMS_ERR_UNSUPPORTED_N
    assert lib.mms_fwd_bf16(*fake, 2, 8, 16, 68, 8, null) == _native.MMS_ERR_UNSUPPORTED_N
    assert lib.mms_fwd_bf16(*([null] * 7), 2, 8, 16, 16, 8, null) == _native.MMS_ERR_INVALID_ARG
    # bf16 arrays need 16-byte alignment (fp32 ones: 16 as before)
    odd = [ctypes.c_void_p(0x10008)] + [ctypes.c_void_p(0x10000)] * 6
    assert lib.mms_fwd_bf16(*odd, 2, 8, 16, 16, 8, null) == _native.MMS_ERR_MISALIGNED
    bargs = [ctypes.c_void_p(0x10000)] * 12
    need = lib.mms_bwd_workspace_size(2, 8, 16, 16, 8)
    ws = ctypes.c_void_p(0x20000)
    assert lib.mms_bwd_bf16(*bargs, ws, need, 2, 8, 16, 16, 16, null) == unsup   # K != 8
    assert lib.mms_bwd_bf16(*bargs, ws, need, 2, 8, 16, 64, 4, null) == unsup    # K != 8
    assert lib.mms_bwd_bf16(*bargs, ws, need, 2, 8, 20, 16, 8, null) == unsup    # D % 8
    assert lib.mms_bwd_bf16(*bargs, ws, need - 1, 2, 8, 16, 16, 8, null) == _native.MMS_ERR_WORKSPACE


def test_bf16_scan_needs_cuda_tensors():
    x, dt, aneg, b_in, c_in, _ = inputs(1, 8, 16, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        selective_scan_bf16(x.bfloat16(), dt.bfloat16(), aneg, b_in, c_in)


def test_workspace_grows_with_long_chunks():
    lib = _native.load()
    base = lib.mms_bwd_workspace_size(16, 512, 2304, 16, 64)
    longer = lib.mms_bwd_workspace_size(16, 512, 2304, 16, 512)
    assert longer > base        # segment-start states of chunks longer than 64 steps


def test_unknown_scan_impl_is_rejected():
    x, dt, aneg, b_in, c_in, _ = inputs(1, 4, 8, 4)
    with pytest.raises(ValueError, match="scan_impl"):
        selective_scan(x, dt, aneg, b_in, c_in, impl="nonsense")


def test_cuda_impls_require_cuda_tensors_and_auto_declines():
    """Reference contract (tests/test_scan.py:74-81): no silent CPU fallback."""
    x, dt, aneg, b_in, c_in, _ = inputs(1, 8, 16, 4)
    for impl in ("cuda", "metal"):
        with pytest.raises(RuntimeError, match="MPS"):
            selective_scan(x, dt, aneg, b_in, c_in, impl=impl)
        with pytest.raises(RuntimeError, match="CUDA"):
            selective_scan(x, dt, aneg, b_in, c_in, impl=impl)
    assert selective_scan(x, dt, aneg, b_in, c_in, impl="auto") is None
    with pytest.raises(RuntimeError, match="CUDA"):
        SelectiveScanCUDA.apply(x, dt, aneg, b_in, c_in, 64, 64, False, "cuda")


def test_torch_impl_is_the_recurrence():
    x, dt, aneg, b_in, c_in, _ = inputs(2, 30, 5, 8, dist="c0")
    y = selective_scan(x, dt, aneg, b_in, c_in, impl="torch")
    y2, h = selective_scan_ref(x, dt, aneg, b_in, c_in, return_state=True)
    assert torch.equal(y, y2) and h.shape == (2, 5, 8)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIB_PATH", tmp_path / "nope.so")
    with pytest.raises(RuntimeError, match="not built"):
        _native.load()
