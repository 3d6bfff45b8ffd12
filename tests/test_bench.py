"""bench.py's accounting on the CPU: the algorithmic units of the step
roofline and the kernel-launch count it reports as `gpu_launches`.

The launch count restates the library's dispatch rules (time segments of the
backward and of the two forwards); these cases pin one shape per rule.
"""
from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("_bench", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_step_bytes_match_the_roofline_units(bench):
    """32·BTD + 24·BTN + 12·DN: 607.6 MB at config 1."""
    bt, t_len, d, n = bench.CONFIGS["c1"][:4]
    fwd, bwd = bench.algorithmic_bytes(bt, t_len, d, n)
    btd, btn, dn = bt * t_len * d, bt * t_len * n, d * n
    assert fwd + bwd == 32 * btd + 24 * btn + 12 * dn
    assert abs((fwd + bwd) / 1e6 - 607.6) < 0.1


@pytest.mark.parametrize("shape,launches", [
    ((16, 512, 2304, 16, 8), 3),     # config 1: whole-state forward, channel-pair backward, reduction
    ((1, 16384, 2048, 16, 8), 7),    # config 3a: both directions cut into time segments
    ((4, 4096, 4096, 16, 8), 3),     # config 4 on two GPUs: G-lane forward and backward unsegmented
    ((1, 16384, 2048, 64, 8), 7),    # config 3b: G-lane forward, channel-pair backward, segmented
    ((4, 4096, 8192, 16, 8), 3),     # config 4 on one GPU
])
def test_launch_count_follows_the_dispatch_rules(bench, shape, launches):
    assert bench.launches_per_step(*shape) == launches


# (N, K, D)
@pytest.mark.parametrize("shape,kernel", [
    ((16, 8, 2304), "bwd_kernel_cp"),       # config 1
    ((16, 8, 2302), "bwd_kernel_w8"),       # config 1's stride with unaligned channel arrays
    ((64, 8, 2048), "bwd_kernel_cp"),       # config 3b
    ((16, 64, 2304), "bwd_kernel_cp"),      # config 1 at the reference's stride
    ((8, 8, 2304), "bwd_kernel_k8"),        # d_state 8
    ((16, 100, 2304), "bwd_kernel"),        # stride beyond 64
    ((32, 16, 2303), "bwd_kernel"),         # unaligned channel count
])
def test_roofline_names_the_backward_kernel_the_library_runs(bench, shape, kernel):
    n, k, d = shape
    assert bench.bwd_kernel_label(n, k, d) == f"mms_bwd ({kernel} + reduce_kernel)"
