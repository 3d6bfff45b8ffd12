"""Fused selective-scan kernels for Mamba on NVIDIA B200 (sm_100a).

Drop-in for Anamaya1729/mamba-metal-scan's `mamba_metal` package: the same
exports, plus `selective_scan_cuda`, the one-token decode step
`selective_scan_step` and `selective_scan_proj` (the scan with the model's dt
and Aneg prologue fused into the kernels), `gated_output` (the block's
(y + D) * silu(z) epilogue as one kernel each way) and `selective_scan_bf16`
(bf16 storage for x, dt and y).
"""
from mamba_metal.model import MambaConfig, TinyMamba
from mamba_metal.scan import (gated_output, selective_scan, selective_scan_bf16, selective_scan_cuda,
                              selective_scan_metal, selective_scan_proj, selective_scan_ref,
                              selective_scan_step, selective_scan_step_ref)

__all__ = ["MambaConfig", "TinyMamba", "gated_output", "selective_scan", "selective_scan_bf16",
           "selective_scan_cuda",
           "selective_scan_metal", "selective_scan_proj", "selective_scan_ref",
           "selective_scan_step", "selective_scan_step_ref"]
