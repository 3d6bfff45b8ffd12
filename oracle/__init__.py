"""CPU oracle for the selective scan -- test infrastructure, not product code.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package, and only as the checker. The product (the CUDA library and the
`mamba_metal` package under mamba-metal-scan_b200/) never imports it.
"""
