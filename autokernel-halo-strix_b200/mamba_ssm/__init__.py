"""Import-compatible shim of `mamba_ssm` exposing only the selective scan.

Code that does `from mamba_ssm.ops.selective_scan_interface import selective_scan_fn`
(e.g. the reference's models/amadeus.py:58-79) gets the B200 kernel.
"""
