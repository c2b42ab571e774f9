"""`selective_scan_fn` / `SelectiveScanFn` backed by the B200 kernel (see kernels.mamba_scan)."""
from kernels.mamba_scan import SelectiveScanFn, selective_scan_fn  # noqa: F401

__all__ = ["SelectiveScanFn", "selective_scan_fn"]
