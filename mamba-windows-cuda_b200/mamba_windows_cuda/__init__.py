"""B200-native (sm_100a) selective scan with the public API of mamba_windows_cuda.

``from mamba_windows_cuda import SelectiveScanCuda, parallel_scan_fn, parallel_scan_ref``
works as with the reference package (mamba_windows_cuda/__init__.py:1-4); the CUDA work
runs in the ahead-of-time built libmwc_b200.so.
"""
from .mamba_cuda import SelectiveScanCuda
from .pscan import parallel_scan_fn, parallel_scan_ref

__all__ = ["SelectiveScanCuda", "parallel_scan_fn", "parallel_scan_ref"]
__version__ = "0.1.0"
