"""B200-native (sm_100a) SSM-scan hot path of dbydd/metal-kernelops.

Drop-in for the reference's hot-path functions, with the same call
signatures (src/metal_kernelops/__init__.py:23-41, cv/__init__.py:15-40):

* ``metal_kernelops_b200.selective_scan`` / ``selective_scan_fn`` -- Mamba-1
  selective scan, forward and backward (``metal_kernelops.selective_scan``)
* ``metal_kernelops_b200.cv.mamba2_chunk_scan`` -- Mamba-2 chunked SSD scan
* ``metal_kernelops_b200.cv.mamba2_state_update`` -- Mamba-2 decode step

The recurrence is mamba_ssm's:

    x_t = exp(dt_t * A) * x_{t-1} + dt_t * B_t * u_t
    y_t = <x_t, C_t>

Every op runs hand-written CUDA kernels from the in-tree library
``libssm_b200.so`` (C ABI: ``include/ssm_b200.h``), registered as torch custom
ops on the CUDA dispatch key under the ``b200ssm`` namespace.  There is no CPU
path: CPU tensors raise ``ValueError``.
"""

from .scan import CHUNK, scan_cuda, selective_scan, selective_scan_fn
from . import cv  # noqa: F401  (registers the Mamba-2 ops)
from ._native import check_errors

__all__ = ["CHUNK", "check_errors", "cv", "scan_cuda", "selective_scan", "selective_scan_fn"]

__version__ = "0.1.0"
