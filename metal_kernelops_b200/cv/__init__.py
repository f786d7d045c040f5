"""Mamba-2 operators (drop-in for the hot-path part of ``metal_kernelops.cv``).

* ``mamba2_chunk_scan`` -- chunked SSD scan (cv/mamba2_chunk.py:617-678)
* ``mamba2_state_update`` -- one decode step (cv/mamba2_state.py:759-819)

The reference's other ``cv`` families (causal conv1d, gated RMSNorm, VMamba
path scan, NSA selection, RoIAlign) are outside this package's scope.
"""

from .mamba2_chunk import last_path, mamba2_chunk_scan
from .mamba2_state import mamba2_state_update

__all__ = ["last_path", "mamba2_chunk_scan", "mamba2_state_update"]
