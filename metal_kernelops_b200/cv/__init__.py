"""Mamba-2 operators (drop-in for the hot-path part of ``metal_kernelops.cv``).

* ``mamba2_chunk_scan`` -- chunked SSD scan (cv/mamba2_chunk.py:617-678)
* ``mamba2_state_update`` -- one decode step (cv/mamba2_state.py:759-819)
* ``ss2d_scan``, ``path_orders`` -- VMamba four-path 2D selective scan
  (cv/path_scan.py:153-163, :546-576), on the Mamba-1 scan kernels
* ``causal_conv1d_fn``, ``causal_conv1d_update`` -- causal depthwise conv1d,
  prefill and decode (cv/causal_conv1d.py:610-756)
* ``rmsnorm_gated`` -- gated RMSNorm, mamba's ``rms_norm_ref``
  (cv/gated_norm.py:647-686)

The reference's other ``cv`` families (NSA selection, RoIAlign) are outside
this package's scope.
"""

from .causal_conv1d import causal_conv1d_fn, causal_conv1d_update
from .gated_norm import rmsnorm_gated
from .mamba2_chunk import last_path, mamba2_chunk_scan, tc_shape
from .mamba2_state import mamba2_state_update
from .path_scan import path_orders, ss2d_scan

__all__ = ["causal_conv1d_fn", "causal_conv1d_update", "last_path", "mamba2_chunk_scan",
           "mamba2_state_update", "path_orders", "rmsnorm_gated", "ss2d_scan", "tc_shape"]
