"""xsake_b200: the HADS block-sparse attention path of Hridambiswas/XSAKE on B200 (sm_100a).

Modules mirror the reference's operator API:
  sparse_attention  -- kernels/pallas/sparse_attention.py
  fused_softmax     -- kernels/pallas/fused_softmax.py
  fused_layernorm   -- kernels/pallas/fused_layernorm.py
  hads_pattern      -- kernels/hads/hads_pattern.py
All compute runs in libxsake_hads.so (include/xsake_hads.h); there is no CPU fallback.
"""

from ._lib import XsakeError, LIB_PATH  # noqa: F401

__all__ = ["sparse_attention", "fused_softmax", "fused_layernorm", "hads_pattern", "XsakeError"]
