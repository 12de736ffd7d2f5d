"""dreamx-creator_b200 -- B200-native (sm_100a) SR-DiT 5B refiner hot path.

Drop-ins for the reference's hot-path interfaces (AMAP-ML/DreamX-Creator,
video_refiner/wan/modules/sr_dit/):
  attention.mask_free_window_attention / attention.run_blockgrid_b200 / install
  fp8_linear.Fp8Linear / convert_linears_to_fp8
  model.SRDiT  -- the 30-block streaming forward, module names as in WanModel

The directory name carries a hyphen, so import it by path:
    import importlib; srdit = importlib.import_module("dreamx-creator_b200")
after which ``dreamx_creator_b200`` is registered as an alias.
"""
from __future__ import annotations

import sys

from . import _lib, blockgrid, ops  # noqa: F401
from . import attention, fp8_linear  # noqa: F401

sys.modules.setdefault("dreamx_creator_b200", sys.modules[__name__])

__all__ = ["attention", "blockgrid", "fp8_linear", "ops"]
