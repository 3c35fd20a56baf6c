"""styx_b200 -- the Qwen3-MoE MoE block of aDirtyScoundrel/styx as sm_100a
CUDA kernels behind a C ABI (include/styx_moe.h, libstyx_moe.so).

    from styx_b200 import ops          # torch-facing operator wrappers (+ ops.Residency:
                                       # budget / pinning / repin host logic)
    from styx_b200 import decode       # the whole decode step (DecodeModel)
    from styx_b200 import gguf         # GGUF reader / writer / model loaders
"""
from ._lib import (BLOCK, IDS_PER_LAYER, Q4_K, Q5_K, Q6_K, Q8_0, QTYPES, SKIP,  # noqa: F401
                   StyxError, row_bytes)

__all__ = ["BLOCK", "IDS_PER_LAYER", "Q4_K", "Q5_K", "Q6_K", "Q8_0", "QTYPES", "SKIP", "StyxError",
           "row_bytes"]
