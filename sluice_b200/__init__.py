"""sluice_b200 — B200-native (sm_100a) MoE expert-offload hot path.

Drop-in for the router-split path of kfirtoledo/sluice: ``Router``
(gate + ``select_experts``), ``sluice_stream_gap`` / ``SlotCache.gap``
(device slot planner + GPU-initiated expert streaming), ``fused_experts``
(tcgen05 grouped GEMMs with SwiGLU and the weighted combine), behind the C ABI
declared in ``include/sluice_b200.h``.
"""

from . import configs
from ._lib import LIB_PATH, SluiceError, lib

__all__ = ["configs", "LIB_PATH", "SluiceError", "lib"]
