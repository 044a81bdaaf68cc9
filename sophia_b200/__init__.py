"""B200-native (sm_100a) Kimi Delta Attention layer for Sophia.

``chunk_kda`` / ``kda_layer`` run hand-written CUDA kernels through the C ABI
of ``include/kda_b200.h``; ``install(model)`` puts them behind Sophia's own
``SophiaKDA`` seams.
"""

from .ops import chunk_kda, fused_recurrent_kda, gated_rms_norm, kda_decode, kda_layer  # noqa: F401
from .integration import install  # noqa: F401
from .packing import document_cu_seqlens  # noqa: F401

__version__ = "0.1.0"
