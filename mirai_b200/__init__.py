"""B200-native (sm_100a) sparse-MoE expert FFN for the seruva19/mirai hot path.

The compute lives in ``libmirai_b200.so`` (hand-written CUDA for sm_100a behind
the C ABI in ``include/mirai_b200.h``).  This package holds the host side that
mirrors the reference's routed-expert interfaces; it has no CPU fallback.
"""

from ._lib import MiraiError, Nf4Weight, Int8Weight, LIB_PATH  # noqa: F401

__all__ = ["MiraiError", "Nf4Weight", "Int8Weight", "LIB_PATH"]
