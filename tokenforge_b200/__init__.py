"""B200-native (sm_100a) backend for TokenForge's quantized-linear hot path.

Importing :mod:`tokenforge_b200.ops` registers the ``torch.ops.tokenforge`` namespace
(``w4a16_linear``, ``w4a16_dequant``, ``rmsnorm_fp8_quant``, ``awq_repack``) on top of the
kernel library ``lib/libtokenforge_b200.so``, whose C ABI is declared in
``include/tokenforge_b200.h``.
"""

from tokenforge_b200.pack import (
    AWQ_ORDER,
    AWQ_REVERSE_ORDER,
    PACK_FACTOR,
    SUPPORTED_GROUP_SIZES,
    W4A16Weights,
)

__all__ = [
    "AWQ_ORDER",
    "AWQ_REVERSE_ORDER",
    "PACK_FACTOR",
    "SUPPORTED_GROUP_SIZES",
    "W4A16Weights",
]
