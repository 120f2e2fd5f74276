"""Drop-in for the reference's planned extension module ``tokenforge.kernels._C``.

The reference's op layer calls ``_C.w4a16_gemv(x2, qweight_t, scales, qzeros, bias,
group_size)`` for decode-sized M when ``TOKENFORGE_BACKEND=cuda`` (tokenforge/kernels/ops.py:
34-40, 86-88) and treats the module's importability as "CUDA extension available". Importing
this module loads the sm_100a kernel library (and raises ImportError if it is not built), so
the reference's availability probe behaves correctly when this module is installed under that
name.

It imports only the direct launchers (``tokenforge_b200.linear``), never
``tokenforge_b200.ops``: the reference keeps its own ``torch.ops.tokenforge.*`` registrations
(their Triton, torch-reference and fake paths) and only its ``cuda_gemv`` route lands here.
"""

from __future__ import annotations

import torch

from tokenforge_b200 import _lib
from tokenforge_b200.linear import w4a16_gemv as _gemv

_lib.lib()  # ImportError here is the "extension unavailable" signal


def w4a16_gemv(
    x2: torch.Tensor,
    qweight_t: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor,
    bias: torch.Tensor | None,
    group_size: int,
) -> torch.Tensor:
    """``x2 [M, K]`` fp16 (M <= 8, unit stride along K) -> ``[M, N]`` fp16."""
    return _gemv(x2, qweight_t, scales, qzeros, bias, group_size)


__all__ = ["w4a16_gemv"]
