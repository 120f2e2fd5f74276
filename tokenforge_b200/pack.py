"""AWQ checkpoint layout and the kernel layout, with the conversions run on the GPU.

Same API and error behaviour as the reference's tokenforge/kernels/pack.py; every tensor
transformation runs in the sm_100a kernel library (CUDA tensors only).

AWQ GEMM layout (the on-disk checkpoint format):

* ``qweight`` int32 ``[K, N/8]``, eight 4-bit values per word packed along N;
* ``qzeros``  int32 ``[K/G, N/8]``, packed the same way;
* ``scales``  fp16  ``[K/G, N]``.

Nibble ``i`` of a word holds offset ``AWQ_ORDER[i]``, so offsets ``2j`` and ``2j+1`` sit in
nibbles ``j`` and ``j+4`` and one mask yields an fp16x2 pair of neighbours.

Kernel layout: ``qweight_t`` int32 ``[N, K/8]`` packed along K with the same interleave;
``scales`` and ``qzeros`` stay in AWQ layout. Dequantization is
``w[n, k] = fp16(q[n, k] - z[k/G, n]) * s[k/G, n]`` with a single rounding.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

AWQ_ORDER: tuple[int, ...] = (0, 2, 4, 6, 1, 3, 5, 7)
"""Nibble ``i`` of a packed word holds offset ``AWQ_ORDER[i]``."""

AWQ_REVERSE_ORDER: tuple[int, ...] = (0, 4, 1, 5, 2, 6, 3, 7)
"""Offset ``j`` lives in nibble ``AWQ_REVERSE_ORDER[j] == (j % 2) * 4 + j // 2``."""

PACK_FACTOR = 8
SUPPORTED_GROUP_SIZES: tuple[int, ...] = (32, 64, 128)


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what}: tokenforge_b200 runs on CUDA tensors only, got {t.device}")


def pack_int4(values: torch.Tensor) -> torch.Tensor:
    """Pack 4-bit values along the last dim into int32 words (AWQ interleave). GPU kernel."""
    if values.shape[-1] % PACK_FACTOR != 0:
        raise ValueError(f"last dim {values.shape[-1]} is not a multiple of {PACK_FACTOR}")
    _require_cuda(values, "pack_int4")
    if values.numel() and (int(values.min()) < 0 or int(values.max()) > 15):
        raise ValueError("int4 values must lie in [0, 15]")
    from tokenforge_b200 import ops

    return ops.pack_int4_cuda(values)


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`pack_int4`: int32 values in [0, 15]. GPU kernel."""
    if packed.dtype != torch.int32:
        raise TypeError(f"packed tensor must be int32, got {packed.dtype}")
    _require_cuda(packed, "unpack_int4")
    from tokenforge_b200 import ops

    return ops.unpack_int4_cuda(packed)


def awq_pack(intweight: torch.Tensor, zeros: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``intweight [K, N]`` and ``zeros [K/G, N]`` in [0, 15] -> AWQ ``(qweight, qzeros)``."""
    return pack_int4(intweight), pack_int4(zeros)


def awq_unpack(qweight: torch.Tensor) -> torch.Tensor:
    """AWQ ``qweight [K, N/8]`` -> int32 ``[K, N]`` (also for ``qzeros``)."""
    return unpack_int4(qweight)


@dataclass(frozen=True)
class W4A16Weights:
    """One linear layer in kernel layout."""

    qweight_t: torch.Tensor  # int32 [N, K/8], packed along K
    scales: torch.Tensor  # fp16 [K/G, N]
    qzeros: torch.Tensor  # int32 [K/G, N/8], AWQ layout
    group_size: int

    @property
    def n(self) -> int:
        return int(self.qweight_t.shape[0])

    @property
    def k(self) -> int:
        return int(self.qweight_t.shape[1]) * PACK_FACTOR

    def to(self, device: torch.device | str) -> W4A16Weights:
        return W4A16Weights(
            self.qweight_t.to(device), self.scales.to(device), self.qzeros.to(device), self.group_size
        )


def repack_awq_to_tf(qweight: torch.Tensor) -> torch.Tensor:
    """AWQ ``qweight [K, N/8]`` -> kernel ``qweight_t [N, K/8]`` (the awq_repack kernel)."""
    import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)

    return torch.ops.tokenforge.awq_repack(qweight)


def repack_tf_to_awq(qweight_t: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`repack_awq_to_tf`."""
    from tokenforge_b200 import ops

    return ops.awq_unrepack_cuda(qweight_t)


def validate_awq(
    qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, group_size: int
) -> None:
    """Raise ``ValueError`` naming the first reason the tensors are not a valid AWQ layer."""
    if qweight.dtype != torch.int32 or qzeros.dtype != torch.int32:
        raise ValueError("qweight and qzeros must be int32")
    if scales.dtype != torch.float16:
        raise ValueError(f"scales must be fp16, got {scales.dtype}")
    if group_size not in SUPPORTED_GROUP_SIZES:
        raise ValueError(f"group_size {group_size} not in {SUPPORTED_GROUP_SIZES}")
    k, n8 = qweight.shape
    if k % group_size != 0:
        raise ValueError(f"K={k} is not a multiple of group_size={group_size}")
    if tuple(qzeros.shape) != (k // group_size, n8):
        raise ValueError(f"qzeros shape {tuple(qzeros.shape)} != {(k // group_size, n8)}")
    if tuple(scales.shape) != (k // group_size, n8 * PACK_FACTOR):
        raise ValueError(
            f"scales shape {tuple(scales.shape)} != {(k // group_size, n8 * PACK_FACTOR)}"
        )


def pack_awq(
    qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, group_size: int
) -> W4A16Weights:
    """Load-time conversion of one AWQ layer into the kernel layout (one repack kernel)."""
    validate_awq(qweight, qzeros, scales, group_size)
    return W4A16Weights(
        qweight_t=repack_awq_to_tf(qweight),
        scales=scales.contiguous(),
        qzeros=qzeros.contiguous(),
        group_size=group_size,
    )


def unpack_to_awq(weights: W4A16Weights) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Inverse of :func:`pack_awq`: ``(qweight, qzeros, scales)``."""
    return repack_tf_to_awq(weights.qweight_t), weights.qzeros, weights.scales


def dequantize_tf(weights: W4A16Weights) -> torch.Tensor:
    """Kernel layout -> fp16 ``[N, K]`` (the w4a16_dequant kernel)."""
    import tokenforge_b200.ops  # noqa: F401

    return torch.ops.tokenforge.w4a16_dequant(
        weights.qweight_t, weights.scales, weights.qzeros, weights.group_size
    )


def awq_dequantize(
    qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, group_size: int
) -> torch.Tensor:
    """AWQ format -> fp16 ``[K, N]`` with the single-rounding dequant rule."""
    return dequantize_tf(pack_awq(qweight, qzeros, scales, group_size)).t()
