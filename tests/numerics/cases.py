"""Deterministic cases: the same seeds and generators as the reference's
tests/numerics/cases.py:17-39, so the inputs here are the reference's inputs.

Weights come from min-max AWQ quantization of ``randn * 0.02`` (the oracle's restatement of
awq_quantize, pinned by the golden vectors), repacked to the kernel layout by the oracle. The
results are CPU tensors; tests move them to the GPU.
"""

from __future__ import annotations

import functools
import zlib

import torch

from oracle import oracle
from tokenforge_b200.pack import W4A16Weights

GROUP_SIZE = 128
TEST_SEEDS = (0,)
CALIBRATION_SEEDS = (0, 1, 2, 3, 4)


def _seed(*parts: object) -> int:
    return zlib.crc32(repr(parts).encode())


@functools.lru_cache(maxsize=16)
def layer_weights(n: int, k: int, seed: int, group_size: int = GROUP_SIZE) -> W4A16Weights:
    gen = torch.Generator().manual_seed(_seed("w", n, k, seed, group_size))
    weight = torch.randn((n, k), generator=gen) * 0.02
    qweight, qzeros, scales = oracle.awq_quantize(weight, group_size)
    return W4A16Weights(oracle.repack_awq_to_tf(qweight), scales, qzeros, group_size)


def activations(m: int, k: int, seed: int) -> torch.Tensor:
    gen = torch.Generator().manual_seed(_seed("x", m, k, seed))
    return torch.randn((m, k), generator=gen).to(torch.float16)


def bias(n: int, seed: int) -> torch.Tensor:
    gen = torch.Generator().manual_seed(_seed("b", n, seed))
    return (torch.randn((n,), generator=gen) * 0.1).to(torch.float16)


def random_awq(n: int, k: int, seed: int, group_size: int = GROUP_SIZE):  # type: ignore[no-untyped-def]
    """Uniform random AWQ layer as BASELINE config 0: q, z uniform in [0, 15], scales
    uniform(0.002, 0.02). Returns (qweight [K, N/8], qzeros [K/G, N/8], scales [K/G, N])."""
    gen = torch.Generator().manual_seed(_seed("awq", n, k, seed, group_size))
    q = torch.randint(0, 16, (k, n), generator=gen, dtype=torch.int32)
    z = torch.randint(0, 16, (k // group_size, n), generator=gen, dtype=torch.int32)
    s = (torch.rand((k // group_size, n), generator=gen) * 0.018 + 0.002).to(torch.float16)
    qweight, qzeros = oracle.awq_pack(q, z)
    return qweight, qzeros, s
