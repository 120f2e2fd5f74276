"""Tensor-parallel sharding of W4A16 layers over one process per GPU.

Qwen2.5-7B decode layers shard Megatron-style:

* column-parallel ``qkv`` and ``gate_up``: rank r owns a contiguous block of output columns
  (whole 8-column words), so it holds ``qweight_t[n0:n1]``, ``scales[:, n0:n1]`` and
  ``qzeros[:, n0/8:n1/8]`` and needs no communication;
* row-parallel ``o`` and ``down``: rank r owns a contiguous block of K made of whole
  quantization groups, ``qweight_t[:, k0/8:k1/8]``, ``scales[g0:g1]``, ``qzeros[g0:g1]``,
  computes an fp16 partial ``[M, N]`` from its slice of the activations, and the ranks sum
  the partials with an NCCL all-reduce (bias added on rank 0 only).

K per rank must be a multiple of the group size. When the group count does not divide by the
world size (o: 28 groups and down: 148 groups at TP = 8) the shards are uneven: the first
``groups % world`` ranks take one extra group. The reference has no multi-GPU code; this module
is the partitioning its BASELINE configs 3 and 4 call for.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from tokenforge_b200.pack import PACK_FACTOR, W4A16Weights


def split_even(total: int, parts: int) -> list[tuple[int, int]]:
    """[start, end) of ``parts`` contiguous chunks of ``total`` units, sizes differing by <= 1
    (larger chunks first)."""
    if parts < 1 or total < 0:
        raise ValueError(f"cannot split {total} units into {parts} parts")
    base, extra = divmod(total, parts)
    out, start = [], 0
    for r in range(parts):
        size = base + (1 if r < extra else 0)
        out.append((start, start + size))
        start += size
    return out


def column_bounds(n: int, world: int) -> list[tuple[int, int]]:
    """Output-column ranges per rank, in whole 8-column words."""
    if n % PACK_FACTOR:
        raise ValueError(f"N={n} is not a multiple of {PACK_FACTOR}")
    return [(a * PACK_FACTOR, b * PACK_FACTOR) for a, b in split_even(n // PACK_FACTOR, world)]


def row_bounds(k: int, group_size: int, world: int) -> list[tuple[int, int]]:
    """K ranges per rank, in whole quantization groups."""
    if k % group_size:
        raise ValueError(f"K={k} is not a multiple of group_size={group_size}")
    return [(a * group_size, b * group_size) for a, b in split_even(k // group_size, world)]


def shard_columns(w: W4A16Weights, n0: int, n1: int) -> W4A16Weights:
    if n0 % PACK_FACTOR or n1 % PACK_FACTOR:
        raise ValueError("column shard bounds must be multiples of 8")
    return W4A16Weights(
        w.qweight_t[n0:n1].contiguous(),
        w.scales[:, n0:n1].contiguous(),
        w.qzeros[:, n0 // PACK_FACTOR : n1 // PACK_FACTOR].contiguous(),
        w.group_size,
    )


def shard_rows(w: W4A16Weights, k0: int, k1: int) -> W4A16Weights:
    g = w.group_size
    if k0 % g or k1 % g:
        raise ValueError(f"row shard bounds must be multiples of group_size={g}")
    return W4A16Weights(
        w.qweight_t[:, k0 // PACK_FACTOR : k1 // PACK_FACTOR].contiguous(),
        w.scales[k0 // g : k1 // g].contiguous(),
        w.qzeros[k0 // g : k1 // g].contiguous(),
        g,
    )


@dataclass(frozen=True)
class LayerShard:
    """One rank's piece of a linear layer."""

    kind: str  # "column" or "row"
    weights: W4A16Weights
    bounds: tuple[int, int]  # columns (column-parallel) or K range (row-parallel)
    bias: torch.Tensor | None


def shard_layer(
    w: W4A16Weights, kind: str, rank: int, world: int, bias: torch.Tensor | None = None
) -> LayerShard:
    if kind == "column":
        n0, n1 = column_bounds(w.n, world)[rank]
        b = None if bias is None else bias[n0:n1].contiguous()
        return LayerShard(kind, shard_columns(w, n0, n1), (n0, n1), b)
    if kind == "row":
        k0, k1 = row_bounds(w.k, w.group_size, world)[rank]
        b = bias if (bias is not None and rank == 0) else None
        return LayerShard(kind, shard_rows(w, k0, k1), (k0, k1), b)
    raise ValueError(f"kind must be 'column' or 'row', got {kind!r}")


def linear_shard(x: torch.Tensor, shard: LayerShard, group=None, linear=None) -> torch.Tensor:  # type: ignore[no-untyped-def]
    """Run one rank's shard. Column-parallel returns this rank's columns; row-parallel takes
    the full activations, uses its K slice, and all-reduces the fp16 partials in place.

    ``linear(x, weights, bias) -> fp16 [M, N]`` computes the local product; by default the
    kernel library's launch table (GEMV for M <= 8, tensor-core GEMM above)."""
    import torch.distributed as dist

    if linear is None:
        from tokenforge_b200.ops import w4a16_gemm

        def linear(xx, w, b):  # type: ignore[no-untyped-def]
            return w4a16_gemm(xx, w.qweight_t, w.scales, w.qzeros, w.group_size, b)

    w = shard.weights
    if shard.kind == "column":
        return linear(x, w, shard.bias)
    k0, k1 = shard.bounds
    y = linear(x[:, k0:k1], w, shard.bias)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y
