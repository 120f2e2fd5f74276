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

Fused column-parallel layers (q|k|v, gate|up) are split part by part (:func:`shard_fused_columns`):
every rank holds its slice of each projection, so a rank's gate and up columns pair up for the
SiLU product, and with group-aligned parts its intermediate slice is exactly the K range of its
down_proj row shard. A q|k|v layer that feeds real attention is split on whole heads instead
(:func:`shard_attention`): the rank's q heads, their KV heads (replicated when there are more
ranks than KV heads) and o_proj's K range over the same q heads.
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
    bounds: tuple[int, int]  # columns (column-parallel; a fused layer's first piece) or K range
    bias: torch.Tensor | None
    # Fused column-parallel layers: the global column range of each piece, in the order the
    # pieces are concatenated in ``weights`` (one range per projection).
    pieces: tuple[tuple[int, int], ...] = ()


def fused_column_bounds(parts: tuple[int, ...] | list[int], rank: int, world: int,
                        group_size: int | None = None) -> list[tuple[int, int]]:
    """Global column ranges of ``rank``'s pieces of a layer whose output concatenates
    projections of widths ``parts``: each projection split on its own, in whole 8-column words,
    or in whole ``group_size``-column groups when given (so that the pieces line up with
    :func:`row_bounds` of the next layer's K)."""
    out, off = [], 0
    for p in parts:
        a, b = (row_bounds(p, group_size, world) if group_size else column_bounds(p, world))[rank]
        out.append((off + a, off + b))
        off += p
    return out


@dataclass(frozen=True)
class AttentionHeads:
    """Head layout of a grouped-query attention block. The fused q|k|v projection's output is
    ``[q (num_heads * head_dim) | k (num_kv_heads * head_dim) | v (same)]`` and o_proj's K is
    the attention output, ``num_heads * head_dim`` wide (Qwen2.5-7B: 28 / 4 heads of 128)."""

    num_heads: int
    num_kv_heads: int
    head_dim: int

    @property
    def parts(self) -> tuple[int, int, int]:
        kv = self.num_kv_heads * self.head_dim
        return (self.num_heads * self.head_dim, kv, kv)


def attention_bounds(heads: AttentionHeads, rank: int, world: int,
                     group_size: int | None = None) -> tuple[list[tuple[int, int]], tuple[int, int]]:
    """Rank ``rank``'s pieces of the fused q|k|v columns (global column ranges, q then k then
    v) and its K range of o_proj, split on whole heads so that the rank's attention output is
    exactly the input of its o_proj shard.

    The rules are the usual tensor-parallel GQA rules (vLLM's): the q heads split evenly, so
    ``world`` must divide ``num_heads``; the KV heads split evenly when ``world <= num_kv_heads``
    (``world`` must divide them), else each KV head is replicated on ``world / num_kv_heads``
    consecutive ranks (``world`` must be a multiple of ``num_kv_heads``). Rank r's q heads then
    read only its own KV heads. With ``group_size``, o's K shard must be whole groups."""
    h, kv, hd = heads.num_heads, heads.num_kv_heads, heads.head_dim
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if h % world:
        raise ValueError(f"{h} attention heads do not split over {world} ranks")
    if world <= kv:
        if kv % world:
            raise ValueError(f"{kv} KV heads do not split over {world} ranks")
        k0, k1 = rank * kv // world, (rank + 1) * kv // world
    else:
        if world % kv:
            raise ValueError(f"{world} ranks cannot replicate {kv} KV heads evenly")
        k0 = rank // (world // kv)
        k1 = k0 + 1
    q0, q1 = rank * h // world, (rank + 1) * h // world
    if group_size and ((q1 - q0) * hd) % group_size:
        raise ValueError(f"o_proj's K shard of {(q1 - q0) * hd} columns is not whole groups of "
                         f"{group_size}")
    qw, kvw = h * hd, kv * hd
    pieces = [(q0 * hd, q1 * hd), (qw + k0 * hd, qw + k1 * hd), (qw + kvw + k0 * hd, qw + kvw + k1 * hd)]
    return pieces, (q0 * hd, q1 * hd)


def shard_column_pieces(w: W4A16Weights, pieces: list[tuple[int, int]],
                        bias: torch.Tensor | None = None) -> LayerShard:
    """Column-parallel shard holding the given global column ranges, concatenated in order."""
    shards = [shard_columns(w, a, b) for a, b in pieces]
    weights = W4A16Weights(
        torch.cat([s.qweight_t for s in shards], dim=0),
        torch.cat([s.scales for s in shards], dim=1),
        torch.cat([s.qzeros for s in shards], dim=1),
        w.group_size,
    )
    b = None if bias is None else torch.cat([bias[a:bb] for a, bb in pieces]).contiguous()
    return LayerShard("column", weights, pieces[0], b, tuple(pieces))


def shard_attention(qkv: W4A16Weights, o: W4A16Weights, heads: AttentionHeads, rank: int,
                    world: int, qkv_bias: torch.Tensor | None = None,
                    o_bias: torch.Tensor | None = None) -> tuple[LayerShard, LayerShard]:
    """Rank ``rank``'s q|k|v and o_proj shards, split on whole heads (:func:`attention_bounds`):
    the q|k|v shard outputs ``[q_r | k_r | v_r]`` and the o shard's K range is the columns of
    q_r's heads."""
    if sum(heads.parts) != qkv.n or heads.parts[0] != o.k:
        raise ValueError(f"heads {heads} do not match q|k|v N={qkv.n} and o K={o.k}")
    pieces, (k0, k1) = attention_bounds(heads, rank, world, o.group_size)
    b = o_bias if (o_bias is not None and rank == 0) else None
    return (shard_column_pieces(qkv, pieces, qkv_bias),
            LayerShard("row", shard_rows(o, k0, k1), (k0, k1), b))


def shard_fused_columns(w: W4A16Weights, parts: tuple[int, ...] | list[int], rank: int, world: int,
                        bias: torch.Tensor | None = None, group_aligned: bool = False) -> LayerShard:
    """Column-parallel shard of a fused layer (q|k|v with parts (q, k, v); gate|up with parts
    (I, I)): rank r holds its slice of every projection, concatenated in part order, so its
    output is [q_r | k_r | v_r] or [gate_r | up_r]. ``group_aligned`` splits each projection in
    whole quantization groups of columns (for gate|up, so that gate_r matches down's K shard).
    This split ignores attention heads: a q|k|v layer feeding real attention is split with
    :func:`shard_attention` instead."""
    if sum(parts) != w.n:
        raise ValueError(f"parts {tuple(parts)} do not add up to N={w.n}")
    pieces = fused_column_bounds(parts, rank, world, w.group_size if group_aligned else None)
    return shard_column_pieces(w, pieces, bias)


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


class PeerMailbox:
    """Per-rank mailboxes for the row-parallel all-reduce fused into the decode GEMV
    (``tf_w4a16_linear_allreduce``): each rank allocates one, the IPC handles are all-gathered
    over ``group`` and every peer's mailbox is mapped into this process. Collective: every rank
    constructs it (and calls :meth:`close`) in the same order. Ranks must sit on distinct GPUs
    (the kernels of different ranks wait on each other)."""

    def __init__(self, group=None, max_m: int = 8, max_n: int = 65536,  # type: ignore[no-untyped-def]
                 device: torch.device | None = None) -> None:
        import ctypes

        import torch.distributed as dist

        from tokenforge_b200 import _lib

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if not 2 <= self.world <= _lib.TF_MAX_PEERS:
            raise ValueError(f"peer all-reduce needs 2..{_lib.TF_MAX_PEERS} ranks, got {self.world}")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        props = torch.cuda.get_device_properties(self.device)
        ids: list[object] = [None] * self.world
        dist.all_gather_object(ids, str(getattr(props, "uuid", self.device)), group=group)
        if len(set(ids)) != self.world:
            raise RuntimeError("peer all-reduce ranks must be on distinct GPUs")
        lib = _lib.lib()
        self.bytes = int(lib.tf_peer_mailbox_bytes(self.world, max_m, max_n))
        if self.bytes == 0:
            raise ValueError(f"bad mailbox shape: world={self.world} max_m={max_m} max_n={max_n}")
        handle = (ctypes.c_char * _lib.TF_IPC_HANDLE_BYTES)()
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check("tf_peer_mailbox_alloc",
                       lib.tf_peer_mailbox_alloc(self.bytes, ctypes.byref(own), handle))
        handles: list[object] = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.peers = _lib.TfPeerSet()
        self.peers.rank, self.peers.world = self.rank, self.world
        self.peers.max_m, self.peers.max_n = max_m, max_n
        self._opened: list[int] = []
        with torch.cuda.device(self.device):
            for q in range(self.world):
                if q == self.rank:
                    self.peers.mailbox[q] = own.value
                    continue
                hq = (ctypes.c_char * _lib.TF_IPC_HANDLE_BYTES).from_buffer_copy(handles[q])  # type: ignore[arg-type]
                mq = ctypes.c_void_p()
                _lib.check("tf_peer_mailbox_open", lib.tf_peer_mailbox_open(hq, ctypes.byref(mq)))
                self.peers.mailbox[q] = mq.value
                self._opened.append(int(mq.value))  # type: ignore[arg-type]
        self._own = int(own.value)  # type: ignore[arg-type]
        dist.barrier(group=group)

    def error(self) -> int:
        """Device-side error word (1 = a peer wait gave up), cleared on read."""
        import ctypes

        from tokenforge_b200 import _lib

        out = ctypes.c_int(0)
        with torch.cuda.device(self.device):
            _lib.check("tf_peer_mailbox_error",
                       _lib.lib().tf_peer_mailbox_error(ctypes.c_void_p(self._own), ctypes.byref(out)))
        return int(out.value)

    def close(self) -> None:
        import torch.distributed as dist

        from tokenforge_b200 import _lib

        if self._own == 0:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no peer still writes into our mailbox
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            for m in self._opened:
                _lib.check("tf_peer_mailbox_close", lib.tf_peer_mailbox_close(m))
            _lib.check("tf_peer_mailbox_free", lib.tf_peer_mailbox_free(self._own))
        self._opened, self._own = [], 0

    def supports(self, m: int, n: int, k: int, group_size: int) -> bool:
        """Whether every rank's row shard of an ``[m, k] x [n, k]`` layer runs the fused kernel
        (the same answer on all ranks, from the global shape alone, so that no rank waits for a
        peer that took the unfused path)."""
        from tokenforge_b200.config import launch_plan

        if m > self.peers.max_m or n > self.peers.max_n:
            return False
        for k0, k1 in row_bounds(k, group_size, self.world):
            try:
                pl = launch_plan(m, n, k1 - k0, group_size)
            except ValueError:
                return False
            if (pl.kernel != "gemv" or pl.split_k != pl.cluster or pl.cluster > 2
                    or pl.grid_x * pl.split_k > 2 * 148):
                return False
        return True

    def linear(self, x: torch.Tensor, w: W4A16Weights, bias: torch.Tensor | None) -> torch.Tensor | None:
        """Fused decode GEMV + all-reduce of this rank's row shard; None when the shape is not
        served by the fused kernel (the caller then uses the plain linear + a collective)."""
        import ctypes

        from tokenforge_b200 import _lib
        from tokenforge_b200.linear import _aligned_rows, _check_inputs, _require

        m, n, k = _check_inputs(x, w.qweight_t, w.scales, w.qzeros, w.group_size)
        for name, t in (("x", x), ("qweight_t", w.qweight_t), ("scales", w.scales),
                        ("qzeros", w.qzeros)):
            _require(t, name)
        y = torch.empty((m, n), dtype=torch.float16, device=x.device)
        x = _aligned_rows(x)
        lib = _lib.lib()
        wsb = int(lib.tf_w4a16_workspace_bytes(m, n, k, w.group_size))
        ws = torch.empty(wsb, dtype=torch.uint8, device=x.device) if wsb else None
        with torch.cuda.device(x.device):
            status = lib.tf_w4a16_linear_allreduce(
                x.data_ptr(), m, k, x.stride(0), w.qweight_t.data_ptr(), w.scales.data_ptr(),
                w.qzeros.data_ptr(), _lib.ptr(None if bias is None else bias.contiguous()), n,
                w.group_size, y.data_ptr(), n, _lib.ptr(ws), wsb, ctypes.byref(self.peers),
                _lib.stream_ptr(x.device))
        if status == _lib.TF_ERR_UNSUPPORTED:
            return None
        _lib.check("tf_w4a16_linear_allreduce", status)
        return y


def linear_shard(x: torch.Tensor, shard: LayerShard, group=None, linear=None,  # type: ignore[no-untyped-def]
                 peers: PeerMailbox | None = None) -> torch.Tensor:
    """Run one rank's shard. Column-parallel returns this rank's columns; row-parallel takes
    the full activations, uses its K slice, and sums the ranks' partials: through ``peers``
    (the all-reduce fused into the decode GEMV) when given and the shape allows it, else with
    an all-reduce of the fp16 partials over ``group``.

    ``linear(x, weights, bias) -> fp16 [M, N]`` computes the local product; by default the
    kernel library's launch table (GEMVs up to M = 16, tensor-core GEMM above)."""
    import torch.distributed as dist

    if linear is None:
        from tokenforge_b200.linear import w4a16_gemm

        def linear(xx, w, b):  # type: ignore[no-untyped-def]
            return w4a16_gemm(xx, w.qweight_t, w.scales, w.qzeros, w.group_size, b)

    w = shard.weights
    if shard.kind == "column":
        return linear(x, w, shard.bias)
    k0, k1 = shard.bounds
    if peers is not None and peers.supports(x.shape[0], w.n, x.shape[1], w.group_size):
        fused = peers.linear(x[:, k0:k1], w, shard.bias)
        if fused is None:
            raise RuntimeError("fused all-reduce refused a shape its plan check admitted")
        return fused
    y = linear(x[:, k0:k1], w, shard.bias)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y
