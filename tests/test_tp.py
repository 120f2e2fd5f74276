"""Tensor-parallel sharding (Qwen2.5-7B decode layers): shard bounds, shard contents against
the unsharded layer, and the row-parallel all-reduce / column-parallel gather over two gloo
ranks on CPU, with the oracle's fp64 product standing in for the kernel (the host logic is
what is under test; the kernels have their own GPU parity suite)."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle
from tests.numerics import cases
from tests.numerics.tolerance import atol
from tokenforge_b200 import tp
from tokenforge_b200.pack import W4A16Weights

G = 128


def test_split_even_sizes_and_order() -> None:
    assert tp.split_even(10, 3) == [(0, 4), (4, 7), (7, 10)]
    assert tp.split_even(4, 4) == [(0, 1), (1, 2), (2, 3), (3, 4)]
    assert tp.split_even(2, 4) == [(0, 1), (1, 2), (2, 2), (2, 2)]
    with pytest.raises(ValueError):
        tp.split_even(5, 0)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("n", [4608, 37888, 3584])
def test_column_bounds_cover_n_in_whole_words(n: int, world: int) -> None:
    b = tp.column_bounds(n, world)
    assert b[0][0] == 0 and b[-1][1] == n
    assert all(hi == lo for (_, hi), (lo, _) in zip(b, b[1:]))
    assert all(lo % 8 == 0 and hi % 8 == 0 for lo, hi in b)
    sizes = [hi - lo for lo, hi in b]
    assert max(sizes) - min(sizes) <= 8


def test_row_bounds_are_group_aligned_and_uneven_at_tp8() -> None:
    # Qwen2.5-7B o (K = 3584, 28 groups) and down (K = 18944, 148 groups) at TP = 8.
    o = tp.row_bounds(3584, G, 8)
    assert [(hi - lo) // G for lo, hi in o] == [4, 4, 4, 4, 3, 3, 3, 3]
    down = tp.row_bounds(18944, G, 8)
    assert [(hi - lo) // G for lo, hi in down] == [19, 19, 19, 19, 18, 18, 18, 18]
    assert tp.row_bounds(3584, G, 2) == [(0, 1792), (1792, 3584)]
    with pytest.raises(ValueError):
        tp.row_bounds(3584 + 64, G, 2)


def test_shards_hold_exactly_the_layer_slices() -> None:
    w = cases.layer_weights(64, 512, 7)
    full = oracle.dequantize_tf(w.qweight_t, w.scales, w.qzeros, G)
    for world in (2, 4):
        for r in range(world):
            col = tp.shard_layer(w, "column", r, world)
            n0, n1 = col.bounds
            got = oracle.dequantize_tf(col.weights.qweight_t, col.weights.scales,
                                       col.weights.qzeros, G)
            assert torch.equal(got.view(torch.int16), full[n0:n1].view(torch.int16))
            row = tp.shard_layer(w, "row", r, world)
            k0, k1 = row.bounds
            got = oracle.dequantize_tf(row.weights.qweight_t, row.weights.scales,
                                       row.weights.qzeros, G)
            assert torch.equal(got.view(torch.int16), full[:, k0:k1].view(torch.int16))


def test_bias_goes_to_column_slices_and_rank0_rows() -> None:
    w = cases.layer_weights(64, 256, 1)
    b = cases.bias(64, 1)
    assert torch.equal(tp.shard_layer(w, "column", 1, 2, b).bias, b[32:])
    assert tp.shard_layer(w, "row", 0, 2, b).bias is b
    assert tp.shard_layer(w, "row", 1, 2, b).bias is None
    with pytest.raises(ValueError):
        tp.shard_layer(w, "diagonal", 0, 2)


def _oracle_linear(x: torch.Tensor, w: W4A16Weights, b: torch.Tensor | None) -> torch.Tensor:
    return oracle.w4a16_reference(x, w.qweight_t, w.scales, w.qzeros, w.group_size, b).to(
        torch.float16)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _rank_main(rank: int, world: int, port: int, out: dict) -> None:  # type: ignore[type-arg]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m, n, k = 3, 64, 1024
        w = cases.layer_weights(n, k, 11)
        b = cases.bias(n, 11)
        x = cases.activations(m, k, 11)
        row = tp.shard_layer(w, "row", rank, world, b)
        y_row = tp.linear_shard(x, row, linear=_oracle_linear)
        col = tp.shard_layer(w, "column", rank, world, b)
        y_col = tp.linear_shard(x, col, linear=_oracle_linear)
        parts = [torch.empty_like(y_col) for _ in range(world)]
        dist.all_gather(parts, y_col)
        if rank == 0:
            out["row"] = y_row
            out["col"] = torch.cat(parts, dim=1)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_two_gloo_ranks_reassemble_the_full_layer(world: int) -> None:
    m, n, k = 3, 64, 1024
    w = cases.layer_weights(n, k, 11)
    b = cases.bias(n, 11)
    x = cases.activations(m, k, 11)
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_rank_main, args=(world, _free_port(), out), nprocs=world,
                           start_method="spawn")
        y_row, y_col = out["row"], out["col"]
    # Row-parallel: the all-reduce sums the ranks' fp16 partials; with two ranks the sum is
    # the same single rounding whatever the order.
    partials = [_oracle_linear(x[:, k0:k1], tp.shard_rows(w, k0, k1), b if r == 0 else None)
                for r, (k0, k1) in enumerate(tp.row_bounds(k, G, world))]
    assert torch.equal(y_row, partials[0] + partials[1])
    # Column-parallel: the gathered columns are the unsharded product, bit for bit.
    full = _oracle_linear(x, w, b)
    assert torch.equal(y_col, full)
    # And the row-parallel result is the full product within the W4A16 tolerance.
    ref = oracle.w4a16_reference(x, w.qweight_t, w.scales, w.qzeros, G, b)
    w16 = oracle.dequantize_tf(w.qweight_t, w.scales, w.qzeros, G)
    assert float((y_row.double() - ref).abs().max()) <= 2 * atol(x, w16, "cpu") + 2e-3


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_column_shards_pair_projections(world: int) -> None:
    """gate|up split part by part and on group boundaries: rank r holds [gate_r | up_r] whose
    dequantised rows are the full layer's, gate_r is the K range of its down shard, and the
    ranks' pieces tile every projection; q|k|v likewise in whole words, bias included."""
    inter, k = 1024, 256
    w = cases.layer_weights(2 * inter, k, 5)
    full = oracle.dequantize_tf(w.qweight_t, w.scales, w.qzeros, w.group_size)
    seen = []
    for rank in range(world):
        sh = tp.shard_fused_columns(w, (inter, inter), rank, world, group_aligned=True)
        (g0, g1), (u0, u1) = sh.pieces
        assert (g0, g1) == tp.row_bounds(inter, w.group_size, world)[rank]
        assert (u0 - inter, u1 - inter) == (g0, g1)
        got = oracle.dequantize_tf(sh.weights.qweight_t, sh.weights.scales, sh.weights.qzeros,
                                   w.group_size)
        assert torch.equal(got, torch.cat([full[g0:g1], full[u0:u1]]))
        seen += [(g0, g1), (u0, u1)]
    cover = sorted(seen)
    assert cover[0][0] == 0 and cover[-1][1] == 2 * inter
    assert all(a[1] == b[0] for a, b in zip(cover, cover[1:]))

    parts = (256, 64, 64)
    wq = cases.layer_weights(sum(parts), k, 6)
    bias = cases.bias(sum(parts), 6)
    fq = oracle.dequantize_tf(wq.qweight_t, wq.scales, wq.qzeros, wq.group_size)
    for rank in range(world):
        sh = tp.shard_fused_columns(wq, parts, rank, world, bias)
        rows = torch.cat([torch.arange(a, b) for a, b in sh.pieces])
        got = oracle.dequantize_tf(sh.weights.qweight_t, sh.weights.scales, sh.weights.qzeros,
                                   wq.group_size)
        assert torch.equal(got, fq[rows])
        assert sh.bias is not None and torch.equal(sh.bias, bias[rows])
    with pytest.raises(ValueError, match="add up"):
        tp.shard_fused_columns(wq, (256, 64), 0, world)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_block_shards_line_up(world: int) -> None:
    """The tensor-parallel block stack's shards at every TP size: the ranks' q/k/v and gate/up
    pieces tile each projection, gate_r and up_r have the width of the rank's down K shard and
    start on the same group, and o's K shards tile the hidden size in whole groups."""
    hidden, kv, inter, g = 3584, 512, 18944, 128
    q_cover, o_cover, gate_cover = [], [], []
    for rank in range(world):
        (q0, q1), (k0, k1), (v0, v1) = tp.fused_column_bounds((hidden, kv, kv), rank, world)
        assert (q1 - q0) % 8 == 0 and (k1 - k0) % 8 == 0 and v1 > v0
        q_cover.append((q0, q1))
        (g0, g1), (u0, u1) = tp.fused_column_bounds((inter, inter), rank, world, g)
        d0, d1 = tp.row_bounds(inter, g, world)[rank]
        assert (g0, g1) == (d0, d1) and (u0 - inter, u1 - inter) == (d0, d1)
        assert d0 % g == 0 and d1 % g == 0
        gate_cover.append((g0, g1))
        o_cover.append(tp.row_bounds(hidden, g, world)[rank])
    for cover, total in ((q_cover, hidden), (gate_cover, inter), (o_cover, hidden)):
        assert cover[0][0] == 0 and cover[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(cover, cover[1:]))


QWEN7B_HEADS = tp.AttentionHeads(28, 4, 128)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_attention_shards_follow_heads(world: int) -> None:
    """Qwen2.5-7B attention at every TP size its heads allow: each rank's q piece is whole heads,
    its width is the rank's o_proj K shard (whole groups), the KV pieces are the KV heads its q
    heads read, and the ranks' q pieces and o K ranges tile the hidden size."""
    h, kv, hd = 28, 4, 128
    q_cover, o_cover = [], []
    for rank in range(world):
        pieces, (k0, k1) = tp.attention_bounds(QWEN7B_HEADS, rank, world, 128)
        (q0, q1), (a0, a1), (b0, b1) = pieces
        assert (q0, q1) == (k0, k1), "q_r must be exactly o's K shard"
        assert q0 % hd == 0 and q1 % hd == 0 and (q1 - q0) % 128 == 0
        assert (a1 - a0) == (b1 - b0) and (a1 - a0) % hd == 0
        assert h * hd <= a0 and a1 <= h * hd + kv * hd and b0 - a0 == kv * hd
        first_kv = (a0 - h * hd) // hd
        for head in range(q0 // hd, q1 // hd):  # every q head reads a KV head the rank holds
            assert first_kv <= head // (h // kv) < first_kv + (a1 - a0) // hd
        q_cover.append((q0, q1))
        o_cover.append((k0, k1))
    for cover in (q_cover, o_cover):
        assert cover[0][0] == 0 and cover[-1][1] == h * hd
        assert all(a[1] == b[0] for a, b in zip(cover, cover[1:]))


def test_attention_shards_replicate_kv_heads_and_refuse_uneven_worlds() -> None:
    small = tp.AttentionHeads(8, 2, 64)
    kv_of = [tp.attention_bounds(small, r, 4)[0][1] for r in range(4)]
    assert kv_of[0] == kv_of[1] != kv_of[2] == kv_of[3]  # each KV head on two ranks
    with pytest.raises(ValueError, match="attention heads do not split"):
        tp.attention_bounds(QWEN7B_HEADS, 0, 8)  # 28 heads over 8 ranks
    with pytest.raises(ValueError, match="replicate"):
        tp.attention_bounds(tp.AttentionHeads(28, 4, 128), 0, 14)  # 14 ranks over 4 KV heads
    with pytest.raises(ValueError, match="whole groups"):
        tp.attention_bounds(tp.AttentionHeads(4, 1, 64), 0, 4, 128)


@pytest.mark.parametrize("world", [2, 4])
def test_shard_attention_holds_the_head_slices(world: int) -> None:
    heads = tp.AttentionHeads(8, 2, 32)
    q, kvw = 8 * 32, 2 * 32
    gen = torch.Generator().manual_seed(world)
    qkv = cases.layer_weights(q + 2 * kvw, 256, world, 64)
    o = cases.layer_weights(256, q, world, 64)
    bias = torch.randn(q + 2 * kvw, generator=gen).half()
    fq = oracle.dequantize_tf(qkv.qweight_t, qkv.scales, qkv.qzeros, 64)
    for rank in range(world):
        s_qkv, s_o = tp.shard_attention(qkv, o, heads, rank, world, bias)
        cols = torch.cat([torch.arange(a, b) for a, b in s_qkv.pieces])
        got = oracle.dequantize_tf(s_qkv.weights.qweight_t, s_qkv.weights.scales,
                                   s_qkv.weights.qzeros, 64)
        assert torch.equal(got, fq[cols])
        assert s_qkv.bias is not None and torch.equal(s_qkv.bias, bias[cols])
        assert s_o.weights.k == s_qkv.pieces[0][1] - s_qkv.pieces[0][0]
        assert s_o.bounds == s_qkv.pieces[0]
