"""Host-side schedule of the persistent decode chain (tf_decode_chain_plan; no GPU needed).

The kernel's correctness rests on these invariants of the unit schedule: every (op, row tile,
chunk) is covered by exactly one unit; each CTA's units are in op order (a CTA publishes its
arrival at op l only after finishing all its units of ops <= l); a tile split across CTAs has
pieces numbered in K order, each piece's sub-units flagged first / last; and the work per CTA is
balanced (whole tile groups where they divide evenly or the op is small, exact stream-K
otherwise)."""

from __future__ import annotations

import collections
import math

import pytest

from tokenforge_b200 import _lib, chain

H, INTER = 3584, 18944
QWEN_LAYER = [(4608, H), (H, H), (2 * INTER, H), (H, INTER)]
FIRST, LAST, SPLIT = 1, 2, 4


def _check_schedule(shapes: list[tuple[int, int]], m: int, ctas: int) -> list[chain.ChainUnit]:
    units = chain.plan(shapes, m, ctas)
    cover: collections.Counter = collections.Counter()
    last_op = collections.defaultdict(lambda: -1)
    pieces: dict[tuple[int, int], list[chain.ChainUnit]] = collections.defaultdict(list)
    for u in units:
        n, k = shapes[u.op]
        tiles, chunks = n // 32, math.ceil(k / 256)
        assert 0 <= u.cta < ctas
        assert u.op >= last_op[u.cta], "a CTA's units must be in op order"
        last_op[u.cta] = u.op
        assert u.rtiles in (1, 2, 4, 8, 16) and u.tile0 % u.rtiles == 0
        assert 0 <= u.c0 < u.c1 <= chunks
        for t in range(u.tile0, min(u.tile0 + u.rtiles, tiles)):
            for c in range(u.c0, u.c1):
                cover[(u.op, t, c)] += 1
        if u.flags & SPLIT:
            pieces[(u.op, u.tile0)].append(u)
        else:
            assert u.piece == -1 and u.pieces == 1
    for op, (n, k) in enumerate(shapes):
        for t in range(n // 32):
            for c in range(math.ceil(k / 256)):
                assert cover[(op, t, c)] == 1, (op, t, c)
    assert sum(cover.values()) == sum((n // 32) * math.ceil(k / 256) for n, k in shapes)
    for (op, _), us in pieces.items():
        us.sort(key=lambda u: u.c0)
        assert len({u.pieces for u in us}) == 1
        count = us[0].pieces
        assert count >= 2 and sorted({u.piece for u in us}) == list(range(count))
        for p in range(count):  # each piece: contiguous sub-units, first and last flagged once
            sub = [u for u in us if u.piece == p]
            assert sub[0].flags & FIRST and sub[-1].flags & LAST
            assert sum(1 for u in sub if u.flags & FIRST) == 1
            assert sum(1 for u in sub if u.flags & LAST) == 1
            assert all(a.c1 == b.c0 for a, b in zip(sub, sub[1:]))
            assert len({u.cta for u in sub}) == 1, "a piece stays on one CTA"
        assert [u.piece for u in us] == sorted(u.piece for u in us), "pieces in K order"
    return units


@pytest.mark.parametrize("m", [1, 2, 4, 8])
def test_qwen_decode_sweep_schedule(m: int) -> None:
    units = _check_schedule(QWEN_LAYER * 2, m, 148)
    per = collections.Counter()
    for u in units:
        per[(u.op, u.cta)] += (u.c1 - u.c0) * u.rtiles
    for op, (n, k) in enumerate(QWEN_LAYER):
        mean = (n // 32) * math.ceil(k / 256) / 148
        worst = max(per[(op, c)] for c in range(148))
        if op == 3:  # down (K = 18944): exact stream-K, 56 chunks on every CTA
            assert worst == mean == 56
        if op == 2:  # gate_up: 1184 tiles = 148 groups of 8, one per CTA
            assert worst == mean == 112
        assert worst <= max(1.35 * mean, 14)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_shards_schedule(world: int) -> None:
    """The shapes of one rank's shards (qkv and gate_up column shards, o and down K shards)."""
    shapes = [(4608 // world // 32 * 32, H), (H, H // world // 128 * 128),
              (2 * INTER // world // 32 * 32, H), (H, INTER // world // 128 * 128)]
    _check_schedule(shapes, 1, 148)


def test_small_and_ragged_shapes() -> None:
    # Qwen2.5-0.5B (K = 896 = 3.5 chunks), tiny N, a K that needs sub-units at M = 8.
    shapes = [(1152, 896), (896, 896), (9728, 896), (896, 4864), (32, 128), (64, 65536),
              (32, 8192)]
    for m in (1, 3, 8):
        units = _check_schedule(shapes, m, 148)
        if m == 8:
            assert any(not (u.flags & LAST) for u in units), "long K ranges are cut into sub-units"
    _check_schedule(shapes, 1, 7)


def test_unsupported_shapes_are_refused() -> None:
    with pytest.raises(_lib.KernelLibraryError, match="not supported"):
        chain.plan([(4600, 3584)], 1)  # N not a multiple of 32
    with pytest.raises(_lib.KernelLibraryError, match="not supported"):
        chain.plan([(4608, 3584 + 64)], 1)  # K not a multiple of 128
    with pytest.raises(_lib.KernelLibraryError, match="invalid argument"):
        chain.plan([(4608, 3584)], 9)  # more than 8 tokens
