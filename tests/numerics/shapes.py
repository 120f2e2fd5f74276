"""Shape suite shared by the numerics tests, the tolerance calibration and the benchmark.

The layer shapes and M values are the reference's (tests/numerics/shapes.py:17-36): vLLM's
fused q/k/v and gate/up shapes of Qwen2.5-0.5B and -7B at TP=1, plus N not divisible by any
tile. The GPU tier runs the full suite.
"""

from __future__ import annotations

from typing import NamedTuple


class LinearShape(NamedTuple):
    model: str
    layer: str
    n: int
    k: int


QWEN25_05B = [
    LinearShape("qwen2.5-0.5b", "qkv_proj", 896 + 2 * 128, 896),
    LinearShape("qwen2.5-0.5b", "o_proj", 896, 896),
    LinearShape("qwen2.5-0.5b", "gate_up_proj", 2 * 4864, 896),
    LinearShape("qwen2.5-0.5b", "down_proj", 896, 4864),
]
QWEN25_7B = [
    LinearShape("qwen2.5-7b", "qkv_proj", 3584 + 2 * 512, 3584),
    LinearShape("qwen2.5-7b", "o_proj", 3584, 3584),
    LinearShape("qwen2.5-7b", "gate_up_proj", 2 * 18944, 3584),
    LinearShape("qwen2.5-7b", "down_proj", 3584, 18944),
]
RAGGED = [
    LinearShape("synthetic", "n_ragged_small", 200, 256),
    LinearShape("synthetic", "n_ragged", 1000, 1024),
]

M_SUITE = (1, 2, 3, 4, 7, 8, 15, 16, 31, 32, 64, 127, 128, 129)


def linear_shapes() -> list[LinearShape]:
    return QWEN25_05B + QWEN25_7B + RAGGED
