"""The tcgen05 GEMM's stream-K schedule: layers whose 128-row tiles do not divide over the 148 SMs
(o and down of Qwen2.5-7B, N = 3584: 28 n-tiles) deal equal runs of K stages to the persistent
CTAs, once each CTA's run covers at least half a tile (M >= 1024 here; fewer tokens keep the
split-K plan); a tile cut between CTAs is written as fp32 partials and summed, with the bias, by the last
CTA to finish its piece, in stage order.

Checks, on every output element: the fp64 product of the oracle's dequantised weights within the
calibrated W4A16 tolerance, with and without bias; repeated calls bit-identical (the sum order
does not depend on which CTA finishes last); the device status word clear.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from oracle import oracle
from tests.numerics import cases
from tests.numerics.tolerance import atol
from tokenforge_b200 import _lib
from tokenforge_b200.config import launch_plan
from tokenforge_b200.pack import W4A16Weights

pytestmark = pytest.mark.gpu
G = 128


def _weights(n: int, k: int, seed: int) -> tuple[W4A16Weights, torch.Tensor]:
    qweight, qzeros, scales = cases.random_awq(n, k, seed)
    w = W4A16Weights(oracle.repack_awq_to_tf(qweight), scales, qzeros, G)
    return w, oracle.dequantize_tf(w.qweight_t, w.scales, w.qzeros, G)


# Shapes and token counts the planner deals as stream-K (tiles not divisible over the SMs, and
# each CTA's run at least half a tile): down and o of Qwen2.5-7B, and a K that cuts tiles at
# other offsets.
@pytest.mark.parametrize("n,k,ms", [
    (3584, 18944, (1024, 2048)),  # down
    (3584, 3584, (1024, 3000)),   # o
    (3584, 7168, (1024, 1500)),
    (3584, 512, (2048,)),         # o's K shard at TP 8 (tiles of 8 stages)
    (3584, 384, (2048,)),
])
def test_stream_k_tiles_match_fp64_and_repeat_bit_identically(
        n: int, k: int, ms: tuple[int, ...], device: torch.device) -> None:
    w, w16 = _weights(n, k, n + k)
    wd = w.to(device)
    w64 = w16.to(device).to(torch.float64)
    bias = cases.bias(n, 3).to(device)
    for m in ms:
        assert launch_plan(m, n, k, G).kernel == "tcgen05_gemm"
        x = cases.activations(m, k, m).to(device)
        ref = x.to(torch.float64) @ w64.t()
        tol = atol(x.cpu(), w16, "cuda")
        for b in (None, bias):
            y = torch.ops.tokenforge.w4a16_linear(x, wd.qweight_t, wd.scales, wd.qzeros, b, G,
                                                  "cuda")
            want = ref if b is None else ref + b.to(torch.float64)
            err = float((y.to(torch.float64) - want).abs().max())
            # The reference's rule scales with sqrt(K); at K = 384-512 it falls below the fp16
            # rounding of the largest outputs (|y| ~ 10), so half an ulp of max|y| is added.
            bound = tol + float(want.abs().max()) * 2.0**-11
            assert err <= bound, f"N={n} K={k} M={m} bias={b is not None}: {err:.3e} > {bound:.3e}"
            again = torch.ops.tokenforge.w4a16_linear(x, wd.qweight_t, wd.scales, wd.qzeros, b, G,
                                                      "cuda")
            assert torch.equal(y, again), f"N={n} K={k} M={m}: repeated call differs"
    code = ctypes.c_int(-1)
    _lib.check("tf_device_error", _lib.lib().tf_device_error(ctypes.byref(code)))
    assert code.value == 0
