"""Full-width parity at the benchmark's own sizes: every output element of the Qwen2.5-7B layers
against the fp64 product of the oracle's dequantised weights, computed on the device.

* BASELINE config 2, the prefill GEMM: gate_up (N 37888, K 3584) and down (N 3584, K 18944) at
  M in {256, 1024, 4096}. These M run the persistent tcgen05 schedule with 256-token tiles and
  several m-tiles per n-tile, which the shape suite (M <= 129) never reaches.
* BASELINE configs 0 and 3, the decode linears qkv, o, gate_up and down at M = 1 and 8 (the
  decode GEMV), 16 (the 16-token GEMV) and 32 / 64 (the small-token tcgen05 GEMM).

Weights follow the configs' distribution (q and z uniform in [0, 15], scales uniform in
[0.002, 0.02]), packed and repacked by the oracle; activations are fp16 ~N(0, 1). The bar is the
reference's: |y - y_fp64| <= c * sqrt(K) * 2^-10 * max|x| * max|w| (tests/numerics/tolerance.py)
with the calibrated cuda constant, on all M * N outputs.
"""

from __future__ import annotations

import functools

import pytest
import torch

import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from oracle import oracle
from tests.numerics import cases
from tests.numerics.tolerance import atol
from tokenforge_b200.config import launch_plan
from tokenforge_b200.pack import W4A16Weights

pytestmark = pytest.mark.gpu
G = 128
QWEN7B = {"qkv": (4608, 3584), "o": (3584, 3584), "gate_up": (37888, 3584), "down": (3584, 18944)}


@functools.lru_cache(maxsize=1)
def _layer(name: str) -> tuple[W4A16Weights, torch.Tensor]:
    """(kernel-layout weights, oracle fp16 dequantisation) on the CPU."""
    n, k = QWEN7B[name]
    qweight, qzeros, scales = cases.random_awq(n, k, 2)
    w = W4A16Weights(oracle.repack_awq_to_tf(qweight), scales, qzeros, G)
    return w, oracle.dequantize_tf(w.qweight_t, w.scales, w.qzeros, G)


def _full_check(name: str, ms: tuple[int, ...], device: torch.device) -> None:
    w, w16 = _layer(name)
    wd = w.to(device)
    w64 = w16.to(device).to(torch.float64)
    for m in ms:
        x = cases.activations(m, w.k, m)
        y = torch.ops.tokenforge.w4a16_linear(x.to(device), wd.qweight_t, wd.scales, wd.qzeros,
                                              None, G, "cuda")
        assert y.shape == (m, w.n) and y.dtype == torch.float16
        ref = x.to(device).to(torch.float64) @ w64.t()
        err = float((y.to(torch.float64) - ref).abs().max())
        tol = atol(x, w16, "cuda")
        assert err <= tol, f"{name} M={m}: max abs err {err:.3e} > tol {tol:.3e} over {m * w.n} outputs"
        assert bool(torch.isfinite(y).all())
        del y, ref
    del w64, wd
    torch.cuda.empty_cache()


@pytest.mark.parametrize("name", ["gate_up", "down"])
def test_config2_prefill_gemm_full_width(name: str, device: torch.device) -> None:
    n, k = QWEN7B[name]
    for m in (256, 1024, 4096):
        plan = launch_plan(m, n, k, G)
        assert plan.kernel == "tcgen05_gemm" and plan.tile_m == 256, plan
    # M = 1024 and 4096 hold 4 and 16 token tiles per weight tile.
    _full_check(name, (256, 1024, 4096), device)


@pytest.mark.parametrize("name", list(QWEN7B))
def test_decode_layers_full_width(name: str, device: torch.device) -> None:
    _full_check(name, (1, 8, 16, 32, 64), device)


def test_m300_route_values(device: torch.device) -> None:
    """The reference routes M > 128 to dequant + cuBLAS and checks its values at M = 300
    (tests/numerics/test_w4a16.py:99-105); here that M runs the tcgen05 GEMM, full width."""
    w = cases.layer_weights(1024, 1024, 0)
    w16 = oracle.dequantize_tf(w.qweight_t, w.scales, w.qzeros, G)
    x = cases.activations(300, 1024, 0)
    wd = w.to(device)
    y = torch.ops.tokenforge.w4a16_linear(x.to(device), wd.qweight_t, wd.scales, wd.qzeros,
                                          None, G, "cuda")
    ref = x.to(torch.float64) @ w16.to(torch.float64).t()
    err = float((y.cpu().to(torch.float64) - ref).abs().max())
    assert err <= atol(x, w16, "cuda")
