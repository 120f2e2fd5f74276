"""GPU parity of the FP8-activation W4A16 linear (torch.ops.tokenforge.w4a16_linear_fp8), the
consumer of rmsnorm_fp8_quant's (e4m3 codes, per-token scale) that the reference lacks, against
the oracle's fp64 product of the decoded activations e4m3(q) * scale.

Tolerance: the decode GEMV stages the codes exactly and scales y in fp32, so it gets the W4A16
bound of tests/numerics/tolerance.py with x = e4m3(q) * scale. Above M = 8 the activations are
rounded once to fp16 (x16 = fp16(e4m3 * scale)) before the regular GEMM, which adds at most
sqrt(K) * 2^-11 * max|x| * max|w| (a random-walk bound on K rounding errors of relative size
2^-11) to that bound."""

from __future__ import annotations

import math

import pytest
import torch

import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from oracle import oracle
from tests.numerics import cases
from tests.numerics.tolerance import atol, error_scale

pytestmark = pytest.mark.gpu


def _fp8_inputs(m: int, k: int, seed: int, device: torch.device):  # type: ignore[no-untyped-def]
    x = cases.activations(m, k, seed).to(device)
    gamma = (1 + 0.1 * torch.randn(k, generator=torch.Generator().manual_seed(seed))).half()
    q, scale = torch.ops.tokenforge.rmsnorm_fp8_quant(x, gamma.to(device), 1e-6, None)
    return q, scale


def _check(y: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, w, bias=None) -> None:  # type: ignore[no-untyped-def]
    m, k = q.shape
    ref = oracle.w4a16_reference_fp8(q.view(torch.uint8).cpu(), scale.cpu(), w.qweight_t,
                                     w.scales, w.qzeros, w.group_size, bias)
    x_real = (oracle.e4m3_values(q.view(torch.uint8).cpu())
              * scale.cpu().double().reshape(-1, 1).expand(m, 1))
    w16 = oracle.dequantize_tf(w.qweight_t, w.scales, w.qzeros, w.group_size)
    tol = atol(x_real, w16, "cuda")
    if m > 8:
        tol += error_scale(x_real, w16) / 2  # sqrt(K) * 2^-11 * max|x| * max|w|
    err = float((y.cpu().double() - ref).abs().max())
    assert err <= tol, f"max abs err {err:.3e} > {tol:.3e} (m={m}, k={k})"


@pytest.mark.parametrize("m", [1, 3, 8, 16, 64])
@pytest.mark.parametrize(("n", "k"), [(4608, 3584), (256, 1024)])
def test_fp8_linear_matches_oracle(m: int, n: int, k: int, device: torch.device) -> None:
    w = cases.layer_weights(n, k, 5)
    q, scale = _fp8_inputs(m, k, m + k, device)
    y = torch.ops.tokenforge.w4a16_linear_fp8(q, scale, w.qweight_t.to(device),
                                              w.scales.to(device), w.qzeros.to(device), None, 128)
    assert y.shape == (m, n) and y.dtype == torch.float16
    _check(y, q, scale, w)


@pytest.mark.parametrize("g", [32, 64])
@pytest.mark.parametrize("m", [2, 24])
def test_fp8_linear_group_sizes_bias_and_static_scale(g: int, m: int, device: torch.device) -> None:
    n, k = 128, 512
    w = cases.layer_weights(n, k, 9, group_size=g)
    b = cases.bias(n, 9)
    x = cases.activations(m, k, 9).to(device)
    static = torch.tensor([0.02], dtype=torch.float32, device=device)
    gamma = torch.ones(k, dtype=torch.float16, device=device)
    q, s = torch.ops.tokenforge.rmsnorm_fp8_quant(x, gamma, 1e-6, static)
    y = torch.ops.tokenforge.w4a16_linear_fp8(q, s, w.qweight_t.to(device), w.scales.to(device),
                                              w.qzeros.to(device), b.to(device), g)
    _check(y, q, s.reshape(1).expand(1), w, b)


def test_fp8_linear_nan_code_stays_in_its_token(device: torch.device) -> None:
    n, k, m = 64, 256, 3
    w = cases.layer_weights(n, k, 2)
    q, scale = _fp8_inputs(m, k, 2, device)
    q = q.view(torch.uint8).clone()
    q[1, 17] = 0x7F  # e4m3fn NaN
    y = torch.ops.tokenforge.w4a16_linear_fp8(q, scale, w.qweight_t.to(device),
                                              w.scales.to(device), w.qzeros.to(device), None, 128)
    assert bool(torch.isnan(y[1]).all())
    assert bool(torch.isfinite(y[0]).all()) and bool(torch.isfinite(y[2]).all())


def test_fp8_linear_rejects_bad_inputs(device: torch.device) -> None:
    w = cases.layer_weights(64, 256, 1)
    args = (w.qweight_t.to(device), w.scales.to(device), w.qzeros.to(device), None, 128)
    q, scale = _fp8_inputs(2, 256, 1, device)
    with pytest.raises(TypeError, match="float8_e4m3fn"):
        torch.ops.tokenforge.w4a16_linear_fp8(q.float(), scale, *args)
    with pytest.raises(TypeError, match="fp32"):
        torch.ops.tokenforge.w4a16_linear_fp8(q, scale.half(), *args)
    with pytest.raises(ValueError, match="one value per token"):
        torch.ops.tokenforge.w4a16_linear_fp8(q, torch.ones(3, device=device), *args)
    assert math.isfinite(float(torch.ops.tokenforge.w4a16_linear_fp8(q, scale, *args).float().sum()))
