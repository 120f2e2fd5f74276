"""GPU parity for fused RMSNorm + e4m3 quantization, mirroring the reference's
tests/numerics/test_rmsnorm_fp8.py, plus the BASELINE config-1 shapes (outlier channels)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import tokenforge_b200.ops  # noqa: F401
from oracle import oracle
from tokenforge_b200.ops import cast_e4m3, rmsnorm_fp8_quant_2d

pytestmark = pytest.mark.gpu
EPS = 1e-6
FP8_MAX = 448.0
GOLDEN = Path(__file__).resolve().parent / "golden"


def _inputs(t: int, h: int, seed: int, scale: float = 2.0) -> tuple[torch.Tensor, torch.Tensor]:
    gen = torch.Generator().manual_seed(seed)
    x = (torch.randn((t, h), generator=gen) * scale).to(torch.float16)
    w = (torch.rand((h,), generator=gen) + 0.5).to(torch.float16)
    return x, w


def _codes(q: torch.Tensor) -> torch.Tensor:
    return q.detach().cpu().view(torch.uint8).to(torch.int16)


def _assert_within_one_code(q: torch.Tensor, ref: torch.Tensor) -> None:
    """Same sign, magnitudes at most one e4m3 code apart, < 5% of codes differing
    (the reference's criterion, test_rmsnorm_fp8.py:41-51)."""
    a, b = _codes(q), ref.to(torch.int16)
    ma, mb = a & 0x7F, b & 0x7F
    sign_ok = ((a & 0x80) == (b & 0x80)) | ((ma == 0) & (mb <= 1)) | ((mb == 0) & (ma <= 1))
    assert bool(sign_ok.all()), "sign mismatch"
    diff = (ma - mb).abs()
    assert int(diff.max()) <= 1, f"max code distance {int(diff.max())}"
    assert float((diff > 0).float().mean()) < 0.05, "too many one-code differences"


def _hf_rmsnorm(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    xf = x.to(torch.float32)
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    return (xf * torch.rsqrt(var + EPS)).to(x.dtype) * w


@pytest.mark.parametrize("h", [896, 3584, 1000, 4096, 5000, 100])
@pytest.mark.parametrize("t", [1, 7, 33])
def test_dynamic_per_token(t: int, h: int, device: torch.device) -> None:
    x, w = _inputs(t, h, seed=t * h)
    q, s = rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS)
    q_ref, s_ref = oracle.rmsnorm_fp8(x, w, EPS)
    assert q.dtype == torch.float8_e4m3fn
    assert s.shape == (t, 1)
    # Bit-exact with the oracle (same IEEE operations, order-independent sum of squares) ...
    assert torch.equal(_codes(q), q_ref.to(torch.int16))
    assert torch.equal(s.cpu(), s_ref)
    # ... and the reference's own acceptance criteria.
    assert float(((s.cpu() - s_ref).abs() / s_ref).max()) <= 1e-3
    _assert_within_one_code(q, q_ref)
    assert bool((q.cpu().float().abs().amax(dim=-1) == FP8_MAX).all())
    y = _hf_rmsnorm(x, w).float()
    deq = q.cpu().float() * s.cpu()
    rel = (deq - y).abs() / y.abs().clamp(min=float(s_ref.max()))
    assert float(rel.max()) <= 2.0**-3


@pytest.mark.parametrize("t", [1, 256, 4096])
def test_config1_outlier_channels(t: int, device: torch.device) -> None:
    """x ~ N(0, 1) with 8 fixed outlier channels x20, gamma ~ N(1, 0.1)."""
    h = 3584
    gen = torch.Generator().manual_seed(2024)
    x = torch.randn((t, h), generator=gen)
    chans = torch.randperm(h, generator=gen)[:8]
    x[:, chans] *= 20
    x = x.to(torch.float16)
    w = (1 + 0.1 * torch.randn(h, generator=gen)).to(torch.float16)
    q, s = rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS)
    q_ref, s_ref = oracle.rmsnorm_fp8(x, w, EPS)
    assert torch.equal(_codes(q), q_ref.to(torch.int16))
    assert torch.equal(s.cpu(), s_ref)


def test_matches_reference_triton_kernel_golden(device: torch.device) -> None:
    """The reference's own Triton kernel outputs (interpreter) for the same inputs."""
    with np.load(GOLDEN / "rmsnorm_fp8.npz") as f:
        for tag in ("a", "b", "c"):
            x = torch.from_numpy(f[f"{tag}_x"].view(np.int16)).view(torch.float16)
            w = torch.from_numpy(f[f"{tag}_w"].view(np.int16)).view(torch.float16)
            static = torch.from_numpy(f[f"{tag}_static"]) if f"{tag}_static" in f.files else None
            q, s = rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS,
                                        None if static is None else static.to(device))
            _assert_within_one_code(q, torch.from_numpy(f[f"{tag}_q_triton"]))
            assert np.allclose(s.cpu().numpy().reshape(-1), f[f"{tag}_s_triton"].reshape(-1), rtol=1e-6)


def test_static_scale_saturates_exactly(device: torch.device) -> None:
    x, w = _inputs(16, 896, seed=11, scale=3.0)
    scale = torch.tensor([2e-3], dtype=torch.float32)
    q, s_out = rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS, scale.to(device))
    q_ref, _ = oracle.rmsnorm_fp8(x, w, EPS, scale)
    assert torch.equal(s_out.cpu(), scale)
    assert torch.equal(_codes(q), q_ref.to(torch.int16))
    y = _hf_rmsnorm(x, w).float() / scale
    saturated = y.abs() >= FP8_MAX
    assert int(saturated.sum()) > 100
    qf = q.cpu().float()
    ref_f = q_ref.view(torch.float8_e4m3fn).float()
    assert torch.equal(qf[saturated], ref_f[saturated])
    assert bool((qf[saturated].abs() == FP8_MAX).all())
    assert not bool(torch.isnan(qf).any())
    _assert_within_one_code(q, q_ref)


def test_e4m3_rounding_is_bit_exact_at_every_midpoint(device: torch.device) -> None:
    """Every e4m3 value, every midpoint and the fp32 values either side of each midpoint, both
    signs and +-0, round exactly as torch's float8_e4m3fn cast (the golden KAT)."""
    with np.load(GOLDEN / "e4m3_kat.npz") as f:
        probe = torch.from_numpy(f["probe"])
        codes = f["codes"]
    out = cast_e4m3(probe.to(device))
    assert np.array_equal(out.cpu().view(torch.uint8).numpy(), codes)


def test_cast_saturates_and_keeps_nan(device: torch.device) -> None:
    v = torch.tensor([500.0, -1e30, float("inf"), float("-inf"), float("nan"), 464.0, 447.9])
    out = cast_e4m3(v.to(device)).cpu().view(torch.uint8).tolist()
    assert out[:4] == [0x7E, 0xFE, 0x7E, 0xFE]
    assert out[4] & 0x7F == 0x7F
    assert out[5] == 0x7E and out[6] == 0x7E


def test_zero_row_uses_min_scale(device: torch.device) -> None:
    x = torch.zeros((2, 256), dtype=torch.float16)
    w = torch.ones(256, dtype=torch.float16)
    q, s = rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS)
    assert bool((q.cpu().float() == 0).all())
    assert torch.equal(s.cpu(), torch.full((2, 1), 1.0 / (448.0 * 512.0)))


def test_op_matches_kernel_and_keeps_leading_dims(device: torch.device) -> None:
    x, w = _inputs(6, 896, seed=3)
    q, s = torch.ops.tokenforge.rmsnorm_fp8_quant(x.reshape(2, 3, 896).to(device), w.to(device), EPS, None)
    assert q.shape == (2, 3, 896)
    assert s.shape == (2, 3, 1)
    qk, sk = rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS)
    assert torch.equal(_codes(q.reshape(6, 896)), _codes(qk))
    assert torch.equal(s.reshape(6, 1).cpu(), sk.cpu())
    # A static scale is returned as a fresh tensor, never an alias of the input.
    st = torch.tensor([1e-2], device=device)
    _, s2 = torch.ops.tokenforge.rmsnorm_fp8_quant(x.to(device), w.to(device), EPS, st)
    assert s2.data_ptr() != st.data_ptr() and torch.equal(s2, st)


def test_misaligned_and_strided_rows(device: torch.device) -> None:
    x, w = _inputs(5, 896, seed=9)
    buf = torch.empty(5 * 896 + 1, dtype=torch.float16, device=device)
    xm = buf[1:].view(5, 896)
    xm.copy_(x.to(device))
    q1, s1 = rmsnorm_fp8_quant_2d(xm, w.to(device), EPS)
    q2, s2 = rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS)
    assert torch.equal(_codes(q1), _codes(q2)) and torch.equal(s1, s2)


def test_rejects_bad_inputs(device: torch.device) -> None:
    x, w = _inputs(2, 128, seed=0)
    with pytest.raises(ValueError, match="2-D"):
        rmsnorm_fp8_quant_2d(x.reshape(-1).to(device), w.to(device), EPS)
    with pytest.raises(ValueError, match="weight shape"):
        rmsnorm_fp8_quant_2d(x.to(device), w[:64].to(device), EPS)
    with pytest.raises(ValueError, match="single fp32"):
        rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS, torch.ones(2, device=device))


@pytest.mark.parametrize("h", [1032, 2048, 3072, 3584, 4096])
@pytest.mark.parametrize("t", [1024, 1029, 2500])
def test_many_rows(t: int, h: int, device: torch.device) -> None:
    """Thousands of rows of 1025-4096 elements (several waves of CTAs, ragged T): codes and
    scales bit-exact against the oracle, dynamic and static scale."""
    gen = torch.Generator().manual_seed(t * 7 + h)
    x = torch.randn((t, h), generator=gen)
    x[:, torch.randperm(h, generator=gen)[:8]] *= 20
    x = x.to(torch.float16)
    w = (1 + 0.1 * torch.randn(h, generator=gen)).to(torch.float16)
    q, s = rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS)
    q_ref, s_ref = oracle.rmsnorm_fp8(x, w, EPS)
    assert torch.equal(_codes(q), q_ref.to(torch.int16))
    assert torch.equal(s.cpu(), s_ref)
    static = torch.tensor([0.05], dtype=torch.float32)
    q, _ = rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS, static.to(device))
    q_ref, _ = oracle.rmsnorm_fp8(x, w, EPS, static)
    assert torch.equal(_codes(q), q_ref.to(torch.int16))
