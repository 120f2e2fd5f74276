"""GPU parity for fused RMSNorm + e4m3 quantization, mirroring the reference's
tests/numerics/test_rmsnorm_fp8.py, plus the BASELINE config-1 shapes (outlier channels)."""

from __future__ import annotations

import ctypes
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


def _ieee_quant(y: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """e4m3(clamp(y / scale)) with torch's IEEE fp32 division (tensor by tensor: torch divides
    by a Python scalar through its reciprocal) and its float8_e4m3fn cast."""
    v = (y.float() / scale.reshape(-1, 1)).clamp(-FP8_MAX, FP8_MAX)
    return v.to(torch.float8_e4m3fn).view(torch.uint8)


def _all_fp16(device: torch.device) -> torch.Tensor:
    return torch.arange(-32768, 32768, dtype=torch.int32, device=device).to(torch.int16).view(
        torch.float16)


def test_quant_division_matches_ieee_for_every_dynamic_scale(device: torch.device) -> None:
    """The quantizer divides by the row scale with FMAs (a reciprocal and residual corrections),
    not an IEEE division per element; dynamic scales take one correction step, which is exact
    for them only as a fact about this finite set. Exhaustive check of that fact through the
    dynamic quantizer itself: for every positive finite fp16 amax h, a row holding h and every
    fp16 value y with |y| <= h (the only quotients the dynamic rule can form), codes bit-exact
    with IEEE division and the float8 cast, and the scale max(h / 448, 1 / (448 * 512)) exact;
    NaN elements give NaN codes."""
    from tokenforge_b200.ops import e4m3_quant_rows

    ys = _all_fp16(device)
    nan_cols = torch.isnan(ys)
    amaxes = torch.arange(1, 0x7C00, dtype=torch.int32, device=device).to(torch.int16).view(
        torch.float16)
    for h in amaxes.split(512):
        y = torch.where(ys.abs().unsqueeze(0) <= h.unsqueeze(1), ys.unsqueeze(0), h.unsqueeze(1))
        y = torch.where(nan_cols.unsqueeze(0), ys.unsqueeze(0), y).contiguous()
        got, scale = e4m3_quant_rows(y)
        hf = h.float()
        want_scale = torch.clamp(hf / torch.full_like(hf, FP8_MAX),
                                 min=1.0 / (FP8_MAX * 512)).unsqueeze(1)
        assert torch.equal(scale, want_scale)
        got = got.view(torch.uint8)
        want = _ieee_quant(y, want_scale)
        assert torch.equal(got[:, ~nan_cols], want[:, ~nan_cols])
        assert bool(((got[:, nan_cols] & 0x7F) == 0x7F).all())
    # the scalar path (C not a multiple of 8), and a row with an Inf (IEEE-division path)
    y = ys[: 3 * 1001].reshape(3, 1001).clone()
    y[1, 5] = float("inf")
    got, scale = e4m3_quant_rows(y)
    fin = ~torch.isnan(y)
    assert torch.equal(got.view(torch.uint8)[fin], _ieee_quant(y, scale)[fin])


def test_quant_division_matches_ieee_for_static_scales(device: torch.device) -> None:
    """Static scales take two correction steps: scales across the FMA path's range [2^-60,
    2^60] (log-uniform), its edges, and outside it (IEEE-division path: tiny, subnormal and huge
    scales), against every fp16 value, bit-exact; also the scalar path (C not a multiple of 8)
    and one scale for all rows."""
    from tokenforge_b200.ops import e4m3_quant_rows

    gen = torch.Generator().manual_seed(4)
    logs = torch.rand(2048, generator=gen, dtype=torch.float64) * 120 - 60
    edges = torch.tensor([2.0**-60, 2.0**60, 2.0**-61, 2.0**61, 1e-30, 1e-40, 3e38, 1.0, 448.0],
                         dtype=torch.float64)
    scales = torch.cat([torch.exp2(logs), edges]).to(torch.float32).to(device)
    ys = _all_fp16(device)
    nan = torch.isnan(ys)
    for s in scales.split(512):
        y = ys.expand(s.numel(), -1).contiguous()
        got = e4m3_quant_rows(y, s)[0].view(torch.uint8)
        want = _ieee_quant(y, s)
        assert torch.equal(got[:, ~nan], want[:, ~nan])
    one = scales[:3]
    y = ys[: 3 * 1001].reshape(3, 1001)
    fin = ~torch.isnan(y)
    got = e4m3_quant_rows(y, one)[0].view(torch.uint8)
    assert torch.equal(got[fin], _ieee_quant(y, one)[fin])
    static = e4m3_quant_rows(y, one[1:2])[0].view(torch.uint8)
    assert torch.equal(static[fin], _ieee_quant(y, one[1:2].expand(3))[fin])


@pytest.mark.parametrize("h", [10000, 16384, 40000])
@pytest.mark.parametrize("t", [3, 1030])
def test_long_rows_bit_exact(t: int, h: int, device: torch.device) -> None:
    """Rows past one vector per thread (H > 8192: two or four vectors per thread) and past the
    CTA-per-row kernel's reach (H = 40000: the generic path), bit-exact with the oracle."""
    x, w = _inputs(t, h, seed=h + t)
    q, s = rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS)
    q_ref, s_ref = oracle.rmsnorm_fp8(x, w, EPS)
    assert torch.equal(_codes(q), q_ref.to(torch.int16))
    assert torch.equal(s.cpu(), s_ref)


@pytest.mark.parametrize("t", [2, 1100])
def test_signed_zeros_tiny_values_and_infinite_products(t: int, device: torch.device) -> None:
    """The FMA division's edge cases, bit-exact with the oracle: +-0 and fp16 subnormal
    activations (the sign of zero), a weight large enough that some products y overflow to Inf
    (dynamic: an Inf row scale; static: the IEEE-division fallback of the threads that hold an
    Inf), and static scales outside the FMA path's range."""
    h = 3584
    x, w = _inputs(t, h, seed=99 + t)
    x[:, :64] = 0.0
    x[:, 1:64:2] = -0.0
    x[:, 64:128] = torch.tensor(6e-8, dtype=torch.float16) * torch.arange(-32, 32)
    x[0, 300] = 100.0
    w[300] = 60000.0
    for static in (None, 1e-30, 2.0**61, 0.05):
        sc = None if static is None else torch.tensor([static], dtype=torch.float32)
        q, s = rmsnorm_fp8_quant_2d(x.to(device), w.to(device), EPS,
                                    None if sc is None else sc.to(device))
        q_ref, s_ref = oracle.rmsnorm_fp8(x, w, EPS, sc)
        ref_nan = torch.isnan(q_ref.view(torch.float8_e4m3fn).float())
        assert torch.equal(torch.isnan(q.cpu().float()), ref_nan), f"static scale {static}"
        assert torch.equal(_codes(q)[~ref_nan], q_ref.to(torch.int16)[~ref_nan]), static
        assert torch.equal(s.cpu(), s_ref)
        if static is None:
            assert float(s_ref[0, 0]) == float("inf"), "row 0 must hold an Inf product"


@pytest.mark.parametrize("h", [1032, 2048, 3000, 3584, 4096])
@pytest.mark.parametrize("t", [600, 5001])
def test_streaming_rows_bit_exact(t: int, h: int, device: torch.device) -> None:
    """Many rows of 1024 to 4096 elements go to the persistent streaming kernel (rows copied
    into per-warp shared-memory rings); dynamic and static scales, a row-strided view, and row
    counts that leave warps of the grid with different numbers of rows. The device status word
    stays clear (no bounded wait gave up)."""
    from tokenforge_b200 import _lib

    x, w = _inputs(t, h, seed=7 * h + t)
    wide = torch.zeros((t, h + 24), dtype=torch.float16)
    wide[:, :h] = x
    xd = wide.to(device)[:, :h]
    q, s = rmsnorm_fp8_quant_2d(xd, w.to(device), EPS)
    q_ref, s_ref = oracle.rmsnorm_fp8(x, w, EPS)
    assert torch.equal(_codes(q), q_ref.to(torch.int16))
    assert torch.equal(s.cpu(), s_ref)
    sc = torch.tensor([0.011], dtype=torch.float32)
    q, _ = rmsnorm_fp8_quant_2d(xd, w.to(device), EPS, sc.to(device))
    q_ref, _ = oracle.rmsnorm_fp8(x, w, EPS, sc)
    assert torch.equal(_codes(q), q_ref.to(torch.int16))
    code = ctypes.c_int(-1)
    _lib.check("tf_device_error", _lib.lib().tf_device_error(ctypes.byref(code)))
    assert code.value == 0
