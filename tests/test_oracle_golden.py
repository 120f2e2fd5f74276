"""The CPU oracle against golden vectors produced by running the reference itself
(tests/golden/make_golden.py). This pins the restatement before it is trusted as the
checker of the CUDA kernels."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.numerics.tolerance import EPS_FP16, load_constant

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


def _t(a: np.ndarray) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.float16)
    return torch.from_numpy(a.copy())


@pytest.fixture(scope="module")
def codec() -> dict[str, np.ndarray]:
    return _load("codec")


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_repack_and_unpack_match_reference(codec, tag: str) -> None:  # type: ignore[no-untyped-def]
    qweight = _t(codec[f"{tag}_qweight"])
    qweight_t = oracle.repack_awq_to_tf(qweight)
    assert np.array_equal(qweight_t.numpy(), codec[f"{tag}_qweight_t"])
    assert np.array_equal(oracle.repack_tf_to_awq(qweight_t).numpy(), codec[f"{tag}_back"])
    assert np.array_equal(oracle.unpack_int4(qweight).numpy(), codec[f"{tag}_unpacked"])


def test_pack_int4_matches_reference(codec) -> None:  # type: ignore[no-untyped-def]
    assert np.array_equal(oracle.pack_int4(_t(codec["ints"])).numpy(), codec["ints_packed"])
    packed = oracle.pack_int4(_t(codec["sign_values"]))
    assert int(packed) == -(2**28) == int(codec["sign_packed"].reshape(-1)[0])  # 0xF0000000 as int32


def _autoawq_pack_loop(intweight: torch.Tensor) -> torch.Tensor:
    """Scalar transcription of AutoAWQ's WQLinear_GEMM pack loop: for each column word,
    nibble i takes column offset order_map[i]."""
    k, n = intweight.shape
    out = torch.zeros((k, n // 8), dtype=torch.int64)
    order_map = [0, 2, 4, 6, 1, 3, 5, 7]
    for col in range(n // 8):
        for i in range(8):
            out[:, col] |= intweight[:, col * 8 + order_map[i]].to(torch.int64) << (i * 4)
    return out.to(torch.int32)


def test_pack_matches_autoawq_loop() -> None:
    gen = torch.Generator().manual_seed(5)
    ints = torch.randint(0, 16, (5, 32), generator=gen, dtype=torch.int32)
    assert torch.equal(oracle.pack_int4(ints), _autoawq_pack_loop(ints))
    assert torch.equal(oracle.unpack_int4(oracle.pack_int4(ints)), ints)


def test_pack_rejects_out_of_range() -> None:
    with pytest.raises(ValueError, match=r"\[0, 15\]"):
        oracle.pack_int4(torch.full((1, 8), 16, dtype=torch.int32))
    with pytest.raises(ValueError, match="multiple of 8"):
        oracle.pack_int4(torch.zeros((1, 7), dtype=torch.int32))


def test_awq_quantize_matches_reference() -> None:
    d = _load("dequant")
    qweight, qzeros, scales = oracle.awq_quantize(_t(d["quant_weight"]), 128)
    assert np.array_equal(qweight.numpy(), d["quant_qweight"])
    assert np.array_equal(qzeros.numpy(), d["quant_qzeros"])
    assert np.array_equal(scales.view(torch.int16).numpy().view(np.uint16), d["quant_scales"])


@pytest.mark.parametrize("g", [32, 64, 128])
def test_dequant_matches_reference_bit_exact(g: int) -> None:
    d = _load("dequant")
    out = oracle.dequantize_tf(_t(d[f"g{g}_qweight_t"]), _t(d[f"g{g}_scales"]), _t(d[f"g{g}_qzeros"]), g)
    assert np.array_equal(out.view(torch.int16).numpy().view(np.uint16), d[f"g{g}_dequant"])


def test_seeded_cases_reproduce_reference_weights() -> None:
    """tests/numerics/cases.py regenerates the reference's layer_weights(200, 384, 0, g)."""
    from tests.numerics import cases

    d = _load("dequant")
    for g in (32, 64, 128):
        w = cases.layer_weights(200, 384, 0, g)
        assert np.array_equal(w.qweight_t.numpy(), d[f"g{g}_qweight_t"])
        assert np.array_equal(w.qzeros.numpy(), d[f"g{g}_qzeros"])
        assert np.array_equal(w.scales.view(torch.int16).numpy().view(np.uint16), d[f"g{g}_scales"])


@pytest.mark.parametrize("m", [1, 3, 8, 16, 33])
def test_w4a16_reference_and_cpu_path(m: int) -> None:
    d = _load("w4a16")
    qw, s, z, b = (_t(d[k]) for k in ("qweight_t", "scales", "qzeros", "bias"))
    x = _t(d[f"m{m}_x"])
    ref = oracle.w4a16_reference(x, qw, s, z, 128, b)
    golden64 = torch.from_numpy(d[f"m{m}_ref64"])
    assert float((ref - golden64).abs().max()) <= 1e-9 * float(golden64.abs().max())
    # The oracle's fp32 CPU path vs the reference's torch CPU path (w4a16_torch): both are
    # within the reference's CPU tolerance of the fp64 result.
    y = oracle.w4a16_cpu(x, qw, s, z, 128, b, threads=2).to(torch.float64)
    w16 = oracle.dequantize_tf(qw, s, z, 128).to(torch.float64)
    tol = load_constant("cpu") * (512**0.5) * EPS_FP16 * float(x.abs().max()) * float(w16.abs().max())
    assert float((y - golden64).abs().max()) <= tol
    torch_path = _t(d[f"m{m}_torch"]).to(torch.float64)
    assert float((torch_path - golden64).abs().max()) <= tol
    if f"m{m}_triton" in d:
        tri = _t(d[f"m{m}_triton"]).to(torch.float64)
        assert float((tri - golden64).abs().max()) <= tol


def _within_one_code(a: torch.Tensor, b: torch.Tensor, max_frac: float = 0.05) -> None:
    a, b = a.to(torch.int16), b.to(torch.int16)
    ma, mb = a & 0x7F, b & 0x7F
    sign_ok = ((a & 0x80) == (b & 0x80)) | ((ma == 0) & (mb <= 1)) | ((mb == 0) & (ma <= 1))
    assert bool(sign_ok.all())
    diff = (ma - mb).abs()
    assert int(diff.max()) <= 1
    assert float((diff > 0).float().mean()) < max_frac


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_rmsnorm_fp8_matches_reference(tag: str) -> None:
    d = _load("rmsnorm_fp8")
    x, w = _t(d[f"{tag}_x"]), _t(d[f"{tag}_w"])
    static = _t(d[f"{tag}_static"]) if f"{tag}_static" in d else None
    q, s = oracle.rmsnorm_fp8(x, w, 1e-6, static)
    # Against the Triton kernel (same IEEE sqrt/div rules): identical codes and scales.
    assert np.array_equal(q.numpy(), d[f"{tag}_q_triton"])
    assert np.array_equal(s.numpy().reshape(-1), d[f"{tag}_s_triton"].reshape(-1))
    # Against the torch reference (rsqrt): the reference's own acceptance criteria.
    _within_one_code(q, torch.from_numpy(d[f"{tag}_q_ref"]))
    s_ref = torch.from_numpy(d[f"{tag}_s_ref"]).reshape(-1)
    assert float(((s.reshape(-1) - s_ref).abs() / s_ref).max()) <= 1e-3


def test_e4m3_rounding_kat() -> None:
    d = _load("e4m3_kat")
    codes = oracle.e4m3_codes(torch.from_numpy(d["probe"]))
    assert np.array_equal(codes.numpy(), d["codes"])


def test_e4m3_decode_matches_torch_for_every_code() -> None:
    """The oracle's e4m3fn decoder (used by the FP8-activation linear's reference) agrees with
    torch.float8_e4m3fn, the arithmetic the reference's FP8 rule is written in."""
    codes = torch.arange(256, dtype=torch.uint8)
    got = oracle.e4m3_values(codes)
    want = codes.view(torch.float8_e4m3fn).to(torch.float64)
    assert bool(((got == want) | (got.isnan() & want.isnan())).all())
    # and the encoder inverts it on every finite code
    finite = ~want.isnan()
    assert torch.equal(oracle.e4m3_codes(want[finite].float()), codes[finite])
