"""GPU parity: AWQ repack, its inverse, the nibble codec and dequantization are bit-exact with
the oracle (and therefore with the reference: tests/test_oracle_golden.py)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from oracle import oracle
from tests.numerics import cases
from tokenforge_b200 import pack

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _bits16(t: torch.Tensor) -> torch.Tensor:
    return t.detach().cpu().view(torch.int16)


def _same_fp16(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bit-identical, except that any two NaNs match (NaN payloads are not specified)."""
    a, b = a.detach().cpu(), b.detach().cpu()
    nan_a, nan_b = torch.isnan(a), torch.isnan(b)
    return bool(torch.equal(nan_a, nan_b)) and bool(
        torch.equal(_bits16(a)[~nan_a], _bits16(b)[~nan_b])
    )


@pytest.mark.parametrize(("k", "n"), [(8, 8), (24, 8), (64, 200), (256, 64), (128, 1000),
                                      (896, 1152), (3584, 4608), (3584, 37888), (18944, 3584),
                                      (3584 + 64, 3584), (2056, 1088), (1032, 96 * 8)])
def test_repack_bit_exact(k: int, n: int, device: torch.device) -> None:
    gen = torch.Generator().manual_seed(k * 131 + n)
    qweight = torch.randint(-(2**31), 2**31 - 1, (k, n // 8), generator=gen, dtype=torch.int32)
    got = torch.ops.tokenforge.awq_repack(qweight.to(device))
    assert got.shape == (n, k // 8)
    assert torch.equal(got.cpu(), oracle.repack_awq_to_tf(qweight))
    back = pack.repack_tf_to_awq(got)
    assert torch.equal(back.cpu(), qweight)


def test_repack_golden(device: torch.device) -> None:
    with np.load(GOLDEN / "codec.npz") as f:
        for tag in ("a", "b", "c"):
            q = torch.from_numpy(f[f"{tag}_qweight"]).to(device)
            assert np.array_equal(torch.ops.tokenforge.awq_repack(q).cpu().numpy(), f[f"{tag}_qweight_t"])
            assert np.array_equal(pack.unpack_int4(q).cpu().numpy(), f[f"{tag}_unpacked"])
        assert np.array_equal(pack.pack_int4(torch.from_numpy(f["ints"]).to(device)).cpu().numpy(),
                              f["ints_packed"])


def test_pack_unpack_roundtrip_and_sign_bit(device: torch.device) -> None:
    gen = torch.Generator().manual_seed(3)
    v = torch.randint(0, 16, (9, 48), generator=gen, dtype=torch.int32)
    p = pack.pack_int4(v.to(device))
    assert torch.equal(p.cpu(), oracle.pack_int4(v))
    assert torch.equal(pack.unpack_int4(p).cpu(), v)
    s = torch.zeros((1, 8), dtype=torch.int32)
    s[0, pack.AWQ_ORDER[7]] = 15
    assert int(pack.pack_int4(s.to(device)).cpu()) == -(2**28)
    with pytest.raises(ValueError, match=r"\[0, 15\]"):
        pack.pack_int4(torch.full((1, 8), 16, dtype=torch.int32, device=device))


def test_pack_awq_roundtrip(device: torch.device) -> None:
    qweight, qzeros, scales = cases.random_awq(64, 3 * 128, 7)
    w = pack.pack_awq(qweight.to(device), qzeros.to(device), scales.to(device), 128)
    assert (w.n, w.k) == (64, 384)
    back = pack.unpack_to_awq(w)
    assert torch.equal(back[0].cpu(), qweight)
    assert torch.equal(back[1].cpu(), qzeros)


@pytest.mark.parametrize("g", [32, 64, 128])
@pytest.mark.parametrize(("n", "k"), [(200, 384), (64, 256), (4608, 3584), (3584, 18944)])
def test_dequant_bit_exact(n: int, k: int, g: int, device: torch.device) -> None:
    qweight, qzeros, scales = cases.random_awq(n, k, 1, g)
    qweight_t = oracle.repack_awq_to_tf(qweight)
    out = torch.ops.tokenforge.w4a16_dequant(qweight_t.to(device), scales.to(device), qzeros.to(device), g)
    ref = oracle.dequantize_tf(qweight_t, scales, qzeros, g)
    assert out.dtype == torch.float16 and out.shape == (n, k)
    assert torch.equal(_bits16(out), _bits16(ref))


@pytest.mark.parametrize("g", [32, 64, 128])
def test_dequant_golden(g: int, device: torch.device) -> None:
    with np.load(GOLDEN / "dequant.npz") as f:
        qw = torch.from_numpy(f[f"g{g}_qweight_t"]).to(device)
        s = torch.from_numpy(f[f"g{g}_scales"].view(np.int16)).view(torch.float16).to(device)
        z = torch.from_numpy(f[f"g{g}_qzeros"]).to(device)
        out = torch.ops.tokenforge.w4a16_dequant(qw, s, z, g)
        assert np.array_equal(_bits16(out).numpy().view(np.uint16), f[f"g{g}_dequant"])


@pytest.mark.parametrize("scale_value", [0.0, 2.0**-24, 6e-6, float("inf")])
def test_dequant_special_scales_bit_exact(scale_value: float, device: torch.device) -> None:
    qweight, qzeros, scales = cases.random_awq(64, 256, 2)
    scales[0, :] = scale_value
    qweight_t = oracle.repack_awq_to_tf(qweight)
    out = torch.ops.tokenforge.w4a16_dequant(qweight_t.to(device), scales.to(device), qzeros.to(device), 128)
    ref = oracle.dequantize_tf(qweight_t, scales, qzeros, 128)
    assert _same_fp16(out, ref)


def test_dequant_size_independent_property_full_layer(device: torch.device) -> None:
    """gate_up at full size: dequant(q, z, s) with s == 1 and z == 0 returns q exactly, and the
    AWQ round trip through repack/unrepack is the identity."""
    n, k = 37888, 3584
    q = torch.randint(-(2**31), 2**31 - 1, (k, n // 8), dtype=torch.int32, device=device)
    qt = torch.ops.tokenforge.awq_repack(q)
    assert torch.equal(pack.repack_tf_to_awq(qt), q)
    ones = torch.ones((k // 128, n), dtype=torch.float16, device=device)
    zeros = torch.zeros((k // 128, n // 8), dtype=torch.int32, device=device)
    deq = torch.ops.tokenforge.w4a16_dequant(qt, ones, zeros, 128)
    assert torch.equal(deq.to(torch.int32), pack.unpack_int4(qt))
