"""GPU check of the SiLU-gated product used by the config-4 block stack:
out = fp16(silu(gate) * up) against torch in fp64 (one fp16 rounding of an fp32 result:
within one fp16 ulp of the fp64 value), with ragged widths and strided rows."""

from __future__ import annotations

import pytest
import torch

from tokenforge_b200 import ops

pytestmark = pytest.mark.gpu


def _ref(gu: torch.Tensor) -> torch.Tensor:
    g, u = gu.double().chunk(2, dim=-1)
    return g * torch.sigmoid(g) * u


@pytest.mark.parametrize(("m", "i"), [(1, 18944), (5, 1000), (64, 37), (3, 8)])
def test_silu_mul_matches_fp64(m: int, i: int, device: torch.device) -> None:
    gen = torch.Generator().manual_seed(m * 7 + i)
    gu = (torch.randn((m, 2 * i), generator=gen) * 3).half()
    y = ops.silu_mul(gu.to(device)).cpu()
    ref = _ref(gu)
    ulp = torch.finfo(torch.float16).eps * ref.abs().clamp_min(2.0**-14)
    assert bool(((y.double() - ref).abs() <= ulp).all())


def test_silu_mul_strided_rows_and_extremes(device: torch.device) -> None:
    base = torch.zeros((4, 40), dtype=torch.float16)
    base[:, :8] = torch.tensor([0.0, -0.0, 30.0, -30.0, 1e-4, -1e-4, 65504.0, -20.0]).half()
    base[:, 16:24] = 0.5
    base[:, 22] = 2.0  # 65504 * 2 overflows fp16: the product saturates to inf as in the reference
    gu = base.to(device)[:, :32]  # row stride 40, width 2 * 16
    y = ops.silu_mul(gu).cpu()
    ref = _ref(base[:, :32])
    assert bool(torch.isfinite(y[:, :6]).all()) and bool(torch.isinf(y[:, 6]).all())
    ulp = torch.finfo(torch.float16).eps * ref.abs().clamp_min(2.0**-14)
    ok = (y.double() - ref).abs() <= ulp
    assert bool(ok[:, :6].all()) and bool(ok[:, 7:16].all())
