"""Host-side contract of the fused decode ops (no GPU needed): argument errors raise the same
kinds of exception as the reference's ops, CPU tensors raise instead of running anywhere, and
the fake (meta) implementations give the output shapes."""

from __future__ import annotations

import pytest
import torch

import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from tests.numerics import cases


def _w():  # type: ignore[no-untyped-def]
    return cases.layer_weights(64, 256, 0)


def test_rmsnorm_fp8_linear_argument_errors() -> None:
    w = _w()
    x = cases.activations(1, 256, 0)
    gamma = torch.ones(256, dtype=torch.float16)
    op = torch.ops.tokenforge.rmsnorm_fp8_w4a16_linear
    with pytest.raises(TypeError, match="fp16"):
        op(x.float(), gamma, 1e-6, None, w.qweight_t, w.scales, w.qzeros, None, 128)
    with pytest.raises(ValueError, match="norm_weight shape"):
        op(x, gamma[:128], 1e-6, None, w.qweight_t, w.scales, w.qzeros, None, 128)
    with pytest.raises(ValueError, match="single fp32"):
        op(x, gamma, 1e-6, torch.ones(2), w.qweight_t, w.scales, w.qzeros, None, 128)
    with pytest.raises(ValueError, match="encodes K"):
        op(x[:, :128], gamma[:128], 1e-6, None, w.qweight_t, w.scales, w.qzeros, None, 128)
    with pytest.raises(RuntimeError, match="CUDA"):  # no CPU path
        op(x, gamma, 1e-6, None, w.qweight_t, w.scales, w.qzeros, None, 128)


def test_silu_mul_linear_argument_errors() -> None:
    w = _w()
    gu = cases.activations(1, 512, 0)
    op = torch.ops.tokenforge.silu_mul_w4a16_linear
    with pytest.raises(ValueError, match="2 \\* K"):
        op(gu[:, :500], w.qweight_t, w.scales, w.qzeros, None, 128)
    with pytest.raises(TypeError, match="fp16"):
        op(gu.float(), w.qweight_t, w.scales, w.qzeros, None, 128)
    with pytest.raises(ValueError, match="divide"):
        op(gu, w.qweight_t, w.scales, w.qzeros, None, 512)
    with pytest.raises(RuntimeError, match="CUDA"):  # no CPU path
        op(gu, w.qweight_t, w.scales, w.qzeros, None, 128)


def test_fused_ops_fake_shapes() -> None:
    from torch._subclasses.fake_tensor import FakeTensorMode

    w = _w()
    with FakeTensorMode() as mode:
        f = mode.from_tensor
        y = torch.ops.tokenforge.rmsnorm_fp8_w4a16_linear(
            f(torch.zeros((2, 3, 256), dtype=torch.float16)), f(torch.ones(256, dtype=torch.float16)),
            1e-6, None, f(w.qweight_t), f(w.scales), f(w.qzeros), None, 128)
        assert y.shape == (2, 3, 64) and y.dtype == torch.float16
        y = torch.ops.tokenforge.silu_mul_w4a16_linear(
            f(torch.zeros((5, 512), dtype=torch.float16)), f(w.qweight_t), f(w.scales),
            f(w.qzeros), None, 128)
        assert y.shape == (5, 64) and y.dtype == torch.float16
