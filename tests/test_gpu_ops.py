"""Custom-op safety on the GPU (the reference's tests/unit/test_ops.py): opcheck (schema,
fake tensor, AOT dispatch), torch.compile fullgraph with no graph breaks, and the bucketed
dispatch under a dynamic-shape graph."""

from __future__ import annotations

import pytest
import torch
from torch.library import opcheck

import tokenforge_b200.ops  # noqa: F401
from tests.numerics import cases
from tokenforge_b200.metrics import KERNEL_CALLS

pytestmark = pytest.mark.gpu
G = cases.GROUP_SIZE
OPCHECK_TESTS = ("test_schema", "test_faketensor", "test_aot_dispatch_dynamic")


def _layer(device, n: int = 64, k: int = 256):  # type: ignore[no-untyped-def]
    w = cases.layer_weights(n, k, 0).to(device)
    return w.qweight_t, w.scales, w.qzeros


@pytest.mark.parametrize("m", [3, 40])
@pytest.mark.parametrize("with_bias", [False, True])
def test_opcheck_w4a16_linear(with_bias: bool, m: int, device: torch.device) -> None:
    qw, s, z = _layer(device)
    x = cases.activations(m, 256, 0).to(device)
    b = cases.bias(64, 0).to(device) if with_bias else None
    opcheck(torch.ops.tokenforge.w4a16_linear.default, (x, qw, s, z, b, G, "cuda"),
            test_utils=OPCHECK_TESTS)


def test_opcheck_dequant_rmsnorm_repack(device: torch.device) -> None:
    qw, s, z = _layer(device)
    opcheck(torch.ops.tokenforge.w4a16_dequant.default, (qw, s, z, G), test_utils=OPCHECK_TESTS)
    x = cases.activations(4, 256, 1).to(device)
    w = torch.ones(256, dtype=torch.float16, device=device)
    opcheck(torch.ops.tokenforge.rmsnorm_fp8_quant.default, (x, w, 1e-6, None),
            test_utils=("test_schema", "test_faketensor"))
    q = torch.randint(-(2**31), 2**31 - 1, (256, 8), dtype=torch.int32, device=device)
    opcheck(torch.ops.tokenforge.awq_repack.default, (q,), test_utils=OPCHECK_TESTS)


class _QLinear(torch.nn.Module):
    def __init__(self, device: torch.device) -> None:
        super().__init__()
        qw, s, z = _layer(device)
        self.register_buffer("qw", qw)
        self.register_buffer("s", s)
        self.register_buffer("z", z)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = torch.ops.tokenforge.w4a16_linear(x, self.qw, self.s, self.z, None, G, "cuda")
        return torch.relu(h) * 2


def test_torch_compile_fullgraph_no_graph_breaks(device: torch.device) -> None:
    mod = _QLinear(device)
    x = cases.activations(5, 256, 2).to(device)
    eager = mod(x)
    compiled = torch.compile(mod, backend="aot_eager", fullgraph=True, dynamic=True)
    assert torch.equal(compiled(x), eager)
    KERNEL_CALLS.reset()
    x2 = cases.activations(17, 256, 3).to(device)
    assert torch.equal(compiled(x2), mod(x2))
    assert KERNEL_CALLS.value(kernel="cuda_gemm", bucket="32") == 2
