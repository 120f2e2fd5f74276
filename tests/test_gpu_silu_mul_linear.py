"""GPU parity of the down projection fused with the SiLU-gated product
(torch.ops.tokenforge.silu_mul_w4a16_linear, C ABI tf_silu_mul_w4a16_linear) against the two
ops it replaces, silu_mul then w4a16_linear: bit-identical outputs, Inf/NaN positions included.
Both ops of the two-op path are checked against their references in test_gpu_silu_mul.py and
test_gpu_w4a16.py."""

from __future__ import annotations

import pytest
import torch

import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from tests.numerics import cases
from tokenforge_b200 import _lib, ops
from tokenforge_b200.config import launch_plan

pytestmark = pytest.mark.gpu


def _gate_up(m: int, k: int, seed: int, device: torch.device) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn((m, 2 * k), generator=gen) * 2).half().to(device)


def _two_op(gu, w, bias=None):  # type: ignore[no-untyped-def]
    return ops.w4a16_gemm(ops.silu_mul(gu), w.qweight_t, w.scales, w.qzeros, w.group_size, bias)


def _abi(gu, w, bias=None):  # type: ignore[no-untyped-def]
    m, k2 = gu.shape
    n = w.qweight_t.shape[0]
    y = torch.empty((m, n), dtype=torch.float16, device=gu.device)
    st = _lib.lib().tf_silu_mul_w4a16_linear(
        gu.data_ptr(), m, k2 // 2, gu.stride(0), w.qweight_t.data_ptr(), w.scales.data_ptr(),
        w.qzeros.data_ptr(), _lib.ptr(bias), n, w.group_size, y.data_ptr(), n, None, 0,
        _lib.stream_ptr(gu.device))
    torch.cuda.synchronize()
    return st, y


@pytest.mark.parametrize("m", [1, 2, 3, 8])
@pytest.mark.parametrize(("n", "k"), [(3584, 18944), (896, 4864), (4608, 3584), (200, 512)])
def test_fused_is_bit_identical_to_the_two_op_path(m: int, n: int, k: int,
                                                   device: torch.device) -> None:
    w = cases.layer_weights(n, k, 21).to(device)
    b = cases.bias(n, 21).to(device)
    gu = _gate_up(m, k, m + n, device)
    for bias in (None, b):
        ref = _two_op(gu, w, bias)
        assert torch.equal(torch.ops.tokenforge.silu_mul_w4a16_linear(
            gu, w.qweight_t, w.scales, w.qzeros, bias, 128), ref)
        plan = launch_plan(m, n, k, 128)
        st, y = _abi(gu, w, bias)
        if plan.kernel == "gemv" and plan.split_k == 1 and plan.cluster == 1:
            assert st == _lib.TF_OK
            assert torch.equal(y, ref)
        else:
            assert st == _lib.TF_ERR_UNSUPPORTED


@pytest.mark.parametrize("g", [32, 64])
def test_fused_group_sizes_and_strided_rows(g: int, device: torch.device) -> None:
    n, k, m = 4608, 3584, 2
    w = cases.layer_weights(n, k, 22, group_size=g).to(device)
    wide = torch.zeros((m, 2 * k + 64), dtype=torch.float16, device=device)
    wide[:, :2 * k] = _gate_up(m, k, 22, device)
    gu = wide[:, :2 * k]  # row stride 2K + 64
    st, y = _abi(gu, w)
    assert st == _lib.TF_OK
    assert torch.equal(y, _two_op(gu.contiguous(), w))


def test_fused_non_finite_match(device: torch.device) -> None:
    n, k, m = 4608, 3584, 2
    w = cases.layer_weights(n, k, 23).to(device)
    gu = _gate_up(m, k, 23, device)
    gu[0, 5] = float("inf")      # gate: silu(inf) * u = inf * u
    gu[1, k + 9] = float("nan")  # up
    st, y = _abi(gu, w)
    assert st == _lib.TF_OK
    ref = _two_op(gu, w)
    assert torch.equal(torch.isnan(y), torch.isnan(ref))
    fin = ~torch.isnan(ref)
    assert torch.equal(y[fin], ref[fin])


def test_fused_graph_replay_identical(device: torch.device) -> None:
    n, k, m = 3584, 18944, 1
    w = cases.layer_weights(n, k, 24).to(device)
    gu = _gate_up(m, k, 24, device)

    def run() -> torch.Tensor:
        return torch.ops.tokenforge.silu_mul_w4a16_linear(gu, w.qweight_t, w.scales, w.qzeros,
                                                          None, 128)

    ref = run()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        run()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = run()
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
