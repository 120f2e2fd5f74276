"""GPU parity of the fused RMSNorm + FP8 + W4A16 decode linear
(torch.ops.tokenforge.rmsnorm_fp8_w4a16_linear, C ABI tf_rmsnorm_fp8_w4a16_linear) against the
two-op path it replaces, rmsnorm_fp8_quant followed by w4a16_linear_fp8: the outputs must be
bit-identical (same codes, same scales, same GEMV sums), including Inf/NaN positions. Both ops of
the two-op path are checked against the oracle in test_gpu_rmsnorm_fp8.py and
test_gpu_fp8_linear.py."""

from __future__ import annotations

import ctypes

import pytest
import torch

import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from tests.numerics import cases
from tokenforge_b200 import _lib
from tokenforge_b200.config import launch_plan

pytestmark = pytest.mark.gpu
EPS = 1e-6


def _inputs(m: int, k: int, seed: int, device: torch.device, outliers: bool = True):  # type: ignore[no-untyped-def]
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn((m, k), generator=gen)
    if outliers:  # 8 seeded outlier channels x20
        x[:, torch.randperm(k, generator=gen)[:8]] *= 20
    gamma = (1 + 0.1 * torch.randn(k, generator=gen)).half()
    return x.half().to(device), gamma.to(device)


def _two_op(x, gamma, scale, w, bias):  # type: ignore[no-untyped-def]
    q, s = torch.ops.tokenforge.rmsnorm_fp8_quant(x, gamma, EPS, scale)
    return torch.ops.tokenforge.w4a16_linear_fp8(q, s, w.qweight_t, w.scales, w.qzeros, bias,
                                                 w.group_size)


def _fused(x, gamma, scale, w, bias):  # type: ignore[no-untyped-def]
    return torch.ops.tokenforge.rmsnorm_fp8_w4a16_linear(x, gamma, EPS, scale, w.qweight_t,
                                                         w.scales, w.qzeros, bias, w.group_size)


def _fused_status(x, gamma, w, scale_out, static=None, bias=None):  # type: ignore[no-untyped-def]
    """The fused kernel through the C ABI at any M (the torch op takes it for one token only)."""
    m, k = x.shape
    n = w.qweight_t.shape[0]
    y = torch.empty((m, n), dtype=torch.float16, device=x.device)
    st = _lib.lib().tf_rmsnorm_fp8_w4a16_linear(
        x.data_ptr(), m, k, k, gamma.data_ptr(), EPS, _lib.ptr(static), _lib.ptr(scale_out),
        w.qweight_t.data_ptr(), w.scales.data_ptr(), w.qzeros.data_ptr(), _lib.ptr(bias), n,
        w.group_size, y.data_ptr(), n, None, 0, _lib.stream_ptr(x.device))
    torch.cuda.synchronize()
    return st, y


@pytest.mark.parametrize("m", [1, 2, 3, 8])
@pytest.mark.parametrize(("n", "k"), [(4608, 3584), (37888, 3584), (3584, 3584), (1152, 896),
                                      (200, 512)])
def test_fused_is_bit_identical_to_the_two_op_path(m: int, n: int, k: int,
                                                   device: torch.device) -> None:
    w = cases.layer_weights(n, k, 11).to(device)
    b = cases.bias(n, 11).to(device)
    x, gamma = _inputs(m, k, m + n, device)
    for bias in (None, b):
        assert torch.equal(_fused(x, gamma, None, w, bias), _two_op(x, gamma, None, w, bias))
    # Through the C ABI: plans that keep K in one CTA take the fused kernel, and the scales it
    # writes are rmsnorm_fp8_quant's; plans that split K are refused (the op then ran two ops).
    plan = launch_plan(m, n, k, 128)
    single_pass = plan.kernel == "gemv" and plan.split_k == 1 and plan.cluster == 1
    scale_out = torch.full((m,), -1.0, dtype=torch.float32, device=device)
    st, y = _fused_status(x, gamma, w, scale_out, bias=b)
    if not single_pass:
        assert st == _lib.TF_ERR_UNSUPPORTED
        return
    assert st == _lib.TF_OK
    _, s_ref = torch.ops.tokenforge.rmsnorm_fp8_quant(x, gamma, EPS, None)
    assert torch.equal(scale_out, s_ref.reshape(-1))
    assert torch.equal(y, _two_op(x, gamma, None, w, b))


@pytest.mark.parametrize("g", [32, 64])
@pytest.mark.parametrize("m", [1, 5])
def test_fused_group_sizes_and_static_scale(g: int, m: int, device: torch.device) -> None:
    n, k = 4608, 3584  # single-pass decode plan
    w = cases.layer_weights(n, k, 12, group_size=g).to(device)
    x, gamma = _inputs(m, k, 12, device)
    static = torch.tensor([0.05], dtype=torch.float32, device=device)
    for scale in (None, static):
        assert torch.equal(_fused(x, gamma, scale, w, None), _two_op(x, gamma, scale, w, None))
        st, y = _fused_status(x, gamma, w, None, static=scale)
        assert st == _lib.TF_OK
        assert torch.equal(y, _two_op(x, gamma, scale, w, None))


def test_fused_non_finite_rows_match(device: torch.device) -> None:
    n, k, m = 4608, 3584, 4
    w = cases.layer_weights(n, k, 13).to(device)
    x, gamma = _inputs(m, k, 13, device, outliers=False)
    x[1, 7] = float("inf")
    x[2, 100] = float("nan")
    st, y_f = _fused_status(x, gamma, w, None)
    assert st == _lib.TF_OK
    y_t = _two_op(x, gamma, None, w, None)
    assert torch.equal(torch.isnan(y_f), torch.isnan(y_t))
    fin = ~torch.isnan(y_t)
    assert torch.equal(y_f[fin], y_t[fin])
    assert bool(torch.isfinite(y_f[[0, 3]]).all())


def test_split_k_plans_are_refused_and_the_op_falls_back(device: torch.device) -> None:
    """down_proj at M = 8 splits K over a cluster: the C entry point launches nothing and says
    so; the torch op then runs the two ops."""
    n, k, m = 3584, 18944, 8
    w = cases.layer_weights(n, k, 14).to(device)
    x, gamma = _inputs(m, k, 14, device)
    scale_out = torch.full((m,), -1.0, dtype=torch.float32, device=device)
    st, _ = _fused_status(x, gamma, w, scale_out)
    assert st == _lib.TF_ERR_UNSUPPORTED
    assert bool((scale_out == -1.0).all())
    assert torch.equal(_fused(x, gamma, None, w, None), _two_op(x, gamma, None, w, None))
    # Prefill sizes take the two-op path too.
    xp, gp = _inputs(24, k, 15, device)
    assert torch.equal(_fused(xp, gp, None, w, None), _two_op(xp, gp, None, w, None))


def test_fused_graph_replay_identical(device: torch.device) -> None:
    n, k, m = 4608, 3584, 1
    w = cases.layer_weights(n, k, 16).to(device)
    x, gamma = _inputs(m, k, 16, device)
    ref = _fused(x, gamma, None, w, None)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _fused(x, gamma, None, w, None)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = _fused(x, gamma, None, w, None)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, ref)


def test_entry_point_rejects_bad_arguments(device: torch.device) -> None:
    n, k = 256, 1024
    w = cases.layer_weights(n, k, 17).to(device)
    x, gamma = _inputs(1, k, 17, device)
    y = torch.empty((1, n), dtype=torch.float16, device=device)
    lib = _lib.lib()
    args = [x.data_ptr(), 1, k, k, gamma.data_ptr(), EPS, None, None, w.qweight_t.data_ptr(),
            w.scales.data_ptr(), w.qzeros.data_ptr(), None, n, 128, y.data_ptr(), n, None, 0,
            _lib.stream_ptr(device)]
    bad = list(args)
    bad[4] = None  # no RMSNorm weight
    assert lib.tf_rmsnorm_fp8_w4a16_linear(*bad) == _lib.TF_ERR_INVALID_ARG
    bad = list(args)
    bad[4] = ctypes.c_void_p(gamma.data_ptr() + 2).value  # misaligned RMSNorm weight
    assert lib.tf_rmsnorm_fp8_w4a16_linear(*bad) == _lib.TF_ERR_ALIGNMENT
    bad = list(args)
    bad[13] = 96  # group size
    assert lib.tf_rmsnorm_fp8_w4a16_linear(*bad) == _lib.TF_ERR_INVALID_ARG
    assert lib.tf_rmsnorm_fp8_w4a16_linear(*args) == _lib.TF_OK


@pytest.mark.parametrize("m", [1, 2])
def test_row_strided_view_keeps_its_stride(m: int, device: torch.device) -> None:
    """x a slice of a wider buffer (row stride > K): the fused path must read row m at
    x + m * stride(0), as the two-op path does."""
    n, k = 1152, 896
    w = cases.layer_weights(n, k, 5).to(device)
    x, gamma = _inputs(m, k, 77, device)
    wide = torch.full((m, k + 64), 1000.0, dtype=torch.float16, device=device)
    wide[:, :k] = x
    view = wide[:, :k]
    assert view.stride(0) == k + 64
    assert torch.equal(_fused(view, gamma, None, w, None), _two_op(x, gamma, None, w, None))
