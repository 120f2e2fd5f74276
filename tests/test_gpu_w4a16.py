"""GPU parity for W4A16 linear, mirroring the reference's tests/numerics/test_w4a16.py: every
shape of the suite and every M against the oracle's fp64 reference within the derived
tolerance, every kernel path, the edge cases (F1 outliers, Inf/NaN, zero and denormal scales,
all-zero weights), layout handling and determinism."""

from __future__ import annotations

import pytest
import torch

import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from oracle import oracle
from tests.numerics import cases
from tests.numerics.shapes import M_SUITE, linear_shapes
from tests.numerics.tolerance import atol
from tokenforge_b200 import ops
from tokenforge_b200.config import launch_plan
from tokenforge_b200.metrics import KERNEL_CALLS
from tokenforge_b200.pack import W4A16Weights

pytestmark = pytest.mark.gpu
G = cases.GROUP_SIZE


def _linear(x: torch.Tensor, w: W4A16Weights, bias: torch.Tensor | None = None,
            backend: str = "cuda") -> torch.Tensor:
    return torch.ops.tokenforge.w4a16_linear(x, w.qweight_t, w.scales, w.qzeros, bias,
                                             w.group_size, backend)


def _cols(w: W4A16Weights, words: torch.Tensor) -> W4A16Weights:
    """The layer restricted to column words ``words`` (8 output columns each)."""
    cols = (words[:, None] * 8 + torch.arange(8)).reshape(-1)
    return W4A16Weights(w.qweight_t[cols].contiguous(), w.scales[:, cols].contiguous(),
                        w.qzeros[:, words].contiguous(), w.group_size)


def _check(y: torch.Tensor, x: torch.Tensor, w: W4A16Weights, bias: torch.Tensor | None = None,
           max_words: int = 64) -> None:
    """Compare y [M, N] with the oracle's fp64 reference on up to ``max_words`` column words
    (all of them for small N), within the derived tolerance of the cuda constant."""
    n8 = w.n // 8
    if n8 <= max_words:
        words = torch.arange(n8)
    else:
        gen = torch.Generator().manual_seed(n8)
        words = torch.cat([torch.tensor([0, n8 - 1]), torch.randperm(n8 - 2, generator=gen)[: max_words - 2] + 1])
    ws = _cols(w, words)
    cols = (words[:, None] * 8 + torch.arange(8)).reshape(-1)
    b = None if bias is None else bias[cols]
    ref = oracle.w4a16_reference(x, ws.qweight_t, ws.scales, ws.qzeros, ws.group_size, b)
    w16 = oracle.dequantize_tf(ws.qweight_t, ws.scales, ws.qzeros, ws.group_size)
    got = y.detach().cpu().reshape(-1, w.n)[:, cols].to(torch.float64)
    tol = atol(x.reshape(-1, w.k), w16, "cuda")
    err = float((got - ref).abs().max()) if got.numel() else 0.0
    assert err <= tol, f"max abs err {err:.3e} > derived tol {tol:.3e}"


SHAPES = linear_shapes()


@pytest.mark.parametrize("m", M_SUITE)
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{s.model}/{s.layer}" for s in SHAPES])
def test_linear_shape_suite(shape, m: int, device: torch.device) -> None:  # type: ignore[no-untyped-def]
    for seed in cases.TEST_SEEDS:
        w = cases.layer_weights(shape.n, shape.k, seed)
        x = cases.activations(m, shape.k, seed)
        y = _linear(x.to(device), w.to(device))
        assert y.shape == (m, shape.n)
        assert y.dtype == torch.float16
        _check(y, x, w)


@pytest.mark.parametrize("with_bias", [False, True])
@pytest.mark.parametrize("g", [32, 64, 128])
@pytest.mark.parametrize("entry", ["gemv", "gemm", "linear"])
@pytest.mark.parametrize("m", [1, 2, 5, 8, 9, 17, 64, 70])
def test_every_kernel_path(entry: str, g: int, m: int, with_bias: bool, device: torch.device) -> None:
    if entry == "gemv" and m > 8:
        pytest.skip("the GEMV serves M <= 8")
    n, k = 200, 512  # N not a multiple of any tile
    w = cases.layer_weights(n, k, 0, g)
    b = cases.bias(n, 0) if with_bias else None
    x = cases.activations(m, k, 0)
    wd = w.to(device)
    fn = {"gemv": ops.w4a16_gemv, "gemm": ops.w4a16_gemm_tc,
          "linear": lambda *a: ops.w4a16_gemm(a[0], a[1], a[2], a[3], a[5], a[4])}[entry]
    y = fn(x.to(device), wd.qweight_t, wd.scales, wd.qzeros, None if b is None else b.to(device), g)
    _check(y, x, w, b)


@pytest.mark.parametrize(("m", "n", "k"), [(8, 3584, 18944), (1, 1024, 16384), (3, 1024, 16384),
                                           (1, 3584, 448 + 64), (2, 200, 4096), (8, 256, 65536)])
def test_split_k_paths(m: int, n: int, k: int, device: torch.device) -> None:
    """Shapes whose launch splits K across CTAs: inside a cluster (partials summed through
    distributed shared memory) and across clusters (fp32 partials + a reduce kernel)."""
    w = cases.layer_weights(n, k, 0)
    b = cases.bias(n, 0)
    x = cases.activations(m, k, 0)
    y = _linear(x.to(device), w.to(device), b.to(device))
    _check(y, x, w, b)
    assert launch_plan(8, 3584, 18944, 128).cluster > 1
    plan = launch_plan(8, 256, 65536, 128)
    assert plan.split_k // plan.cluster > 1


def test_leading_dims_and_bias_through_op(device: torch.device) -> None:
    w = cases.layer_weights(64, 256, 0)
    b = cases.bias(64, 0)
    x = cases.activations(6, 256, 0)
    y = _linear(x.reshape(2, 3, 256).to(device), w.to(device), b.to(device))
    assert y.shape == (2, 3, 64)
    _check(y.reshape(6, 64), x, w, b)


def test_zero_rows(device: torch.device) -> None:
    w = cases.layer_weights(64, 256, 0).to(device)
    y = _linear(torch.empty((0, 256), dtype=torch.float16, device=device), w)
    assert y.shape == (0, 64)


def test_non_contiguous_and_misaligned_inputs_are_handled(device: torch.device) -> None:
    w = cases.layer_weights(64, 256, 0)
    wd = w.to(device)
    x = cases.activations(4, 256, 0)
    x_cm = x.t().contiguous().t().to(device)
    assert x_cm.stride(1) != 1
    _check(_linear(x_cm, wd), x, w)
    buf = torch.empty(4 * 256 + 1, dtype=torch.float16, device=device)
    x_mis = buf[1:].view(4, 256)
    x_mis.copy_(x.to(device))
    assert x_mis.data_ptr() % 16 != 0
    _check(_linear(x_mis, wd), x, w)
    # Row-strided view (a slice of a wider activation buffer).
    wide = torch.zeros((4, 256 + 8), dtype=torch.float16, device=device)
    wide[:, :256] = x.to(device)
    _check(_linear(wide[:, :256], wd), x, w)


def _weights_from_ints(q: torch.Tensor, z: torch.Tensor, s: torch.Tensor) -> W4A16Weights:
    qweight, qzeros = oracle.awq_pack(q.to(torch.int32), z.to(torch.int32))
    return W4A16Weights(oracle.repack_awq_to_tf(qweight), s.to(torch.float16), qzeros, G)


@pytest.mark.parametrize("m", [1, 2, 16])
def test_f1_outliers_cancel_without_fp16_overflow(m: int, device: torch.device) -> None:
    """Products of 6e4 x 1.6 overflow fp16; fp32 products and accumulation must cancel them."""
    k, n = 256, 64
    gen = torch.Generator().manual_seed(0)
    q = torch.randint(0, 16, (k, n), generator=gen)
    q[1] = q[0] = 15
    z = torch.full((k // G, n), 7)
    s = torch.full((k // G, n), 0.2)
    w = _weights_from_ints(q, z, s)
    x = (torch.randn((max(m, 2), k), generator=gen) * 0.5).to(torch.float16)
    x[:, 0], x[:, 1] = 6e4, -6e4
    x = x[:m]
    y = _linear(x.to(device), w.to(device))
    assert bool(torch.isfinite(y).all())
    _check(y, x, w)


@pytest.mark.parametrize("m", [3, 8, 16])
def test_f1_real_inf_and_nan_propagate(m: int, device: torch.device) -> None:
    w = cases.layer_weights(64, 256, 0)
    x = cases.activations(16, 256, 0)
    x[0, 5] = float("inf")
    x[1, 7] = float("-inf")
    x[2, 9] = float("nan")
    ref16 = oracle.w4a16_reference(x, w.qweight_t, w.scales, w.qzeros, G).to(torch.float16)
    rows = x[:m]
    y = _linear(rows.to(device), w.to(device)).cpu()
    r = ref16[:m]
    assert torch.equal(torch.isnan(y), torch.isnan(r))
    assert torch.equal(torch.isposinf(y), torch.isposinf(r))
    assert torch.equal(torch.isneginf(y), torch.isneginf(r))
    assert bool(torch.isfinite(y[3:]).all()), "Inf leaked into clean rows"


@pytest.mark.parametrize("scale_value", [0.0, 2.0**-24, 6e-6])
@pytest.mark.parametrize("m", [1, 4, 16])
def test_zero_and_denormal_scales(scale_value: float, m: int, device: torch.device) -> None:
    k, n = 256, 64
    gen = torch.Generator().manual_seed(1)
    q = torch.randint(0, 16, (k, n), generator=gen)
    z = torch.randint(0, 16, (k // G, n), generator=gen)
    s = torch.rand((k // G, n), generator=gen) * 0.01 + 1e-3
    s[0, :] = scale_value
    w = _weights_from_ints(q, z, s)
    x = cases.activations(m, k, 0)
    y = _linear(x.to(device), w.to(device))
    assert bool(torch.isfinite(y).all())
    _check(y, x, w)


@pytest.mark.parametrize("m", [2, 24])
def test_all_zero_weights_are_exact(m: int, device: torch.device) -> None:
    k, n = 128, 16
    w = _weights_from_ints(torch.full((k, n), 9), torch.full((1, n), 9), torch.full((1, n), 0.5))
    y = _linear(cases.activations(m, k, 0).to(device), w.to(device))
    assert bool((y == 0).all())


@pytest.mark.parametrize("m", [1, 8, 64])
def test_deterministic_and_graph_replay_identical(m: int, device: torch.device) -> None:
    w = cases.layer_weights(896, 4864, 0).to(device)
    x = cases.activations(m, 4864, 0).to(device)
    y1 = _linear(x, w)
    y2 = _linear(x, w)
    assert torch.equal(y1, y2)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _linear(x, w)  # warm the allocator for capture
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y_graph = _linear(x, w)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y_graph, y1)


def test_dispatch_counts_buckets(device: torch.device) -> None:
    KERNEL_CALLS.reset()
    w = cases.layer_weights(128, 256, 0).to(device)
    _linear(cases.activations(3, 256, 0).to(device), w)
    x300 = cases.activations(300, 256, 0)
    y300 = _linear(x300.to(device), w, backend="triton")
    assert KERNEL_CALLS.value(kernel="cuda_gemv", bucket="4") == 1
    assert KERNEL_CALLS.value(kernel="cuda_gemm", bucket="512") == 1
    # The values of the M > 128 route, as the reference checks them (test_w4a16.py:99-105).
    _check(y300, x300, cases.layer_weights(128, 256, 0))


def test_drop_in_extension_module(device: torch.device) -> None:
    """tokenforge_b200._C provides the reference's planned `_C.w4a16_gemv` contract."""
    from tokenforge_b200 import _C

    w = cases.layer_weights(200, 512, 0)
    b = cases.bias(200, 0)
    x = cases.activations(3, 512, 0)
    wd = w.to(device)
    y = _C.w4a16_gemv(x.to(device), wd.qweight_t, wd.scales, wd.qzeros, b.to(device), G)
    _check(y, x, w, b)


@pytest.mark.parametrize(("m", "n", "k"), [(12, 3584, 18944), (16, 3584, 18944), (9, 256, 65536),
                                           (16, 1000, 1024), (13, 4608, 3584)])
def test_16_token_gemv_split_k_paths(m: int, n: int, k: int, device: torch.device) -> None:
    """M = 9..16 on the 16-token GEMV: K split inside a cluster and across clusters (fp32
    partials + the reduce kernel), ragged N, bias."""
    plan = launch_plan(m, n, k, G)
    assert plan.kernel == "gemv" and plan.tile_m == 16
    w = cases.layer_weights(n, k, 0)
    b = cases.bias(n, 0)
    x = cases.activations(m, k, 0)
    y = _linear(x.to(device), w.to(device), b.to(device))
    _check(y, x, w, b)


def test_16_token_gemv_non_finite_in_either_n_tile(device: torch.device) -> None:
    w = cases.layer_weights(64, 256, 0)
    x = cases.activations(14, 256, 0)
    x[2, 5] = float("inf")     # first n-tile (tokens 0-7)
    x[10, 7] = float("-inf")   # second n-tile (tokens 8-15)
    x[12, 9] = float("nan")
    ref16 = oracle.w4a16_reference(x, w.qweight_t, w.scales, w.qzeros, G).to(torch.float16)
    y = _linear(x.to(device), w.to(device)).cpu()
    assert torch.equal(torch.isnan(y), torch.isnan(ref16))
    assert torch.equal(torch.isposinf(y), torch.isposinf(ref16))
    assert torch.equal(torch.isneginf(y), torch.isneginf(ref16))
    clean = [i for i in range(14) if i not in (2, 10, 12)]
    assert bool(torch.isfinite(y[clean]).all())
    _check(y[clean].to(device), x[clean], w)


@pytest.mark.parametrize("m", [11, 16])
def test_16_token_gemv_deterministic_and_graph_replay(m: int, device: torch.device) -> None:
    w = cases.layer_weights(3584, 3584, 0).to(device)
    x = cases.activations(m, 3584, 0).to(device)
    y1 = _linear(x, w)
    assert torch.equal(_linear(x, w), y1)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _linear(x, w)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y_graph = _linear(x, w)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y_graph, y1)
