"""GPU parity of the persistent decode chain (tokenforge_b200.chain.DecodeChain, C ABI
tf_decode_chain_*).

Every op of a chain is checked over its full output against the fp64 product of the oracle's
dequantised weights, within the W4A16 tolerance (the reference's rule, calibrated cuda
constant), and against tf_w4a16_linear on the same inputs within the same tolerance (the chain
splits K differently, so the two agree to rounding, not bit for bit). Dependent ops (an op whose
activations are an earlier op's output) are checked against the fp64 product of the chain's
own earlier output. Runs are deterministic: repeated runs and CUDA-graph replays are
bit-identical, which also exercises the counters carried from run to run.
"""

from __future__ import annotations

import functools

import pytest
import torch

import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from oracle import oracle
from tests.numerics import cases
from tests.numerics.tolerance import atol
from tokenforge_b200.chain import ChainLinear, DecodeChain
from tokenforge_b200.pack import W4A16Weights

pytestmark = pytest.mark.gpu
G = 128
QWEN7B = [(4608, 3584), (3584, 3584), (37888, 3584), (3584, 18944)]


@functools.lru_cache(maxsize=8)
def _weights(n: int, k: int, seed: int) -> tuple[W4A16Weights, torch.Tensor]:
    qweight, qzeros, scales = cases.random_awq(n, k, seed)
    w = W4A16Weights(oracle.repack_awq_to_tf(qweight), scales, qzeros, G)
    return w, oracle.dequantize_tf(w.qweight_t, w.scales, w.qzeros, G)


def _check_op(y: torch.Tensor, x: torch.Tensor, w16: torch.Tensor, bias: torch.Tensor | None,
              what: str) -> None:
    ref = x.to(torch.float64) @ w16.to(y.device).to(torch.float64).t()
    if bias is not None:
        ref = ref + bias.to(torch.float64)
    err = float((y.to(torch.float64) - ref).abs().max())
    tol = atol(x.cpu(), w16, "cuda")
    assert err <= tol, f"{what}: max abs err {err:.3e} > tol {tol:.3e}"


def _linear(x: torch.Tensor, w: W4A16Weights, bias: torch.Tensor | None) -> torch.Tensor:
    return torch.ops.tokenforge.w4a16_linear(x, w.qweight_t, w.scales, w.qzeros, bias, G, "cuda")


@pytest.mark.parametrize("m", [1, 2, 4, 8])
def test_qwen_layer_chain_matches_oracle_and_linear(m: int, device: torch.device) -> None:
    """One Qwen2.5-7B decoder layer's four linears (independent inputs) as one chain."""
    ops, refs = [], []
    for i, (n, k) in enumerate(QWEN7B):
        w, w16 = _weights(n, k, i)
        wd = w.to(device)
        x = cases.activations(m, k, 10 + i).to(device)
        y = torch.full((m, n), float("nan"), dtype=torch.float16, device=device)
        ops.append(ChainLinear(x, wd, y, wait=i > 0))
        refs.append((x, w16, wd))
    with DecodeChain(ops) as ch:
        ch.run()
        torch.cuda.synchronize()
        assert ch.error() == 0
        for i, (op, (x, w16, wd)) in enumerate(zip(ops, refs)):
            assert not torch.isnan(op.y).any(), f"op {i}: output not fully written"
            _check_op(op.y, x, w16, None, f"op {i} M={m}")
            y_lin = _linear(x, wd, None)
            diff = float((op.y.double() - y_lin.double()).abs().max())
            assert diff <= atol(x.cpu(), w16, "cuda"), f"op {i}: chain vs linear {diff:.3e}"


@pytest.mark.parametrize("m", [1, 3, 8])
def test_dependent_ops_read_the_previous_output(m: int, device: torch.device) -> None:
    """o -> o -> down-shaped chain where each op reads the previous op's output (wait set),
    with bias, a row-strided input view and ragged K (896 = 3.5 chunks)."""
    shapes = [(3584, 896), (896 * 8, 3584), (3584, 7168)]
    ws = [_weights(n, k, 20 + i) for i, (n, k) in enumerate(shapes)]
    wide = torch.zeros((m, 896 + 64), dtype=torch.float16, device=device)
    wide[:, :896] = cases.activations(m, 896, 3).to(device)
    x0 = wide[:, :896]
    ys = [torch.empty((m, n), dtype=torch.float16, device=device) for n, _ in shapes]
    biases = [cases.bias(n, 7 + i).to(device) for i, (n, _) in enumerate(shapes)]
    ops = [ChainLinear(x0, ws[0][0].to(device), ys[0], biases[0], wait=False),
           ChainLinear(ys[0], ws[1][0].to(device), ys[1], biases[1]),
           ChainLinear(ys[1], ws[2][0].to(device), ys[2], biases[2])]
    with DecodeChain(ops) as ch:
        ch.run()
        torch.cuda.synchronize()
        assert ch.error() == 0
    inputs = [x0, ys[0], ys[1]]
    for i in range(3):
        _check_op(ys[i], inputs[i], ws[i][1], biases[i], f"op {i} M={m}")


def test_runs_and_graph_replays_are_bit_identical(device: torch.device) -> None:
    ops = []
    for i, (n, k) in enumerate(QWEN7B * 2):
        w, _ = _weights(n, k, i % 4)
        x = cases.activations(2, k, 30 + i).to(device)
        ops.append(ChainLinear(x, w.to(device), torch.empty((2, n), dtype=torch.float16,
                                                            device=device), wait=i > 0))
    with DecodeChain(ops) as ch:
        ch.run()
        first = [op.y.clone() for op in ops]
        for _ in range(5):  # counters carry from run to run (epochs)
            ch.run()
        torch.cuda.synchronize()
        assert all(torch.equal(a, op.y) for a, op in zip(first, ops))
        for op in ops:
            op.y.zero_()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ch.run()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ch.run()
            ch.run()
        for op in ops:
            op.y.zero_()
        graph.replay()
        graph.replay()
        torch.cuda.synchronize()
        assert all(torch.equal(a, op.y) for a, op in zip(first, ops))
        assert ch.error() == 0
        del graph


def test_non_finite_activations_propagate_like_the_linear(device: torch.device) -> None:
    w, _ = _weights(3584, 18944, 3)
    wd = w.to(device)
    x = cases.activations(4, 18944, 5)
    x[0, 100] = float("inf")
    x[1, 18000] = float("-inf")
    x[2, 7] = float("nan")
    xd = x.to(device)
    y = torch.empty((4, 3584), dtype=torch.float16, device=device)
    with DecodeChain([ChainLinear(xd, wd, y, wait=False)]) as ch:
        ch.run()
        torch.cuda.synchronize()
    ref = _linear(xd, wd, None)
    assert torch.equal(torch.isnan(y), torch.isnan(ref))
    assert torch.equal(torch.isposinf(y), torch.isposinf(ref))
    assert torch.equal(torch.isneginf(y), torch.isneginf(ref))
    assert bool(torch.isfinite(y[3]).all())


def test_invalid_chains_are_refused(device: torch.device) -> None:
    from tokenforge_b200._lib import KernelLibraryError

    w, _ = _weights(3584, 3584, 1)
    wd = w.to(device)
    x = torch.zeros((9, 3584), dtype=torch.float16, device=device)
    y = torch.zeros((9, 3584), dtype=torch.float16, device=device)
    with pytest.raises(ValueError, match="1 to 8 tokens"):
        DecodeChain([ChainLinear(x, wd, y)])
    with pytest.raises(ValueError, match="x must be"):
        DecodeChain([ChainLinear(x[:2, :128], wd, y[:2])])
    mis = torch.zeros(2 * 3584 + 8, dtype=torch.float16, device=device)[1:1 + 2 * 3584].view(2, 3584)
    with pytest.raises(KernelLibraryError, match="aligned"):
        DecodeChain([ChainLinear(mis, wd, y[:2])])
