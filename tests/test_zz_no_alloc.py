"""GPU check of tf_w4a16_linear_noalloc, the W4A16 linear entry point whose split-K partials live
in the library's fixed device buffer instead of a caller workspace.

Called through the C ABI. Each shape runs twice in a row through the fixed-scratch entry point
and is compared with tf_w4a16_linear given a torch-allocated workspace; both follow the same
launch plan and the same fixed-order split-K sums, so the outputs must be bit-identical (and
therefore also within the W4A16 test tolerance, which is checked as well). Shapes cover the decode GEMV with and without a cross-cluster split, the 64-token
MMA kernel with split K, and the tensor-core GEMM with split K. This file is named to be
collected last, so it also runs after the rest of the GPU suite has used the library.
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle
from tests.numerics import cases
from tests.numerics.tolerance import atol
from tokenforge_b200 import _lib
from tokenforge_b200.config import launch_plan, workspace_bytes

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20  # TF_NOALLOC_SCRATCH_BYTES

# (M, N, K): kernel and split taken by each (see the assertions in the test).
SHAPES = [
    (1, 4608, 3584),     # GEMV, K split inside one cluster: no partials
    (8, 256, 65536),     # GEMV, K split across clusters: fp32 partials + reduce
    (40, 1000, 4096),    # 64-token MMA kernel (N % 32 != 0) with split K
    (64, 3584, 18944),   # tcgen05 GEMM with split K (4.6 MB of partials)
]


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _noalloc(x, w, bias, y, stream) -> int:  # type: ignore[no-untyped-def]
    m, k = x.shape
    return _lib.lib().tf_w4a16_linear_noalloc(
        x.data_ptr(), m, k, x.stride(0), w.qweight_t.data_ptr(), w.scales.data_ptr(),
        w.qzeros.data_ptr(), _ptr(bias), w.n, w.group_size, y.data_ptr(), y.stride(0), stream)


def _with_workspace(x, w, bias, y, stream) -> None:  # type: ignore[no-untyped-def]
    m, k = x.shape
    wsb = workspace_bytes(m, w.n, k, w.group_size)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=x.device)
    status = _lib.lib().tf_w4a16_linear(
        x.data_ptr(), m, k, x.stride(0), w.qweight_t.data_ptr(), w.scales.data_ptr(),
        w.qzeros.data_ptr(), _ptr(bias), w.n, w.group_size, y.data_ptr(), y.stride(0),
        ws.data_ptr(), wsb, stream)
    _lib.check("tf_w4a16_linear", status)


@pytest.mark.parametrize("with_bias", [False, True])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
def test_noalloc_matches_workspace_entry(shape, with_bias: bool, device: torch.device) -> None:  # type: ignore[no-untyped-def]
    m, n, k = shape
    plan = launch_plan(m, n, k, cases.GROUP_SIZE)
    if shape[1:] in ((256, 65536), (1000, 4096), (3584, 18944)):
        # These shapes exercise the scratch: split-K partials, or the tensor-core GEMM's
        # stream-K partials and tickets (reported with split_k 1).
        assert workspace_bytes(m, n, k, cases.GROUP_SIZE) > 0, plan
    seed = n * 7 + k
    w = cases.layer_weights(n, k, seed).to(device)
    x = cases.activations(m, k, seed).to(device)
    bias = cases.bias(n, seed).to(device) if with_bias else None
    stream = torch.cuda.current_stream(device).cuda_stream

    ref = torch.empty(m, n, dtype=torch.float16, device=device)
    _with_workspace(x, w, bias, ref, stream)
    w16 = oracle.dequantize_tf(w.qweight_t.cpu(), w.scales.cpu(), w.qzeros.cpu(), w.group_size)
    tol = atol(x.cpu(), w16, "cuda")

    for call in range(2):
        y = torch.full((m, n), float("nan"), dtype=torch.float16, device=device)
        torch.cuda.synchronize(device)
        status = _noalloc(x, w, bias, y, stream)
        _lib.check("tf_w4a16_linear_noalloc", status)
        torch.cuda.synchronize(device)
        assert not torch.isnan(y).any(), f"call {call}: output not fully written"
        err = float((y.float() - ref.float()).abs().max())
        assert err <= tol, f"call {call}: max abs diff {err:.3e} > tol {tol:.3e}"
        assert torch.equal(y, ref), f"call {call}: not bit-identical to the workspace entry"


def test_noalloc_leaves_device_memory_alone(device: torch.device) -> None:
    """After the first call on the device, a call changes no device allocation."""
    m, n, k = 64, 3584, 18944
    w = cases.layer_weights(n, k, 3).to(device)
    x = cases.activations(m, k, 3).to(device)
    y = torch.empty(m, n, dtype=torch.float16, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream
    _lib.check("tf_w4a16_linear_noalloc", _noalloc(x, w, None, y, stream))
    torch.cuda.synchronize(device)
    free_before = torch.cuda.mem_get_info(device)[0]
    _lib.check("tf_w4a16_linear_noalloc", _noalloc(x, w, None, y, stream))
    torch.cuda.synchronize(device)
    assert torch.cuda.mem_get_info(device)[0] == free_before


def test_noalloc_rejects_plans_beyond_the_scratch(device: torch.device) -> None:
    m, n, k = 1024, 3584, 18944
    assert workspace_bytes(m, n, k, cases.GROUP_SIZE) > SCRATCH_BYTES
    w = cases.layer_weights(n, k, 5).to(device)
    x = cases.activations(m, k, 5).to(device)
    y = torch.zeros(m, n, dtype=torch.float16, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream
    status = _noalloc(x, w, None, y, stream)
    assert status == _lib.TF_ERR_TOO_LARGE, _lib.status_string(status)
    assert "capacity" in _lib.status_string(status)
    torch.cuda.synchronize(device)
    assert not y.any(), "a refused call must not launch"


def test_noalloc_handles_empty_and_invalid_input(device: torch.device) -> None:
    stream = torch.cuda.current_stream(device).cuda_stream
    fn = _lib.lib().tf_w4a16_linear_noalloc
    assert fn(None, 0, 4096, 4096, None, None, None, None, 4608, 128, None, 4608, stream) == _lib.TF_OK
    assert fn(None, 1, 4096, 4096, None, None, None, None, 4608, 128, None, 4608, stream) == _lib.TF_ERR_INVALID_ARG
    assert fn(None, 1, 4096, 4096, None, None, None, None, 4608, 100, None, 4608, stream) == _lib.TF_ERR_INVALID_ARG
