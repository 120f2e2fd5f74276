"""Direct launchers of the W4A16 linear kernels, with no ``torch.library`` registration.

``tokenforge_b200.ops`` builds the ``torch.ops.tokenforge.*`` custom ops on these functions;
``tokenforge_b200._C`` (the drop-in for the reference's ``tokenforge.kernels._C``) uses them
directly, so importing it next to the reference leaves the reference's own custom ops in place.

Validation follows the reference's contract (tokenforge/kernels/triton/w4a16.py:149-175: same
checks, same matchable message substrings). Every call enqueues on the current CUDA stream of
the input's device through the C ABI; the only allocations are the output and the optional
split-K workspace, both from PyTorch's caching allocator. CPU tensors raise.
"""

from __future__ import annotations

import torch

from tokenforge_b200 import _lib
from tokenforge_b200.pack import PACK_FACTOR

_VEC = 16  # bytes: alignment the vectorised kernels require


def _require(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (tokenforge_b200 has no CPU path)")


def _aligned_rows(x2: torch.Tensor) -> torch.Tensor:
    """x2 with unit stride along K, a 16-byte aligned base and a row stride multiple of 8."""
    if x2.stride(-1) != 1 or x2.data_ptr() % _VEC != 0 or (x2.shape[0] > 1 and x2.stride(0) % 8):
        x2 = x2.clone(memory_format=torch.contiguous_format)
    return x2


def _check_inputs(
    x: torch.Tensor,
    qweight_t: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor,
    group_size: int,
) -> tuple[int, int, int]:
    """Shape/dtype/layout contract of the reference (triton/w4a16.py:149-175)."""
    if x.dim() != 2:
        raise ValueError(f"x must be 2-D [M, K], got shape {tuple(x.shape)}")
    if x.dtype != torch.float16:
        raise TypeError(f"x must be fp16, got {x.dtype}")
    m, k = x.shape
    n = qweight_t.shape[0]
    if qweight_t.dtype != torch.int32 or qzeros.dtype != torch.int32:
        raise TypeError("qweight_t and qzeros must be int32")
    if scales.dtype != torch.float16:
        raise TypeError(f"scales must be fp16, got {scales.dtype}")
    if qweight_t.shape[1] * PACK_FACTOR != k:
        raise ValueError(f"x has K={k} but qweight_t encodes K={qweight_t.shape[1] * PACK_FACTOR}")
    if group_size not in (32, 64, 128):
        raise ValueError(f"group_size {group_size} must be 32, 64 or 128 and divide K")
    if k % group_size != 0:
        raise ValueError(f"K={k} is not a multiple of group_size={group_size}")
    if n % PACK_FACTOR != 0:
        raise ValueError(f"N={n} is not a multiple of {PACK_FACTOR}")
    if tuple(scales.shape) != (k // group_size, n):
        raise ValueError(f"scales shape {tuple(scales.shape)} != {(k // group_size, n)}")
    if tuple(qzeros.shape) != (k // group_size, n // PACK_FACTOR):
        raise ValueError(
            f"qzeros shape {tuple(qzeros.shape)} != {(k // group_size, n // PACK_FACTOR)}"
        )
    for name, t in (("qweight_t", qweight_t), ("scales", scales), ("qzeros", qzeros)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if x.stride(1) != 1:
        raise ValueError("x must be contiguous along K (stride(1) == 1)")
    return m, n, k


_LINEAR_ENTRY = {"linear": "tf_w4a16_linear", "gemv": "tf_w4a16_gemv", "gemm": "tf_w4a16_gemm"}


def _launch_linear(
    entry: str,
    x2: torch.Tensor,
    qweight_t: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor,
    bias: torch.Tensor | None,
    group_size: int,
) -> torch.Tensor:
    m, n, k = _check_inputs(x2, qweight_t, scales, qzeros, group_size)
    for name, t in (("x", x2), ("qweight_t", qweight_t), ("scales", scales), ("qzeros", qzeros)):
        _require(t, name)
    if bias is not None:
        _require(bias, "bias")
        if tuple(bias.shape) != (n,):
            raise ValueError(f"bias shape {tuple(bias.shape)} != {(n,)}")
        if bias.dtype != torch.float16:
            raise TypeError(f"bias must be fp16, got {bias.dtype}")
        bias = bias.contiguous()
    y = torch.empty((m, n), dtype=torch.float16, device=x2.device)
    if m == 0:
        return y
    x2 = _aligned_rows(x2)
    lib = _lib.lib()
    ws_bytes = int(lib.tf_w4a16_workspace_bytes(m, n, k, group_size))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x2.device) if ws_bytes else None
    with torch.cuda.device(x2.device):
        status = getattr(lib, _LINEAR_ENTRY[entry])(
            x2.data_ptr(), m, k, x2.stride(0),
            qweight_t.data_ptr(), scales.data_ptr(), qzeros.data_ptr(), _lib.ptr(bias),
            n, group_size, y.data_ptr(), n, _lib.ptr(ws), ws_bytes, _lib.stream_ptr(x2.device),
        )  # fmt: skip
    _lib.check(_LINEAR_ENTRY[entry], status)
    return y


def w4a16_gemm(
    x: torch.Tensor,
    qweight_t: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor,
    group_size: int,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """``x [M, K] fp16 @ dequant(W)^T (+ bias) -> [M, N] fp16`` through the launch table."""
    return _launch_linear("linear", x, qweight_t, scales, qzeros, bias, group_size)


def w4a16_gemv(x, qweight_t, scales, qzeros, bias, group_size):  # type: ignore[no-untyped-def]
    """Decode entry (M <= 8): the ``_C.w4a16_gemv`` contract of the reference (ops.py:86-88)."""
    return _launch_linear("gemv", x, qweight_t, scales, qzeros, bias, group_size)


def w4a16_gemm_tc(x, qweight_t, scales, qzeros, bias, group_size):  # type: ignore[no-untyped-def]
    """Prefill entry: the tensor-core GEMM for any M (used by tests to pin each kernel)."""
    return _launch_linear("gemm", x, qweight_t, scales, qzeros, bias, group_size)
