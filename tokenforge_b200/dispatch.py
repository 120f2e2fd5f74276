"""Host-side kernel dispatch for the CUDA backend (mirrors tokenforge/kernels/dispatch.py).

Two decisions, as in the reference:

* :func:`layer_support` runs once per layer at weight-load time and names the reason a layer
  cannot be served (the caller keeps its own AWQ path for it and counts the fallback).
* :func:`select` runs per call on ``M`` only, reads no tensor values and never synchronises,
  so it is safe under CUDA-graph capture and opaque to torch.compile.

Routing differs from the reference by design: every supported call runs a CUDA kernel.
``M <= 8`` goes to the decode GEMV (``cuda_gemv``), larger ``M`` to the kernel library's launch
table (``cuda_gemm``: the 16-token GEMV up to ``M = 16`` at group size 128, the tensor-core
GEMM above). There is no Triton path, no dequant+cuBLAS path and no CPU fallback: a call
on CPU tensors, or without the kernel library, raises.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Final, Literal, get_args

from tokenforge_b200.config import MAX_GEMV_M, bucket_label
from tokenforge_b200.metrics import FALLBACKS, KERNEL_CALLS
from tokenforge_b200.pack import PACK_FACTOR, SUPPORTED_GROUP_SIZES

Backend = Literal["triton", "cuda", "marlin"]
Kernel = Literal["cuda_gemv", "cuda_gemm"]
FallbackReason = Literal[
    "kill_switch",
    "unsupported_dtype",
    "unsupported_group_size",
    "unsupported_shape",
    "unsupported_arch",
    "cuda_ext_unavailable",
]

BACKENDS: Final[tuple[str, ...]] = get_args(Backend)
BACKEND_ENV: Final = "TOKENFORGE_BACKEND"
MIN_SM: Final = 100  # the kernels are built for sm_100a only


def backend_from_env() -> Backend:
    """The layer-level backend a process asks for. ``triton`` is refused: this package carries
    no Triton kernels, so a process that asked for them would otherwise get CUDA without being
    told. (The op-level ``backend`` argument still accepts ``"triton"``, as the reference's op
    schema does, and serves it with the CUDA kernels: that string names a route, not a
    toolchain the caller depends on.)"""
    value = os.environ.get(BACKEND_ENV, "cuda").strip().lower()
    if value == "triton":
        raise ValueError(
            f"{BACKEND_ENV}=triton: tokenforge_b200 has no Triton path; use 'cuda', or 'marlin' "
            "to keep the serving engine's own AWQ kernels"
        )
    if value not in BACKENDS:
        raise ValueError(f"{BACKEND_ENV}={value!r} is not one of {BACKENDS}")
    return value  # type: ignore[return-value]


def layer_support(
    n: int, k: int, group_size: int, dtype: str, sm: int | None, backend: Backend
) -> FallbackReason | None:
    """``None`` if this backend can serve the layer, else the reason it cannot."""
    if backend == "marlin":
        return "kill_switch"
    if dtype not in ("float16", "torch.float16"):
        return "unsupported_dtype"
    if group_size not in SUPPORTED_GROUP_SIZES:
        return "unsupported_group_size"
    if n <= 0 or n % PACK_FACTOR or k % PACK_FACTOR or k % group_size:
        return "unsupported_shape"
    if sm is not None and sm < MIN_SM:
        return "unsupported_arch"
    return None


def record_layer_fallback(reason: FallbackReason) -> None:
    FALLBACKS.inc(reason=reason)


@dataclass(frozen=True)
class Decision:
    kernel: Kernel
    bucket: str
    fallback: FallbackReason | None = None


class BackendUnavailableError(RuntimeError):
    """The CUDA backend cannot run this call (CPU tensors or no kernel library)."""


def select(m: int, *, backend: Backend, on_gpu: bool, cuda_ext_available: bool) -> Decision:
    """Kernel for one call with ``m`` rows; the layer has already passed :func:`layer_support`."""
    if backend == "marlin":
        raise ValueError("backend 'marlin' is resolved per layer, not per call")
    if m < 1:
        raise ValueError(f"M must be >= 1, got {m}")
    if not on_gpu:
        raise BackendUnavailableError(
            "tokenforge_b200 runs on CUDA tensors only (sm_100a); got CPU tensors"
        )
    if not cuda_ext_available:
        raise BackendUnavailableError("tokenforge_b200 kernel library is not available")
    kernel: Kernel = "cuda_gemv" if m <= MAX_GEMV_M else "cuda_gemm"
    return Decision(kernel, bucket_label(m))


def record(decision: Decision) -> None:
    KERNEL_CALLS.inc(kernel=decision.kernel, bucket=decision.bucket)
    if decision.fallback is not None:
        FALLBACKS.inc(reason=decision.fallback)
