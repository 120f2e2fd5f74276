"""ctypes binding of the sm_100a kernel library (C ABI declared in ``include/tokenforge_b200.h``).

The library is the only compute path of this package: there is no CPU or Triton fallback. If
the shared object is missing, :func:`lib` raises with the command that builds it.
"""

from __future__ import annotations

import ctypes
import functools
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libtokenforge_b200.so"

TF_OK = 0
TF_ERR_INVALID_ARG = 1
TF_ERR_ALIGNMENT = 2
TF_ERR_WORKSPACE = 3
TF_ERR_UNSUPPORTED = 4
TF_ERR_CUDA = 5
TF_ERR_NO_DEVICE = 6
TF_ERR_TOO_LARGE = 7

TF_LAUNCH_PDL = 1

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_SZ = ctypes.c_size_t
_F32 = ctypes.c_float

# name -> (restype, argtypes); mirrors include/tokenforge_b200.h
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "tf_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "tf_last_cuda_error": (ctypes.c_int, []),
    "tf_abi_version": (ctypes.c_int, []),
    "tf_set_launch_flags": (None, [ctypes.c_uint32]),
    "tf_get_launch_flags": (ctypes.c_uint32, []),
    "tf_awq_repack": (ctypes.c_int, [_P, _I64, _I64, _P, _P]),
    "tf_awq_unrepack": (ctypes.c_int, [_P, _I64, _I64, _P, _P]),
    "tf_pack_int4": (ctypes.c_int, [_P, _I64, _P, _P]),
    "tf_unpack_int4": (ctypes.c_int, [_P, _I64, _P, _P]),
    "tf_w4a16_dequant": (ctypes.c_int, [_P, _P, _P, _I64, _I64, _I32, _P, _P]),
    "tf_w4a16_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I32]),
    "tf_w4a16_gemv": (
        ctypes.c_int,
        [_P, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _I32, _P, _I64, _P, _SZ, _P],
    ),
    "tf_w4a16_gemm": (
        ctypes.c_int,
        [_P, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _I32, _P, _I64, _P, _SZ, _P],
    ),
    "tf_w4a16_linear": (
        ctypes.c_int,
        [_P, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _I32, _P, _I64, _P, _SZ, _P],
    ),
    "tf_w4a16_linear_noalloc": (
        ctypes.c_int,
        [_P, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _I32, _P, _I64, _P],
    ),
    "tf_w4a16_fp8_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I32]),
    "tf_w4a16_linear_fp8": (
        ctypes.c_int,
        [_P, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _I32, _P, _I64, _P, _SZ, _P],
    ),
    "tf_rmsnorm_fp8_w4a16_linear": (
        ctypes.c_int,
        [_P, _I64, _I64, _I64, _P, _F32, _P, _P, _P, _P, _P, _P, _I64, _I32, _P, _I64, _P, _SZ,
         _P],
    ),
    "tf_silu_mul": (ctypes.c_int, [_P, _I64, _I64, _I64, _P, _I64, _P]),
    "tf_silu_mul_w4a16_linear": (
        ctypes.c_int,
        [_P, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _I32, _P, _I64, _P, _SZ, _P],
    ),
    "tf_peer_mailbox_bytes": (_SZ, [_I32, _I32, _I32]),
    "tf_peer_mailbox_alloc": (ctypes.c_int, [_SZ, _P, _P]),
    "tf_peer_mailbox_open": (ctypes.c_int, [_P, _P]),
    "tf_peer_mailbox_close": (ctypes.c_int, [_P]),
    "tf_peer_mailbox_free": (ctypes.c_int, [_P]),
    "tf_peer_mailbox_error": (ctypes.c_int, [_P, _P]),
    "tf_peer_trace": (ctypes.c_int, [_P]),
    "tf_w4a16_linear_allreduce": (
        ctypes.c_int,
        [_P, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _I32, _P, _I64, _P, _SZ, _P, _P],
    ),
    "tf_launch_plan": (ctypes.c_int, [_I64, _I64, _I64, _I32, _P]),
    "tf_rmsnorm_fp8_quant": (ctypes.c_int, [_P, _I64, _I64, _I64, _P, _F32, _P, _P, _P, _P]),
    "tf_cast_e4m3": (ctypes.c_int, [_P, _I64, _P, _P]),
    "tf_e4m3_quant_rows": (ctypes.c_int, [_P, _I64, _I64, _I64, _P, _I64, _P, _P, _P]),
    "tf_device_error": (ctypes.c_int, [_P]),
    "tf_reset_device_error": (ctypes.c_int, []),
    "tf_decode_chain_create": (ctypes.c_int, [_P, _I32, _I64, _I32, _P]),
    "tf_decode_chain_run": (ctypes.c_int, [_P, _P]),
    "tf_decode_chain_error": (ctypes.c_int, [_P, _P]),
    "tf_decode_chain_destroy": (ctypes.c_int, [_P]),
    "tf_decode_chain_plan": (ctypes.c_int, [_P, _P, _I32, _I64, _I32, _P, _I32, _P]),
}

TF_MAX_PEERS = 8
TF_IPC_HANDLE_BYTES = 64


class TfPeerSet(ctypes.Structure):
    """Mirror of ``TfPeerSet`` in include/tokenforge_b200.h."""

    _fields_ = [
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("max_m", ctypes.c_int32),
        ("max_n", ctypes.c_int32),
        ("mailbox", ctypes.c_void_p * TF_MAX_PEERS),
    ]


class TfChainOp(ctypes.Structure):
    """Mirror of ``TfChainOp`` in include/tokenforge_b200.h."""

    _fields_ = [
        ("x", ctypes.c_void_p),
        ("ldx", ctypes.c_int64),
        ("qweight_t", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("qzeros", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("ldy", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("wait", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class TfChainUnitInfo(ctypes.Structure):
    """Mirror of ``TfChainUnitInfo`` in include/tokenforge_b200.h."""

    _fields_ = [(name, ctypes.c_int32) for name in
                ("cta", "op", "tile0", "rtiles", "c0", "c1", "piece", "pieces", "flags")]


_lock = threading.Lock()


class KernelLibraryError(RuntimeError):
    """A kernel-library call returned a non-zero status."""

    def __init__(self, fn: str, status: int, detail: str) -> None:
        super().__init__(f"{fn} failed: {detail} (status {status})")
        self.fn = fn
        self.status = status


@functools.cache
def lib() -> ctypes.CDLL:
    """Load the kernel library once per process; raise if it has not been built."""
    if not LIB_PATH.exists():
        raise ImportError(
            f"tokenforge_b200 kernel library not found at {LIB_PATH}; build it with "
            "`python -m tokenforge_b200._build` (requires nvcc)"
        )
    with _lock:
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
    return handle


def status_string(status: int) -> str:
    return lib().tf_status_string(status).decode()


def check(fn: str, status: int) -> None:
    if status == TF_OK:
        return
    detail = status_string(status)
    if status == TF_ERR_CUDA:
        detail += f" (cudaError {lib().tf_last_cuda_error()})"
    raise KernelLibraryError(fn, status, detail)


def stream_ptr(device: torch.device) -> int:
    """Raw handle of the current CUDA stream on ``device`` (work is enqueued there)."""
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def set_launch_flags(flags: int) -> None:
    lib().tf_set_launch_flags(flags)


def get_launch_flags() -> int:
    return int(lib().tf_get_launch_flags())


def device_error() -> int:
    """Device-side status word of kernels with bounded waits (synchronises the device)."""
    out = ctypes.c_int(0)
    check("tf_device_error", lib().tf_device_error(ctypes.byref(out)))
    return int(out.value)
