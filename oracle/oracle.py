"""CPU oracle for the quantized-linear path: ctypes wrapper of ``tf_oracle.c`` plus the AWQ
fixture generator.

TEST INFRASTRUCTURE ONLY. Imported by ``tests/``, ``__graft_entry__.smoke()`` (as the checker)
and ``bench.py`` (the timed CPU baseline); never by the product package ``tokenforge_b200``.

Every function restates a reference function (saransh-debugs/TokenForge; cited per function)
and is pinned against golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``, checked by ``tests/test_oracle_golden.py``). Inputs and
outputs are CPU torch tensors; fp16 data crosses into C as raw bit patterns.
"""

from __future__ import annotations

import ctypes
import functools
import os
import subprocess
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
SRC = HERE / "tf_oracle.c"
LIB = HERE / "_build" / "libtf_oracle.so"

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SIG = {
    "oracle_unpack_int4": (None, [_P, _I64, _P]),
    "oracle_pack_int4": (None, [_P, _I64, _P]),
    "oracle_repack_awq_to_tf": (None, [_P, _I64, _I64, _P]),
    "oracle_dequantize_tf": (None, [_P, _P, _P, _I64, _I64, _I64, _P]),
    "oracle_w4a16_ref_f64": (None, [_P, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _P]),
    "oracle_w4a16_cpu_f32": (None, [_P, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _P, _P, _I64]),
    "oracle_e4m3": (ctypes.c_uint8, [ctypes.c_float]),
    "oracle_e4m3_value": (ctypes.c_double, [ctypes.c_uint8]),
    "oracle_w4a16_ref_fp8_f64": (None, [_P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _P]),
    "oracle_rmsnorm_fp8": (None, [_P, _I64, _I64, _P, ctypes.c_float, _P, _P, _P]),
}

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)  # pack.py:32
AWQ_REVERSE_ORDER = (0, 4, 1, 5, 2, 6, 3, 7)  # pack.py:35
FP8_E4M3_MAX = 448.0  # reference.py:9
MIN_SCALE = 1.0 / (FP8_E4M3_MAX * 512.0)  # reference.py:10


def build(force: bool = False) -> Path:
    """Compile the C restatement with gcc (OpenMP) into ``oracle/_build``."""
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        LIB.parent.mkdir(exist_ok=True)
        tmp = LIB.with_suffix(f".{os.getpid()}.tmp")
        subprocess.run(
            ["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-o", str(tmp), str(SRC), "-lm"],
            check=True,
        )
        os.replace(tmp, LIB)
    return LIB


@functools.cache
def _lib() -> ctypes.CDLL:
    handle = ctypes.CDLL(str(build()))
    for name, (res, args) in _SIG.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    return handle


def _np(t: torch.Tensor | np.ndarray, dtype: np.dtype) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        t = t.detach().cpu()
        if t.dtype == torch.float16:
            t = t.view(torch.int16)
        t = t.numpy()
    return np.ascontiguousarray(t).view(dtype) if t.dtype.itemsize == np.dtype(dtype).itemsize else np.ascontiguousarray(t.astype(dtype))


def _addr(a: np.ndarray | None) -> int | None:
    return None if a is None else a.ctypes.data


def _f16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.view(np.int16).copy()).view(torch.float16)


# ----------------------------------------------------------------------------- codec


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """unpack_int4, pack.py:57-67."""
    p = _np(packed, np.int32)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 8,), dtype=np.int32)
    _lib().oracle_unpack_int4(_addr(p), p.size, _addr(out))
    return torch.from_numpy(out)


def pack_int4(values: torch.Tensor) -> torch.Tensor:
    """pack_int4, pack.py:42-54 (range errors as the reference)."""
    if values.shape[-1] % 8 != 0:
        raise ValueError(f"last dim {values.shape[-1]} is not a multiple of 8")
    v = _np(values.to(torch.int32), np.int32)
    if v.size and (int(v.min()) < 0 or int(v.max()) > 15):
        raise ValueError("int4 values must lie in [0, 15]")
    out = np.empty(v.shape[:-1] + (v.shape[-1] // 8,), dtype=np.int32)
    _lib().oracle_pack_int4(_addr(v), out.size, _addr(out))
    return torch.from_numpy(out)


def awq_pack(intweight: torch.Tensor, zeros: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """awq_pack, pack.py:73-75."""
    return pack_int4(intweight), pack_int4(zeros)


def repack_awq_to_tf(qweight: torch.Tensor) -> torch.Tensor:
    """repack_awq_to_tf, pack.py:141-143: [K, N/8] -> [N, K/8]."""
    q = _np(qweight, np.int32)
    k, n8 = q.shape
    out = np.empty((n8 * 8, k // 8), dtype=np.int32)
    _lib().oracle_repack_awq_to_tf(_addr(q), k, n8 * 8, _addr(out))
    return torch.from_numpy(out)


def repack_tf_to_awq(qweight_t: torch.Tensor) -> torch.Tensor:
    """repack_tf_to_awq, pack.py:146-148: the same transform with K and N exchanged."""
    return repack_awq_to_tf(qweight_t)


# ----------------------------------------------------------------------------- dequant / GEMM


def dequantize_tf(qweight_t: torch.Tensor, scales: torch.Tensor, qzeros: torch.Tensor,
                  group_size: int) -> torch.Tensor:
    """dequantize_tf, pack.py:189-194: fp16 [N, K]."""
    q, s, z = _np(qweight_t, np.int32), _np(scales, np.uint16), _np(qzeros, np.int32)
    n, k = q.shape[0], q.shape[1] * 8
    out = np.empty((n, k), dtype=np.uint16)
    _lib().oracle_dequantize_tf(_addr(q), _addr(s), _addr(z), n, k, group_size, _addr(out))
    return _f16(out)


def w4a16_reference(x: torch.Tensor, qweight_t: torch.Tensor, scales: torch.Tensor,
                    qzeros: torch.Tensor, group_size: int,
                    bias: torch.Tensor | None = None) -> torch.Tensor:
    """w4a16_reference, reference.py:13-21: fp64 [M, N]."""
    xs = _np(x.reshape(-1, x.shape[-1]), np.uint16)
    q, s, z = _np(qweight_t, np.int32), _np(scales, np.uint16), _np(qzeros, np.int32)
    b = None if bias is None else _np(bias, np.uint16)
    m, k = xs.shape
    n = q.shape[0]
    out = np.empty((m, n), dtype=np.float64)
    _lib().oracle_w4a16_ref_f64(_addr(xs), m, k, _addr(q), _addr(s), _addr(z), _addr(b), n,
                                group_size, _addr(out))
    return torch.from_numpy(out)


def w4a16_cpu(x: torch.Tensor, qweight_t: torch.Tensor, scales: torch.Tensor,
              qzeros: torch.Tensor, group_size: int, bias: torch.Tensor | None = None,
              threads: int | None = None) -> torch.Tensor:
    """w4a16_torch, reference.py:24-32 (dequant + fp32 matmul): fp16 [M, N]."""
    xs = _np(x.reshape(-1, x.shape[-1]), np.uint16)
    q, s, z = _np(qweight_t, np.int32), _np(scales, np.uint16), _np(qzeros, np.int32)
    b = None if bias is None else _np(bias, np.uint16)
    m, k = xs.shape
    n = q.shape[0]
    nt = threads or os.cpu_count() or 1
    scratch = np.empty(nt * k, dtype=np.float32)
    out = np.empty((m, n), dtype=np.uint16)
    _lib().oracle_w4a16_cpu_f32(_addr(xs), m, k, _addr(q), _addr(s), _addr(z), _addr(b), n,
                                group_size, _addr(out), _addr(scratch), nt)
    return _f16(out)


# ----------------------------------------------------------------------------- RMSNorm + FP8


def e4m3_codes(values: torch.Tensor) -> torch.Tensor:
    """Saturating round-to-nearest-even fp32 -> e4m3fn codes (reference.py:49)."""
    v = values.detach().cpu().to(torch.float32).reshape(-1).tolist()
    f = _lib().oracle_e4m3
    return torch.tensor([f(x) for x in v], dtype=torch.uint8).reshape(values.shape)


def e4m3_values(codes: torch.Tensor) -> torch.Tensor:
    """Values of e4m3fn codes (uint8) as fp64, decoded from the format's bit fields."""
    f = _lib().oracle_e4m3_value
    c = codes.detach().cpu().to(torch.uint8).reshape(-1).tolist()
    return torch.tensor([f(v) for v in c], dtype=torch.float64).reshape(codes.shape)


def w4a16_reference_fp8(xq: torch.Tensor, x_scale: torch.Tensor, qweight_t: torch.Tensor,
                        scales: torch.Tensor, qzeros: torch.Tensor, group_size: int,
                        bias: torch.Tensor | None = None) -> torch.Tensor:
    """FP8-activation linear in fp64: (e4m3(xq) * x_scale) @ dequant(W)^T + bias. x_scale holds
    one fp32 value per token ([M] or [M, 1]) or a single static value."""
    q8 = _np(xq.reshape(-1, xq.shape[-1]), np.uint8)
    sc = _np(x_scale.reshape(-1).to(torch.float32), np.float32)
    stride = 0 if sc.size == 1 else 1
    q, s, z = _np(qweight_t, np.int32), _np(scales, np.uint16), _np(qzeros, np.int32)
    b = None if bias is None else _np(bias, np.uint16)
    m, k = q8.shape
    n = q.shape[0]
    out = np.empty((m, n), dtype=np.float64)
    _lib().oracle_w4a16_ref_fp8_f64(_addr(q8), _addr(sc), stride, m, k, _addr(q), _addr(s),
                                    _addr(z), _addr(b), n, group_size, _addr(out))
    return torch.from_numpy(out)


def rmsnorm_fp8(x: torch.Tensor, weight: torch.Tensor, eps: float,
                scale: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """rmsnorm_fp8_reference, reference.py:35-56 with the fp32 operations of
    triton/rmsnorm_fp8.py:57-73. Returns (e4m3 codes as uint8 [T, H], scale)."""
    xs = _np(x.reshape(-1, x.shape[-1]), np.uint16)
    w = _np(weight, np.uint16)
    t, h = xs.shape
    q = np.empty((t, h), dtype=np.uint8)
    s_out = np.empty((t, 1), dtype=np.float32)
    st = None if scale is None else _np(scale.reshape(1).to(torch.float32), np.float32)
    _lib().oracle_rmsnorm_fp8(_addr(xs), t, h, _addr(w), eps, _addr(st), _addr(q), _addr(s_out))
    return torch.from_numpy(q), (torch.from_numpy(s_out) if scale is None else scale.clone())


# ----------------------------------------------------------------------------- fixtures


def awq_quantize(weight: torch.Tensor, group_size: int
                 ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Min-max asymmetric int4 quantization of an ``[N, K]`` weight into AWQ format
    (awq_quantize, pack.py:83-107): scales = fp16((max - min).clamp(1e-5) / 15),
    zeros = clamp(-round(min / s), 0, 15), q = clamp(round(w / s) + zeros, 0, 15).
    Returns ``(qweight [K, N/8], qzeros [K/G, N/8], scales [K/G, N])``."""
    n, k = weight.shape
    if k % group_size != 0:
        raise ValueError(f"K={k} is not a multiple of group_size={group_size}")
    w = weight.to(torch.float32).reshape(n, k // group_size, group_size)
    hi = w.amax(dim=-1, keepdim=True)
    lo = w.amin(dim=-1, keepdim=True)
    s = ((hi - lo).clamp(min=1e-5) / 15).to(torch.float16).to(torch.float32)
    z = (-torch.round(lo / s)).clamp(0, 15)
    q = (torch.round(w / s) + z).clamp(0, 15)
    intweight = q.reshape(n, k).t().contiguous().to(torch.int32)
    zeros = z.squeeze(-1).t().contiguous().to(torch.int32)
    scales = s.squeeze(-1).t().contiguous().to(torch.float16)
    qweight, qzeros = awq_pack(intweight, zeros)
    return qweight, qzeros, scales
