"""Persistent decode chain: a fixed sequence of W4A16 linears run as one kernel launch.

At decode sizes (1 to 8 tokens) a linear layer streams a few MB of int4 weights, which on B200
takes about as long as the fixed cost of launching and draining a kernel. A :class:`DecodeChain`
records the sequence once (weights, activation and output buffers, and which ops read an
earlier op's output) and then runs it as ONE persistent kernel (C ABI ``tf_decode_chain_*``):
one CTA per SM streams weight chunks with TMA into shared-memory rings that keep loading the
next layers while the current one finishes, and layer-to-layer dependencies are device-side
counters with bounded waits. Every op computes what ``torch.ops.tokenforge.w4a16_linear``
computes for it, within the W4A16 tolerance (the K split, hence the fp32 sum order, differs);
a chain's results are deterministic.

The chain keeps the addresses it was built with: reuse the same input and output tensors
across runs (as a CUDA graph does). No reference counterpart: the reference calls the linear op
once per layer (tokenforge/kernels/ops.py:48).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from tokenforge_b200 import _lib
from tokenforge_b200.pack import W4A16Weights

MAX_TOKENS = 8
GROUP_SIZE = 128


@dataclass
class ChainLinear:
    """One op of a chain: ``y = x @ dequant(weights)^T (+ bias)``. ``wait``: ``x`` is (or
    depends on) an earlier op's output, so the op reads it only after every earlier op of the
    chain has finished."""

    x: torch.Tensor  # fp16 [M, K], unit stride along K
    weights: W4A16Weights
    y: torch.Tensor  # fp16 [M, N], unit stride along N
    bias: torch.Tensor | None = None
    wait: bool = True


@dataclass(frozen=True)
class ChainUnit:
    """One unit of the schedule (see ``tf_decode_chain_plan``)."""

    cta: int
    op: int
    tile0: int
    rtiles: int
    c0: int
    c1: int
    piece: int
    pieces: int
    flags: int


def plan(shapes: list[tuple[int, int]], m: int, num_ctas: int = 148) -> list[ChainUnit]:
    """The unit schedule of a chain of ``(N, K)`` ops at ``m`` tokens on ``num_ctas`` SMs,
    computed on the host (no GPU needed)."""
    lib = _lib.lib()
    n = (ctypes.c_int64 * len(shapes))(*[s[0] for s in shapes])
    k = (ctypes.c_int64 * len(shapes))(*[s[1] for s in shapes])
    count = ctypes.c_int32(0)
    st = lib.tf_decode_chain_plan(n, k, len(shapes), m, num_ctas, None, 0, ctypes.byref(count))
    _lib.check("tf_decode_chain_plan", st)
    out = (_lib.TfChainUnitInfo * max(count.value, 1))()
    st = lib.tf_decode_chain_plan(n, k, len(shapes), m, num_ctas, out, count.value,
                                  ctypes.byref(count))
    _lib.check("tf_decode_chain_plan", st)
    return [ChainUnit(*(getattr(u, f) for f, _ in _lib.TfChainUnitInfo._fields_))
            for u in out[: count.value]]


class DecodeChain:
    """A recorded sequence of decode linears run as one persistent kernel (see the module
    docstring). Build it once; :meth:`run` enqueues one launch on the current stream."""

    def __init__(self, linears: list[ChainLinear]) -> None:
        if not linears:
            raise ValueError("a chain needs at least one linear")
        m = linears[0].x.shape[0]
        device = linears[0].x.device
        if not 1 <= m <= MAX_TOKENS:
            raise ValueError(f"a decode chain serves 1 to {MAX_TOKENS} tokens, got M={m}")
        ops = (_lib.TfChainOp * len(linears))()
        for i, op in enumerate(linears):
            w = op.weights
            if w.group_size != GROUP_SIZE:
                raise ValueError(f"op {i}: a decode chain serves group size {GROUP_SIZE}")
            if op.x.dim() != 2 or op.x.shape != (m, w.k) or op.x.dtype != torch.float16:
                raise ValueError(f"op {i}: x must be fp16 [{m}, {w.k}], got "
                                 f"{op.x.dtype} {tuple(op.x.shape)}")
            if op.y.dim() != 2 or op.y.shape != (m, w.n) or op.y.dtype != torch.float16:
                raise ValueError(f"op {i}: y must be fp16 [{m}, {w.n}], got "
                                 f"{op.y.dtype} {tuple(op.y.shape)}")
            if op.x.stride(1) != 1 or op.y.stride(1) != 1:
                raise ValueError(f"op {i}: x and y must have unit stride along their last dim")
            for name, t in (("x", op.x), ("y", op.y), ("qweight_t", w.qweight_t),
                            ("scales", w.scales), ("qzeros", w.qzeros)):
                if t.device != device:
                    raise ValueError(f"op {i}: {name} is on {t.device}, the chain on {device}")
            if op.bias is not None and (op.bias.shape != (w.n,) or op.bias.dtype != torch.float16
                                        or not op.bias.is_contiguous()):
                raise ValueError(f"op {i}: bias must be contiguous fp16 [{w.n}]")
            ops[i].x = op.x.data_ptr()
            ops[i].ldx = op.x.stride(0) if m > 1 else w.k
            ops[i].qweight_t = w.qweight_t.data_ptr()
            ops[i].scales = w.scales.data_ptr()
            ops[i].qzeros = w.qzeros.data_ptr()
            ops[i].bias = _lib.ptr(op.bias)
            ops[i].y = op.y.data_ptr()
            ops[i].ldy = op.y.stride(0) if m > 1 else w.n
            ops[i].N = w.n
            ops[i].K = w.k
            ops[i].wait = 1 if op.wait else 0
        self.device = device
        self.m = m
        self.linears = list(linears)  # keeps every recorded buffer alive
        self._handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            st = _lib.lib().tf_decode_chain_create(ops, len(linears), m, GROUP_SIZE,
                                                   ctypes.byref(self._handle))
        _lib.check("tf_decode_chain_create", st)

    def run(self) -> None:
        """Enqueue one run of the chain on the device's current stream."""
        if not self._handle:
            raise RuntimeError("the chain was closed")
        with torch.cuda.device(self.device):
            st = _lib.lib().tf_decode_chain_run(self._handle, _lib.stream_ptr(self.device))
        _lib.check("tf_decode_chain_run", st)

    def error(self) -> int:
        """The chain's device error word (0: no bounded wait gave up), cleared on read.
        Synchronises the device."""
        out = ctypes.c_int(0)
        with torch.cuda.device(self.device):
            st = _lib.lib().tf_decode_chain_error(self._handle, ctypes.byref(out))
        _lib.check("tf_decode_chain_error", st)
        return int(out.value)

    def close(self) -> None:
        if self._handle:
            torch.cuda.synchronize(self.device)
            with torch.cuda.device(self.device):
                st = _lib.lib().tf_decode_chain_destroy(self._handle)
            self._handle = ctypes.c_void_p()
            _lib.check("tf_decode_chain_destroy", st)

    def __enter__(self) -> DecodeChain:
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()
