"""``torch.ops.tokenforge.*`` custom ops backed by the sm_100a kernel library.

Same op names, schemas, fake implementations and error messages as the reference's
tokenforge/kernels/ops.py (ADR 0004: custom ops with fakes, no host syncs, no host reads of
tensor values, shape-only dispatch), plus ``tokenforge::awq_repack``:

* ``tokenforge::w4a16_linear(x, qweight_t, scales, qzeros, bias, group_size, backend) -> y``
* ``tokenforge::w4a16_dequant(qweight_t, scales, qzeros, group_size) -> w [N, K] fp16``
* ``tokenforge::rmsnorm_fp8_quant(x, weight, eps, scale) -> (q e4m3, scale fp32)``
* ``tokenforge::awq_repack(qweight) -> qweight_t``

Every real implementation enqueues kernels on the current CUDA stream through the C ABI; the
only allocations are outputs and the optional split-K workspace, both from PyTorch's caching
allocator. CPU tensors raise: there is no CPU fallback.
"""

from __future__ import annotations

import functools

import torch

from tokenforge_b200 import _lib, dispatch
from tokenforge_b200.linear import (  # noqa: F401  (re-exported launch API)
    _VEC,
    _aligned_rows,
    _check_inputs,
    _launch_linear,
    _require,
    w4a16_gemm,
    w4a16_gemm_tc,
    w4a16_gemv,
)
from tokenforge_b200.pack import PACK_FACTOR


def cuda_ext_available() -> bool:
    """The kernel library is built and loadable."""
    return _ext() is not None


@functools.cache
def _ext():  # type: ignore[no-untyped-def]
    try:
        return _lib.lib()
    except (ImportError, OSError):
        return None


@torch.library.custom_op("tokenforge::w4a16_linear", mutates_args=())
def w4a16_linear(
    x: torch.Tensor,
    qweight_t: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor,
    bias: torch.Tensor | None,
    group_size: int,
    backend: str,
) -> torch.Tensor:
    k = x.shape[-1]
    n = qweight_t.shape[0]
    out_shape = (*x.shape[:-1], n)
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m = x2.shape[0]
    if m == 0:
        return x.new_empty(out_shape)
    if backend not in ("triton", "cuda"):
        raise ValueError(f"backend must be 'triton' or 'cuda' at op level, got {backend!r}")
    decision = dispatch.select(
        m, backend=backend, on_gpu=x.is_cuda, cuda_ext_available=cuda_ext_available()  # type: ignore[arg-type]
    )
    dispatch.record(decision)
    # M <= 8: the reference's _C.w4a16_gemv contract; larger M: the launch table (the 16-token
    # GEMV up to M = 16 with group size 128, the tensor-core GEMM above).
    entry = "gemv" if decision.kernel == "cuda_gemv" else "linear"
    return _launch_linear(entry, x2, qweight_t, scales, qzeros, bias, group_size).reshape(out_shape)


@w4a16_linear.register_fake
def _w4a16_linear_fake(x, qweight_t, scales, qzeros, bias, group_size, backend):  # type: ignore[no-untyped-def]
    return x.new_empty((*x.shape[:-1], qweight_t.shape[0]))


@torch.library.custom_op("tokenforge::w4a16_dequant", mutates_args=())
def w4a16_dequant(
    qweight_t: torch.Tensor, scales: torch.Tensor, qzeros: torch.Tensor, group_size: int
) -> torch.Tensor:
    for name, t in (("qweight_t", qweight_t), ("scales", scales), ("qzeros", qzeros)):
        _require(t, name)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    n, k = qweight_t.shape[0], qweight_t.shape[1] * PACK_FACTOR
    if group_size not in (32, 64, 128) or k % group_size:
        raise ValueError(f"K={k} is not a multiple of group_size={group_size}")
    if tuple(scales.shape) != (k // group_size, n) or tuple(qzeros.shape) != (
        k // group_size,
        n // PACK_FACTOR,
    ):
        raise ValueError("scales/qzeros shape does not match qweight_t")
    out = torch.empty((n, k), dtype=torch.float16, device=qweight_t.device)
    with torch.cuda.device(qweight_t.device):
        status = _lib.lib().tf_w4a16_dequant(
            qweight_t.data_ptr(), scales.data_ptr(), qzeros.data_ptr(), n, k, group_size,
            out.data_ptr(), _lib.stream_ptr(qweight_t.device),
        )  # fmt: skip
    _lib.check("tf_w4a16_dequant", status)
    return out


@w4a16_dequant.register_fake
def _w4a16_dequant_fake(qweight_t, scales, qzeros, group_size):  # type: ignore[no-untyped-def]
    return qweight_t.new_empty((qweight_t.shape[0], qweight_t.shape[1] * 8), dtype=torch.float16)


@torch.library.custom_op("tokenforge::w4a16_linear_fp8", mutates_args=())
def w4a16_linear_fp8(
    xq: torch.Tensor,
    x_scale: torch.Tensor,
    qweight_t: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor,
    bias: torch.Tensor | None,
    group_size: int,
) -> torch.Tensor:
    """W4A16 linear on FP8 activations, the consumer of ``rmsnorm_fp8_quant``'s output:
    ``x = e4m3(xq) * x_scale`` with ``x_scale`` one fp32 per token (``[..., 1]``) or a single
    static value. No reference counterpart (the reference produces e4m3 activations only)."""
    k = xq.shape[-1]
    n = qweight_t.shape[0]
    out_shape = (*xq.shape[:-1], n)
    if xq.dtype not in (torch.float8_e4m3fn, torch.uint8):
        raise TypeError(f"xq must be float8_e4m3fn (or its uint8 codes), got {xq.dtype}")
    if x_scale.dtype != torch.float32:
        raise TypeError(f"x_scale must be fp32, got {x_scale.dtype}")
    x2 = xq.reshape(-1, k)
    m = x2.shape[0]
    if m == 0:
        return torch.empty(out_shape, dtype=torch.float16, device=xq.device)
    if x_scale.numel() not in (1, m):
        raise ValueError(f"x_scale must hold one value per token ({m}) or a single value, "
                         f"got {x_scale.numel()}")
    _check_inputs(torch.empty((m, k), dtype=torch.float16, device="meta"), qweight_t, scales,
                  qzeros, group_size)
    for name, t in (("xq", xq), ("x_scale", x_scale), ("qweight_t", qweight_t),
                    ("scales", scales), ("qzeros", qzeros)):
        _require(t, name)
    if bias is not None:
        _require(bias, "bias")
        if tuple(bias.shape) != (n,) or bias.dtype != torch.float16:
            raise ValueError(f"bias must be fp16 [{n}]")
        bias = bias.contiguous()
    x2 = x2.view(torch.uint8)
    if x2.stride(-1) != 1 or x2.data_ptr() % 8 or (m > 1 and x2.stride(0) % 8):
        x2 = x2.contiguous()
        if x2.data_ptr() % 8:
            x2 = x2.clone()
    sc = x_scale.reshape(-1).contiguous()
    y = torch.empty((m, n), dtype=torch.float16, device=xq.device)
    lib = _lib.lib()
    wsb = int(lib.tf_w4a16_fp8_workspace_bytes(m, n, k, group_size))
    ws = torch.empty(wsb, dtype=torch.uint8, device=xq.device) if wsb else None
    with torch.cuda.device(xq.device):
        status = lib.tf_w4a16_linear_fp8(
            x2.data_ptr(), sc.data_ptr(), 0 if sc.numel() == 1 else 1, m, k, x2.stride(0),
            qweight_t.data_ptr(), scales.data_ptr(), qzeros.data_ptr(), _lib.ptr(bias), n,
            group_size, y.data_ptr(), n, _lib.ptr(ws), wsb, _lib.stream_ptr(xq.device),
        )  # fmt: skip
    _lib.check("tf_w4a16_linear_fp8", status)
    return y.reshape(out_shape)


@w4a16_linear_fp8.register_fake
def _w4a16_linear_fp8_fake(xq, x_scale, qweight_t, scales, qzeros, bias, group_size):  # type: ignore[no-untyped-def]
    return torch.empty((*xq.shape[:-1], qweight_t.shape[0]), dtype=torch.float16,
                       device=xq.device)


@torch.library.custom_op("tokenforge::rmsnorm_fp8_w4a16_linear", mutates_args=())
def rmsnorm_fp8_w4a16_linear(
    x: torch.Tensor,
    norm_weight: torch.Tensor,
    eps: float,
    scale: torch.Tensor | None,
    qweight_t: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor,
    bias: torch.Tensor | None,
    group_size: int,
) -> torch.Tensor:
    """``w4a16_linear_fp8(*rmsnorm_fp8_quant(x, norm_weight, eps, scale), ...)``. For one or two
    tokens on a layer whose decode plan keeps K in one CTA, this is one kernel: the normalised
    and quantised activations stay in shared memory, and y is bit-identical to the two-op path.
    Otherwise the two ops run (both on the GPU): every CTA of the fused kernel normalises all
    M rows itself, which on B200 costs more than the saved launch from M = 4 on (measured in
    the config-4 block stack: +10.6% tokens/s at M = 1, +3.1% at 2, -6% at 4, -17% at 8).
    No reference counterpart."""
    k = x.shape[-1]
    n = qweight_t.shape[0]
    out_shape = (*x.shape[:-1], n)
    x2 = x.reshape(-1, k)
    m = x2.shape[0]
    if m == 0:
        return torch.empty(out_shape, dtype=torch.float16, device=x.device)
    if x.dtype != torch.float16 or norm_weight.dtype != torch.float16:
        raise TypeError("x and norm_weight must be fp16")
    if tuple(norm_weight.shape) != (k,):
        raise ValueError(f"norm_weight shape {tuple(norm_weight.shape)} != {(k,)}")
    if scale is not None and (scale.numel() != 1 or scale.dtype != torch.float32):
        raise ValueError("static scale must be a single fp32 element")
    _check_inputs(x2, qweight_t, scales, qzeros, group_size)
    for name, t in (("x", x), ("norm_weight", norm_weight), ("qweight_t", qweight_t),
                    ("scales", scales), ("qzeros", qzeros)):
        _require(t, name)
    if bias is not None:
        _require(bias, "bias")
        if tuple(bias.shape) != (n,) or bias.dtype != torch.float16:
            raise ValueError(f"bias must be fp16 [{n}]")
        bias = bias.contiguous()
    if m <= 2:
        # The kernel reads row m at x + m * ldx: a row-strided view keeps its own stride.
        xc = _aligned_rows(x2)
        nw = norm_weight.contiguous()
        if nw.data_ptr() % _VEC:
            nw = nw.clone()
        if scale is not None:
            _require(scale, "scale")
        y = torch.empty((m, n), dtype=torch.float16, device=x.device)
        with torch.cuda.device(x.device):
            status = _lib.lib().tf_rmsnorm_fp8_w4a16_linear(
                xc.data_ptr(), m, k, xc.stride(0) if m > 1 else k, nw.data_ptr(), float(eps),
                _lib.ptr(scale), None, qweight_t.data_ptr(), scales.data_ptr(),
                qzeros.data_ptr(), _lib.ptr(bias), n, group_size, y.data_ptr(), n, None, 0,
                _lib.stream_ptr(x.device),
            )  # fmt: skip
        if status == _lib.TF_OK:
            return y.reshape(out_shape)
        if status != _lib.TF_ERR_UNSUPPORTED:
            _lib.check("tf_rmsnorm_fp8_w4a16_linear", status)
    q, s = rmsnorm_fp8_quant(x2, norm_weight, eps, scale)
    return w4a16_linear_fp8(q, s, qweight_t, scales, qzeros, bias, group_size).reshape(out_shape)


@rmsnorm_fp8_w4a16_linear.register_fake
def _rmsnorm_fp8_w4a16_linear_fake(x, norm_weight, eps, scale, qweight_t, scales, qzeros, bias,  # type: ignore[no-untyped-def]
                                   group_size):
    return torch.empty((*x.shape[:-1], qweight_t.shape[0]), dtype=torch.float16,
                       device=x.device)


# Fuse up to this many tokens: every CTA of down computes silu(g) * u (an exp and an IEEE
# division) for its whole K range before its first tensor-core step; measured in the config-4
# block stack, +1.4% tokens/s at M = 1 (within run-to-run spread), -4.5% at M = 2.
SILU_FUSE_MAX_M = 1


@torch.library.custom_op("tokenforge::silu_mul_w4a16_linear", mutates_args=())
def silu_mul_w4a16_linear(
    gate_up: torch.Tensor,
    qweight_t: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor,
    bias: torch.Tensor | None,
    group_size: int,
) -> torch.Tensor:
    """``w4a16_linear(silu_mul(gate_up), ...)``: the MLP's down projection on the SiLU-gated
    product of its gate_up output [..., 2K]. For small M on layers whose decode plan keeps K in
    one CTA this is one kernel that forms the products while staging its activations (the
    intermediate never reaches HBM); y is bit-identical to the two ops, which run otherwise.
    No reference counterpart."""
    k = qweight_t.shape[1] * PACK_FACTOR
    n = qweight_t.shape[0]
    if gate_up.shape[-1] != 2 * k:
        raise ValueError(f"gate_up's last dimension {gate_up.shape[-1]} != 2 * K = {2 * k}")
    if gate_up.dtype != torch.float16:
        raise TypeError(f"gate_up must be fp16, got {gate_up.dtype}")
    out_shape = (*gate_up.shape[:-1], n)
    g2 = gate_up.reshape(-1, 2 * k)
    m = g2.shape[0]
    if m == 0:
        return torch.empty(out_shape, dtype=torch.float16, device=gate_up.device)
    _check_inputs(torch.empty((m, k), dtype=torch.float16, device="meta"), qweight_t, scales,
                  qzeros, group_size)
    for name, t in (("gate_up", gate_up), ("qweight_t", qweight_t), ("scales", scales),
                    ("qzeros", qzeros)):
        _require(t, name)
    if bias is not None:
        _require(bias, "bias")
        if tuple(bias.shape) != (n,) or bias.dtype != torch.float16:
            raise ValueError(f"bias must be fp16 [{n}]")
        bias = bias.contiguous()
    if m <= SILU_FUSE_MAX_M:
        gc = g2
        if gc.stride(-1) != 1 or gc.data_ptr() % _VEC or (m > 1 and gc.stride(0) % 8):
            gc = g2.contiguous()
            if gc.data_ptr() % _VEC:
                gc = gc.clone()
        y = torch.empty((m, n), dtype=torch.float16, device=gate_up.device)
        with torch.cuda.device(gate_up.device):
            status = _lib.lib().tf_silu_mul_w4a16_linear(
                gc.data_ptr(), m, k, gc.stride(0) if m > 1 else 2 * k, qweight_t.data_ptr(),
                scales.data_ptr(), qzeros.data_ptr(), _lib.ptr(bias), n, group_size,
                y.data_ptr(), n, None, 0, _lib.stream_ptr(gate_up.device),
            )  # fmt: skip
        if status == _lib.TF_OK:
            return y.reshape(out_shape)
        if status != _lib.TF_ERR_UNSUPPORTED:
            _lib.check("tf_silu_mul_w4a16_linear", status)
    a = silu_mul(g2)
    return w4a16_gemm(a, qweight_t, scales, qzeros, group_size, bias).reshape(out_shape)


@silu_mul_w4a16_linear.register_fake
def _silu_mul_w4a16_linear_fake(gate_up, qweight_t, scales, qzeros, bias, group_size):  # type: ignore[no-untyped-def]
    return torch.empty((*gate_up.shape[:-1], qweight_t.shape[0]), dtype=torch.float16,
                       device=gate_up.device)


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """``gate_up [..., 2I] fp16 -> silu(gate) * up [..., I] fp16`` (fp32 inside, one rounding)."""
    if gate_up.dtype != torch.float16:
        raise TypeError(f"gate_up must be fp16, got {gate_up.dtype}")
    if gate_up.shape[-1] % 2:
        raise ValueError("gate_up's last dimension must be even (gate and up halves)")
    _require(gate_up, "gate_up")
    i = gate_up.shape[-1] // 2
    g2 = gate_up.reshape(-1, 2 * i)
    if g2.stride(-1) != 1:
        g2 = g2.contiguous()
    out = torch.empty((g2.shape[0], i), dtype=torch.float16, device=gate_up.device)
    with torch.cuda.device(gate_up.device):
        status = _lib.lib().tf_silu_mul(g2.data_ptr(), g2.shape[0], i, g2.stride(0),
                                        out.data_ptr(), i, _lib.stream_ptr(gate_up.device))
    _lib.check("tf_silu_mul", status)
    return out.reshape(*gate_up.shape[:-1], i)


def rmsnorm_fp8_quant_2d(
    x: torch.Tensor, weight: torch.Tensor, eps: float, scale: torch.Tensor | None = None
) -> tuple[torch.Tensor, torch.Tensor]:
    """``x [T, H]`` -> ``(q [T, H] e4m3, scale)``; contract of triton/rmsnorm_fp8.py:76-117.

    ``scale`` is ``[T, 1]`` fp32 (dynamic per token) or the given single-element fp32 tensor
    (static per tensor), which is returned as is.
    """
    if x.dim() != 2:
        raise ValueError(f"x must be 2-D [T, H], got {tuple(x.shape)}")
    t, h = x.shape
    if tuple(weight.shape) != (h,):
        raise ValueError(f"weight shape {tuple(weight.shape)} != {(h,)}")
    if x.stride(1) != 1:
        raise ValueError("x must be contiguous along H")
    if x.dtype != torch.float16 or weight.dtype != torch.float16:
        raise TypeError("x and weight must be fp16")
    if scale is not None and (scale.numel() != 1 or scale.dtype != torch.float32):
        raise ValueError("static scale must be a single fp32 element")
    _require(x, "x")
    _require(weight, "weight")
    out = torch.empty((t, h), dtype=torch.float8_e4m3fn, device=x.device)
    scale_out = torch.empty((t, 1), dtype=torch.float32, device=x.device) if scale is None else scale
    if t == 0:
        return out, scale_out
    if scale is not None:
        _require(scale, "scale")
    if x.data_ptr() % _VEC or (t > 1 and x.stride(0) % 8):
        x = x.clone(memory_format=torch.contiguous_format)
    weight = weight.contiguous()
    with torch.cuda.device(x.device):
        status = _lib.lib().tf_rmsnorm_fp8_quant(
            x.data_ptr(), t, h, x.stride(0) if t > 1 else h, weight.data_ptr(), float(eps),
            _lib.ptr(scale), out.data_ptr(), None if scale is not None else scale_out.data_ptr(),
            _lib.stream_ptr(x.device),
        )  # fmt: skip
    _lib.check("tf_rmsnorm_fp8_quant", status)
    return out, scale_out


@torch.library.custom_op("tokenforge::rmsnorm_fp8_quant", mutates_args=())
def rmsnorm_fp8_quant(
    x: torch.Tensor, weight: torch.Tensor, eps: float, scale: torch.Tensor | None
) -> tuple[torch.Tensor, torch.Tensor]:
    h = x.shape[-1]
    x2 = x.reshape(-1, h)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    q, s = rmsnorm_fp8_quant_2d(x2, weight, eps, scale)
    if scale is not None:
        s = s.clone()  # a custom op may not return an alias of an input
    return q.reshape(x.shape), s.reshape((*x.shape[:-1], 1)) if scale is None else s


@rmsnorm_fp8_quant.register_fake
def _rmsnorm_fp8_quant_fake(x, weight, eps, scale):  # type: ignore[no-untyped-def]
    q = x.new_empty(x.shape, dtype=torch.float8_e4m3fn)
    if scale is None:
        return q, x.new_empty((*x.shape[:-1], 1), dtype=torch.float32)
    return q, torch.empty_like(scale)


def _check_packed(t: torch.Tensor, name: str) -> None:
    if t.dim() != 2:
        raise ValueError(f"{name} must be 2-D, got shape {tuple(t.shape)}")
    if t.dtype != torch.int32:
        raise TypeError(f"{name} must be int32, got {t.dtype}")
    _require(t, name)


@torch.library.custom_op("tokenforge::awq_repack", mutates_args=())
def awq_repack(qweight: torch.Tensor) -> torch.Tensor:
    """AWQ ``qweight [K, N/8]`` -> ``qweight_t [N, K/8]``, bit-exact with repack_awq_to_tf."""
    _check_packed(qweight, "qweight")
    k, n8 = qweight.shape
    if k % PACK_FACTOR:
        raise ValueError(f"K={k} is not a multiple of {PACK_FACTOR}")
    qweight = qweight.contiguous()
    out = torch.empty((n8 * PACK_FACTOR, k // PACK_FACTOR), dtype=torch.int32, device=qweight.device)
    with torch.cuda.device(qweight.device):
        status = _lib.lib().tf_awq_repack(
            qweight.data_ptr(), k, n8 * PACK_FACTOR, out.data_ptr(), _lib.stream_ptr(qweight.device)
        )
    _lib.check("tf_awq_repack", status)
    return out


@awq_repack.register_fake
def _awq_repack_fake(qweight):  # type: ignore[no-untyped-def]
    return qweight.new_empty((qweight.shape[1] * 8, qweight.shape[0] // 8))


def awq_unrepack_cuda(qweight_t: torch.Tensor) -> torch.Tensor:
    """Kernel ``qweight_t [N, K/8]`` -> AWQ ``qweight [K, N/8]`` (repack_tf_to_awq)."""
    _check_packed(qweight_t, "qweight_t")
    n, k8 = qweight_t.shape
    if n % PACK_FACTOR:
        raise ValueError(f"N={n} is not a multiple of {PACK_FACTOR}")
    qweight_t = qweight_t.contiguous()
    out = torch.empty((k8 * PACK_FACTOR, n // PACK_FACTOR), dtype=torch.int32, device=qweight_t.device)
    with torch.cuda.device(qweight_t.device):
        status = _lib.lib().tf_awq_unrepack(
            qweight_t.data_ptr(), n, k8 * PACK_FACTOR, out.data_ptr(),
            _lib.stream_ptr(qweight_t.device),
        )  # fmt: skip
    _lib.check("tf_awq_unrepack", status)
    return out


def unpack_int4_cuda(packed: torch.Tensor) -> torch.Tensor:
    _require(packed, "packed")
    p = packed.contiguous()
    out = torch.empty((*p.shape[:-1], p.shape[-1] * PACK_FACTOR), dtype=torch.int32, device=p.device)
    with torch.cuda.device(p.device):
        status = _lib.lib().tf_unpack_int4(
            p.data_ptr(), p.numel(), out.data_ptr(), _lib.stream_ptr(p.device)
        )
    _lib.check("tf_unpack_int4", status)
    return out


def pack_int4_cuda(values: torch.Tensor) -> torch.Tensor:
    _require(values, "values")
    v = values.to(torch.int32).contiguous()
    if v.data_ptr() % _VEC:
        v = v.clone()
    out = torch.empty((*v.shape[:-1], v.shape[-1] // PACK_FACTOR), dtype=torch.int32, device=v.device)
    with torch.cuda.device(v.device):
        status = _lib.lib().tf_pack_int4(
            v.data_ptr(), out.numel(), out.data_ptr(), _lib.stream_ptr(v.device)
        )
    _lib.check("tf_pack_int4", status)
    return out


def cast_e4m3(values: torch.Tensor) -> torch.Tensor:
    """fp32 -> e4m3 with the quantizer's rounding (RNE, saturating, NaN kept)."""
    _require(values, "values")
    v = values.to(torch.float32).contiguous()
    out = torch.empty(v.shape, dtype=torch.float8_e4m3fn, device=v.device)
    with torch.cuda.device(v.device):
        status = _lib.lib().tf_cast_e4m3(v.data_ptr(), v.numel(), out.data_ptr(), _lib.stream_ptr(v.device))
    _lib.check("tf_cast_e4m3", status)
    return out


def e4m3_quant_rows(y: torch.Tensor, scale: torch.Tensor | None = None
                    ) -> tuple[torch.Tensor, torch.Tensor]:
    """e4m3(clamp(y / scale, -448, 448)) of fp16 activations [R, C] already normalised: the
    quantization step of ``rmsnorm_fp8_quant`` on its own (C ABI ``tf_e4m3_quant_rows``).
    ``scale``: one static fp32 value, one per row ([R] or [R, 1]), or None for the dynamic
    per-row scale max(amax / 448, 1 / (448 * 512)). Returns (codes, scale [R, 1] or the given
    scale)."""
    _require(y, "y")
    if y.dim() != 2 or y.dtype != torch.float16 or y.stride(1) != 1:
        raise ValueError(f"y must be fp16 [R, C] with unit stride along C, got {y.dtype} "
                         f"{tuple(y.shape)}")
    r, c = y.shape
    out = torch.empty((r, c), dtype=torch.float8_e4m3fn, device=y.device)
    ldy = y.stride(0) if r > 1 else c
    if scale is None:
        sc, stride = None, 0
        s_out = torch.empty((r, 1), dtype=torch.float32, device=y.device)
    else:
        sc = scale.reshape(-1)
        if sc.dtype != torch.float32 or sc.device != y.device or sc.numel() not in (1, r):
            raise ValueError(f"scale must be fp32 on {y.device} with 1 or {r} elements")
        sc, stride, s_out = sc.contiguous(), 0 if sc.numel() == 1 else 1, scale
    with torch.cuda.device(y.device):
        status = _lib.lib().tf_e4m3_quant_rows(
            y.data_ptr(), r, c, ldy, _lib.ptr(sc), stride, out.data_ptr(),
            s_out.data_ptr() if scale is None else None, _lib.stream_ptr(y.device))
    _lib.check("tf_e4m3_quant_rows", status)
    return out, s_out
